"""Pins the CPU oracle against the reference's own known-answer tests and golden vectors.

Every case cites the reference test it restates.  Tolerances are the
reference's: `assert_tensor` is |a-e| <= 1e-6*max(|e|,1) (tests/tensor_ops.rs:9-22).
"""
import math

import numpy as np
import pytest

import oracle
from tests import llama_host as lh

F32MAX = np.finfo(np.float32).max


def close(actual, expected, tol=1e-6):
    a = np.asarray(actual, dtype=np.float32).ravel()
    e = np.asarray(expected, dtype=np.float32).ravel()
    assert a.shape == e.shape
    assert np.all(np.isfinite(a))
    assert np.all(np.abs(a - e) <= tol * np.maximum(np.abs(e), 1.0)), (a, e)


# ---- matmul: tests/tensor_ops.rs:24-88 ---------------------------------------

def test_matmul_hand_values():
    close(oracle.matmul([[1, 2, 3], [4, 5, 6]], [[7, 8], [9, 10], [11, 12]]),
          [58, 64, 139, 154])
    close(oracle.matmul([[-3.0]], [[4.0]]), [-12])


def test_matmul_large_matches_f64_reference():
    rows, shared, cols = 96, 80, 64
    left = np.array([((i * 17 % 101) - 50.0) / 13.0 for i in range(rows * shared)],
                    dtype=np.float32).reshape(rows, shared)
    right = np.array([((i * 29 % 97) - 48.0) / 11.0 for i in range(shared * cols)],
                     dtype=np.float32).reshape(shared, cols)
    expected = (left.astype(np.float64) @ right.astype(np.float64)).astype(np.float32)
    close(oracle.matmul(left, right), expected, 3e-5)


def test_matmul_accumulates_sequentially_in_f32():
    # tests/tensor_ops.rs:80-84: 2^24 + 1 - 2^24 == 0 in sequential f32
    close(oracle.matmul([[16777216.0, 1.0, -16777216.0]], [[1.0], [1.0], [1.0]]), [0.0])


# ---- softmax: tests/tensor_ops.rs:304-438 ------------------------------------

LOW, MID, HIGH = 0.09003057, 0.24472848, 0.66524094


def test_softmax_hand_values():
    close(oracle.softmax(np.array([[1, 2, 3], [0, 0, 0]], np.float32), 1),
          [LOW, MID, HIGH, 1 / 3, 1 / 3, 1 / 3])
    close(oracle.softmax(np.array([[0, 2], [0, 2]], np.float32), 0), [0.5] * 4)


def test_softmax_middle_axis():
    x = np.array([0, 2, 1, 1, 2, 0, 2, 0, 1, 1, 0, 2], np.float32).reshape(2, 3, 2)
    close(oracle.softmax(x, 1),
          [LOW, HIGH, MID, MID, HIGH, LOW, HIGH, LOW, MID, MID, LOW, HIGH])


def test_softmax_stability_and_extremes():
    for vals in ([1000, 1001, 1002], [-1002, -1001, -1000]):
        close(oracle.softmax(np.array(vals, np.float32), 0), [LOW, MID, HIGH])
    close(oracle.softmax(np.array([-F32MAX, 0, F32MAX], np.float32), 0), [0, 0, 1])


def test_softmax_large_slice_matches_f64():
    vals = np.array([-((i % 113)) / 7.0 for i in range(16384)], dtype=np.float32)
    e = np.exp(vals.astype(np.float64))
    expected = (e / e.sum()).astype(np.float32)
    actual = oracle.softmax(vals, 0)
    close(actual, expected, 1e-9)
    assert abs(actual.astype(np.float64).sum() - 1.0) < 1e-7


def test_softmax_infinities():
    ninf, pinf = -np.inf, np.inf
    close(oracle.softmax(np.array([[ninf, 0], [ninf, 0]], np.float32), 0), [0.5] * 4)
    close(oracle.softmax(np.array([0, ninf, 0], np.float32), 0), [0.5, 0, 0.5])
    close(oracle.softmax(np.array([[pinf, 2, pinf], [0, pinf, ninf]], np.float32), 1),
          [0.5, 0, 0.5, 0, 1, 0])
    close(oracle.softmax(np.array([[-3.0], [8.0]], np.float32), 1), [1, 1])


def test_softmax_rejects_nan_and_bad_axis():
    for vals in ([0, np.nan], [np.inf, np.nan]):
        with pytest.raises(oracle.OracleError, match="NaN"):
            oracle.softmax(np.array(vals, np.float32), 0)
    with pytest.raises(oracle.OracleError, match="out of bounds"):
        oracle.softmax(np.ones((2, 3), np.float32), 2)


# ---- rope: tests/tensor_ops.rs:670-801, 897-999; tests/transformer_layers.rs:541-582 ----

def test_rope_position_zero_is_identity():
    x = np.array([[1, 2, 3, 4]], np.float32)
    close(oracle.rope(x, 4, 0, 10000.0), x)
    big = np.array([[F32MAX, -F32MAX]], np.float32)
    assert np.array_equal(oracle.rope(big, 2, 0, 10000.0), big)


def test_rope_interleaved_pairs_hand_values():
    close(oracle.rope(np.array([[1, 0, 0, 1]], np.float32), 4, 1, 100.0),
          [0.5403023, 0.84147096, -0.099833414, 0.9950042])


def test_rope_multisequence_multihead():
    x = np.array([1, 0, 0, 1, 0, 1, 1, 0, 1, 0, 0, 1, 0, 1, 1, 0], np.float32).reshape(2, 2, 4)
    close(oracle.rope(x, 4, 1, 100.0),
          [0.5403023, 0.84147096, -0.099833414, 0.9950042, -0.84147096, 0.5403023, 0.9950042,
           0.099833414, -0.41614684, 0.9092974, -0.19866933, 0.9800666, -0.9092974,
           -0.41614684, 0.9800666, 0.19866933])


def test_rope_flattens_intermediate_dims():
    x = np.array([1, 0, 1, 0, 1, 0, 1, 0], np.float32).reshape(1, 2, 2, 2)
    close(oracle.rope(x, 2, 1, 10000.0), [0.5403023, 0.84147096] * 4)


def test_rope_preserves_pair_magnitudes():
    x = np.array([(i % 31) - 15.0 for i in range(32 * 3 * 8)], np.float32).reshape(32, 3, 8)
    y = oracle.rope(x, 8, 123, 10000.0)
    b = x.reshape(-1, 2).astype(np.float64)
    a = y.reshape(-1, 2).astype(np.float64)
    nb, na = (b ** 2).sum(1), (a ** 2).sum(1)
    assert np.all(np.abs(nb - na) <= 2e-7 * np.maximum(nb, 1.0))


def _llama_normal(x, hd, pos, theta):
    out = []
    for s, chunk in enumerate(x.reshape(-1, hd)):
        p = float(pos + s)
        for i in range(hd // 2):
            f = theta ** (-2.0 * i / hd)
            sn, cs = math.sin(p * f), math.cos(p * f)
            a, b = float(chunk[2 * i]), float(chunk[2 * i + 1])
            out += [a * cs - b * sn, a * sn + b * cs]
    return np.array(out, np.float32)


def _hf_rotate_half(x, hd, pos, theta):
    out = np.zeros(x.size, np.float32)
    half = hd // 2
    for s, chunk in enumerate(x.reshape(-1, hd)):
        p = float(pos + s)
        for i in range(half):
            f = theta ** (-2.0 * i / hd)
            sn, cs = math.sin(p * f), math.cos(p * f)
            a, b = float(chunk[i]), float(chunk[i + half])
            out[s * hd + i] = a * cs - b * sn
            out[s * hd + i + half] = a * sn + b * cs
    return out


def test_rope_matches_llamacpp_normal_and_rejects_rotate_half():
    x = np.arange(1, 17, dtype=np.float32).reshape(2, 8)
    close(oracle.rope(x, 8, 1, 10000.0), _llama_normal(x, 8, 1, 10000.0))
    x = np.array([[-2.0, 0.33333334, -1.6666667, 0.6666667, -1.3333334, 1.0, -1.0, 1.3333334]],
                 np.float32)
    y = oracle.rope(x, 8, 1, 10000.0)
    normal, neox = _llama_normal(x, 8, 1, 10000.0), _hf_rotate_half(x, 8, 1, 10000.0)
    assert np.abs(normal - neox).max() > 0.5
    close(y, normal)
    assert np.abs(y.ravel() - neox).max() > 0.5


def test_rope_attention_pairing_kat():
    # tests/transformer_layers.rs:541-582
    y = oracle.rope(np.array([[1, 2, 3, 4]], np.float32), 4, 1, 10000.0).ravel()
    c1, s1, c2, s2 = math.cos(1), math.sin(1), math.cos(0.01), math.sin(0.01)
    exp = [c1 - 2 * s1, s1 + 2 * c1, 3 * c2 - 4 * s2, 3 * s2 + 4 * c2]
    assert np.all(np.abs(y - np.array(exp, np.float32)) <= 1e-6)
    assert abs(y[1] - (2 * c2 - 4 * s2)) > 1e-3


def test_rope_validation():
    with pytest.raises(oracle.OracleError):
        oracle.rope(np.ones((2, 3), np.float32), 3, 0, 100.0)
    for theta in (0.0, -1.0, float("nan"), float("inf"), float("-inf")):
        with pytest.raises(oracle.OracleError, match="theta"):
            oracle.rope(np.ones((1, 2), np.float32), 2, 0, theta)
    y = oracle.rope(np.ones((1, 4), np.float32), 4, 1, float(np.float32(1e-45)))
    assert np.all(np.isfinite(y))
    assert np.all(np.isnan(oracle.rope(np.array([[np.nan, 1]], np.float32), 2, 1, 100.0)))


def test_rope_against_numpy_reference_golden(golden):
    """scripts/numpy_forward_reference.py rope/rotate_rows on the bench head sizes."""
    i = 0
    while f"rope/{i}/x" in golden.files:
        x = golden[f"rope/{i}/x"]
        hd, start = (int(v) for v in golden[f"rope/{i}/params"])
        theta = float(golden[f"rope/{i}/theta"][0])
        y = oracle.rope(x, hd, start, theta)
        ref = golden[f"rope/{i}/y"].astype(np.float32)
        # f64 rotation cast to f32 on both sides: within one f32 ulp.
        assert np.all(np.abs(y - ref) <= 2.5e-7 * np.maximum(np.abs(ref), 1.0)), i
        i += 1
    assert i >= 5


# ---- mask: src/transformer/layers.rs:509-531 ---------------------------------

def test_causal_mask_offset():
    s = oracle.causal_mask_offset(np.zeros((2, 5), np.float32), 2)
    assert np.isneginf(s[0, 3:]).all() and (s[0, :3] == 0).all()
    assert np.isneginf(s[1, 4:]).all() and (s[1, :4] == 0).all()
    with pytest.raises(oracle.OracleError, match="cannot cover"):
        oracle.causal_mask_offset(np.zeros((2, 3), np.float32), 2)


# ---- element formats ---------------------------------------------------------

def test_f16_and_bf16_rounding_match_numpy_and_torch():
    import torch

    rng = np.random.default_rng(7)
    bits = rng.integers(0, 2 ** 32, size=20000, dtype=np.uint64).astype(np.uint32)
    x = bits.view(np.float32)
    x = x[np.isfinite(x)]
    special = np.array([65504, 65519.99, 65520, 6.1e-5, 5.96e-8, 2.98e-8, 2.9802322e-08,
                        1e-8, -0.0, 0.0, 1.0, -2.5, 3.0e38], np.float32)
    x = np.concatenate([x, special, rng.normal(0, 1, 4000).astype(np.float32)])
    assert np.array_equal(oracle.f32_to_f16_bits(x), x.astype(np.float16).view(np.uint16))
    tb = torch.from_numpy(x.copy()).to(torch.bfloat16).view(torch.int16).numpy().view(np.uint16)
    assert np.array_equal(oracle.f32_to_bf16_bits(x), tb)


def test_q8_0_quantizer_rules():
    x = np.zeros(64, np.float32)
    x[:32] = np.linspace(-3, 3, 32)
    x[40] = 0.5
    qs, sc = oracle.q8_0_quantize(x)
    d = np.float32(3.0) / np.float32(127.0)
    assert sc[0] == np.float16(d).view(np.uint16)
    assert qs[0] == -127 and qs[31] == 127
    assert sc[1] == np.float16(np.float32(0.5) / np.float32(127)).view(np.uint16)
    assert qs[40] == 127 and np.count_nonzero(qs[32:]) == 1
    # round half away from zero: 63.5 -> 64 when id*x lands exactly on .5
    y = np.zeros(32, np.float32)
    y[0], y[1] = 127.0, 63.5
    q, _ = oracle.q8_0_quantize(y)
    assert q[1] == 64
    back = oracle.store_roundtrip(oracle.Q8_0, x, 32)
    assert np.abs(back - x).max() <= 3.0 / 127 / 2 + 1e-6


# ---- KvCache: tests/kv_cache.rs (all cases) ----------------------------------

def staged(n, heads, dim, offset):
    t = np.empty((n, heads, dim), np.float32)
    for i in range(n):
        for h in range(heads):
            for d in range(dim):
                t[i, h, d] = (offset + i) * 100 + h * 10 + d
    return t


def assert_k_at(cache, layer, positions, heads, dim):
    k, v = cache.get(layer, positions)
    assert k.shape == (len(positions), heads, dim) and v.shape == k.shape
    for r, p in enumerate(positions):
        exp = staged(1, heads, dim, p)[0]
        assert np.array_equal(k[r], exp) and np.array_equal(v[r], exp)


def test_kv_update_get_append_clear():
    c = oracle.KvCache(2, 16, 4, 8)
    c.update(0, staged(3, 4, 8, 0), staged(3, 4, 8, 0), [0, 1, 2])
    assert c.seq_len() == 3
    assert_k_at(c, 0, [0, 1, 2], 4, 8)
    c = oracle.KvCache(1, 16, 2, 4)
    c.update(0, staged(2, 2, 4, 0), staged(2, 2, 4, 0), [0, 1])
    c.update(0, staged(2, 2, 4, 2), staged(2, 2, 4, 2), [2, 3])
    assert c.seq_len() == 4
    assert_k_at(c, 0, [0, 1, 2, 3], 2, 4)
    k, v = c.get(0, [])
    assert k.shape == (0, 2, 4)
    c.clear()
    assert c.seq_len() == 0
    with pytest.raises(oracle.OracleError, match="written prefix"):
        c.get(0, [0])
    c.update(0, staged(1, 2, 4, 0), staged(1, 2, 4, 0), [0])
    assert c.seq_len() == 1


def test_kv_update_rejections():
    c = oracle.KvCache(1, 8, 2, 4)
    good = staged(1, 2, 4, 0)
    with pytest.raises(oracle.OracleError) as e:
        c.update(0, staged(1, 4, 4, 0), good, [0])
    assert "[1, 4, 4]" in str(e.value) and "[_, 2, 4]" in str(e.value)
    for k, v in ((staged(1, 2, 6, 0), good), (good, staged(1, 2, 6, 0)),
                 (np.ones((2, 4), np.float32), good)):
        with pytest.raises(oracle.OracleError):
            c.update(0, k, v, [0])
    with pytest.raises(oracle.OracleError) as e:
        c.update(0, staged(2, 2, 4, 0), staged(2, 2, 4, 0), [0])
    assert "2 token(s)" in str(e.value) and "1 position" in str(e.value)
    c.update(0, staged(2, 2, 4, 0), staged(2, 2, 4, 0), [0, 1])
    for pos in ([3], [1], [0]):
        with pytest.raises(oracle.OracleError, match="must continue"):
            c.update(0, good, good, pos)
    with pytest.raises(oracle.OracleError):
        c.update(0, staged(2, 2, 4, 0), staged(2, 2, 4, 0), [2, 4])
    assert c.seq_len() == 2


def test_kv_capacity_negative_and_layers():
    c = oracle.KvCache(1, 4, 2, 4)
    c.update(0, staged(4, 2, 4, 0), staged(4, 2, 4, 0), [0, 1, 2, 3])
    with pytest.raises(oracle.OracleError, match="capacity 4"):
        c.update(0, staged(1, 2, 4, 0), staged(1, 2, 4, 0), [4])
    f = oracle.KvCache(1, 4, 2, 4)
    for pos in ([99], [-1]):
        with pytest.raises(oracle.OracleError):
            f.update(0, staged(1, 2, 4, 0), staged(1, 2, 4, 0), pos)
    c = oracle.KvCache(1, 8, 2, 4)
    with pytest.raises(oracle.OracleError) as e:
        c.update(1, staged(1, 2, 4, 0), staged(1, 2, 4, 0), [0])
    assert "layer index 1" in str(e.value) and "1 layers" in str(e.value)


def test_kv_failed_update_is_transactional():
    c = oracle.KvCache(1, 8, 2, 4)
    c.update(0, staged(2, 2, 4, 0), staged(2, 2, 4, 0), [0, 1])
    with pytest.raises(oracle.OracleError):
        c.update(0, staged(1, 4, 4, 0), staged(1, 2, 4, 0), [2])
    assert c.seq_len() == 2
    with pytest.raises(oracle.OracleError):
        c.get(0, [2])
    assert_k_at(c, 0, [0, 1], 2, 4)
    c.update(0, staged(1, 2, 4, 2), staged(1, 2, 4, 2), [2])
    assert c.seq_len() == 3
    assert_k_at(c, 0, [0, 1, 2], 2, 4)


def test_kv_get_rejections_layers_independent_and_order():
    c = oracle.KvCache(2, 8, 2, 4)
    c.update(0, staged(2, 2, 4, 0), staged(2, 2, 4, 0), [0, 1])
    for pos in ([-1], [8], [2]):
        with pytest.raises(oracle.OracleError):
            c.get(0, pos)
    with pytest.raises(oracle.OracleError, match="layer index 2"):
        c.get(2, [0])
    c.update(1, staged(1, 2, 4, 0), staged(1, 2, 4, 0), [0])
    assert c.seq_len() == 2
    assert_k_at(c, 1, [0], 2, 4)
    with pytest.raises(oracle.OracleError):
        c.get(1, [1])
    c = oracle.KvCache(1, 8, 2, 4)
    c.update(0, staged(3, 2, 4, 0), staged(3, 2, 4, 0), [0, 1, 2])
    assert_k_at(c, 0, [2, 0], 2, 4)
    assert_k_at(c, 0, [1, 1], 2, 4)


def test_kv_no_layers_clear_all_layers_empty_batch():
    c = oracle.KvCache(0, 8, 2, 4)
    assert c.seq_len() == 0
    with pytest.raises(oracle.OracleError):
        c.get(0, [0])
    with pytest.raises(oracle.OracleError):
        c.update(0, staged(1, 2, 4, 0), staged(1, 2, 4, 0), [0])
    c = oracle.KvCache(2, 8, 2, 4)
    c.update(0, staged(3, 2, 4, 0), staged(3, 2, 4, 0), [0, 1, 2])
    c.update(1, staged(1, 2, 4, 0), staged(1, 2, 4, 0), [0])
    c.clear()
    for layer in (0, 1):
        with pytest.raises(oracle.OracleError):
            c.get(layer, [0])
        c.update(layer, staged(1, 2, 4, 0), staged(1, 2, 4, 0), [0])
    assert c.seq_len() == 1
    c = oracle.KvCache(1, 8, 2, 4)
    c.update(0, staged(2, 2, 4, 0), staged(2, 2, 4, 0), [0, 1])
    c.update(0, staged(0, 2, 4, 0), staged(0, 2, 4, 0), [])
    assert c.seq_len() == 2
    assert_k_at(c, 0, [0, 1], 2, 4)


# ---- attention: tests/transformer_layers.rs:355-538 ---------------------------

def _attn_full(x_q, x_k, x_v, hq, hkv, hd, start=0, theta=10000.0):
    n = x_q.shape[0]
    return oracle.attention_full(x_q.reshape(n, hq, hd), x_k.reshape(n, hkv, hd),
                                 x_v.reshape(n, hkv, hd), start, hq, hkv, hd, theta)


def test_attention_hand_cases():
    x = np.array([[1, 2, 3, 4]], np.float32)
    # single token identity; head columns in place (:355-411)
    assert _attn_full(x, x, x, 2, 2, 2).ravel().tolist() == [1, 2, 3, 4]
    # GQA sharing (:460-489): kv head = first two features of x
    kv = x[:, :2]
    assert _attn_full(x, kv, kv, 2, 1, 2).ravel().tolist() == [1, 2, 1, 2]
    # causal masking (:413-458)
    f = _attn_full(*(np.array([[1, 0], [7, 9]], np.float32),) * 3, 1, 1, 2)
    s = _attn_full(*(np.array([[1, 0], [-3, 5]], np.float32),) * 3, 1, 1, 2)
    assert f[0].tolist() == [1, 0] and f[0].tolist() == s[0].tolist()
    assert f[1].tolist() != s[1].tolist()
    w = _attn_full(*(np.array([[10, 0], [1, 1]], np.float32),) * 3, 1, 1, 2)
    st = _attn_full(*(np.array([[20, 0], [1, 1]], np.float32),) * 3, 1, 1, 2)
    assert w[1].tolist() != st[1].tolist()


def _lcg_matrix(rows, cols, seed):
    state = seed
    out = np.empty((rows, cols), np.float64)
    for r in range(rows):
        for c in range(cols):
            state = (state * 6364136223846793005 + 1442695040888963407) % (1 << 64)
            out[r, c] = (state >> 40) / float(1 << 24) - 0.5
    return out


def _f64_reference_attention(x, wq, wk, wv, wo, hq, hkv, hd, start, theta):
    """Restates tests/transformer_layers.rs:808-898 (independent f64 attention)."""
    n = x.shape[0]
    q, k, v = x @ wq.T, x @ wk.T, x @ wv.T

    def rotate(t, heads):
        t = t.copy()
        for p in range(n):
            for h in range(heads):
                for i in range(hd // 2):
                    f = theta ** (-2.0 * i / hd)
                    sn, cs = math.sin((start + p) * f), math.cos((start + p) * f)
                    a, b = t[p, h * hd + 2 * i], t[p, h * hd + 2 * i + 1]
                    t[p, h * hd + 2 * i], t[p, h * hd + 2 * i + 1] = a * cs - b * sn, a * sn + b * cs
        return t

    q, k = rotate(q, hq), rotate(k, hkv)
    group, scale = hq // hkv, 1.0 / math.sqrt(hd)
    merged = np.zeros((n, hq * hd))
    for h in range(hq):
        kvh = h // group
        for i in range(n):
            sc = np.array([q[i, h * hd:(h + 1) * hd] @ k[j, kvh * hd:(kvh + 1) * hd] * scale
                           if j <= i else -np.inf for j in range(n)])
            e = np.exp(sc - sc.max())
            merged[i, h * hd:(h + 1) * hd] = (e / e.sum()) @ v[:, kvh * hd:(kvh + 1) * hd]
    return merged @ wo.T


@pytest.mark.parametrize("seq,hidden,hq,hkv,start", [(2, 4, 2, 2, 0), (3, 4, 2, 1, 0),
                                                     (2, 6, 3, 3, 2)])
def test_attention_matches_independent_f64_reference(seq, hidden, hq, hkv, start):
    hd = hidden // hq
    wq = _lcg_matrix(hidden, hidden, 0x51AA0001).astype(np.float32)
    wk = _lcg_matrix(hkv * hd, hidden, 0x51AA0002).astype(np.float32)
    wv = _lcg_matrix(hkv * hd, hidden, 0x51AA0003).astype(np.float32)
    wo = _lcg_matrix(hidden, hidden, 0x51AA0004).astype(np.float32)
    x = _lcg_matrix(seq, hidden, 0x51AA0005).astype(np.float32)
    q, k, v = lh.linear(x, wq), lh.linear(x, wk), lh.linear(x, wv)
    a = oracle.attention_full(q.reshape(seq, hq, hd), k.reshape(seq, hkv, hd),
                              v.reshape(seq, hkv, hd), start, hq, hkv, hd, 10000.0)
    out = lh.linear(a, wo)
    exp = _f64_reference_attention(x.astype(np.float64), wq.astype(np.float64),
                                   wk.astype(np.float64), wv.astype(np.float64),
                                   wo.astype(np.float64), hq, hkv, hd, start, 10000.0)
    assert np.abs(out - exp.astype(np.float32)).max() <= 1e-4


def test_attention_rejects_bad_heads():
    x = np.ones((1, 3, 2), np.float32)
    with pytest.raises(oracle.OracleError, match="divisible"):
        oracle.attention_full(x, np.ones((1, 2, 2), np.float32), np.ones((1, 2, 2), np.float32),
                              0, 3, 2, 2, 10000.0)


# ---- cached path: tests/transformer_forward.rs:665-946 -----------------------

def _rand_qkv(rng, n, hq, hkv, hd):
    return (rng.normal(0, 1, (n, hq, hd)).astype(np.float32),
            rng.normal(0, 1, (n, hkv, hd)).astype(np.float32),
            rng.normal(0, 1, (n, hkv, hd)).astype(np.float32))


@pytest.mark.parametrize("hq,hkv", [(2, 2), (4, 2)])
def test_cached_prefill_is_bit_identical_and_splits_match(hq, hkv):
    rng = np.random.default_rng(3)
    hd, n = 8, 5
    q, k, v = _rand_qkv(rng, n, hq, hkv, hd)
    full = oracle.attention_full(q, k, v, 0, hq, hkv, hd, 10000.0)
    c = oracle.KvCache(1, 16, hkv, hd)
    cached = oracle.attention_with_cache(c, 0, q, k, v, 0, hq, hkv, hd, 10000.0)
    assert np.array_equal(cached, full)  # transformer_forward.rs:751-769
    assert c.seq_len() == n
    for splits in ([1, 1, 1, 1, 1], [1, 2, 2], [2, 3], [3, 1, 1], [5], [4, 1]):
        c = oracle.KvCache(1, 16, hkv, hd)
        rows, pos = [], 0
        for b in splits:
            rows.append(oracle.attention_with_cache(c, 0, q[pos:pos + b], k[pos:pos + b],
                                                    v[pos:pos + b], pos, hq, hkv, hd, 10000.0))
            pos += b
        got = np.concatenate(rows)
        assert np.abs(got - full).max() <= 1e-5, splits  # PATH_TOLERANCE


def test_cached_repeated_prefill_and_empty_batch():
    rng = np.random.default_rng(4)
    q, k, v = _rand_qkv(rng, 3, 2, 2, 4)
    c = oracle.KvCache(1, 8, 2, 4)
    oracle.attention_with_cache(c, 0, q, k, v, 0, 2, 2, 4, 10000.0)
    with pytest.raises(oracle.OracleError, match="must continue"):
        oracle.attention_with_cache(c, 0, q, k, v, 0, 2, 2, 4, 10000.0)
    assert c.seq_len() == 3
    e = oracle.attention_with_cache(c, 0, q[:0], k[:0], v[:0], 3, 2, 2, 4, 10000.0)
    assert e.shape == (0, 8) and c.seq_len() == 3
    nxt = oracle.attention_with_cache(c, 0, q[:1], k[:1], v[:1], 3, 2, 2, 4, 10000.0)
    assert nxt.shape == (1, 8) and c.seq_len() == 4


# ---- end to end against the reference's golden logits --------------------------

def test_tiny_llama_expected_logits(golden):
    """tests/transformer_from_gguf.rs:148-182: EXPECTED_LOGITS at 1e-4, every row."""
    model = lh.tiny_from_golden(golden)
    for tag in ("a", "b"):
        ids = golden[f"tiny/ids_{tag}"]
        ref = golden[f"tiny/logits_{tag}"]
        full = model.forward(ids, 0, lh.oracle_full_attend(model))
        assert np.abs(full - ref).max() <= 1e-4
        cache = oracle.KvCache(model.n_layers, 128, model.n_kv, model.hd)
        rows, pos = [], 0
        for b in ([1] * len(ids) if tag == "a" else [4, 1, 3, 1, 2]):
            rows.append(model.forward(ids[pos:pos + b], pos, lh.oracle_cached_attend(model, cache)))
            pos += b
        assert np.abs(np.concatenate(rows) - ref).max() <= 1e-4
    exp_head = [0.241964, 0.266576, -0.563725, 0.346897, -0.285221, 0.133072]
    assert np.abs(golden["tiny/logits_a"][-1][:6] - np.array(exp_head)).max() <= 1e-6


def test_numpy_reference_forward_golden(golden):
    """scripts/numpy_forward_reference.py forward (f64) vs the f32 restatement, 1e-3."""
    model = lh.npref_from_golden(golden)
    ids = golden["npref/ids"]
    ref = golden["npref/logits"]
    cache = oracle.KvCache(model.n_layers, 64, model.n_kv, model.hd)
    rows, pos = [], 0
    for b in (6, 1, 1, 3, 2):
        rows.append(model.forward(ids[pos:pos + b], pos, lh.oracle_cached_attend(model, cache)))
        pos += b
    got = np.concatenate(rows)
    assert np.abs(got - ref).max() <= 1e-3
