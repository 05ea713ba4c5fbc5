"""Parity of the CUDA path (through the C ABI) with the CPU oracle.

Tolerances (max-abs on attention outputs, against the oracle run on the same
rounded inputs and the same cache storage format):
  f16 / bf16 KV: 2e-3;  Q8_0 KV: 2e-3 against the oracle on the dequantised
  cache and 1e-2 against the oracle on the unquantised values.
Integer/byte work (cache contents after append, Q8_0 quantisation) is bit-exact.
"""
import zlib

import numpy as np
import pytest
import torch

import oracle
import qllama_b200 as qb
from tests import gpu_util as gu
from tests import llama_host as lh

pytestmark = pytest.mark.gpu

TOL_16 = 2e-3
TOL_Q8_DEQ = 2e-3
TOL_Q8_RAW = 1e-2


@pytest.fixture(scope="module")
def ctx():
    return qb.Context(0)


# ---- KvCache contract on the device (tests/kv_cache.rs) ------------------------

def staged(n, heads, dim, offset):
    i = np.arange(n)[:, None, None] + offset
    h = np.arange(heads)[None, :, None]
    d = np.arange(dim)[None, None, :]
    return (i * 100 + h * 10 + d).astype(np.float32)


@pytest.mark.parametrize("storage", ["f32", "f16"])
def test_device_kv_cache_contract(ctx, storage):
    c = qb.KvCache(ctx, 2, 16, 4, 8, storage, max_batch=2)
    c.update(0, staged(3, 4, 8, 0), staged(3, 4, 8, 0), [0, 1, 2])
    assert c.seq_len() == 3
    k, v = c.get(0, [0, 1, 2])
    assert np.array_equal(k, staged(3, 4, 8, 0)) and np.array_equal(v, k)
    c.update(0, staged(2, 4, 8, 3), staged(2, 4, 8, 3), [3, 4])
    k, _ = c.get(0, [4, 0, 4])
    assert np.array_equal(k[0], staged(1, 4, 8, 4)[0]) and np.array_equal(k[1], staged(1, 4, 8, 0)[0])
    assert np.array_equal(k[2], k[0])
    with pytest.raises(qb.QllamaError, match="must continue"):
        c.update(0, staged(1, 4, 8, 0), staged(1, 4, 8, 0), [7])
    with pytest.raises(qb.QllamaError) as e:
        c.update(0, staged(1, 2, 8, 0), staged(1, 2, 8, 0), [5])
    assert "[1, 2, 8]" in str(e.value) and "[_, 4, 8]" in str(e.value)
    with pytest.raises(qb.QllamaError, match="2 token"):
        c.update(0, staged(2, 4, 8, 0), staged(2, 4, 8, 0), [5])
    with pytest.raises(qb.QllamaError, match="layer index 2"):
        c.get(2, [0])
    with pytest.raises(qb.QllamaError, match="written prefix"):
        c.get(0, [5])
    assert c.seq_len() == 5 and c.layer_len(1) == 0
    c.update(0, staged(0, 4, 8, 0), staged(0, 4, 8, 0), [])
    assert c.seq_len() == 5
    # capacity (16): fill to the end, then one more must fail
    c.update(0, staged(11, 4, 8, 5), staged(11, 4, 8, 5), list(range(5, 16)))
    with pytest.raises(qb.QllamaError, match="capacity 16"):
        c.update(0, staged(1, 4, 8, 16), staged(1, 4, 8, 16), [16])
    c.clear()
    assert c.seq_len() == 0
    with pytest.raises(qb.QllamaError, match="written prefix"):
        c.get(0, [0])
    # sequence slots are independent
    c.update(0, staged(2, 4, 8, 0), staged(2, 4, 8, 0), [0, 1], seq=1)
    assert c.seq_len(1) == 2 and c.seq_len(0) == 0


@pytest.mark.parametrize("storage", ["f32", "f16", "bf16", "q8_0"])
def test_append_and_quantisation_bit_exact(ctx, storage):
    """Rows written by update() and by the fused append read back exactly as the oracle stores them."""
    rng = np.random.default_rng(11)
    hkv, hd, hq, theta = 2, 64, 8, 10000.0
    p = gu.Pair(ctx, storage, 1, 256, hkv, hd, 1)
    p.prefill_rows(rng, 0, 0, 70, theta)
    # one prefill chunk and two decode steps through the operator (RoPE inside)
    for n in (5, 1, 1):
        start = p.gpu.seq_len(0)
        q, k, v = (gu.normal(rng, (1, n, h, hd)) for h in (hq, hkv, hkv))
        qb.attention_forward(p.gpu, 0, gu.to_device(q, "f32"), gu.to_device(k, "f32"),
                             gu.to_device(v, "f32"), [start], hq, hkv, hd, theta)
        p.oracle_forward(0, q, k, v, [start], hq, theta)
    L = p.gpu.seq_len(0)
    assert L == 77
    kg, vg = p.gpu.get(0, np.arange(L))
    ko, vo = p.orc[0].get(0, np.arange(L))
    assert np.array_equal(kg.view(np.uint32), ko.view(np.uint32))
    assert np.array_equal(vg.view(np.uint32), vo.view(np.uint32))


CASES = [
    # storage, in_dtype, hd, hq, hkv, lens
    ("f16", "f16", 128, 32, 32, [1, 63, 64, 65, 700]),
    ("f16", "f32", 128, 8, 1, [129, 2000]),
    ("f16", "f16", 64, 32, 4, [5, 511, 767]),
    ("bf16", "bf16", 128, 32, 8, [1, 100, 1500]),
    ("bf16", "bf16", 64, 16, 4, [3, 333]),
    ("q8_0", "f16", 128, 64, 8, [1, 64, 1000, 3000]),
    ("q8_0", "bf16", 128, 16, 16, [17, 900]),
    # one sequence: a cluster of one-tile CTAs (more than 8, merged 16 wide)
    ("f16", "f16", 64, 32, 4, [700]),
    # one long sequence: clustered CTAs of several tiles (next tile's QK^T issued early)
    ("bf16", "bf16", 64, 32, 4, [4000]),
    # few long sequences at head_dim 128: the wide kernel (two groups per CTA)
    ("f16", "f16", 128, 32, 8, [6000, 5000]),
]


@pytest.mark.parametrize("storage,in_dt,hd,hq,hkv,lens", CASES)
def test_decode_parity(ctx, storage, in_dt, hd, hq, hkv, lens):
    rng = np.random.default_rng(zlib.crc32(repr((storage, in_dt, hd, hq, hkv)).encode()))
    theta, B = 10000.0, len(lens)
    p = gu.Pair(ctx, storage, 1, max(lens) + 8, hkv, hd, B)
    for s, L in enumerate(lens):
        p.prefill_rows(rng, 0, s, L - 1, theta)  # the step appends position L-1
    starts = np.array([L - 1 for L in lens])
    for _ in range(2):  # two consecutive decode steps
        q = gu.rounded(gu.normal(rng, (B, 1, hq, hd)), in_dt)
        k = gu.rounded(gu.normal(rng, (B, 1, hkv, hd)), in_dt)
        v = gu.rounded(gu.normal(rng, (B, 1, hkv, hd)), in_dt)
        out = qb.attention_forward(p.gpu, 0, gu.to_device(q, in_dt), gu.to_device(k, in_dt),
                                   gu.to_device(v, in_dt), starts, hq, hkv, hd, theta)
        torch.cuda.synchronize()
        ref = p.oracle_forward(0, q, k, v, starts, hq, theta)
        err = gu.max_err(out, ref)
        tol = TOL_Q8_DEQ if storage == "q8_0" else TOL_16
        assert err <= tol, (storage, err)
        starts = starts + 1
    p.gpu.ctx.synchronize()


def test_q8_0_against_unquantised_oracle(ctx):
    rng = np.random.default_rng(5)
    hd, hq, hkv, theta, lens = 128, 64, 8, 10000.0, [2048, 300]
    q8 = gu.Pair(ctx, "q8_0", 1, 2100, hkv, hd, len(lens))
    raw = [oracle.KvCache(1, 2100, hkv, hd, oracle.F32) for _ in lens]
    for s, L in enumerate(lens):
        k = gu.normal(rng, (L - 1, hkv, hd))
        v = gu.normal(rng, (L - 1, hkv, hd))
        kr = oracle.rope(k, hd, 0, theta)
        q8.gpu.update(0, kr, v, np.arange(L - 1), seq=s)
        raw[s].update(0, kr, v, np.arange(L - 1))
    q = gu.normal(rng, (2, 1, hq, hd))
    k = gu.normal(rng, (2, 1, hkv, hd))
    v = gu.normal(rng, (2, 1, hkv, hd))
    starts = [L - 1 for L in lens]
    out = qb.attention_forward(q8.gpu, 0, gu.to_device(q, "f32"), gu.to_device(k, "f32"),
                               gu.to_device(v, "f32"), starts, hq, hkv, hd, theta)
    ref = np.stack([oracle.attention_with_cache(raw[b], 0, q[b], k[b], v[b], starts[b], hq, hkv,
                                                hd, theta) for b in range(2)])
    assert gu.max_err(out, ref) <= TOL_Q8_RAW


@pytest.mark.parametrize("storage,hd,hq,hkv", [("f16", 128, 32, 8), ("bf16", 64, 32, 4),
                                              ("q8_0", 128, 16, 2), ("f16", 64, 8, 8)])
def test_prefill_chunks_parity(ctx, storage, hd, hq, hkv):
    """Multi-token batches at zero and non-zero start (tests/transformer_forward.rs:772-850)."""
    rng = np.random.default_rng(hd + hq)
    theta, B = 500000.0, 3
    p = gu.Pair(ctx, storage, 2, 512, hkv, hd, B)
    starts = np.zeros(B, np.int64)
    for n in (37, 1, 64, 5):
        q = gu.rounded(gu.normal(rng, (B, n, hq, hd)), "bf16")
        k = gu.rounded(gu.normal(rng, (B, n, hkv, hd)), "bf16")
        v = gu.rounded(gu.normal(rng, (B, n, hkv, hd)), "bf16")
        out = qb.attention_forward(p.gpu, 1, gu.to_device(q, "bf16"), gu.to_device(k, "bf16"),
                                   gu.to_device(v, "bf16"), starts, hq, hkv, hd, theta)
        ref = p.oracle_forward(1, q, k, v, starts, hq, theta)
        tol = TOL_Q8_DEQ if storage == "q8_0" else TOL_16
        assert gu.max_err(out, ref) <= tol, n
        starts = starts + n
    assert p.gpu.layer_len(1, 2) == 107 and p.gpu.layer_len(0, 2) == 0


def test_generic_f32_path_tracks_reference_bits(ctx):
    """f32 cache, head_dim 48 (the generic kernel): reference op order on the GPU."""
    rng = np.random.default_rng(9)
    hd, hq, hkv, theta = 48, 6, 6, 10000.0
    p = gu.Pair(ctx, "f32", 1, 256, hkv, hd, 2)
    starts = np.zeros(2, np.int64)
    exact = total = 0
    for n in (32, 1, 1, 3):
        q, k, v = (gu.normal(rng, (2, n, h, hd)) for h in (hq, hkv, hkv))
        out = qb.attention_forward(p.gpu, 0, q, k, v, starts, hq, hkv, hd, theta)
        ref = p.oracle_forward(0, q, k, v, starts, hq, theta)
        assert np.abs(out - ref).max() <= 1e-6
        exact += int((out.view(np.uint32) == ref.view(np.uint32)).sum())
        total += out.size
        starts = starts + n
    assert exact >= 0.999 * total, (exact, total)


def test_host_buffers_round_trip(ctx):
    """QL_MEM_HOST: numpy in, numpy out, copies inside the call."""
    rng = np.random.default_rng(1)
    hd, hq, hkv, theta = 128, 16, 2, 10000.0
    p = gu.Pair(ctx, "f16", 1, 600, hkv, hd, 1)
    p.prefill_rows(rng, 0, 0, 500, theta)
    q, k, v = (gu.rounded(gu.normal(rng, (1, 1, h, hd)), "f16").astype(np.float16)
               for h in (hq, hkv, hkv))
    out = qb.attention_forward(p.gpu, 0, q, k, v, [500], hq, hkv, hd, theta)
    assert isinstance(out, np.ndarray) and out.shape == (1, 1, hq * hd)
    ref = p.oracle_forward(0, q.astype(np.float32), k.astype(np.float32), v.astype(np.float32),
                           [500], hq, theta)
    assert np.abs(out - ref).max() <= TOL_16


def test_operator_errors_are_transactional(ctx):
    hd, hq, hkv, theta = 64, 8, 2, 10000.0
    c = qb.KvCache(ctx, 2, 128, hkv, hd, "f16", max_batch=2)
    rng = np.random.default_rng(0)
    q, k, v = (gu.to_device(gu.normal(rng, (1, 4, h, hd)), "f16") for h in (hq, hkv, hkv))
    qb.attention_forward(c, 0, q, k, v, [0], hq, hkv, hd, theta)
    with pytest.raises(qb.QllamaError, match="must continue"):  # repeated prefill
        qb.attention_forward(c, 0, q, k, v, [0], hq, hkv, hd, theta)
    assert c.seq_len() == 4
    with pytest.raises(qb.QllamaError, match="divisible"):
        qb.attention_forward(c, 0, q, k, v, [4], 6, 4, hd, theta)
    with pytest.raises(qb.QllamaError, match="theta"):
        qb.attention_forward(c, 0, q, k, v, [4], hq, hkv, hd, float("nan"))
    with pytest.raises(qb.QllamaError, match="layer index 5"):
        qb.attention_forward(c, 5, q, k, v, [4], hq, hkv, hd, theta)
    zeros = np.zeros((122, hkv, hd), np.float32)
    c.update(0, zeros, zeros, np.arange(4, 126))
    with pytest.raises(qb.QllamaError, match="capacity 128"):
        qb.attention_forward(c, 0, q, k, v, [126], hq, hkv, hd, theta)
    assert c.seq_len() == 126
    e = qb.attention_forward(c, 0, q[:, :0], k[:, :0], v[:, :0], [126], hq, hkv, hd, theta)
    assert tuple(e.shape) == (1, 0, hq * hd) and c.seq_len() == 126
    # a sequence named twice in one call is rejected, and the next calls that
    # name each sequence once go through
    q2, k2, v2 = (gu.to_device(gu.normal(rng, (2, 1, h, hd)), "f16") for h in (hq, hkv, hkv))
    with pytest.raises(qb.QllamaError, match="appears twice"):
        qb.attention_forward(c, 1, q2, k2, v2, [0, 0], hq, hkv, hd, theta, seq_ids=[1, 1])
    for pos in range(2):
        qb.attention_forward(c, 1, q2, k2, v2, [pos, pos], hq, hkv, hd, theta, seq_ids=[1, 0])
    assert c.layer_len(1, 1) == 2 and c.layer_len(1, 0) == 2


def test_tiny_llama_end_to_end_on_gpu(ctx, golden):
    """The reference's tiny-llama fixture with attention on the GPU (f32 cache)."""
    model = lh.tiny_from_golden(golden)
    ids = golden["tiny/ids_b"]
    ref = golden["tiny/logits_b"]
    cache = qb.KvCache(ctx, model.n_layers, 128, model.n_kv, model.hd, "f32")
    ocache = oracle.KvCache(model.n_layers, 128, model.n_kv, model.hd)

    def attend(layer, q, k, v, start):
        return qb.attention_forward(cache, layer, q, k, v, [start], model.n_head, model.n_kv,
                                    model.hd, model.theta)

    rows_g, rows_o, pos = [], [], 0
    for b in (4, 1, 3, 1, 2):
        rows_g.append(model.forward(ids[pos:pos + b], pos, attend))
        rows_o.append(model.forward(ids[pos:pos + b], pos, lh.oracle_cached_attend(model, ocache)))
        pos += b
    g, o = np.concatenate(rows_g), np.concatenate(rows_o)
    assert np.abs(g - ref).max() <= 1e-4
    assert np.abs(g - o).max() <= 1e-6
    assert np.array_equal(g.argmax(1), o.argmax(1))


def test_long_context_q8_0_decode_sample(ctx):
    """Llama-3-70B-shaped decode sample: 64/8 heads, hd 128, Q8_0 KV at length 32768."""
    rng = np.random.default_rng(70)
    hd, hq, hkv, theta, L = 128, 64, 8, 500000.0, 32768
    p = gu.Pair(ctx, "q8_0", 1, L, hkv, hd, 2, page=256)
    for s in range(2):
        p.prefill_rows(rng, 0, s, L - 1, theta)
    q = gu.rounded(gu.normal(rng, (2, 1, hq, hd)), "bf16")
    k = gu.rounded(gu.normal(rng, (2, 1, hkv, hd)), "bf16")
    v = gu.rounded(gu.normal(rng, (2, 1, hkv, hd)), "bf16")
    out = qb.attention_forward(p.gpu, 0, gu.to_device(q, "bf16"), gu.to_device(k, "bf16"),
                               gu.to_device(v, "bf16"), [L - 1, L - 1], hq, hkv, hd, theta)
    ref = p.oracle_forward(0, q, k, v, [L - 1, L - 1], hq, theta)
    assert gu.max_err(out, ref) <= TOL_Q8_DEQ
    assert p.gpu.seq_len(1) == L
    with pytest.raises(qb.QllamaError, match="capacity"):
        qb.attention_forward(p.gpu, 0, gu.to_device(q, "bf16"), gu.to_device(k, "bf16"),
                             gu.to_device(v, "bf16"), [L, L], hq, hkv, hd, theta)


@pytest.mark.parametrize("storage", ["f16", "bf16", "q8_0"])
@pytest.mark.parametrize("batch,n,start,hq,hkv,hd", [
    (2, 200, 0, 8, 2, 128),      # ragged last 128-row tile, GQA 4
    (1, 512, 100, 16, 4, 128),   # non-zero start: offset causal mask
    (3, 128, 37, 4, 4, 128),     # MHA, start inside a KV tile
    (1, 1500, 0, 8, 8, 128),     # many KV tiles: pipeline wrap, O rescaling
    (1, 64, 0, 8, 1, 128),       # one half-filled tile, GQA 8
    (8, 1024, 0, 32, 8, 128),    # enough CTAs for two heads per CTA
    (2, 200, 0, 8, 2, 64),       # head_dim 64: one 128-byte box per row
    (1, 512, 100, 32, 4, 64),    # TinyLlama-shaped chunk at an offset
    (1, 1500, 0, 8, 8, 64),
    (4, 1024, 0, 32, 4, 64),     # two heads per CTA at head_dim 64
])
def test_tcgen05_prefill_parity(ctx, storage, batch, n, start, hq, hkv, hd):
    """Multi-token calls on an f16, bf16 or Q8_0 cache with head_dim 64 or 128 run
    the tcgen05/TMEM kernel (bf16 and Q8_0 keys first copied as f16 tiles; Q8_0
    against the oracle on the dequantised cache)."""
    rng = np.random.default_rng(n * 7 + start + hd)
    theta = 500000.0
    p = gu.Pair(ctx, storage, 1, start + n + 64, hkv, hd, batch)
    for s in range(batch):
        if start:
            p.prefill_rows(rng, 0, s, start, theta)
    q = gu.rounded(gu.normal(rng, (batch, n, hq, hd)), "bf16")
    k = gu.rounded(gu.normal(rng, (batch, n, hkv, hd)), "bf16")
    v = gu.rounded(gu.normal(rng, (batch, n, hkv, hd)), "bf16")
    starts = np.full(batch, start, np.int64)
    out = qb.attention_forward(p.gpu, 0, gu.to_device(q, "bf16"), gu.to_device(k, "bf16"),
                               gu.to_device(v, "bf16"), starts, hq, hkv, hd, theta)
    p.gpu.ctx.synchronize()
    ref = p.oracle_forward(0, q, k, v, starts, hq, theta)
    tol = TOL_Q8_DEQ if storage == "q8_0" else TOL_16
    assert gu.max_err(out, ref) <= tol
    # a decode step after the prefill sees the appended rows
    q1 = gu.rounded(gu.normal(rng, (batch, 1, hq, hd)), "bf16")
    k1 = gu.rounded(gu.normal(rng, (batch, 1, hkv, hd)), "bf16")
    out1 = qb.attention_forward(p.gpu, 0, gu.to_device(q1, "bf16"), gu.to_device(k1, "bf16"),
                                gu.to_device(k1, "bf16"), starts + n, hq, hkv, hd, theta)
    ref1 = p.oracle_forward(0, q1, k1, k1, starts + n, hq, theta)
    assert gu.max_err(out1, ref1) <= tol


@pytest.mark.parametrize("storage", ["f16", "bf16"])
def test_tcgen05_prefill_ignores_stale_rows_past_the_end(ctx, storage):
    """Pages keep old rows after a roll-back; keys past the end must not reach O.

    Positions 0..255 are first written with Inf/NaN K and V (and, in a bf16
    cache, huge finite values) and rolled back, so the last 128-key tile of a
    200-token prefill reads them (keys 200..255) from the same pages. Their
    probabilities are exactly 0, and 0 * Inf must not turn the visible rows
    into NaN; nor may their magnitudes set the f16 range of the tile's
    operands."""
    rng = np.random.default_rng(23)
    hd, hq, hkv, theta, n = 128, 8, 2, 500000.0, 200
    p = gu.Pair(ctx, storage, 1, 320, hkv, hd, 1)
    bad = np.full((256, hkv, hd), np.inf, np.float32)
    bad[:, :, 1::3] = np.nan
    bad[:, :, 2::3] = -np.inf if storage == "f16" else -1e30
    p.gpu.update(0, bad, bad, np.arange(256))
    p.gpu.truncate(0, 0)
    assert p.gpu.seq_len(0) == 0
    q, k, v = (gu.rounded(gu.normal(rng, (1, n, h, hd)), "bf16") for h in (hq, hkv, hkv))
    out = qb.attention_forward(p.gpu, 0, gu.to_device(q, "bf16"), gu.to_device(k, "bf16"),
                               gu.to_device(v, "bf16"), [0], hq, hkv, hd, theta)
    p.gpu.ctx.synchronize()
    ref = p.oracle_forward(0, q, k, v, [0], hq, theta)
    assert np.isfinite(out.float().cpu().numpy()).all()
    assert gu.max_err(out, ref) <= TOL_16
    # the split-KV decode step reads the same stale tail (keys 201..255)
    q1, k1, v1 = (gu.rounded(gu.normal(rng, (1, 1, h, hd)), "bf16") for h in (hq, hkv, hkv))
    out1 = qb.attention_forward(p.gpu, 0, gu.to_device(q1, "bf16"), gu.to_device(k1, "bf16"),
                                gu.to_device(v1, "bf16"), [n], hq, hkv, hd, theta)
    ref1 = p.oracle_forward(0, q1, k1, v1, [n], hq, theta)
    assert np.isfinite(out1.float().cpu().numpy()).all()
    assert gu.max_err(out1, ref1) <= TOL_16


@pytest.mark.parametrize("scenario", ["small_q", "large_q"])
@pytest.mark.parametrize("hd", [64, 128])
def test_tcgen05_bf16_prefill_keeps_the_bf16_range(ctx, hd, scenario):
    """A bf16 cache holds magnitudes far outside f16's; the tensor-core prefill
    divides each K/V tile (and each rotated q row) by a power of two that puts
    it in the f16 operand range and folds the factor back, so such values
    neither overflow nor underflow nor disturb the other tiles.

    small_q: q x 2^-16 everywhere, K of keys 128..255 x 2^16 (those scores stay
    O(1)), V of keys 256..383 x 2^20, K of keys 384..511 and V of keys
    512..599 x 2^-20.  large_q: q of every third token x 2^18 with all K
    x 2^-18, V of keys 256..383 x 2^20.  Scores stay O(1) in both (large
    scores would make the softmax an argmax, where any rounding of q picks
    between near-ties)."""
    rng = np.random.default_rng(hd + 3)
    hq, hkv, theta, n = 8, 2, 500000.0, 600
    p = gu.Pair(ctx, "bf16", 1, n + 64, hkv, hd, 1)
    q = gu.normal(rng, (1, n, hq, hd))
    k = gu.normal(rng, (1, n, hkv, hd))
    v = gu.normal(rng, (1, n, hkv, hd))
    if scenario == "small_q":
        q *= 2.0 ** -16
        k[:, 128:256] *= 2.0 ** 16
        k[:, 384:512] *= 2.0 ** -20
        v[:, 512:] *= 2.0 ** -20
    else:
        q[:, ::3] *= 2.0 ** 18
        k *= 2.0 ** -18
    v[:, 256:384] *= 2.0 ** 20
    q, k, v = (gu.rounded(x, "bf16") for x in (q, k, v))
    out = qb.attention_forward(p.gpu, 0, gu.to_device(q, "bf16"), gu.to_device(k, "bf16"),
                               gu.to_device(v, "bf16"), [0], hq, hkv, hd, theta,
                               out_dtype="f32")
    p.gpu.ctx.synchronize()
    ref = p.oracle_forward(0, q, k, v, [0], hq, theta)
    got = out.float().cpu().numpy().reshape(ref.shape)
    assert np.isfinite(got).all()
    # 2e-3 of each token's output magnitude (at least 1): tokens that see the
    # scaled V carry values near 2^20
    err = np.abs(got.astype(np.float64) - ref).reshape(n, -1).max(axis=1)
    mag = np.maximum(1.0, np.abs(ref).reshape(n, -1).max(axis=1))
    assert (err / mag).max() <= TOL_16
    assert err[:256].max() <= TOL_16  # before the scaled V: absolute


def test_truncate_rolls_back_and_rewrites(ctx):
    """ql_kv_truncate: roll a sequence back, write new rows over the old positions."""
    rng = np.random.default_rng(21)
    hd, hq, hkv, theta = 64, 8, 2, 10000.0
    p = gu.Pair(ctx, "f16", 2, 256, hkv, hd, 1)
    for layer in (0, 1):
        p.prefill_rows(rng, layer, 0, 100, theta)
    with pytest.raises(qb.QllamaError, match="cannot truncate"):
        p.gpu.truncate(0, 101)
    p.gpu.truncate(0, 60)
    assert p.gpu.seq_len(0) == 60 and p.gpu.layer_len(1, 0) == 60
    # the oracle has no roll-back: rebuild its cache with the first 60 rows
    kg, vg = p.gpu.get(0, np.arange(60))
    fresh = oracle.KvCache(2, 256, hkv, hd, oracle.F16)
    fresh.update(0, kg, vg, np.arange(60))
    q, k, v = (gu.normal(rng, (1, 1, h, hd)) for h in (hq, hkv, hkv))
    out = qb.attention_forward(p.gpu, 0, gu.to_device(q, "f32"), gu.to_device(k, "f32"),
                               gu.to_device(v, "f32"), [60], hq, hkv, hd, theta)
    ref = oracle.attention_with_cache(fresh, 0, q[0], k[0], v[0], 60, hq, hkv, hd, theta)
    assert gu.max_err(out[0], ref) <= TOL_16
    assert p.gpu.layer_len(0, 0) == 61 and p.gpu.layer_len(1, 0) == 60


def test_page_crossing_decode_never_waits_for_the_gpu(ctx):
    """A ragged decode loop where some sequence enters a new page on every step.

    The new block-table entries travel to the device in stream order (a table
    patch launch), so the call returns while the GPU is still busy with work
    queued before it: a long sleep kernel is queued first on the context's
    stream, and the stream must still be busy when the call returns.  Every
    step is checked against the oracle (cache.rs:83-170 semantics: the step
    appends at current_len)."""
    rng = np.random.default_rng(77)
    hq, hkv, hd, theta, B = 16, 2, 64, 10000.0, 12
    # step 0 warms up (RoPE table, workspace); sequence b enters a new
    # 64-position page at step b + 1
    starts = np.array([64 * (b % 3 + 1) - b - 1 for b in range(B)], np.int64)
    p = gu.Pair(ctx, "f16", 2, 320, hkv, hd, B)
    for s in range(B):
        for layer in range(2):
            p.prefill_rows(rng, layer, s, int(starts[s]), theta)
    stream = torch.cuda.Stream()
    ctx.set_stream(stream.cuda_stream)
    try:
        for step in range(B + 1):
            crossing = [b for b in range(B) if (starts[b] % 64) == 0]
            assert crossing == ([step - 1] if step else [])
            for layer in range(2):
                q, k, v = (gu.rounded(gu.normal(rng, (B, 1, h, hd)), "f16")
                           for h in (hq, hkv, hkv))
                dq, dk, dv = (gu.to_device(x, "f16") for x in (q, k, v))
                out = torch.empty(B, 1, hq * hd, device="cuda", dtype=torch.float32)
                torch.cuda.synchronize()
                with torch.cuda.stream(stream):
                    torch.cuda._sleep(200_000_000)  # ~0.1 s of GPU time queued first
                qb.attention_forward(p.gpu, layer, dq, dk, dv, starts, hq, hkv, hd, theta,
                                     out=out)
                if step:
                    assert not stream.query(), "the call waited for the GPU"
                stream.synchronize()
                ref = p.oracle_forward(layer, q, k, v, starts, hq, theta)
                assert gu.max_err(out, ref) <= TOL_16, (step, layer)
            starts = starts + 1
        ctx.synchronize()
    finally:
        ctx.set_stream(None)
