"""Host-side pieces of the model path, on the CPU: the oracle's sampler
against the reference's sampler tests (tests/sampler.rs, deterministic cases
exactly, statistical cases with seeded uniform draws), and the GGUF reader's
validation (src/gguf/parser.rs, config.rs), which runs before any device is
needed."""
import ctypes

import numpy as np
import pytest

import oracle
import qllama_b200 as qb
from tests import model_util as mu


def samp(logits, context, temperature, top_k, top_p, penalty, r=0.5):
    return oracle.sample(np.asarray(logits, np.float32), context, temperature, top_k, top_p,
                         penalty, r)


def counts(logits, sampler, rounds, seed):
    u = np.random.default_rng(seed).random(rounds)
    c = np.zeros(len(logits), int)
    for r in u:
        c[samp(logits, [], *sampler, r)] += 1
    return c


def test_oracle_sampler_deterministic_cases():
    assert samp([0.1, 0.9, 0.2], [], 0.0, 0, 1.0, 1.0) == 1
    assert samp([-1.0, -2.0, -0.5], [], 0.0, 0, 1.0, 1.0) == 2
    assert samp([0.5, 0.5, 0.1], [], 0.0, 0, 1.0, 1.0) == 0
    assert samp([-0.0, 0.0], [], 0.0, 0, 1.0, 1.0) == 1  # total order: +0 above -0
    for r in np.linspace(0, 0.999, 8):
        assert samp([1.0, 2.0, 3.0], [], 1e-6, 0, 1.0, 1.0, r) == 2
        assert samp([0.1, 5.0, 0.2], [], 1.0, 1, 1.0, 1.0, r) == 1
        assert samp([10.0, 1.0, 1.0], [], 1.0, 0, 0.5, 1.0, r) == 0
        assert samp([0.5, 0.3], [0], 1.0, 1, 1.0, 2.0, r) == 1
    assert samp([0.3, 0.5], [1], 0.0, 0, 1.0, 2.0) == 0
    assert samp([-1.0, -0.5], [0], 0.0, 0, 1.0, 4.0) == 1
    assert samp([0.25, 0.5], [1], 0.0, 0, 1.0, 1.0) == 1
    assert samp([0.4, 0.5], [1], 0.0, 0, 1.0, 2.0) == 0
    assert samp([0.4, 0.5], [], 0.0, 0, 1.0, 2.0) == 1
    assert samp([0.3, 0.5], [1, 1, 1], 0.0, 0, 1.0, 2.0) == 0
    assert samp([0.25, 0.5], [7, -1], 0.0, 0, 1.0, 2.0) == 1


def test_oracle_sampler_statistics():
    c = counts([0.0, 0.0], (1.0, 0, 1.0, 1.0), 2000, 7)
    assert 933 < c[0] < 1067 and 933 < c[1] < 1067
    c = counts([10.0, 9.0, 0.0], (1.0, 2, 1.0, 1.0), 500, 2024)
    assert c[2] == 0 and 94 < c[1] < 174
    for k in (0, 10):
        c = counts([1.0, 1.0, 1.0], (1.0, k, 1.0, 1.0), 300, 2024)
        assert all(67 < x < 133 for x in c)
    lg = [0.0, -float(np.log(np.float32(18.0))), -float(np.log(np.float32(18.0)))]
    c = counts(lg, (1.0, 0, 0.91, 1.0), 1000, 11)
    assert c[2] == 0 and 24 < c[1] < 81
    c = counts(lg, (1.0, 0, 0.89, 1.0), 200, 11)
    assert c[1] == 0 and c[2] == 0
    c = counts([1.0, 1.0, 1.0], (1.0, 0, 0.5, 1.0), 300, 2024)
    assert c[2] == 0 and 115 < c[0] < 185 and 115 < c[1] < 185


def test_oracle_sampler_errors():
    with pytest.raises(oracle.OracleError, match="finite"):
        samp([0.1, float("nan")], [], 0.0, 0, 1.0, 1.0)
    with pytest.raises(oracle.OracleError, match="temperature"):
        samp([0.1], [], float("inf"), 0, 1.0, 1.0)
    with pytest.raises(oracle.OracleError, match="repeat_penalty"):
        samp([0.1], [], 1.0, 0, 1.0, -1.0)
    with pytest.raises(oracle.OracleError, match="non-empty"):
        samp([], [], 1.0, 0, 1.0, 1.0)


def _load(path):
    L = qb.load()
    h = ctypes.c_void_p()
    rc = L.ql_llama_load_gguf(None, str(path).encode(), ctypes.byref(h))
    return rc, L.ql_last_error().decode()


def test_gguf_reader_validates_before_any_device_work(golden, tmp_path):
    t, cfg = mu.tiny_tensors(golden)
    good = tmp_path / "tiny.gguf"
    mu.write_gguf(good, t, cfg["heads"], cfg["kv_heads"], cfg["layers"], cfg["ff"],
                  cfg["max_pos"], cfg["eps"], cfg["theta"])
    rc, msg = _load(good)  # parses and checks everything; then wants a context
    assert rc == qb.ERR_INVALID and "NULL context" in msg
    raw = bytearray(good.read_bytes())
    bad = tmp_path / "bad.gguf"
    bad.write_bytes(b"GGUX" + raw[4:])
    assert _load(bad) == (qb.ERR_INVALID, "Invalid GGUF magic")
    bad.write_bytes(raw[:4] + (0).to_bytes(4, "little") + raw[8:])
    assert _load(bad) == (qb.ERR_INVALID, "Bad GGUF version: 0")
    bad.write_bytes(raw[:4] + (0x30000).to_bytes(4, "little") + raw[8:])
    assert "big-endian" in _load(bad)[1]
    bad.write_bytes(raw[:4] + (9).to_bytes(4, "little") + raw[8:])
    assert "exceeds supported version" in _load(bad)[1]
    bad.write_bytes(raw[:200])
    assert "end of file" in _load(bad)[1]
    # a missing epsilon, a head count that does not divide, quantised weights
    no_eps = tmp_path / "noeps.gguf"
    import gguf

    w = gguf.GGUFWriter(str(no_eps), "llama")
    w.add_block_count(1)
    w.add_context_length(16)
    w.add_embedding_length(16)
    w.add_feed_forward_length(32)
    w.add_head_count(4)
    w.add_tensor("token_embd.weight", np.zeros((8, 16), np.float32))
    w.write_header_to_file()
    w.write_kv_data_to_file()
    w.write_tensors_to_file()
    w.close()
    rc, msg = _load(no_eps)
    assert rc == qb.ERR_INVALID and "llama.attention.layer_norm_rms_epsilon" in msg
    t2 = dict(t)
    mu.write_gguf(bad, t2, 3, 3, cfg["layers"], cfg["ff"], 128, cfg["eps"], cfg["theta"])
    assert "not divisible by attention.head_count" in _load(bad)[1]
    assert "cannot open" in _load(tmp_path / "missing.gguf")[1]
    # string-array metadata (the token list) is skipped over, and its length
    # must agree with the embedding's rows (config.rs:98-108)
    for n_tokens, ok in ((cfg["vocab"], True), (cfg["vocab"] - 1, False)):
        w = gguf.GGUFWriter(str(bad), "llama")
        w.add_block_count(cfg["layers"])
        w.add_context_length(128)
        w.add_embedding_length(cfg["dim"])
        w.add_feed_forward_length(cfg["ff"])
        w.add_head_count(cfg["heads"])
        w.add_head_count_kv(cfg["kv_heads"])
        w.add_layer_norm_rms_eps(cfg["eps"])
        w.add_token_list([f"tok{i}" for i in range(n_tokens)])
        for name, a in t.items():
            w.add_tensor(name, np.ascontiguousarray(a, np.float32))
        w.write_header_to_file()
        w.write_kv_data_to_file()
        w.write_tensors_to_file()
        w.close()
        rc, msg = _load(bad)
        if ok:
            assert rc == qb.ERR_INVALID and "NULL context" in msg, msg
        else:
            assert "tokenizer.ggml.tokens has" in msg, msg
