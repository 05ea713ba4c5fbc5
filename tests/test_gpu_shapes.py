"""Parity at the shapes the benchmark times, against the CPU oracle.

Each test runs the benchmark workload's own shapes through the C ABI and
checks the results against the oracle (the restatement of the reference's
attention, src/transformer/layers.rs:397-455) at the tolerances of the other
GPU tests:
  * the TinyLlama-1.1B-shaped job: a 512-token prefill at head_dim 64 on an
    f16 cache, then single-token decode steps to position 767, two layers;
  * the Llama-2-7B-shaped MHA decode: 32/32 heads, head_dim 128, batch 16 at
    ragged lengths drawn from U[1024, 4096];
  * the Llama-3-8B-shaped GQA prefill at full length: 8192 tokens, 32/8
    heads, head_dim 128, theta 5e5.  The GPU runs the whole call; the oracle
    checks a seeded sample of query rows of every head (a row of the
    reference's computation depends only on its own query and the keys up to
    its position, so one row is the oracle's attention core on that row).
"""
import numpy as np
import pytest
import torch

import oracle
import qllama_b200 as qb
from tests import gpu_util as gu

pytestmark = pytest.mark.gpu

TOL_16 = 2e-3


@pytest.fixture(scope="module")
def ctx():
    return qb.Context(0)


def test_tinyllama_job_prefill_512_then_decode_to_767(ctx):
    """22-layer TinyLlama-shaped job, two of its layers: 32/4 heads, hd 64, f16 KV."""
    rng = np.random.default_rng(1100)
    hq, hkv, hd, theta, P, D, layers = 32, 4, 64, 10000.0, 512, 256, 2
    p = gu.Pair(ctx, "f16", layers, P + D, hkv, hd, 1)
    for layer in range(layers):
        q, k, v = (gu.rounded(gu.normal(rng, (1, P, h, hd)), "f16") for h in (hq, hkv, hkv))
        out = qb.attention_forward(p.gpu, layer, gu.to_device(q, "f16"), gu.to_device(k, "f16"),
                                   gu.to_device(v, "f16"), [0], hq, hkv, hd, theta)
        ref = p.oracle_forward(layer, q, k, v, [0], hq, theta)
        assert gu.max_err(out, ref) <= TOL_16, ("prefill", layer)
    worst = 0.0
    for step in range(D):
        for layer in range(layers):
            q, k, v = (gu.rounded(gu.normal(rng, (1, 1, h, hd)), "f16") for h in (hq, hkv, hkv))
            out = qb.attention_forward(p.gpu, layer, gu.to_device(q, "f16"),
                                       gu.to_device(k, "f16"), gu.to_device(v, "f16"), [P + step],
                                       hq, hkv, hd, theta)
            ref = p.oracle_forward(layer, q, k, v, [P + step], hq, theta)
            worst = max(worst, gu.max_err(out, ref))
    assert worst <= TOL_16, worst
    assert p.gpu.seq_len(0) == P + D == 768
    p.gpu.ctx.synchronize()


def test_llama2_mha_decode_batch16_ragged(ctx):
    """Llama-2-7B-shaped decode: 32/32 heads, hd 128, f16 KV, batch 16, L ~ U[1024, 4096]."""
    rng = np.random.default_rng(4096)
    hq = hkv = 32
    hd, theta, B = 128, 10000.0, 16
    lens = rng.integers(1024, 4097, size=B)
    p = gu.Pair(ctx, "f16", 1, int(lens.max()) + 4, hkv, hd, B)
    for s, L in enumerate(lens):
        p.prefill_rows(rng, 0, s, int(L) - 1, theta)
    starts = lens - 1
    for _ in range(2):
        q, k, v = (gu.rounded(gu.normal(rng, (B, 1, h, hd)), "f16") for h in (hq, hkv, hkv))
        out = qb.attention_forward(p.gpu, 0, gu.to_device(q, "f16"), gu.to_device(k, "f16"),
                                   gu.to_device(v, "f16"), starts, hq, hkv, hd, theta)
        ref = p.oracle_forward(0, q, k, v, starts, hq, theta)
        assert gu.max_err(out, ref) <= TOL_16
        starts = starts + 1
    p.gpu.ctx.synchronize()


def _sampled_rows(rng, n, count):
    edges = [0, 1, 2, 63, 64, 127, 128, 129, 255, 4095, 4096, n - 2, n - 1]
    rest = rng.choice(np.arange(n), size=count - len(edges), replace=False)
    return np.unique(np.concatenate([edges, rest]))


@pytest.mark.parametrize("storage", ["f16", "bf16"])
def test_llama3_prefill_8192_full_length(ctx, storage):
    """One 8192-token sequence at the Llama-3-8B shape, checked on sampled rows."""
    rng = np.random.default_rng(8192)
    hq, hkv, hd, theta, n = 32, 8, 128, 500000.0, 8192
    q, k, v = (gu.rounded(gu.normal(rng, (1, n, h, hd)), "bf16") for h in (hq, hkv, hkv))
    cache = qb.KvCache(ctx, 1, n, hkv, hd, storage, 64, 1)
    out = qb.attention_forward(cache, 0, gu.to_device(q, "bf16"), gu.to_device(k, "bf16"),
                               gu.to_device(v, "bf16"), [0], hq, hkv, hd, theta)
    ctx.synchronize()
    out = out[0].float().cpu().numpy()
    # the oracle's cache after the same append: rotated K and V in the same storage
    orc = oracle.KvCache(1, n, hkv, hd, oracle.STORAGE[storage])
    orc.update(0, oracle.rope(k[0], hd, 0, theta), v[0], np.arange(n))
    kc, vc = orc.get(0, np.arange(n))
    # and the device cache holds exactly those rows
    kg, vg = cache.get(0, np.arange(0, n, 97))
    assert np.array_equal(kg.view(np.uint32), kc[::97].view(np.uint32))
    assert np.array_equal(vg.view(np.uint32), vc[::97].view(np.uint32))
    qr = oracle.rope(q[0], hd, 0, theta)
    rows = _sampled_rows(rng, n, 48)
    worst = 0.0
    for i in rows:
        ref = oracle.attention_core(qr[i:i + 1], kc[:i + 1], vc[:i + 1], int(i), hq, hkv, hd)
        worst = max(worst, float(np.abs(out[i] - ref[0]).max()))
    assert worst <= TOL_16, worst
    assert cache.seq_len(0) == n
    cache.close()
