"""ql_attn_decode_noalloc: single-token decode whose scratch is a static device array.

Some callers cannot allocate device memory once they are serving: a runtime
that gives all GPU memory to its own allocator at start-up, or a loop that
promises no cudaMalloc/cudaFree after warm-up.  This entry point is for them.
The test drives it through the C ABI next to ql_attn_forward, on two caches
holding the same rows, and checks two consecutive decode steps against the
existing entry point and against the CPU oracle at the parity tolerance of
the other GPU tests (2e-3), including a ragged batch whose split partials
would not fit the static array.
It lives in a file of its own that pytest collects last.
"""
import ctypes

import numpy as np
import pytest
import torch

import oracle
import qllama_b200 as qb

pytestmark = pytest.mark.gpu

TOL = 2e-3


def _args(layer, q, k, v, out, seqs, starts, hq, hkv, hd, theta, mem=qb.MEM_DEVICE, new_len=1):
    codes = {torch.float16: qb.F16, torch.bfloat16: qb.BF16, torch.float32: qb.F32}
    return qb.AttnArgs(layer, q.shape[0], new_len,
                       seqs.ctypes.data_as(ctypes.POINTER(ctypes.c_int32)),
                       starts.ctypes.data_as(ctypes.POINTER(ctypes.c_int64)), hq, hkv, hd, theta,
                       codes[q.dtype], codes[out.dtype], mem, q.data_ptr(), k.data_ptr(),
                       v.data_ptr(), out.data_ptr())


@pytest.mark.parametrize("storage,hd,hq,hkv,lens", [
    ("f16", 128, 64, 8, [3000, 700, 64]),   # several KV splits: partials and counters in use
    ("bf16", 64, 32, 4, [1, 513]),
    ("q8_0", 128, 16, 2, [2049, 37]),
    # one long sequence among 63 short ones: the split plan's partials for 64
    # sequences x 8 KV heads would overflow the static array, so the entry
    # point falls back to fewer, longer splits
    ("f16", 128, 64, 8, [16384] + [40] * 63),
])
def test_noalloc_decode_matches_forward(storage, hd, hq, hkv, lens):
    L = qb.load()
    ctx = qb.Context(0)
    rng = np.random.default_rng(2024)
    theta, B = 10000.0, len(lens)
    pages = sum((n + 2 + 63) // 64 for n in lens) + 8
    caches = [qb.KvCache(ctx, 1, max(lens) + 4, hkv, hd, storage, 64, B, pages) for _ in range(2)]
    orc = [oracle.KvCache(1, max(lens) + 4, hkv, hd, oracle.STORAGE[storage]) for _ in lens]
    for s, n in enumerate(lens):
        k = rng.standard_normal((n - 1, hkv, hd)).astype(np.float32)
        v = rng.standard_normal((n - 1, hkv, hd)).astype(np.float32)
        kr = oracle.rope(k, hd, 0, theta)
        for c in caches:
            c.update(0, kr, v, np.arange(n - 1), seq=s)
        orc[s].update(0, kr, v, np.arange(n - 1))
    seqs = np.arange(B, dtype=np.int32)
    starts = np.array([n - 1 for n in lens], dtype=np.int64)
    dt = torch.bfloat16 if storage == "bf16" else torch.float16
    gen = torch.Generator(device="cuda")
    gen.manual_seed(7)
    for step in range(2):  # two calls in a row
        q, k, v = (torch.randn(B, 1, h, hd, device="cuda", generator=gen).to(dt)
                   for h in (hq, hkv, hkv))
        out_ref = torch.empty(B, 1, hq * hd, device="cuda", dtype=torch.float32)
        out_new = torch.full_like(out_ref, float("nan"))
        rc = L.ql_attn_forward(ctx._h, caches[0]._h,
                               ctypes.byref(_args(0, q, k, v, out_ref, seqs, starts, hq, hkv, hd,
                                                  theta)))
        assert rc == qb.OK, L.ql_last_error()
        rc = L.ql_attn_decode_noalloc(ctx._h, caches[1]._h,
                                      ctypes.byref(_args(0, q, k, v, out_new, seqs, starts, hq,
                                                         hkv, hd, theta)))
        assert rc == qb.OK, L.ql_last_error()
        ctx.synchronize()
        err = (out_new - out_ref).abs().max().item()
        assert err <= TOL, (step, err)
        # and against the oracle, the restatement of the reference's attention
        qn, kn, vn = (x.float().cpu().numpy() for x in (q, k, v))
        ref = np.stack([oracle.attention_with_cache(orc[b], 0, qn[b], kn[b], vn[b],
                                                    int(starts[b]), hq, hkv, hd, theta)
                        for b in range(B)])
        err_o = float(np.abs(out_new.cpu().numpy().astype(np.float64) - ref).max())
        assert err_o <= TOL, (step, err_o)
        starts = starts + 1
    assert caches[1].seq_len(0) == lens[0] + 1
    # The rows this entry point appended (K rotated with angles evaluated on the
    # device in f64) against the oracle's rows (angles from libm, as the
    # reference computes them): identical but for rare last-place differences.
    same = total = 0
    for b in range(min(B, 4)):
        new_pos = np.arange(lens[b] - 1, lens[b] + 1)
        kg, vg = caches[1].get(0, new_pos, seq=b)
        ko, vo = orc[b].get(0, new_pos)
        assert np.array_equal(vg.view(np.uint32), vo.view(np.uint32))
        assert np.abs(kg - ko).max() <= 1e-2 * max(1.0, float(np.abs(ko).max()))
        same += int((kg.view(np.uint32) == ko.view(np.uint32)).sum())
        total += kg.size
    assert same >= 0.99 * total, (same, total)
    for c in caches:
        c.close()
    ctx.close()


def test_noalloc_rejects_what_it_cannot_serve():
    L = qb.load()
    ctx = qb.Context(0)
    hq, hkv, hd, theta = 8, 2, 64, 10000.0
    cache = qb.KvCache(ctx, 1, 128, hkv, hd, "f16", 64, 1)
    seqs, starts = np.zeros(1, np.int32), np.zeros(1, np.int64)
    q = torch.randn(1, 2, hq, hd, device="cuda").half()
    k = torch.randn(1, 2, hkv, hd, device="cuda").half()
    out = torch.empty(1, 2, hq * hd, device="cuda")
    rc = L.ql_attn_decode_noalloc(ctx._h, cache._h,
                                  ctypes.byref(_args(0, q, k, k, out, seqs, starts, hq, hkv, hd,
                                                     theta, new_len=2)))
    assert rc == qb.ERR_INVALID and b"new_len 1" in L.ql_last_error()
    rc = L.ql_attn_decode_noalloc(ctx._h, cache._h,
                                  ctypes.byref(_args(0, q, k, k, out, seqs, starts, hq, hkv, hd,
                                                     theta, mem=qb.MEM_HOST)))
    assert rc == qb.ERR_INVALID and b"device buffers" in L.ql_last_error()
    assert cache.seq_len(0) == 0
    # more (sequence, KV head) pairs than the scratch has counters for
    big_hkv, batch = 128, 129
    wide = qb.KvCache(ctx, 1, 64, big_hkv, hd, "f16", 64, batch)
    qs = torch.randn(batch, 1, big_hkv, hd, device="cuda").half()
    outs = torch.empty(batch, 1, big_hkv * hd, device="cuda")
    rc = L.ql_attn_decode_noalloc(ctx._h, wide._h,
                                  ctypes.byref(_args(0, qs, qs, qs, outs,
                                                     np.arange(batch, dtype=np.int32),
                                                     np.zeros(batch, np.int64), big_hkv, big_hkv,
                                                     hd, theta)))
    assert rc == qb.ERR_INVALID and b"no-allocation limit" in L.ql_last_error()
    wide.close()
    cache.close()
    ctx.close()
