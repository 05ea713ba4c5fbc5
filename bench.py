#!/usr/bin/env python
"""Benchmark of the Qllama attention hot path on B200.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
                    [--workload c2|c3|c4|c5]

Workloads (seeded synthetic N(0,1) inputs of the named shapes; cache contents
random where the shape says "pre-filled"):
  c2 (default) TinyLlama-1.1B-shaped attention stack: 22 layers, 32 query /
     4 KV heads (GQA 8:1), head_dim 64, theta 1e4, f16 KV, batch 1; a step is
     the whole job -- causal prefill of 512 tokens, then 256 decode steps,
     every layer (5,654 attention calls).  value: tokens/s.
  c3 Llama-2-7B-shaped MHA decode: 32 layers, 32/32 heads, head_dim 128, f16
     KV pre-filled to ragged lengths U[1024, 4096] for 16 sequences; a step is
     128 decode steps of all 16 sequences through the 32 layers.  value: KV
     GB/s (algorithmic bytes read); tokens/s beside it.
  c4 Llama-3-8B-shaped GQA prefill: 32/8 heads, head_dim 128, theta 5e5, bf16
     Q/K/V (f16 cache), 4 sequences x 8192 tokens; a step is one layer's causal
     prefill.  value: TFLOP/s counting unmasked pairs only.
  c5 Llama-3-70B-shaped GQA decode: 64/8 heads, head_dim 128, Q8_0 KV of
     length 32768, 64 sequences; a step is 16 decode steps of one layer (80
     layers do not fit one GPU).  value: KV GB/s.
value is measured with the inputs resident in HBM: the API's launches for a
step are captured once into CUDA graphs and replayed, the L2 flushed between
steps (outside the timed events).  e2e repeats the step through the C ABI from
a native loop (qlb_run_job: one ql_attn_forward per layer per token step),
with the step's Q/K/V copied from pinned host memory and its outputs copied
back inside the timed region (on a copy stream, in chunks of layers or token
steps that overlap the calls).  Multi-GPU (torchrun): every rank runs its own
replica (weak scaling, no data-path collective); times are the max over ranks.
--impl reference times the CPU oracle (the restatement of the reference's Rust
CPU attention) on this host's cores on a bounded sample of the same workload.
"""
from __future__ import annotations

import argparse
import ctypes
import json
import os
import statistics
import subprocess
import sys
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

METRIC = "decode attn KV GB/s + prefill TFLOP/s (% roofline), tok/s at 1/2/4/8 B200"

WORKLOADS = {
    "c2": dict(kind="job", unit="tok/s",
               desc="TinyLlama-1.1B-shaped attention: 22 layers, 32 Q / 4 KV heads, head_dim 64, "
                    "theta 1e4, f16 KV, batch 1, causal prefill 512 then 256 decode steps",
               layers=22, hq=32, hkv=4, hd=64, theta=10000.0, kv="f16", batch=1, prefill=512,
               decode=256, in_dtype="f16", out_dtype="f16", page=64),
    "c3": dict(kind="decode", unit="GB/s",
               desc="Llama-2-7B-shaped MHA decode: 32 layers, 32/32 heads, head_dim 128, f16 KV "
                    "pre-filled to ragged lengths U[1024,4096], batch 16, 128 decode steps",
               layers=32, hq=32, hkv=32, hd=128, theta=10000.0, kv="f16", batch=16, prefill=0,
               len_lo=1024, len_hi=4096, decode=128, in_dtype="f16", out_dtype="f16", page=64),
    "c4": dict(kind="prefill", unit="TFLOP/s",
               desc="Llama-3-8B-shaped GQA causal prefill: 32/8 heads, head_dim 128, theta 5e5, "
                    "bf16 Q/K/V, f16 KV, batch 4 x 8192 tokens, one layer",
               layers=1, hq=32, hkv=8, hd=128, theta=500000.0, kv="f16", batch=4, prefill=8192,
               decode=0, in_dtype="bf16", out_dtype="bf16", page=64),
    "c5": dict(kind="decode", unit="GB/s",
               desc="Llama-3-70B-shaped GQA decode: 64/8 heads, head_dim 128, Q8_0 KV at length "
                    "32768, batch 64, one layer of 80",
               layers=1, hq=64, hkv=8, hd=128, theta=500000.0, kv="q8_0", batch=64, prefill=0,
               len_lo=32768 - 16, len_hi=32768 - 16, decode=16, in_dtype="bf16",
               out_dtype="bf16", page=64, shard=True),
}

KV_BYTES = {"f16": 2.0, "bf16": 2.0, "f32": 4.0, "q8_0": 34.0 / 32.0}
IO_BYTES = {"f16": 2, "bf16": 2, "f32": 4}


def peaks():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        d = json.load(open(p))
        return float(d["hbm_gbs"]), float(d["bf16_tflops"]), "measured"
    return 6650.0, 1590.0, "fallback"


def ncu_traffic(workload, batch, alg_bytes):
    """DRAM bytes per launch of the dominant kernel, scaled from the small-case
    ncu capture in profiles/dram_traffic.txt (None when there is none)."""
    path = os.path.join(ROOT, "profiles", "dram_traffic.txt")
    if not os.path.exists(path):
        return None
    for line in open(path):
        f = line.split()
        if not f or f[0].startswith("#") or f[0] != workload:
            continue
        case_batch, rd, wr, case_alg = int(f[2]), float(f[3]), float(f[4]), float(f[5])
        if WORKLOADS[workload]["kind"] == "prefill":
            return (rd + wr) * batch / case_batch
        return (rd + wr) / case_alg * alg_bytes
    return None


def seq_lengths(w, rank=0):
    """Cached lengths of the sequences before the first decode step (seeded)."""
    if w["kind"] != "decode":
        return np.zeros(w["batch"], np.int64)
    rng = np.random.default_rng(4096 + rank)
    return rng.integers(w["len_lo"], w["len_hi"] + 1, size=w["batch"]).astype(np.int64)


# ---------------------------------------------------------------- clocks ----

class ClockSampler:
    FIELDS = ("clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.hw_slowdown,"
              "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,"
              "clocks_event_reasons.sw_power_cap")
    NAMES = ("hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap")

    def __init__(self, gpu_index: int):
        self.idx = gpu_index
        self.proc = None

    def start(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", "-i", str(self.idx), "--query-gpu=" + self.FIELDS,
                 "--format=csv,noheader,nounits", "-lms", "200"],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except OSError:
            self.proc = None

    def stop(self):
        if not self.proc:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"]}
        self.proc.terminate()
        out, _ = self.proc.communicate(timeout=10)
        sm, mx, reasons = [], None, set()
        for line in out.strip().splitlines():
            parts = [x.strip() for x in line.split(",")]
            if len(parts) < 7:
                continue
            try:
                sm.append(float(parts[0]))
                mx = float(parts[1])
            except ValueError:
                continue
            for name, val in zip(self.NAMES, parts[3:7]):
                if val.lower() == "active":
                    reasons.add(name)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": mx,
                "reasons": sorted(reasons), "samples": len(sm)}


# ------------------------------------------------------------ CPU oracle ----

def _cpu_inputs(rng, m, heads, hd):
    return rng.standard_normal((m, heads, hd)).astype(np.float16).astype(np.float32)


def cpu_sample(w, layers=None, seed=7):
    """A bounded sample of the workload on the host through the CPU oracle.

    Returns the value the reference's CPU path reaches on it, in the
    workload's unit, with a description of what was run and how it scales.
    """
    import oracle

    threads = os.cpu_count() or 1
    oracle.set_threads(threads)
    rng = np.random.default_rng(seed)
    hq, hkv, hd, th = w["hq"], w["hkv"], w["hd"], w["theta"]
    if w["kind"] == "job":
        P, D = w["prefill"], w["decode"]
        n = w["layers"] if layers is None else layers
        cache = oracle.KvCache(n, P + D, hkv, hd, oracle.F32)
        t = 0.0
        for layer in range(n):
            q, k, v = (_cpu_inputs(rng, P, h, hd) for h in (hq, hkv, hkv))
            dec = [tuple(_cpu_inputs(rng, 1, h, hd) for h in (hq, hkv, hkv)) for _ in range(D)]
            t0 = time.perf_counter()
            oracle.attention_with_cache(cache, layer, q, k, v, 0, hq, hkv, hd, th)
            for s, (dq, dk, dv) in enumerate(dec):
                oracle.attention_with_cache(cache, layer, dq, dk, dv, P + s, hq, hkv, hd, th)
            t += time.perf_counter() - t0
        t_job = t * w["layers"] / n
        return {"value": w["batch"] * (P + D) / t_job, "unit": "tok/s", "cores": threads,
                "kind": "port",
                "sample": f"{n} of {w['layers']} layers of the job (prefill {P} + {D} decode "
                          f"steps each, {t:.1f} s), scaled by layers"}
    if w["kind"] == "prefill":
        S, g = w["prefill"], hq // hkv
        cache = oracle.KvCache(1, S, 1, hd, oracle.F32)
        q, k, v = _cpu_inputs(rng, S, g, hd), _cpu_inputs(rng, S, 1, hd), _cpu_inputs(rng, S, 1, hd)
        t0 = time.perf_counter()
        oracle.attention_with_cache(cache, 0, q, k, v, 0, g, 1, hd, th)
        t = time.perf_counter() - t0
        flops = 4.0 * g * hd * S * (S + 1) / 2
        return {"value": flops / t / 1e12, "unit": "TFLOP/s", "cores": threads, "kind": "port",
                "sample": f"1 sequence x 1 KV group ({g} query heads) x {S} tokens ({t:.1f} s); "
                          f"the rate stands for all {w['batch']} sequences x {hkv} groups"}
    lens = seq_lengths(w)
    nseq = min(len(lens), 16 if w["kv"] != "q8_0" else 2)
    t, byts = 0.0, 0.0
    for b in range(nseq):
        L = int(lens[b])
        cache = oracle.KvCache(1, L + 1, hkv, hd, oracle.F32)
        kk, vv = _cpu_inputs(rng, L, hkv, hd), _cpu_inputs(rng, L, hkv, hd)
        cache.update(0, oracle.rope(kk, hd, 0, th), vv, np.arange(L))
        q, k, v = (_cpu_inputs(rng, 1, h, hd) for h in (hq, hkv, hkv))
        t0 = time.perf_counter()
        oracle.attention_with_cache(cache, 0, q, k, v, L, hq, hkv, hd, th)
        t += time.perf_counter() - t0
        byts += (L + 1) * hkv * hd * 2 * KV_BYTES[w["kv"]]
    return {"value": byts / t / 1e9, "unit": "GB/s", "cores": threads, "kind": "port",
            "sample": f"1 decode step of 1 layer for {nseq} of {len(lens)} sequences "
                      f"({t:.1f} s); algorithmic {w['kv']} KV bytes over that time"}


def run_reference(args, w):
    if int(os.environ.get("RANK", "0")) != 0:
        return
    vals, last = [], None
    for i in range(args.warmup + args.steps):
        last = cpu_sample(w, layers=4 if w["kind"] == "job" else None, seed=100 + i)
        if i >= args.warmup:
            vals.append(last["value"])
    value = statistics.median(vals)
    cb = {k: last[k] for k in ("unit", "cores", "kind", "sample")}
    cb["value"] = value
    print(json.dumps({
        "impl": "reference", "metric": METRIC, "value": value, "unit": w["unit"],
        "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup, "ms_per_step": None,
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32",
        "data": "synthetic", "config": {"workload": args.workload, "desc": w["desc"]},
        "cpu_baseline": cb,
        "e2e": {"value": value, "unit": w["unit"], "h2d_bytes_per_step": 0,
                "d2h_bytes_per_step": 0}}), flush=True)


# ------------------------------------------------------------------ GPU -----

def run_ours(args, w):
    import torch
    import torch.distributed as dist

    import qllama_b200 as qb

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    if world > 1:
        import datetime

        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300),
                                device_id=torch.device("cuda", local))
    dev = torch.device("cuda", local)
    qb.load()
    blib = ctypes.CDLL(qb.build.BENCH_LIB)
    vp, i32 = ctypes.c_void_p, ctypes.c_int32
    blib.qlb_run_job.argtypes = [vp, vp, i32, i32, i32, i32, vp, i32, i32, i32, ctypes.c_float,
                                 i32, i32] + [vp] * 8 + [vp, i32, i32]
    blib.qlb_run_job.restype = ctypes.c_int

    kind = w["kind"]
    Lyr, hq, hkv, hd, B = w["layers"], w["hq"], w["hkv"], w["hd"], w["batch"]
    # Under torchrun the 70B-shaped decode splits its KV heads over the GPUs
    # (strong scaling, outputs all-gathered inside the decode kernel); the
    # other workloads run one independent replica per GPU (weak scaling).
    shard = world > 1 and (args.shard == "heads" or (args.shard == "auto" and w.get("shard")))
    if shard:
        qb.shard_heads(hq, hkv, world, rank)  # raises unless the heads split evenly
    hq_r, hkv_r = (hq // world, hkv // world) if shard else (hq, hkv)  # this rank's heads
    P, D = w["prefill"], w["decode"]
    tdt = {"f16": torch.float16, "bf16": torch.bfloat16, "f32": torch.float32}
    in_t, out_t = tdt[w["in_dtype"]], tdt[w["out_dtype"]]
    code = {"f32": qb.F32, "f16": qb.F16, "bf16": qb.BF16}
    gen = torch.Generator(device=dev)
    gen.manual_seed(1234 + rank)

    def rnd(*shape):
        if 0 in shape:
            return torch.empty(0, device=dev, dtype=in_t)
        return torch.randn(*shape, generator=gen, device=dev, dtype=torch.float32).to(in_t)

    ctx = qb.Context(local)
    stream = torch.cuda.Stream(device=dev)
    ctx.set_stream(stream.cuda_stream)
    lens0 = seq_lengths(w, 0 if shard else rank)  # lengths before the step's first new token
    kv = qb.KvCache(ctx, Lyr, int(lens0.max()) + P + D, hkv_r, hd, w["kv"], w["page"], B)
    comm = None
    if shard:
        uid = [qb.comm_unique_id() if rank == 0 else None]
        dist.broadcast_object_list(uid, src=0)
        comm = qb.Comm(ctx, world, rank, uid[0], B * max(P, 1) * hq * hd * 4, "p2p")
    if kind == "decode":  # pre-fill: seeded N(0,1) rotated keys and values
        for layer in range(Lyr):
            for b in range(B):
                L = int(lens0[b])
                kk = torch.randn(L, hkv_r, hd, generator=gen, device=dev, dtype=torch.float16)
                kv.update(layer, kk, kk.flip(0), np.arange(L), seq=b)
        torch.cuda.synchronize(dev)

    pq, pk, pv = rnd(Lyr, B, P, hq_r, hd), rnd(Lyr, B, P, hkv_r, hd), rnd(Lyr, B, P, hkv_r, hd)
    dq = rnd(D, Lyr, B, 1, hq_r, hd)
    dk, dv = rnd(D, Lyr, B, 1, hkv_r, hd), rnd(D, Lyr, B, 1, hkv_r, hd)
    pout = torch.empty(Lyr, B, P, hq * hd, device=dev, dtype=out_t)
    dout = torch.empty(D, Lyr, B, 1, hq * hd, device=dev, dtype=out_t)
    bufs = (pq, pk, pv, pout, dq, dk, dv, dout)

    def job(prefill, steps):
        """One phase through the C ABI: `prefill` tokens from position 0, or
        `steps` single-token steps from each sequence's length after the prefill."""
        st = np.ascontiguousarray(lens0 + P, dtype=np.int64)
        ptrs = [t.data_ptr() if t.numel() else None for t in bufs]
        rc = blib.qlb_run_job(ctx._h, kv._h, Lyr, B, prefill, steps, st.ctypes.data, hq_r, hkv_r,
                              hd, w["theta"], code[w["in_dtype"]], code[w["out_dtype"]], *ptrs,
                              comm._h if comm else None, hq, 0)
        if rc != 0:
            raise qb.QllamaError(rc, qb.load().ql_last_error().decode())

    def rewind():
        """Back to the state before the step (pages kept), so it can be issued again."""
        if kind == "decode":
            for b in range(B):
                kv.truncate(b, int(lens0[b]))
        else:
            kv.clear()

    phases = []
    if P:
        phases.append(("prefill", lambda: job(P, 0)))
    if D:
        phases.append(("decode", lambda: job(0, D)))

    # warm-up through the API (pages, workspace, RoPE table, kernel attributes),
    # then capture the same launches, one graph per phase
    with torch.cuda.stream(stream):
        for _, fn in phases:
            fn()
    stream.synchronize()
    ctx.synchronize()
    rewind()
    graphs = []
    for name, fn in phases:
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, stream=stream):
            fn()
        graphs.append((name, g))
    rewind()
    launches = {"job": Lyr * 2 + D * Lyr, "prefill": Lyr * 3, "decode": D * Lyr}[kind]

    flush = torch.empty(256 * 1024 * 1024, dtype=torch.uint8, device=dev)

    def barrier():
        torch.cuda.synchronize(dev)
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize(dev)

    for _ in range(args.warmup):
        with torch.cuda.stream(stream):
            for _, g in graphs:
                g.replay()
    stream.synchronize()
    ctx.synchronize()
    nph = len(graphs)
    ev = [[torch.cuda.Event(enable_timing=True) for _ in range(nph + 1)] for _ in range(args.steps)]
    gpu_index = local
    cvd = os.environ.get("CUDA_VISIBLE_DEVICES")
    if cvd:
        gpu_index = int(cvd.split(",")[local])
    sampler = ClockSampler(gpu_index)
    barrier()
    sampler.start()
    time.sleep(0.3)
    for i in range(args.steps):
        with torch.cuda.stream(stream):
            flush.zero_()  # evict the previous step's data from L2 (outside the events)
            ev[i][0].record(stream)
            for p, (_, g) in enumerate(graphs):
                g.replay()
                ev[i][p + 1].record(stream)
    barrier()
    clocks = sampler.stop()
    ctx.synchronize()
    t_ph = [sum(e[p].elapsed_time(e[p + 1]) for e in ev) / 1e3 for p in range(nph)]
    if world > 1:
        tt = torch.tensor(t_ph, device=dev, dtype=torch.float64)
        dist.all_reduce(tt, op=dist.ReduceOp.MAX)
        t_ph = tt.tolist()
    t_tot = sum(t_ph)
    ph = dict(zip([n for n, _ in graphs], t_ph))

    # ---- algorithmic work of one step
    hbm, bf16, which = peaks()
    eb, ib, ob = KV_BYTES[w["kv"]], IO_BYTES[w["in_dtype"]], IO_BYTES[w["out_dtype"]]
    dec_bytes = 0.0
    for s in range(D):
        dec_bytes += Lyr * float(np.sum(lens0 + P + s + 1)) * hkv_r * hd * 2 * eb
    dec_bytes += D * Lyr * B * ((hq_r + 4 * hkv_r) * hd * ib + hq * hd * ob)
    pre_flops = 4.0 * B * hq_r * hd * P * (P + 1) / 2 * Lyr
    tokens = B * (P + D)
    # bytes and FLOPs add up over the ranks; with sharded heads the tokens do not
    tok_mult = 1 if shard else world
    step_value = {"job": tokens, "prefill": pre_flops / 1e12, "decode": dec_bytes / 1e9}[kind]
    value = (tok_mult if kind == "job" else world) * args.steps * step_value / t_tot

    # ---- e2e through the C ABI from pinned host memory
    # The step's inputs come from pinned host memory and its outputs go back
    # to it, every step, inside the timed region.  The copies run on a copy
    # stream in chunks (the prefill inputs a few layers at a time, then the
    # decode inputs a few token steps at a time) so that they overlap the
    # calls, which wait for their chunk's inputs; each chunk's outputs are
    # copied back once its calls end.
    host_in = [t.cpu().pin_memory() for t in (pq, pk, pv, dq, dk, dv)]
    host_out = [torch.empty(t.shape, dtype=t.dtype, pin_memory=True) for t in (pout, dout)]
    h2d = sum(t.numel() * t.element_size() for t in host_in)
    d2h = sum(t.numel() * t.element_size() for t in host_out)
    e2e_reps = max(1, min(args.steps, 3))
    cstream = torch.cuda.Stream(device=dev)
    chunk = max(1, (D + 7) // 8)  # decode steps per copy chunk
    dchunks = [(c0, min(D, c0 + chunk)) for c0 in range(0, D, chunk)]
    lchunk = max(1, (Lyr + 7) // 8)  # prefill layers per copy chunk
    pchunks = [(c0, min(Lyr, c0 + lchunk)) for c0 in range(0, Lyr, lchunk)] if P else []

    def job_steps(s0, s1):
        """Decode steps [s0, s1) through the C ABI (inputs and outputs of those steps)."""
        st = np.ascontiguousarray(lens0 + P + s0, dtype=np.int64)
        ptrs = [None] * 4 + [t[s0].data_ptr() for t in (dq, dk, dv, dout)]
        rc = blib.qlb_run_job(ctx._h, kv._h, Lyr, B, 0, s1 - s0, st.ctypes.data, hq_r, hkv_r, hd,
                              w["theta"], code[w["in_dtype"]], code[w["out_dtype"]], *ptrs,
                              comm._h if comm else None, hq, 0)
        if rc != 0:
            raise qb.QllamaError(rc, qb.load().ql_last_error().decode())

    def job_layers(l0, l1):
        """The prefill of cache layers [l0, l1) through the C ABI."""
        st = np.ascontiguousarray(lens0 + P, dtype=np.int64)
        ptrs = [t[l0].data_ptr() for t in (pq, pk, pv, pout)] + [None] * 4
        rc = blib.qlb_run_job(ctx._h, kv._h, l1 - l0, B, P, 0, st.ctypes.data, hq_r, hkv_r, hd,
                              w["theta"], code[w["in_dtype"]], code[w["out_dtype"]], *ptrs,
                              comm._h if comm else None, hq, l0)
        if rc != 0:
            raise qb.QllamaError(rc, qb.load().ql_last_error().decode())

    def e2e_step():
        """One step: chunked copies in on `cstream`, the calls on `stream`, copies out."""
        ev_c = torch.cuda.Event()
        ev_c.record(stream)
        cstream.wait_event(ev_c)  # the previous step's calls are done with the buffers
        ready = []
        with torch.cuda.stream(cstream):
            for l0, l1 in pchunks:
                for dst, src in zip((pq, pk, pv), host_in[:3]):
                    dst[l0:l1].copy_(src[l0:l1], non_blocking=True)
                e = torch.cuda.Event()
                e.record(cstream)
                ready.append(e)
            for s0, s1 in dchunks:
                for dst, src in zip((dq, dk, dv), host_in[3:]):
                    dst[s0:s1].copy_(src[s0:s1], non_blocking=True)
                e = torch.cuda.Event()
                e.record(cstream)
                ready.append(e)
        with torch.cuda.stream(stream):
            rewind()
            k = 0
            for l0, l1 in pchunks:
                stream.wait_event(ready[k])
                k += 1
                job_layers(l0, l1)
                e = torch.cuda.Event()
                e.record(stream)
                cstream.wait_event(e)
                with torch.cuda.stream(cstream):
                    host_out[0][l0:l1].copy_(pout[l0:l1], non_blocking=True)
            for s0, s1 in dchunks:
                stream.wait_event(ready[k])
                k += 1
                job_steps(s0, s1)
                e = torch.cuda.Event()
                e.record(stream)
                cstream.wait_event(e)
                with torch.cuda.stream(cstream):
                    host_out[1][s0:s1].copy_(dout[s0:s1], non_blocking=True)
        done = torch.cuda.Event()
        done.record(cstream)
        stream.wait_event(done)  # the step ends when its outputs are in host memory

    t0 = torch.cuda.Event(enable_timing=True)
    t1 = torch.cuda.Event(enable_timing=True)
    for it in range(1 + e2e_reps):
        if it == 1:
            barrier()
            t0.record(stream)
        e2e_step()
    t1.record(stream)
    barrier()
    ctx.synchronize()
    t_e2e = t0.elapsed_time(t1) / 1e3
    if world > 1:
        tt = torch.tensor([t_e2e], device=dev, dtype=torch.float64)
        dist.all_reduce(tt, op=dist.ReduceOp.MAX)
        t_e2e = tt.item()
    e2e_value = (tok_mult if kind == "job" else world) * e2e_reps * step_value / t_e2e

    # ---- roofline of the dominant kernel
    if kind == "prefill":
        t_pre = ph["prefill"] / args.steps
        achieved = pre_flops / t_pre / 1e12
        roof = {"kernel": "prefill_tc_kernel<128> (tcgen05/TMEM causal attention)",
                "bound": "tensor", "achieved": achieved, "peak": bf16, "unit": "TFLOP/s",
                "frac": achieved / bf16, "peak_source": which,
                "traffic": ncu_traffic(args.workload, B, None),
                "flops_per_launch": pre_flops / Lyr, "launch_us": 1e6 * t_pre / Lyr,
                "timed": "the whole call: append, rotated-q and attention kernels"}
    else:
        t_dec = ph["decode"] / args.steps
        achieved = dec_bytes / t_dec / 1e9
        roof = {"kernel": f"splitkv_kernel<{hd},{w['kv']}> (fused RoPE+append+decode attention)",
                "bound": "hbm", "achieved": achieved, "peak": hbm, "unit": "GB/s",
                "frac": achieved / hbm, "peak_source": which,
                "traffic": ncu_traffic(args.workload, B, dec_bytes / (D * Lyr)),
                "bytes_per_launch": dec_bytes / (D * Lyr), "launch_us": 1e6 * t_dec / (D * Lyr),
                "timed": "decode phase / launches, graph gaps included"}
    if rank == 0:
        phases_out = {}
        if P:
            tf = world * args.steps * pre_flops / ph["prefill"] / 1e12
            phases_out["prefill"] = {"ms_per_step": 1e3 * ph["prefill"] / args.steps,
                                     "tflops": tf, "frac_bf16_peak": tf / bf16}
        if D:
            gbs = world * args.steps * dec_bytes / ph["decode"] / 1e9
            phases_out["decode"] = {"ms_per_step": 1e3 * ph["decode"] / args.steps,
                                    "kv_gbs": gbs, "frac_hbm": gbs / hbm,
                                    "tok_s": tok_mult * args.steps * B * D / ph["decode"]}
        line = {
            "metric": METRIC, "value": value, "unit": w["unit"], "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": 1e3 * t_tot / args.steps,
            "higher_is_better": True, "scaling": "strong" if shard else "weak",
            "vs_baseline": None,
            "dtype": "q8_0/f16" if w["kv"] == "q8_0" else "f16", "data": "synthetic",
            "config": {"workload": args.workload, "desc": w["desc"], "layers": Lyr,
                       "num_heads": hq, "num_kv_heads": hkv, "head_dim": hd, "kv_dtype": w["kv"],
                       "batch_per_gpu": B, "prefill": P, "decode_steps": D,
                       "page_size": w["page"],
                       "l2": "flushed between steps (256 MB write outside the timed events)",
                       "parallelism": (f"KV heads split over {world} GPUs ({hkv_r} KV / {hq_r} "
                                       f"query heads each), outputs all-gathered over NVLink "
                                       f"inside the decode kernel" if shard else
                                       f"{world} independent replica(s), one per GPU"),
                       "timing": "CUDA events around CUDA-graph replays of the API's launches"},
            "roofline": roof, "phases": phases_out,
            "e2e": {"value": e2e_value, "unit": w["unit"], "h2d_bytes_per_step": h2d,
                    "d2h_bytes_per_step": d2h,
                    "path": "qlb_run_job -> ql_attn_forward" + ("_sharded" if shard else "") +
                            " per layer per token step (C ABI)"},
            "gpu_launches": launches * args.steps,
            "clocks": clocks,
        }
        if world == 1 and not args.no_cpu_baseline:
            cb = cpu_sample(w)
            line["cpu_baseline"] = {k: cb[k] for k in ("value", "unit", "cores", "kind",
                                                       "sample")}
        print(json.dumps(line), flush=True)
    del graphs
    if comm:
        comm.close()
    kv.close()
    ctx.close()
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


def main():
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawTextHelpFormatter)
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=5)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", choices=("ours", "reference"), default="ours")
    ap.add_argument("--workload", choices=sorted(WORKLOADS), default="c2")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--batch", type=int, default=None,
                    help="override the workload's batch (a smaller case of the same shapes, "
                         "e.g. for an ncu capture; the line then names the changed config)")
    ap.add_argument("--layers", type=int, default=None, help="override the layer count")
    ap.add_argument("--shard", choices=("auto", "heads", "replicas"), default="auto",
                    help="with several GPUs: split the KV heads (auto: the 70B-shaped decode) "
                         "or run independent replicas")
    args = ap.parse_args()
    w = dict(WORKLOADS[args.workload])
    for key in ("batch", "layers"):
        if getattr(args, key) is not None:
            w[key] = getattr(args, key)
            w["desc"] += f" [{key} overridden to {w[key]}]"
    if args.impl == "reference":
        run_reference(args, w)
    else:
        run_ours(args, w)


if __name__ == "__main__":
    main()
