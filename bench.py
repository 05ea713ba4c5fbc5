#!/usr/bin/env python
"""Benchmark of the Qllama attention hot path on B200.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
                    [--workload c2|c3|c4|c5] [--only]

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
     Q/K/V (bf16 cache), 4 sequences x 8192 tokens; a step is one layer's causal
     prefill.  value: TFLOP/s counting unmasked pairs only.
  c5 Llama-3-70B-shaped GQA decode: 64/8 heads, head_dim 128, Q8_0 KV of
     length 32768, 64 sequences; a step is 16 decode steps of one layer (80
     layers do not fit one GPU).  value: KV GB/s.

The line's headline is the chosen workload (c2 by default).  Unless --only is
given, the same run also measures the other workloads and reports them under
"workloads": on one GPU c3, c4 and c5 (fewer timed steps, stated per entry);
under torchrun the 70B-shaped decode with its KV heads split over the GPUs,
once with the exchange fused into the decode kernel (NVLink peer stores) and
once with the NCCL all-gather baseline, after a check of the sharded output
against a single-GPU call over all heads on rank 0.

value is measured with the inputs resident in HBM: the API's launches for a
step are captured once into CUDA graphs and replayed, the L2 flushed between
steps (outside the timed events).  e2e repeats the step through the C ABI from
a native loop (qlb_run_job: one ql_attn_forward per layer per token step),
with the step's Q/K/V copied from pinned host memory and its outputs copied
back inside the timed region (on a copy stream, in chunks that overlap the
calls).  The e2e steps also pay for page reservation: decode workloads keep
going from where the previous step ended (sequences enter new pages as they
grow) and whole jobs release their pages between steps (ql_kv_clear_seq).

Multi-GPU (torchrun): the headline runs one replica of the TinyLlama-shaped
job per GPU (weak scaling); "workloads" adds its head split over 2 or 4 GPUs
(strong scaling, outputs all-gathered over NVLink inside the kernels) and the
70B-shaped decode split over every GPU; times are the max over ranks.
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
    # shard_upto: the most GPUs the workload splits its KV heads over in the
    # line's headline (0: replicas).  The batch-1 job is bound by per-call
    # latency, which a per-layer exchange between GPUs only lengthens, so its
    # headline runs one replica per GPU and its head split is reported beside it.
    "c2": dict(kind="job", unit="tok/s",
               desc="TinyLlama-1.1B-shaped attention: 22 layers, 32 Q / 4 KV heads, head_dim 64, "
                    "theta 1e4, f16 KV, batch 1, causal prefill 512 then 256 decode steps",
               layers=22, hq=32, hkv=4, hd=64, theta=10000.0, kv="f16", batch=1, prefill=512,
               decode=256, in_dtype="f16", out_dtype="f16", page=64, shard_upto=0),
    "c3": dict(kind="decode", unit="GB/s",
               desc="Llama-2-7B-shaped MHA decode: 32 layers, 32/32 heads, head_dim 128, f16 KV "
                    "pre-filled to ragged lengths U[1024,4096], batch 16, 128 decode steps",
               layers=32, hq=32, hkv=32, hd=128, theta=10000.0, kv="f16", batch=16, prefill=0,
               len_lo=1024, len_hi=4096, decode=128, in_dtype="f16", out_dtype="f16", page=64,
               shard_upto=0),
    "c4": dict(kind="prefill", unit="TFLOP/s",
               desc="Llama-3-8B-shaped GQA causal prefill: 32/8 heads, head_dim 128, theta 5e5, "
                    "bf16 Q/K/V, bf16 KV, batch 4 x 8192 tokens, one layer",
               layers=1, hq=32, hkv=8, hd=128, theta=500000.0, kv="bf16", batch=4, prefill=8192,
               decode=0, in_dtype="bf16", out_dtype="bf16", page=64, shard_upto=0),
    "c5": dict(kind="decode", unit="GB/s",
               desc="Llama-3-70B-shaped GQA decode: 64/8 heads, head_dim 128, Q8_0 KV at length "
                    "32768, batch 64, one layer of 80",
               layers=1, hq=64, hkv=8, hd=128, theta=500000.0, kv="q8_0", batch=64, prefill=0,
               len_lo=32768 - 16, len_hi=32768 - 16, decode=16, in_dtype="bf16",
               out_dtype="bf16", page=64, shard_upto=8),
}

KV_BYTES = {"f16": 2.0, "bf16": 2.0, "f32": 4.0, "q8_0": 34.0 / 32.0}
IO_BYTES = {"f16": 2, "bf16": 2, "f32": 4}
# The oracle's CPU sample of the job workload: this many of its layers, scaled.
CPU_JOB_LAYERS = 4


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


def sharded(w, world):
    """Whether the workload splits its KV heads over `world` GPUs (else replicas)."""
    return 1 < world <= w["shard_upto"] and w["hkv"] % world == 0


def parallelism(w, world):
    if world == 1:
        return "1 GPU"
    if sharded(w, world):
        hkv_r, hq_r = w["hkv"] // world, w["hq"] // world
        return (f"KV heads split over {world} GPUs ({hkv_r} KV / {hq_r} query heads each), "
                f"outputs all-gathered over NVLink inside the kernels")
    return f"{world} independent replicas, one per GPU"


def config_of(name, w, world):
    """The workload a line measures; both arms print the same dict."""
    return {"workload": name, "desc": w["desc"], "layers": w["layers"], "num_heads": w["hq"],
            "num_kv_heads": w["hkv"], "head_dim": w["hd"], "kv_dtype": w["kv"],
            "batch": w["batch"], "prefill": w["prefill"], "decode_steps": w["decode"],
            "page_size": w["page"], "parallelism": parallelism(w, world)}


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


def cpu_sample(w, seed=7):
    """A bounded sample of the workload on the host through the CPU oracle.

    Returns the value the reference's CPU path reaches on it, in the
    workload's unit, with a description of what was run and how it scales.
    Both arms of the benchmark report this same sample.
    """
    import oracle

    threads = os.cpu_count() or 1
    oracle.set_threads(threads)
    rng = np.random.default_rng(seed)
    hq, hkv, hd, th = w["hq"], w["hkv"], w["hd"], w["theta"]
    if w["kind"] == "job":
        P, D = w["prefill"], w["decode"]
        n = min(w["layers"], CPU_JOB_LAYERS)
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
    world = int(os.environ.get("WORLD_SIZE", str(args.gpus)))
    vals, last = [], None
    for i in range(args.warmup + args.steps):
        last = cpu_sample(w, seed=100 + i)
        if i >= args.warmup:
            vals.append(last["value"])
    value = statistics.median(vals)
    cb = {k: last[k] for k in ("unit", "cores", "kind", "sample")}
    cb["value"] = value
    print(json.dumps({
        "impl": "reference", "metric": METRIC, "value": value, "unit": w["unit"],
        "n_gpus": world, "steps": args.steps, "warmup": args.warmup, "ms_per_step": None,
        "higher_is_better": True, "scaling": "strong" if sharded(w, world) else "weak",
        "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "config": config_of(args.workload, w, world),
        "cpu_baseline": cb,
        "e2e": {"value": value, "unit": w["unit"], "h2d_bytes_per_step": 0,
                "d2h_bytes_per_step": 0}}), flush=True)


# ------------------------------------------------------------------ GPU -----

class Env:
    """Process-wide state of one GPU rank."""

    def __init__(self):
        import torch
        import torch.distributed as dist

        import qllama_b200 as qb

        self.torch, self.dist, self.qb = torch, dist, qb
        self.world = int(os.environ.get("WORLD_SIZE", "1"))
        self.rank = int(os.environ.get("RANK", "0"))
        self.local = int(os.environ.get("LOCAL_RANK", "0"))
        torch.cuda.set_device(self.local)
        self.dev = torch.device("cuda", self.local)
        # No NVLink multicast objects: the exchange uses plain peer stores, and
        # NCCL's NVLS buffers are not needed for the gathers measured here.
        os.environ.setdefault("NCCL_NVLS_ENABLE", "0")
        if self.world > 1:
            import datetime

            dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300),
                                    device_id=self.dev)
        qb.load()
        blib = ctypes.CDLL(qb.build.BENCH_LIB)
        vp, i32 = ctypes.c_void_p, ctypes.c_int32
        blib.qlb_run_job.argtypes = [vp, vp, i32, i32, i32, i32, vp, i32, i32, i32,
                                     ctypes.c_float, i32, i32] + [vp] * 8 + [vp, i32, i32]
        blib.qlb_run_job.restype = ctypes.c_int
        self.blib = blib
        self.ctx = qb.Context(self.local)
        self.stream = torch.cuda.Stream(device=self.dev)
        self.ctx.set_stream(self.stream.cuda_stream)
        gpu_index = self.local
        cvd = os.environ.get("CUDA_VISIBLE_DEVICES")
        if cvd:
            gpu_index = int(cvd.split(",")[self.local])
        self.gpu_index = gpu_index
        self.flush = torch.empty(256 * 1024 * 1024, dtype=torch.uint8, device=self.dev)

    def barrier(self):
        self.torch.cuda.synchronize(self.dev)
        if self.world > 1:
            self.dist.barrier()
        self.torch.cuda.synchronize(self.dev)

    def max_over_ranks(self, values):
        if self.world == 1:
            return list(values)
        t = self.torch.tensor(list(values), device=self.dev, dtype=self.torch.float64)
        self.dist.all_reduce(t, op=self.dist.ReduceOp.MAX)
        return t.tolist()

    def comm(self, max_bytes, mode):
        uid = [self.qb.comm_unique_id() if self.rank == 0 else None]
        self.dist.broadcast_object_list(uid, src=0)
        return self.qb.Comm(self.ctx, self.world, self.rank, uid[0], max_bytes, mode)

    def close(self):
        self.ctx.close()
        if self.world > 1:
            self.dist.barrier()
            self.dist.destroy_process_group()


def graph_kernel_nodes(g):
    """Kernel launches a captured CUDA graph holds (None if it cannot be read)."""
    try:
        from cuda.bindings import runtime as rt

        graph = rt.cudaGraph_t(init_value=g.raw_cuda_graph())
        err, _, n = rt.cudaGraphGetNodes(graph, 0)
        if err != rt.cudaError_t.cudaSuccess:
            return None
        err, nodes, n = rt.cudaGraphGetNodes(graph, n)
        if err != rt.cudaError_t.cudaSuccess:
            return None
        count = 0
        for node in nodes[:n]:
            err, typ = rt.cudaGraphNodeGetType(node)
            if err == rt.cudaError_t.cudaSuccess and typ == rt.cudaGraphNodeType.cudaGraphNodeTypeKernel:
                count += 1
        return count
    except Exception:  # an older cuda-python: the count is computed instead
        return None


def measure(env, name, w, steps, warmup, comm_mode="p2p", with_e2e=True):
    """One workload on this rank: device-timed graph replays, then e2e."""
    torch, qb = env.torch, env.qb
    world, rank, dev = env.world, env.rank, env.dev
    kind = w["kind"]
    Lyr, hq, hkv, hd, B = w["layers"], w["hq"], w["hkv"], w["hd"], w["batch"]
    shard = sharded(w, world)
    if shard:
        qb.shard_heads(hq, hkv, world, rank)  # raises unless the heads split evenly
    hq_r, hkv_r = (hq // world, hkv // world) if shard else (hq, hkv)  # this rank's heads
    P, D = w["prefill"], w["decode"]
    tdt = {"f16": torch.float16, "bf16": torch.bfloat16, "f32": torch.float32}
    in_t, out_t = tdt[w["in_dtype"]], tdt[w["out_dtype"]]
    code = {"f32": qb.F32, "f16": qb.F16, "bf16": qb.BF16}
    gen = torch.Generator(device=dev)
    gen.manual_seed(1234 + rank)
    ctx, stream, blib = env.ctx, env.stream, env.blib

    def rnd(*shape):
        if 0 in shape:
            return torch.empty(0, device=dev, dtype=in_t)
        return torch.randn(*shape, generator=gen, device=dev, dtype=torch.float32).to(in_t)

    e2e_reps = max(1, min(steps, 3))
    lens0 = seq_lengths(w, 0 if shard else rank)  # lengths before the step's first new token
    # decode e2e steps continue past the graph-replayed step (1 untimed + e2e_reps)
    cap = int(lens0.max()) + P + D * (2 + e2e_reps if kind == "decode" else 1)
    kv = qb.KvCache(ctx, Lyr, cap, hkv_r, hd, w["kv"], w["page"], B)
    comm = env.comm(B * max(P, 1) * hq * hd * 4, comm_mode) if shard else None
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

    def run_job(layer0, layers, prefill, steps_, starts, ptrs):
        st = np.ascontiguousarray(starts, dtype=np.int64)
        rc = blib.qlb_run_job(ctx._h, kv._h, layers, B, prefill, steps_, st.ctypes.data, hq_r,
                              hkv_r, hd, w["theta"], code[w["in_dtype"]], code[w["out_dtype"]],
                              *ptrs, comm._h if comm else None, hq, layer0)
        if rc != 0:
            raise qb.QllamaError(rc, qb.load().ql_last_error().decode())

    def ptrs_all():
        return [t.data_ptr() if t.numel() else None
                for t in (pq, pk, pv, pout, dq, dk, dv, dout)]

    def rewind():
        """Back to the state before the step (pages kept), so it can be issued again."""
        if kind == "decode":
            for b in range(B):
                kv.truncate(b, int(lens0[b]))
        else:
            kv.clear()

    phases = []
    if P:
        phases.append(("prefill", lambda: run_job(0, Lyr, P, 0, lens0 + P, ptrs_all())))
    if D:
        phases.append(("decode", lambda: run_job(0, Lyr, 0, D, lens0 + P, ptrs_all())))

    # warm-up through the API (pages, workspace, RoPE table, kernel attributes),
    # then capture the same launches, one graph per phase
    with torch.cuda.stream(stream):
        for _, fn in phases:
            fn()
    stream.synchronize()
    ctx.synchronize()
    rewind()
    def capture(fn):
        graph = torch.cuda.CUDAGraph(keep_graph=True)  # kept, so its nodes can be counted
        with torch.cuda.graph(graph, stream=stream):
            fn()
        return graph

    graphs = [(pname, capture(fn)) for pname, fn in phases]
    rewind()
    counted = [graph_kernel_nodes(gr) for _, gr in graphs]
    for entry in graphs:
        entry[1].instantiate()
    if all(c is not None for c in counted):
        launches, launch_src = sum(counted), "kernel nodes of the captured graphs"
    else:
        per_prefill = 2  # tcgen05 prefill: prologue + attention; else append + split-KV
        launches = Lyr * per_prefill * (P > 0) + D * Lyr
        if shard and P:
            launches += Lyr  # the peer copy kernel of each prefill call
        launch_src = "computed from the dispatch rules"

    for _ in range(warmup):
        with torch.cuda.stream(stream):
            for entry in graphs:
                entry[1].replay()
    stream.synchronize()
    ctx.synchronize()
    nph = len(graphs)
    ev = [[torch.cuda.Event(enable_timing=True) for _ in range(nph + 1)] for _ in range(steps)]
    sampler = ClockSampler(env.gpu_index)
    env.barrier()
    sampler.start()
    time.sleep(0.3)
    for i in range(steps):
        with torch.cuda.stream(stream):
            env.flush.zero_()  # evict the previous step's data from L2 (outside the events)
            ev[i][0].record(stream)
            for p, entry in enumerate(graphs):
                entry[1].replay()
                ev[i][p + 1].record(stream)
    env.barrier()
    clocks = sampler.stop()
    ctx.synchronize()
    t_ph = [sum(e[p].elapsed_time(e[p + 1]) for e in ev) / 1e3 for p in range(nph)]
    t_ph = env.max_over_ranks(t_ph)
    t_tot = sum(t_ph)
    ph = dict(zip([n for n, _ in graphs], t_ph))
    # Every reference to the graphs goes before the communicator: a graph that
    # holds NCCL calls keeps the communicator busy, and its destroy would wait.
    del graphs, entry
    torch.cuda.synchronize(dev)

    # ---- algorithmic work of one step (this rank's share)
    hbm, bf16, which = peaks()
    eb, ib, ob = KV_BYTES[w["kv"]], IO_BYTES[w["in_dtype"]], IO_BYTES[w["out_dtype"]]

    def decode_bytes(start_lens):
        tot = 0.0
        for s in range(D):
            tot += Lyr * float(np.sum(start_lens + s + 1)) * hkv_r * hd * 2 * eb
        return tot + D * Lyr * B * ((hq_r + 4 * hkv_r) * hd * ib + hq * hd * ob)

    dec_bytes = decode_bytes(lens0 + P)
    pre_flops = 4.0 * B * hq_r * hd * P * (P + 1) / 2 * Lyr
    tokens = B * (P + D)
    # bytes and FLOPs add up over the ranks; with sharded heads the tokens do not
    tok_mult = 1 if shard else world
    step_value = {"job": tokens * tok_mult, "prefill": world * pre_flops / 1e12,
                  "decode": world * dec_bytes / 1e9}[kind]
    value = steps * step_value / t_tot

    # ---- e2e through the C ABI from pinned host memory
    e2e = None
    if with_e2e:
        host_in = [t.cpu().pin_memory() for t in (pq, pk, pv, dq, dk, dv)]
        host_out = [torch.empty(t.shape, dtype=t.dtype, pin_memory=True) for t in (pout, dout)]
        h2d = sum(t.numel() * t.element_size() for t in host_in)
        d2h = sum(t.numel() * t.element_size() for t in host_out)
        cstream = torch.cuda.Stream(device=dev)
        chunk = max(1, (D + 7) // 8)  # decode steps per copy chunk
        dchunks = [(c0, min(D, c0 + chunk)) for c0 in range(0, D, chunk)]
        lchunk = max(1, (Lyr + 7) // 8)  # prefill layers per copy chunk
        pchunks = [(c0, min(Lyr, c0 + lchunk)) for c0 in range(0, Lyr, lchunk)] if P else []
        # decode workloads: each e2e step continues where the last one ended
        e2e_start = [lens0 + P + (D * it if kind == "decode" else 0) for it in range(1 + e2e_reps)]

        def e2e_step(it):
            """Chunked copies in on `cstream`, the calls on `stream`, copies out."""
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
                if kind != "decode":  # a new job: its pages go back to the pool
                    for b in range(B):
                        kv.clear_seq(b)
                k = 0
                for l0, l1 in pchunks:
                    stream.wait_event(ready[k])
                    k += 1
                    run_job(l0, l1 - l0, P, 0, lens0 + P,
                            [t[l0].data_ptr() for t in (pq, pk, pv, pout)] + [None] * 4)
                    e = torch.cuda.Event()
                    e.record(stream)
                    cstream.wait_event(e)
                    with torch.cuda.stream(cstream):
                        host_out[0][l0:l1].copy_(pout[l0:l1], non_blocking=True)
                for s0, s1 in dchunks:
                    stream.wait_event(ready[k])
                    k += 1
                    run_job(0, Lyr, 0, s1 - s0, e2e_start[it] + s0,
                            [None] * 4 + [t[s0].data_ptr() for t in (dq, dk, dv, dout)])
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
                env.barrier()
                t0.record(stream)
            e2e_step(it)
        t1.record(stream)
        env.barrier()
        ctx.synchronize()
        t_e2e = env.max_over_ranks([t0.elapsed_time(t1) / 1e3])[0]
        if kind == "decode":
            e2e_work = world * sum(decode_bytes(e2e_start[it]) for it in range(1, 1 + e2e_reps)) / 1e9
        else:
            e2e_work = e2e_reps * step_value
        e2e = {"value": e2e_work / t_e2e, "unit": w["unit"], "h2d_bytes_per_step": h2d,
               "d2h_bytes_per_step": d2h,
               "path": "qlb_run_job -> ql_attn_forward" + ("_sharded" if shard else "") +
                       " per layer per token step (C ABI)",
               "pages": ("decode steps continue past the timed step: sequences enter new pages"
                         if kind == "decode" else
                         "every step releases its pages (ql_kv_clear_seq) and reserves them again")}

    # ---- roofline of the dominant kernel (per GPU)
    if kind == "prefill":
        t_pre = ph["prefill"] / steps
        achieved = pre_flops / t_pre / 1e12
        roof = {"kernel": f"prefill_tc_kernel<{hd}> (tcgen05/TMEM causal attention)",
                "bound": "tensor", "achieved": achieved, "peak": bf16, "unit": "TFLOP/s",
                "frac": achieved / bf16, "peak_source": which,
                "traffic": ncu_traffic(name, B, None) if not shard else None,
                "flops_per_launch": pre_flops / Lyr, "launch_us": 1e6 * t_pre / Lyr,
                "timed": "the whole call: append, rotated-q" +
                         (", bf16-to-f16 tile conversion" if w["kv"] == "bf16" else "") +
                         " and attention kernels"}
    else:
        t_dec = ph["decode"] / steps
        achieved = dec_bytes / t_dec / 1e9
        roof = {"kernel": f"splitkv_kernel<{hd},{w['kv']}> (fused RoPE+append+decode attention)",
                "bound": "hbm", "achieved": achieved, "peak": hbm, "unit": "GB/s",
                "frac": achieved / hbm, "peak_source": which,
                "traffic": ncu_traffic(name, B, dec_bytes / (D * Lyr)) if not shard else None,
                "bytes_per_launch": dec_bytes / (D * Lyr), "launch_us": 1e6 * t_dec / (D * Lyr),
                "timed": "decode phase / launches, graph gaps included"}
    phases_out = {}
    if P:
        tf = pre_flops / (ph["prefill"] / steps) / 1e12  # per GPU
        phases_out["prefill"] = {"ms_per_step": 1e3 * ph["prefill"] / steps,
                                 "tflops_per_gpu": tf, "frac_bf16_peak": tf / bf16}
    if D:
        gbs = dec_bytes / (ph["decode"] / steps) / 1e9  # per GPU
        phases_out["decode"] = {"ms_per_step": 1e3 * ph["decode"] / steps,
                                "kv_gbs_per_gpu": gbs, "frac_hbm": gbs / hbm,
                                "tok_s": tok_mult * steps * B * D / ph["decode"]}
    res = {"value": value, "unit": w["unit"], "steps": steps, "warmup": warmup,
           "ms_per_step": 1e3 * t_tot / steps, "scaling": "strong" if shard else "weak",
           "config": config_of(name, w, world), "roofline": roof, "phases": phases_out,
           "e2e": e2e, "gpu_launches": launches * steps, "gpu_launches_source": launch_src,
           "clocks": clocks}
    if shard:
        res["exchange"] = {"p2p": "attention kernel stores its rows into every rank's buffer "
                                  "over NVLink (CUDA IPC mappings), bounded flag waits",
                           "nccl": "local attention, ncclAllGather, head-major permute"}[comm_mode]
    if comm:
        comm.close()
    kv.close()
    del pq, pk, pv, dq, dk, dv, pout, dout
    torch.cuda.empty_cache()
    return res


def check_sharded(env, mode):
    """Max-abs difference between a head-sharded call's gathered output and one
    GPU's call over all heads (rank 0), on the same seeded inputs: a decode step
    (fused exchange) and a 64-token chunk (exchange after the attention)."""
    torch, qb = env.torch, env.qb
    world, rank = env.world, env.rank
    hq, hkv, hd, theta, B, L = 64, 8, 128, 500000.0, 4, 1000
    rng = np.random.default_rng(99)  # the same on every rank
    kfull = rng.standard_normal((B, L, hkv, hd)).astype(np.float32)
    vfull = rng.standard_normal((B, L, hkv, hd)).astype(np.float32)
    qr, kr = qb.shard_heads(hq, hkv, world, rank)
    mine = qb.KvCache(env.ctx, 1, L + 80, len(kr), hd, "f16", 64, B)
    full = qb.KvCache(env.ctx, 1, L + 80, hkv, hd, "f16", 64, B) if rank == 0 else None
    for b in range(B):  # the same cached rows in both (update() stores K as given)
        mine.update(0, np.ascontiguousarray(kfull[b][:, kr.start:kr.stop]),
                    np.ascontiguousarray(vfull[b][:, kr.start:kr.stop]), np.arange(L), seq=b)
        if full:
            full.update(0, kfull[b], vfull[b], np.arange(L), seq=b)
    comm = env.comm(B * 64 * hq * hd * 4, mode)
    worst = 0.0
    start = L
    for n in (1, 64):
        q = rng.standard_normal((B, n, hq, hd)).astype(np.float32)
        k = rng.standard_normal((B, n, hkv, hd)).astype(np.float32)
        v = rng.standard_normal((B, n, hkv, hd)).astype(np.float32)
        dq = torch.from_numpy(np.ascontiguousarray(q[:, :, qr.start:qr.stop])).to(env.dev).half()
        dk = torch.from_numpy(np.ascontiguousarray(k[:, :, kr.start:kr.stop])).to(env.dev).half()
        dv = torch.from_numpy(np.ascontiguousarray(v[:, :, kr.start:kr.stop])).to(env.dev).half()
        with torch.cuda.stream(env.stream):
            out = qb.attention_forward_sharded(comm, mine, 0, dq, dk, dv, [start] * B, len(qr),
                                               len(kr), hd, theta, out_dtype="f32")
        env.ctx.synchronize()
        if full:
            fq, fk, fv = (torch.from_numpy(x).to(env.dev).half() for x in (q, k, v))
            with torch.cuda.stream(env.stream):
                ref = qb.attention_forward(full, 0, fq, fk, fv, [start] * B, hq, hkv, hd, theta,
                                           out_dtype="f32")
            env.ctx.synchronize()
            worst = max(worst, float((out - ref).abs().max().item()))
        start += n
    env.barrier()
    comm.close()
    mine.close()
    if full:
        full.close()
    return worst if rank == 0 else None


def run_ours(args, w):
    env = Env()
    world, rank = env.world, env.rank
    steps, warmup = args.steps, args.warmup
    head = measure(env, args.workload, w, steps, warmup)
    extra = {}
    if not args.only:
        sub_steps, sub_warm = min(steps, 5), 3
        if world == 1:
            for name in ("c2", "c3", "c4", "c5"):
                if name == args.workload:
                    continue
                r = measure(env, name, dict(WORKLOADS[name]), sub_steps, sub_warm)
                if rank == 0 and not args.no_cpu_baseline:
                    cb = cpu_sample(WORKLOADS[name])
                    r["cpu_baseline"] = {k: cb[k] for k in ("value", "unit", "cores", "kind",
                                                            "sample")}
                extra[name] = r
        else:
            # the head split of the path's partition by KV heads, beside the replicas:
            # the TinyLlama-shaped job where its 4 KV heads divide the GPUs, and
            # the 70B-shaped decode through the fused exchange and through NCCL
            w2 = dict(WORKLOADS["c2"], shard_upto=4)
            if sharded(w2, world):
                extra["c2_heads"] = measure(env, "c2", w2, sub_steps, sub_warm)
            w5 = dict(WORKLOADS["c5"])
            if sharded(w5, world):
                for mode in ("p2p", "nccl"):
                    r = measure(env, "c5", w5, sub_steps, sub_warm, comm_mode=mode)
                    r["check_max_abs_err_vs_1gpu"] = check_sharded(env, mode)
                    extra[f"c5_{mode}"] = r
    if rank == 0:
        hbm, bf16, which = peaks()
        line = {
            "metric": METRIC, "value": head["value"], "unit": head["unit"], "n_gpus": world,
            "steps": steps, "warmup": warmup, "ms_per_step": head["ms_per_step"],
            "higher_is_better": True, "scaling": head["scaling"], "vs_baseline": None,
            "dtype": "q8_0/f16" if w["kv"] == "q8_0" else "f16", "data": "synthetic",
            "config": head["config"],
            "l2": "flushed between steps (256 MB write outside the timed events)",
            "timing": "CUDA events around CUDA-graph replays of the API's launches, max over ranks",
            "roofline": head["roofline"], "phases": head["phases"], "e2e": head["e2e"],
            "gpu_launches": head["gpu_launches"],
            "gpu_launches_source": head["gpu_launches_source"], "clocks": head["clocks"],
            "peaks": {"hbm_gbs": hbm, "bf16_tflops": bf16, "source": which},
        }
        if "exchange" in head:
            line["exchange"] = head["exchange"]
        if extra:
            line["workloads"] = extra
        if world == 1 and not args.no_cpu_baseline:
            cb = cpu_sample(w)
            line["cpu_baseline"] = {k: cb[k] for k in ("value", "unit", "cores", "kind",
                                                       "sample")}
        print(json.dumps(line), flush=True)
    env.close()


def main():
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawTextHelpFormatter)
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=5)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", choices=("ours", "reference"), default="ours")
    ap.add_argument("--workload", choices=sorted(WORKLOADS), default="c2")
    ap.add_argument("--only", action="store_true",
                    help="measure the chosen workload alone (no 'workloads' entries)")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--batch", type=int, default=None,
                    help="override the workload's batch (a smaller case of the same shapes, "
                         "e.g. for an ncu capture; the line then names the changed config)")
    ap.add_argument("--layers", type=int, default=None, help="override the layer count")
    ap.add_argument("--kv", choices=("f32", "f16", "bf16", "q8_0"), default=None,
                    help="override the KV cache storage type")
    ap.add_argument("--shard", choices=("auto", "heads", "replicas"), default="auto",
                    help="with several GPUs: the workload's own choice (auto), its KV heads "
                         "split over the GPUs, or replicas")
    args = ap.parse_args()
    args.warmup = max(3, args.warmup)  # at least three untimed steps
    w = dict(WORKLOADS[args.workload])
    for key in ("batch", "layers", "kv"):
        if getattr(args, key) is not None:
            w[key] = getattr(args, key)
            w["desc"] += f" [{key} overridden to {w[key]}]"
    if args.shard != "auto":
        w["shard_upto"] = 0 if args.shard == "replicas" else 8
    if args.impl == "reference":
        run_reference(args, w)
    else:
        run_ours(args, w)


if __name__ == "__main__":
    main()
