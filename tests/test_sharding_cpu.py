"""Head-sharded layers on the CPU: world-size-2 gloo groups, no GPU.

The GPU path splits a layer's KV heads evenly over the ranks (each KV head
keeps its group of query heads, layers.rs:436) and all-gathers the outputs
into the reference's head-major layout (layers.rs:447-455).  Attention of one
head never reads another head's data, so running the oracle per rank on its
heads and gathering must reproduce the full layer bit for bit; these tests
check that plan and the host-side failure detection of the multi-rank path.
"""
from __future__ import annotations

import multiprocessing as mp
import socket

import numpy as np
import pytest

import oracle
import qllama_b200 as qb
from tests import sharding_workers as sw


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _run(target, world, *args, timeout=120):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=target, args=(r, world, port, *args, q)) for r in range(world)]
    for p in procs:
        p.start()
    results = {}
    try:
        for _ in range(world):
            rank, status, payload, extra = q.get(timeout=timeout)
            results[rank] = (status, payload, extra)
    finally:
        for p in procs:
            p.join(timeout=30)
            if p.is_alive():
                p.kill()
    return results


def test_shard_heads_partition():
    for hq, hkv, n in [(64, 8, 8), (64, 8, 2), (32, 32, 4), (32, 8, 4), (6, 6, 3)]:
        q_ranges, kv_ranges = zip(*(qb.shard_heads(hq, hkv, n, r) for r in range(n)))
        assert [h for r in q_ranges for h in r] == list(range(hq))
        assert [h for r in kv_ranges for h in r] == list(range(hkv))
        group = hq // hkv
        for qr, kr in zip(q_ranges, kv_ranges):  # every query head stays with its KV head
            assert [h // group for h in qr] == [h for h in kr for _ in range(group)]
    with pytest.raises(qb.QllamaError, match="split evenly"):
        qb.shard_heads(32, 4, 8, 0)  # 4 KV heads over 8 GPUs: replicas instead
    with pytest.raises(qb.QllamaError, match="outside"):
        qb.shard_heads(32, 8, 2, 2)


def test_head_sharded_oracle_matches_full_layer():
    cfg = dict(hq=16, hkv=4, hd=64, theta=500000.0, seed=7, prefill=37, decode=3,
               storages=["f32", "q8_0"])
    res = _run(sw.oracle_sharded_worker, 2, cfg)
    for rank, (status, payload, _) in res.items():
        assert status == "ok", payload
    assert res[0][2] == 2.0  # max over ranks
    steps = sw.case_inputs(cfg["seed"], cfg["prefill"], cfg["decode"], cfg["hq"], cfg["hkv"],
                           cfg["hd"])
    for storage in cfg["storages"]:
        kv = oracle.KvCache(1, 512, cfg["hkv"], cfg["hd"], oracle.STORAGE[storage])
        pos = 0
        for (q, k, v), got in zip(steps, res[0][1][storage]):
            full = oracle.attention_with_cache(kv, 0, q, k, v, pos, cfg["hq"], cfg["hkv"],
                                               cfg["hd"], cfg["theta"])
            assert np.array_equal(got.view(np.uint32), full.view(np.uint32)), storage
            pos += q.shape[0]


def test_absent_rank_is_detected_not_waited_for():
    res = _run(sw.absent_rank_worker, 2, timeout=60)
    assert res[1][0] == "left"
    assert res[0][0] == "detected", res[0]
