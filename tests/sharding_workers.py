"""Process bodies of the multi-rank tests (started with the spawn method).

Each function runs as one rank of a torch.distributed group, so it must live
at module level to be importable by the child process.
"""
from __future__ import annotations

import datetime
import os
import traceback

import numpy as np


def _init(rank: int, world: int, port: int, backend: str, timeout_s: float):
    import torch.distributed as dist

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group(backend, rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=timeout_s))
    return dist


def case_inputs(seed, n_prefill, n_decode, hq, hkv, hd):
    """Seeded full-width Q/K/V of one sequence: a prefill chunk, then single tokens."""
    rng = np.random.default_rng(seed)
    steps = [n_prefill] + [1] * n_decode
    return [tuple((rng.standard_normal((n, h, hd))).astype(np.float32) for h in (hq, hkv, hkv))
            for n in steps]


def oracle_sharded_worker(rank, world, port, cfg, queue):
    """One rank of the head-sharded layer on the CPU: the oracle over this
    rank's heads, outputs all-gathered (gloo) into the head-major layout."""
    try:
        import torch

        import oracle
        import qllama_b200 as qb

        dist = _init(rank, world, port, "gloo", 30.0)
        hq, hkv, hd, theta = cfg["hq"], cfg["hkv"], cfg["hd"], cfg["theta"]
        qr, kr = qb.shard_heads(hq, hkv, world, rank)
        outs = {}
        for storage in cfg["storages"]:
            kv = oracle.KvCache(1, 512, len(kr), hd, oracle.STORAGE[storage])
            pos, outs[storage] = 0, []
            for q, k, v in case_inputs(cfg["seed"], cfg["prefill"], cfg["decode"], hq, hkv, hd):
                local = oracle.attention_with_cache(kv, 0, q[:, qr.start:qr.stop],
                                                    k[:, kr.start:kr.stop],
                                                    v[:, kr.start:kr.stop], pos, len(qr),
                                                    len(kr), hd, theta)
                parts = [torch.empty_like(torch.from_numpy(local)) for _ in range(world)]
                dist.all_gather(parts, torch.from_numpy(local))
                # rank-major parts -> head-major rows: rank r's heads are columns
                # [r*len(qr)*hd, (r+1)*len(qr)*hd) of every row
                outs[storage].append(torch.cat(parts, dim=-1).numpy())
                pos += q.shape[0]
        # the timing rule of the bench: the maximum over ranks
        t = torch.tensor([float(rank + 1)], dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        dist.barrier()
        dist.destroy_process_group()
        queue.put((rank, "ok", outs if rank == 0 else None, t.item()))
    except Exception:  # reported to the test, never swallowed
        queue.put((rank, "error", traceback.format_exc(), None))


def absent_rank_worker(rank, world, port, queue):
    """Rank 1 leaves between steps without joining the collective; rank 0 must
    get an error from its next collective instead of waiting for ever."""
    try:
        import torch

        dist = _init(rank, world, port, "gloo", 3.0)
        dist.barrier()
        if rank == 1:
            queue.put((rank, "left", None, None))
            queue.close()
            queue.join_thread()  # the message is out before the process vanishes
            os._exit(0)  # no destroy_process_group: the rank just disappears
        try:
            dist.all_reduce(torch.ones(4))
            queue.put((rank, "no error", None, None))
        except Exception as e:  # the detection this test wants
            queue.put((rank, "detected", type(e).__name__, None))
    except Exception:
        queue.put((rank, "error", traceback.format_exc(), None))


def gpu_sharded_worker(rank, world, port, cfg, queue):
    """One GPU of a head-sharded layer: its KV heads in its own cache, the
    outputs exchanged by the library; every rank checks the whole layer's
    output against the oracle over all heads."""
    try:
        os.environ.setdefault("NCCL_NVLS_ENABLE", "0")
        import torch

        import oracle
        import qllama_b200 as qb
        from tests import gpu_util as gu

        torch.cuda.set_device(rank)
        dist = _init(rank, world, port, "gloo", 60.0)
        hq, hkv, hd, theta = cfg["hq"], cfg["hkv"], cfg["hd"], cfg["theta"]
        B, storage, mode = cfg["batch"], cfg["storage"], cfg["mode"]
        qr, kr = qb.shard_heads(hq, hkv, world, rank)
        uid = [qb.comm_unique_id() if rank == 0 else None]
        dist.broadcast_object_list(uid, src=0)
        ctx = qb.Context(rank)
        steps = [cfg["prefill"]] + [1] * cfg["decode"]
        max_rows = B * max(steps)
        comm = qb.Comm(ctx, world, rank, uid[0], max_rows * hq * hd * 4, mode)
        kv = qb.KvCache(ctx, 1, sum(steps) + 8, len(kr), hd, storage, 64, B)
        orc = [oracle.KvCache(1, sum(steps) + 8, hkv, hd, oracle.STORAGE[storage])
               for _ in range(B)]
        rng = np.random.default_rng(cfg["seed"])
        pos, worst = 0, 0.0
        for n in steps:
            q, k, v = (gu.rounded(gu.normal(rng, (B, n, h, hd)), "bf16") for h in (hq, hkv, hkv))
            dq, dk, dv = (gu.to_device(np.ascontiguousarray(x[:, :, r.start:r.stop]), "bf16")
                          for x, r in ((q, qr), (k, kr), (v, kr)))
            dist.barrier()  # the ranks issue the call together
            out = qb.attention_forward_sharded(comm, kv, 0, dq, dk, dv, [pos] * B, len(qr),
                                               len(kr), hd, theta, out_dtype="f32")
            ctx.synchronize()
            got = out.cpu().numpy()
            ref = np.stack([oracle.attention_with_cache(orc[b], 0, q[b], k[b], v[b], pos, hq,
                                                        hkv, hd, theta) for b in range(B)])
            worst = max(worst, float(np.abs(got - ref).max()))
            pos += n
        timed_out = None
        if cfg.get("absent_rank_step") and mode == "p2p":
            # rank 1 skips one decode call; rank 0's kernel gives up waiting for it
            q, k, v = (gu.rounded(gu.normal(rng, (B, 1, h, hd)), "bf16") for h in (hq, hkv, hkv))
            dist.barrier()
            if rank == 0:
                dq, dk, dv = (gu.to_device(np.ascontiguousarray(x[:, :, r.start:r.stop]),
                                           "bf16") for x, r in ((q, qr), (k, kr), (v, kr)))
                qb.attention_forward_sharded(comm, kv, 0, dq, dk, dv, [pos] * B, len(qr),
                                             len(kr), hd, theta, out_dtype="f32")
                try:
                    ctx.synchronize()
                    timed_out = "no error"
                except qb.QllamaError as e:
                    timed_out = f"{e.code}:{e}"
            dist.barrier()
        comm.close()
        dist.barrier()
        dist.destroy_process_group()
        queue.put((rank, "ok", worst, timed_out))
    except Exception:
        queue.put((rank, "error", traceback.format_exc(), None))
