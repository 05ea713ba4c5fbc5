"""Head-sharded layers on two GPUs: the fused NVLink exchange and the NCCL
baseline against the oracle over all heads (skipped with fewer than 2 GPUs).

Each rank owns half of the KV heads (with their query heads) in its own
cache; ql_attn_forward_sharded returns the whole layer's output on every
rank in the head-major layout of layers.rs:447-455.  A prefill chunk takes
the local kernels plus the push exchange, the single-token decodes the
split-KV kernel that stores into every rank's output itself.
"""
from __future__ import annotations

import pytest
import torch

from tests import sharding_workers as sw
from tests.test_sharding_cpu import _run

TOL_16 = 2e-3  # f16 / bf16 cache, and Q8_0 against its dequantised rows

pytestmark = [
    pytest.mark.gpu,
    pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two GPUs"),
]


@pytest.mark.parametrize("storage,mode,prefill", [
    ("f16", "p2p", 130),   # tcgen05 prefill + push, then fused decodes
    ("bf16", "p2p", 130),  # the same on a bf16 cache (tiles converted to f16 operands)
    ("q8_0", "p2p", 70),   # split-KV prefill + push, then fused decodes
    ("f16", "nccl", 130),  # the library baseline
])
def test_sharded_layer_matches_oracle(storage, mode, prefill):
    cfg = dict(hq=16, hkv=4, hd=128, theta=500000.0, batch=2, prefill=prefill, decode=3,
               storage=storage, mode=mode, seed=31)
    res = _run(sw.gpu_sharded_worker, 2, cfg, timeout=240)
    for rank, (status, worst, _) in res.items():
        assert status == "ok", worst
        assert worst <= TOL_16, (rank, worst)


def test_sharded_peer_wait_runs_out_instead_of_hanging():
    """Rank 1 skips a call: rank 0's kernel stops waiting after its bound and the
    context reports QL_ERR_DEVICE at the next synchronize."""
    cfg = dict(hq=16, hkv=4, hd=128, theta=500000.0, batch=1, prefill=64, decode=1,
               storage="f16", mode="p2p", seed=5, absent_rank_step=True)
    res = _run(sw.gpu_sharded_worker, 2, cfg, timeout=240)
    for rank, (status, payload, _) in res.items():
        assert status == "ok", payload
    code_msg = res[0][2]
    assert code_msg.startswith("6:") and "another GPU" in code_msg, code_msg
