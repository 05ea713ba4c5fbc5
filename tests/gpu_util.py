"""Helpers shared by the GPU parity tests: matching device and oracle caches."""
from __future__ import annotations

import numpy as np
import torch

import oracle
import qllama_b200 as qb

TORCH_DT = {"f32": torch.float32, "f16": torch.float16, "bf16": torch.bfloat16}


def rounded(x: np.ndarray, in_dtype: str) -> np.ndarray:
    """The f32 values an input of dtype `in_dtype` carries (what the oracle receives)."""
    return torch.from_numpy(np.ascontiguousarray(x, np.float32)).to(TORCH_DT[in_dtype]).float().numpy()


def to_device(x: np.ndarray, in_dtype: str) -> torch.Tensor:
    return torch.from_numpy(np.ascontiguousarray(x, np.float32)).to("cuda").to(TORCH_DT[in_dtype])


def normal(rng, shape, scale=1.0) -> np.ndarray:
    return (rng.standard_normal(shape) * scale).astype(np.float32)


class Pair:
    """A device KvCache and one oracle KvCache per sequence holding the same rows."""

    def __init__(self, ctx, storage, layers, max_seq, hkv, hd, batch, page=64, num_pages=0):
        self.storage, self.hkv, self.hd = storage, hkv, hd
        self.gpu = qb.KvCache(ctx, layers, max_seq, hkv, hd, storage, page, batch, num_pages)
        self.orc = [oracle.KvCache(layers, max_seq, hkv, hd, oracle.STORAGE[storage])
                    for _ in range(batch)]

    def prefill_rows(self, rng, layer, seq, length, theta, scale=1.0):
        """Writes `length` rotated-K / V rows of N(0, scale) into both caches via update()."""
        k = normal(rng, (length, self.hkv, self.hd), scale)
        v = normal(rng, (length, self.hkv, self.hd), scale)
        kr = oracle.rope(k, self.hd, 0, theta)
        pos = np.arange(length, dtype=np.int32)
        self.gpu.update(layer, kr, v, pos, seq=seq)
        self.orc[seq].update(layer, kr, v, pos)

    def oracle_forward(self, layer, q, k, v, starts, hq, theta):
        """oracle attention_with_cache per sequence; q/k/v [B, n, H, hd] f32."""
        outs = []
        for b in range(q.shape[0]):
            outs.append(oracle.attention_with_cache(self.orc[b], layer, q[b], k[b], v[b],
                                                    int(starts[b]), hq, self.hkv, self.hd,
                                                    theta))
        return np.stack(outs)


def max_err(a, b) -> float:
    a = a.float().cpu().numpy() if isinstance(a, torch.Tensor) else np.asarray(a, np.float32)
    return float(np.abs(a.astype(np.float64) - np.asarray(b, np.float64)).max())
