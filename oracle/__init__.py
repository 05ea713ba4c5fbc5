"""CPU oracle for the Qllama attention hot path -- TEST INFRASTRUCTURE ONLY.

A ctypes view of ``libqlo.so`` (built from ``qlo.c`` by ``make -C oracle``),
which restates the reference's CPU arithmetic:

* ``rope``            -- src/tensor/ops.rs:168-220
* ``matmul``          -- src/tensor/ops.rs:63-94
* ``softmax_*``       -- src/tensor/ops.rs:138-166, 292-319
* ``causal_mask_offset`` -- src/transformer/layers.rs:509-531
* ``KvCache``         -- src/kv_cache/cache.rs:47-247
* ``attention_with_cache`` -- src/transformer/layers.rs:397-455
* ``attention_full``  -- src/transformer/layers.rs:293-351
* ``silu``            -- src/tensor/ops.rs:222-239 (end-to-end model parity)
* ``sample``          -- src/sampler/sampler.rs:119-325 (with the uniform draw given)

Only the tests, ``__graft_entry__.smoke`` and the CPU-baseline leg of
``bench.py`` may import this package.  The product library never does.
"""
from __future__ import annotations

import ctypes
import os
import subprocess

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))
_LIB_PATH = os.path.join(_HERE, "libqlo.so")

F32, F16, BF16, Q8_0 = 0, 1, 2, 3
STORAGE = {"f32": F32, "f16": F16, "bf16": BF16, "q8_0": Q8_0}

_lib = None
_c_size_p = ctypes.POINTER(ctypes.c_size_t)
_c_f32_p = ctypes.POINTER(ctypes.c_float)


class OracleError(RuntimeError):
    """An error the reference would have returned as ``Err(String)``."""


def build() -> str:
    """Compile libqlo.so with the committed Makefile (no-op when up to date)."""
    subprocess.run(["make", "-s", "-C", _HERE], check=True)
    return _LIB_PATH


def lib() -> ctypes.CDLL:
    global _lib
    if _lib is None:
        if not os.path.exists(_LIB_PATH):
            build()
        L = ctypes.CDLL(_LIB_PATH)
        sz, i32p, vp = ctypes.c_size_t, ctypes.POINTER(ctypes.c_int32), ctypes.c_void_p
        f32p, cp = _c_f32_p, ctypes.c_char_p
        L.qlo_f32_to_f16.argtypes = [ctypes.c_float]
        L.qlo_f32_to_f16.restype = ctypes.c_uint16
        L.qlo_f16_to_f32.argtypes = [ctypes.c_uint16]
        L.qlo_f16_to_f32.restype = ctypes.c_float
        L.qlo_f32_to_bf16.argtypes = [ctypes.c_float]
        L.qlo_f32_to_bf16.restype = ctypes.c_uint16
        L.qlo_bf16_to_f32.argtypes = [ctypes.c_uint16]
        L.qlo_bf16_to_f32.restype = ctypes.c_float
        L.qlo_q8_0_quantize.argtypes = [f32p, sz, vp, vp]
        L.qlo_q8_0_dequantize.argtypes = [vp, vp, sz, f32p]
        L.qlo_store_roundtrip.argtypes = [ctypes.c_int, f32p, sz, sz, f32p]
        L.qlo_rope.argtypes = [f32p, sz, sz, sz, sz, ctypes.c_float, f32p, cp, sz]
        L.qlo_matmul.argtypes = [f32p, f32p, sz, sz, sz, f32p]
        L.qlo_scale.argtypes = [f32p, sz, ctypes.c_float, f32p]
        L.qlo_softmax_rows.argtypes = [f32p, sz, sz, f32p, cp, sz]
        L.qlo_softmax_axis.argtypes = [f32p, _c_size_p, sz, sz, f32p, cp, sz]
        L.qlo_causal_mask_offset.argtypes = [f32p, sz, sz, sz, cp, sz]
        L.qlo_kv_new.argtypes = [sz, sz, sz, sz, ctypes.c_int]
        L.qlo_kv_new.restype = vp
        L.qlo_kv_free.argtypes = [vp]
        L.qlo_kv_update.argtypes = [vp, sz, f32p, _c_size_p, sz, f32p, _c_size_p, sz, i32p, sz,
                                    cp, sz]
        L.qlo_kv_get.argtypes = [vp, sz, i32p, sz, f32p, f32p, cp, sz]
        L.qlo_kv_clear.argtypes = [vp]
        L.qlo_kv_seq_len.argtypes = [vp]
        L.qlo_kv_seq_len.restype = sz
        L.qlo_kv_layer_len.argtypes = [vp, sz]
        L.qlo_kv_layer_len.restype = sz
        L.qlo_attention_with_cache.argtypes = [vp, sz, f32p, f32p, f32p, sz, sz, sz, sz, sz,
                                               ctypes.c_float, f32p, cp, sz]
        L.qlo_attention_full.argtypes = [f32p, f32p, f32p, sz, sz, sz, sz, sz, ctypes.c_float,
                                         f32p, cp, sz]
        L.qlo_attention_core.argtypes = [f32p, f32p, f32p, sz, sz, sz, sz, sz, sz, f32p, cp, sz]
        L.qlo_set_threads.argtypes = [ctypes.c_int]
        L.qlo_get_threads.restype = ctypes.c_int
        L.qlo_batch_attention_core.argtypes = [f32p, ctypes.POINTER(f32p), ctypes.POINTER(f32p),
                                               _c_size_p, sz, sz, sz, sz, sz, f32p, ctypes.c_int]
        L.qlo_silu.argtypes = [f32p, sz, f32p]
        L.qlo_sample.argtypes = [f32p, sz, i32p, sz, ctypes.c_float, sz, ctypes.c_float,
                                 ctypes.c_float, ctypes.c_double, i32p, cp, sz]
        _lib = L
    return _lib


def _f32(a) -> np.ndarray:
    return np.ascontiguousarray(a, dtype=np.float32)


def _fp(a: np.ndarray):
    return a.ctypes.data_as(_c_f32_p)


def _err():
    return ctypes.create_string_buffer(512)


def _check(rc: int, err) -> None:
    if rc:
        raise OracleError(err.value.decode())


# ---- element formats -------------------------------------------------------

def f32_to_f16_bits(x) -> np.ndarray:
    x = _f32(x).ravel()
    return np.array([lib().qlo_f32_to_f16(float(v)) for v in x], dtype=np.uint16)


def f32_to_bf16_bits(x) -> np.ndarray:
    x = _f32(x).ravel()
    return np.array([lib().qlo_f32_to_bf16(float(v)) for v in x], dtype=np.uint16)


def store_roundtrip(storage: int, x, head_dim: int) -> np.ndarray:
    x = _f32(x)
    out = np.empty_like(x)
    lib().qlo_store_roundtrip(storage, _fp(x), x.size, head_dim, _fp(out))
    return out


def q8_0_quantize(x):
    """Returns (int8 values, f16 scale bits) for a length-32k vector."""
    x = _f32(x).ravel()
    nb = x.size // 32
    qs = np.empty(nb * 32, dtype=np.int8)
    sc = np.empty(nb, dtype=np.uint16)
    lib().qlo_q8_0_quantize(_fp(x), nb, qs.ctypes.data, sc.ctypes.data)
    return qs, sc


# ---- tensor ops ------------------------------------------------------------

def rope(x, head_dim: int, start_pos: int, theta: float) -> np.ndarray:
    """ops.rs rope on a [seq, ..., head_dim] tensor."""
    x = _f32(x)
    if x.ndim < 2:
        raise OracleError(
            "RoPE requires shape [seq_len, ..., head_dim] with a positive even head_dim")
    if x.shape[-1] != head_dim:
        raise OracleError(
            "RoPE requires shape [seq_len, ..., head_dim] with a positive even head_dim")
    seq = x.shape[0]
    inner = int(np.prod(x.shape[1:])) if x.ndim > 1 else 0
    out = np.empty_like(x)
    e = _err()
    _check(lib().qlo_rope(_fp(x), seq, inner, head_dim, start_pos, theta, _fp(out), e, 512), e)
    return out


def matmul(a, b) -> np.ndarray:
    a, b = _f32(a), _f32(b)
    m, k = a.shape
    k2, n = b.shape
    assert k == k2
    out = np.empty((m, n), dtype=np.float32)
    lib().qlo_matmul(_fp(a), _fp(b), m, k, n, _fp(out))
    return out


def softmax(x, axis: int) -> np.ndarray:
    x = _f32(x)
    dims = (ctypes.c_size_t * max(1, x.ndim))(*x.shape)
    out = np.empty_like(x)
    e = _err()
    _check(lib().qlo_softmax_axis(_fp(x), dims, x.ndim, axis, _fp(out), e, 512), e)
    return out


def causal_mask_offset(scores, offset: int) -> np.ndarray:
    s = _f32(scores).copy()
    e = _err()
    _check(lib().qlo_causal_mask_offset(_fp(s), s.shape[0], s.shape[1], offset, e, 512), e)
    return s


def set_threads(n: int) -> None:
    lib().qlo_set_threads(int(n))


# ---- KV cache ------------------------------------------------------------

class KvCache:
    """cache.rs KvCache: per layer [max_seq_len, num_kv_heads, head_dim]."""

    def __init__(self, num_layers, max_seq_len, num_kv_heads, head_dim, storage=F32):
        self.num_kv_heads, self.head_dim = num_kv_heads, head_dim
        self._h = lib().qlo_kv_new(num_layers, max_seq_len, num_kv_heads, head_dim, storage)

    def __del__(self):
        if getattr(self, "_h", None):
            lib().qlo_kv_free(self._h)
            self._h = None

    def update(self, layer: int, k, v, positions) -> None:
        k, v = _f32(k), _f32(v)
        pos = np.ascontiguousarray(positions, dtype=np.int32)
        kd = (ctypes.c_size_t * max(1, k.ndim))(*k.shape)
        vd = (ctypes.c_size_t * max(1, v.ndim))(*v.shape)
        e = _err()
        _check(lib().qlo_kv_update(self._h, layer, _fp(k), kd, k.ndim, _fp(v), vd, v.ndim,
                                   pos.ctypes.data_as(ctypes.POINTER(ctypes.c_int32)), pos.size,
                                   e, 512), e)

    def get(self, layer: int, positions):
        pos = np.ascontiguousarray(positions, dtype=np.int32)
        shape = (pos.size, self.num_kv_heads, self.head_dim)
        k = np.empty(shape, dtype=np.float32)
        v = np.empty(shape, dtype=np.float32)
        e = _err()
        _check(lib().qlo_kv_get(self._h, layer, pos.ctypes.data_as(ctypes.POINTER(ctypes.c_int32)),
                                pos.size, _fp(k), _fp(v), e, 512), e)
        return k, v

    def clear(self) -> None:
        lib().qlo_kv_clear(self._h)

    def seq_len(self) -> int:
        return int(lib().qlo_kv_seq_len(self._h))

    def layer_len(self, layer: int) -> int:
        return int(lib().qlo_kv_layer_len(self._h, layer))


# ---- attention -------------------------------------------------------------

def attention_with_cache(kv: KvCache, layer: int, q, k, v, start_pos: int, num_heads: int,
                         num_kv_heads: int, head_dim: int, theta: float) -> np.ndarray:
    """layers.rs:397-455 on pre-RoPE q [n,Hq,hd], k/v [n,Hkv,hd]; returns [n, Hq*hd]."""
    q, k, v = _f32(q), _f32(k), _f32(v)
    n = q.shape[0]
    out = np.empty((n, num_heads * head_dim), dtype=np.float32)
    e = _err()
    _check(lib().qlo_attention_with_cache(kv._h, layer, _fp(q), _fp(k), _fp(v), n, start_pos,
                                          num_heads, num_kv_heads, head_dim, theta, _fp(out), e,
                                          512), e)
    return out


def attention_full(q, k, v, start_pos: int, num_heads: int, num_kv_heads: int, head_dim: int,
                   theta: float) -> np.ndarray:
    """layers.rs:293-351 (uncached) on pre-RoPE q/k/v; returns [seq, Hq*hd]."""
    q, k, v = _f32(q), _f32(k), _f32(v)
    n = q.shape[0]
    out = np.empty((n, num_heads * head_dim), dtype=np.float32)
    e = _err()
    _check(lib().qlo_attention_full(_fp(q), _fp(k), _fp(v), n, start_pos, num_heads,
                                    num_kv_heads, head_dim, theta, _fp(out), e, 512), e)
    return out


def attention_core(q_roped, k_cache, v_cache, start_pos: int, num_heads: int, num_kv_heads: int,
                   head_dim: int) -> np.ndarray:
    """layers.rs:425-455 on post-RoPE queries and cached keys/values."""
    q, kc, vc = _f32(q_roped), _f32(k_cache), _f32(v_cache)
    n, total = q.shape[0], kc.shape[0]
    out = np.empty((n, num_heads * head_dim), dtype=np.float32)
    e = _err()
    _check(lib().qlo_attention_core(_fp(q), _fp(kc), _fp(vc), n, total, start_pos, num_heads,
                                    num_kv_heads, head_dim, _fp(out), e, 512), e)
    return out


def batch_attention_core(q_roped, k_caches, v_caches, num_heads, num_kv_heads, head_dim,
                         threads: int) -> np.ndarray:
    """Independent sequences' attention cores on `threads` host threads (CPU baseline)."""
    q = _f32(q_roped)
    batch, n = q.shape[0], q.shape[1]
    kcs = [_f32(k) for k in k_caches]
    vcs = [_f32(v) for v in v_caches]
    kp = (_c_f32_p * batch)(*[_fp(k) for k in kcs])
    vp = (_c_f32_p * batch)(*[_fp(v) for v in vcs])
    lens = (ctypes.c_size_t * batch)(*[k.shape[0] for k in kcs])
    out = np.empty((batch, n, num_heads * head_dim), dtype=np.float32)
    rc = lib().qlo_batch_attention_core(_fp(q), kp, vp, lens, batch, n, num_heads, num_kv_heads,
                                        head_dim, _fp(out), int(threads))
    if rc:
        raise OracleError("batched attention core failed")
    return out


# ---- model-host pieces (end-to-end parity) --------------------------------

def silu(x) -> np.ndarray:
    """ops.rs:222-239 with libm expf, as Rust's f32::exp calls it."""
    x = _f32(x)
    out = np.empty_like(x)
    lib().qlo_silu(_fp(x), x.size, _fp(out))
    return out


def sample(logits, context, temperature: float, top_k: int, top_p: float,
           repeat_penalty: float, r: float) -> int:
    """Sampler::sample_slice (sampler.rs:119-325) with the uniform draw r in [0, 1)."""
    lg = _f32(logits).ravel()
    ctx = np.ascontiguousarray(np.asarray(context, dtype=np.int32).ravel())
    out = ctypes.c_int32()
    e = _err()
    _check(lib().qlo_sample(_fp(lg), lg.size, ctx.ctypes.data_as(ctypes.POINTER(ctypes.c_int32)),
                            ctx.size, temperature, top_k, top_p, repeat_penalty, r,
                            ctypes.byref(out), e, 512), e)
    return out.value
