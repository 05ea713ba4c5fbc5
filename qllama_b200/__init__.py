"""qllama_b200 -- the Qllama attention hot path on B200 (sm_100a).

Python view of the C ABI in include/qllama_attn.h (libqllama_attn.so, built
in-tree by qllama_b200.build).  The classes mirror the reference's interface
for this path:

* ``KvCache``  -- src/kv_cache/cache.rs (new / update / get / clear / seq_len),
  device resident and paged, with f32, f16, bf16 or Q8_0 storage and several
  sequence slots;
* ``attention_forward`` -- steps 3-7 of ``Attention::forward_with_cache``
  (src/transformer/layers.rs:397-455) on already projected Q/K/V;
* ``Comm`` / ``attention_forward_sharded`` -- the same operator with the KV
  heads split over several GPUs (one process each) and the outputs
  all-gathered into the reference's head-major layout (layers.rs:447-455).

``qllama_b200.model`` holds the model host of include/qllama_model.h: the
device ``Llama`` (Transformer, GGUF loading, generate), the device sampler and
the fused Q/K/V projection.

There is no CPU fallback: without the compiled library or a CUDA device the
calls raise.
"""
from __future__ import annotations

import ctypes
import os

import numpy as np

from . import build as _build

F32, F16, BF16, Q8_0 = 0, 1, 2, 3
DTYPES = {"f32": F32, "f16": F16, "bf16": BF16, "q8_0": Q8_0}
MEM_DEVICE, MEM_HOST = 0, 1

OK, ERR_INVALID, ERR_CUDA, ERR_OOM, ERR_NO_DEVICE, ERR_UNSUPPORTED, ERR_DEVICE = range(7)

# Every symbol include/qllama_attn.h declares.
EXPORTS = (
    "ql_version", "ql_last_error", "ql_ctx_create", "ql_ctx_destroy", "ql_ctx_set_stream",
    "ql_ctx_synchronize", "ql_kv_create", "ql_kv_destroy", "ql_kv_clear", "ql_kv_clear_seq",
    "ql_kv_seq_len", "ql_kv_layer_len", "ql_kv_update", "ql_kv_get", "ql_attn_forward",
    "ql_attn_decode_noalloc", "ql_kv_truncate", "ql_comm_unique_id", "ql_comm_create",
    "ql_comm_destroy", "ql_comm_buffer", "ql_attn_forward_sharded",
    # include/qllama_model.h
    "ql_llama_create", "ql_llama_destroy", "ql_llama_get_config", "ql_llama_set_tensor",
    "ql_llama_load_gguf", "ql_llama_forward", "ql_sample", "ql_llama_generate",
    "ql_qkv_rope_append", "ql_attn_forward_appended",
)

COMM_P2P, COMM_NCCL = 0, 1
COMM_MODES = {"p2p": COMM_P2P, "nccl": COMM_NCCL}
COMM_ID_BYTES = 128
MAX_RANKS = 8


class QllamaError(RuntimeError):
    """A non-zero status from the C ABI, with the library's message."""

    def __init__(self, code: int, message: str):
        super().__init__(message)
        self.code = code


class KvConfig(ctypes.Structure):
    _fields_ = [("num_layers", ctypes.c_int32), ("max_seq_len", ctypes.c_int32),
                ("num_kv_heads", ctypes.c_int32), ("head_dim", ctypes.c_int32),
                ("dtype", ctypes.c_int32), ("page_size", ctypes.c_int32),
                ("max_batch", ctypes.c_int32), ("num_pages", ctypes.c_int32)]


class AttnArgs(ctypes.Structure):
    _fields_ = [("layer_idx", ctypes.c_int32), ("batch", ctypes.c_int32),
                ("new_len", ctypes.c_int32), ("seq_ids", ctypes.POINTER(ctypes.c_int32)),
                ("start_pos", ctypes.POINTER(ctypes.c_int64)), ("num_heads", ctypes.c_int32),
                ("num_kv_heads", ctypes.c_int32), ("head_dim", ctypes.c_int32),
                ("rope_theta", ctypes.c_float), ("in_dtype", ctypes.c_int32),
                ("out_dtype", ctypes.c_int32), ("mem", ctypes.c_int32),
                ("q", ctypes.c_void_p), ("k", ctypes.c_void_p), ("v", ctypes.c_void_p),
                ("out", ctypes.c_void_p)]


class CommId(ctypes.Structure):
    _fields_ = [("bytes", ctypes.c_char * COMM_ID_BYTES)]


_lib = None


def lib_path() -> str:
    return _build.LIB


def load(build_if_missing: bool = True) -> ctypes.CDLL:
    """Loads libqllama_attn.so (building it if absent); raises if it cannot."""
    global _lib
    if _lib is not None:
        return _lib
    path = _build.LIB
    if not os.path.exists(path):
        if not build_if_missing:
            raise QllamaError(ERR_UNSUPPORTED, f"{path} is not built")
        _build.build()
    L = ctypes.CDLL(path)
    vp, i32, i64 = ctypes.c_void_p, ctypes.c_int32, ctypes.c_int64
    i32p, i64p = ctypes.POINTER(i32), ctypes.POINTER(i64)
    L.ql_version.restype = ctypes.c_char_p
    L.ql_last_error.restype = ctypes.c_char_p
    L.ql_ctx_create.argtypes = [ctypes.c_int, ctypes.POINTER(vp)]
    L.ql_ctx_destroy.argtypes = [vp]
    L.ql_ctx_set_stream.argtypes = [vp, vp]
    L.ql_ctx_synchronize.argtypes = [vp]
    L.ql_kv_create.argtypes = [vp, ctypes.POINTER(KvConfig), ctypes.POINTER(vp)]
    L.ql_kv_destroy.argtypes = [vp]
    L.ql_kv_clear.argtypes = [vp]
    L.ql_kv_clear_seq.argtypes = [vp, i32]
    L.ql_kv_truncate.argtypes = [vp, i32, i64]
    L.ql_kv_seq_len.argtypes = [vp, i32, i64p]
    L.ql_kv_layer_len.argtypes = [vp, i32, i32, i64p]
    L.ql_kv_update.argtypes = [vp, vp, i32, i32, vp, i64p, i32, vp, i64p, i32, i32, i32p, i64,
                               i32]
    L.ql_kv_get.argtypes = [vp, vp, i32, i32, i32p, i64, vp, vp, i32]
    L.ql_attn_forward.argtypes = [vp, vp, ctypes.POINTER(AttnArgs)]
    L.ql_attn_decode_noalloc.argtypes = [vp, vp, ctypes.POINTER(AttnArgs)]
    L.ql_comm_unique_id.argtypes = [ctypes.POINTER(CommId)]
    L.ql_comm_create.argtypes = [vp, ctypes.c_int, ctypes.c_int, ctypes.POINTER(CommId),
                                 ctypes.c_uint64, ctypes.c_int, ctypes.POINTER(vp)]
    L.ql_comm_destroy.argtypes = [vp]
    L.ql_comm_buffer.argtypes = [vp, ctypes.POINTER(vp), ctypes.POINTER(ctypes.c_uint64)]
    L.ql_attn_forward_sharded.argtypes = [vp, vp, vp, ctypes.POINTER(AttnArgs)]
    from . import model as _model

    _model.bind(L)
    for name in EXPORTS:
        if name not in ("ql_version", "ql_last_error"):
            getattr(L, name).restype = ctypes.c_int
    _lib = L
    return L


def _check(rc: int) -> None:
    if rc != OK:
        raise QllamaError(rc, load().ql_last_error().decode())


def _dtype_code(x) -> int:
    """QL element type of a numpy array or torch tensor (f32/f16/bf16)."""
    name = str(getattr(x, "dtype", ""))
    if name.endswith("float32"):
        return F32
    if name.endswith("float16") and "b" not in name.split(".")[-1]:
        return F16
    if name.endswith("bfloat16"):
        return BF16
    raise QllamaError(ERR_INVALID, f"unsupported element type {name}")


def _buffer(x):
    """(pointer, memory kind, keep-alive) of a contiguous numpy array or torch tensor."""
    if isinstance(x, np.ndarray):
        x = np.ascontiguousarray(x)
        return x.ctypes.data, MEM_HOST, x
    import torch

    if not x.is_contiguous():
        x = x.contiguous()
    return x.data_ptr(), (MEM_DEVICE if x.is_cuda else MEM_HOST), x


class Context:
    """One CUDA device and its stream/workspace (ql_ctx)."""

    def __init__(self, device: int = 0):
        L = load()
        h = ctypes.c_void_p()
        _check(L.ql_ctx_create(device, ctypes.byref(h)))
        self._h = h
        self.device = device

    def set_stream(self, stream_handle: int | None) -> None:
        _check(load().ql_ctx_set_stream(self._h, stream_handle))

    def synchronize(self) -> None:
        _check(load().ql_ctx_synchronize(self._h))

    def close(self) -> None:
        if getattr(self, "_h", None):
            load().ql_ctx_destroy(self._h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:  # interpreter shutdown: the library may already be gone
            pass


class KvCache:
    """KvCache::new(num_layers, max_seq_len, num_kv_heads, head_dim) on the device.

    Extra arguments: storage dtype ("f32", "f16", "bf16", "q8_0"), page_size,
    max_batch (sequence slots), num_pages (0 = enough for every slot).
    """

    def __init__(self, ctx: Context, num_layers: int, max_seq_len: int, num_kv_heads: int,
                 head_dim: int, dtype: str = "f16", page_size: int = 64, max_batch: int = 1,
                 num_pages: int = 0):
        self.ctx = ctx
        self.num_kv_heads, self.head_dim = num_kv_heads, head_dim
        cfg = KvConfig(num_layers, max_seq_len, num_kv_heads, head_dim, DTYPES[dtype], page_size,
                       max_batch, num_pages)
        h = ctypes.c_void_p()
        _check(load().ql_kv_create(ctx._h, ctypes.byref(cfg), ctypes.byref(h)))
        self._h = h

    def update(self, layer: int, k, v, positions, seq: int = 0) -> None:
        """cache.rs:83-170 -- k already rotated; shapes are checked as the reference does."""
        kp, mem, kk = _buffer(k)
        vp, mem2, vv = _buffer(v)
        if mem != mem2:
            raise QllamaError(ERR_INVALID, "k and v must live in the same memory")
        kd = (ctypes.c_int64 * max(1, len(kk.shape)))(*kk.shape)
        vd = (ctypes.c_int64 * max(1, len(vv.shape)))(*vv.shape)
        pos = np.ascontiguousarray(positions, dtype=np.int32)
        _check(load().ql_kv_update(self.ctx._h, self._h, layer, seq, kp, kd, len(kk.shape), vp,
                                   vd, len(vv.shape), _dtype_code(kk),
                                   pos.ctypes.data_as(ctypes.POINTER(ctypes.c_int32)), pos.size,
                                   mem))

    def get(self, layer: int, positions, seq: int = 0):
        """cache.rs:185-229 -- returns f32 numpy arrays [n, num_kv_heads, head_dim]."""
        pos = np.ascontiguousarray(positions, dtype=np.int32)
        shape = (pos.size, self.num_kv_heads, self.head_dim)
        k = np.empty(shape, np.float32)
        v = np.empty(shape, np.float32)
        _check(load().ql_kv_get(self.ctx._h, self._h, layer, seq,
                                pos.ctypes.data_as(ctypes.POINTER(ctypes.c_int32)), pos.size,
                                k.ctypes.data, v.ctypes.data, MEM_HOST))
        return k, v

    def clear(self) -> None:
        _check(load().ql_kv_clear(self._h))

    def clear_seq(self, seq: int) -> None:
        _check(load().ql_kv_clear_seq(self._h, seq))

    def truncate(self, seq: int, new_len: int) -> None:
        """Roll sequence `seq` back to `new_len` positions in every layer (pages kept)."""
        _check(load().ql_kv_truncate(self._h, seq, new_len))

    def seq_len(self, seq: int = 0) -> int:
        out = ctypes.c_int64()
        _check(load().ql_kv_seq_len(self._h, seq, ctypes.byref(out)))
        return out.value

    def layer_len(self, layer: int, seq: int = 0) -> int:
        out = ctypes.c_int64()
        _check(load().ql_kv_layer_len(self._h, layer, seq, ctypes.byref(out)))
        return out.value

    def close(self) -> None:
        if getattr(self, "_h", None):
            load().ql_kv_destroy(self._h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:  # interpreter shutdown: the library may already be gone
            pass


def _attn_call(q, k, v, start_pos, num_heads, num_kv_heads, head_dim, rope_theta, layer,
               seq_ids, out, out_dtype, out_heads):
    """(AttnArgs, out, single, keep-alive) for one operator call."""
    single = len(q.shape) == 3
    if single:
        q, k, v = q[None], k[None], v[None]
    batch, new_len = int(q.shape[0]), int(q.shape[1])
    starts = np.atleast_1d(np.asarray(start_pos, dtype=np.int64))
    if starts.size == 1 and batch > 1:
        starts = np.repeat(starts, batch)
    seqs = np.arange(batch, dtype=np.int32) if seq_ids is None else np.asarray(seq_ids, np.int32)
    qp, mem, qq = _buffer(q)
    kp, _, kk = _buffer(k)
    vp, _, vv = _buffer(v)
    in_dt = _dtype_code(qq)
    od = DTYPES[out_dtype] if out_dtype else F32
    if out is None:
        shape = (batch, new_len, out_heads * head_dim)
        if mem == MEM_HOST:
            out = np.empty(shape, {F32: np.float32, F16: np.float16}.get(od, np.float32))
            if od == BF16:
                raise QllamaError(ERR_INVALID, "bf16 host output needs a torch tensor")
        else:
            import torch

            tdt = {F32: torch.float32, F16: torch.float16, BF16: torch.bfloat16}[od]
            out = torch.empty(shape, dtype=tdt, device=qq.device)
    op, _, oo = _buffer(out)
    od = _dtype_code(oo)
    args = AttnArgs(layer, batch, new_len, seqs.ctypes.data_as(ctypes.POINTER(ctypes.c_int32)),
                    starts.ctypes.data_as(ctypes.POINTER(ctypes.c_int64)), num_heads,
                    num_kv_heads, head_dim, rope_theta, in_dt, od, mem, qp, kp, vp, op)
    return args, out, single, (qq, kk, vv, oo, starts, seqs)


def attention_forward(kv: KvCache, layer: int, q, k, v, start_pos, num_heads: int,
                      num_kv_heads: int, head_dim: int, rope_theta: float, seq_ids=None,
                      out=None, out_dtype: str | None = None):
    """Steps 3-7 of Attention::forward_with_cache for a batch of sequences.

    q: [batch, new_len, num_heads, head_dim] (or [new_len, H, hd] for one
    sequence), k/v: [..., num_kv_heads, head_dim], pre-RoPE.  numpy arrays are
    host buffers (copied in and out inside the call); torch CUDA tensors are
    used in place.  Returns out [batch, new_len, num_heads*head_dim].
    """
    args, out, single, keep = _attn_call(q, k, v, start_pos, num_heads, num_kv_heads, head_dim,
                                         rope_theta, layer, seq_ids, out, out_dtype, num_heads)
    _check(load().ql_attn_forward(kv.ctx._h, kv._h, ctypes.byref(args)))
    return out[0] if single else out


# ------------------------------------------------------------ several GPUs --

def shard_heads(num_heads: int, num_kv_heads: int, nranks: int, rank: int):
    """(query-head range, KV-head range) rank `rank` owns when a layer's KV
    heads are split evenly over `nranks` GPUs; each KV head keeps its group of
    num_heads/num_kv_heads query heads (layers.rs:436)."""
    if nranks < 1 or not 0 <= rank < nranks:
        raise QllamaError(ERR_INVALID, f"rank {rank} is outside 0..{nranks - 1}")
    if num_heads % num_kv_heads or num_kv_heads % nranks:
        raise QllamaError(ERR_INVALID, f"{num_kv_heads} KV heads do not split evenly over "
                                       f"{nranks} GPUs (or num_heads is not divisible)")
    hkv = num_kv_heads // nranks
    hq = hkv * (num_heads // num_kv_heads)
    return range(rank * hq, (rank + 1) * hq), range(rank * hkv, (rank + 1) * hkv)


def comm_unique_id() -> bytes:
    """A fresh communicator id (made on one rank, handed to the others)."""
    cid = CommId()
    _check(load().ql_comm_unique_id(ctypes.byref(cid)))
    return ctypes.string_at(ctypes.addressof(cid), COMM_ID_BYTES)  # all bytes, NULs included


class Comm:
    """ql_comm: this process's member of a head-sharded group of GPUs."""

    def __init__(self, ctx: Context, nranks: int, rank: int, unique_id: bytes,
                 max_out_bytes: int, mode: str = "p2p"):
        if len(unique_id) != COMM_ID_BYTES:
            raise QllamaError(ERR_INVALID, f"a communicator id has {COMM_ID_BYTES} bytes")
        cid = CommId()
        ctypes.memmove(ctypes.addressof(cid), bytes(unique_id), COMM_ID_BYTES)
        h = ctypes.c_void_p()
        _check(load().ql_comm_create(ctx._h, nranks, rank, ctypes.byref(cid), max_out_bytes,
                                     COMM_MODES[mode], ctypes.byref(h)))
        self._h, self.ctx, self.nranks, self.rank = h, ctx, nranks, rank

    def buffer(self):
        """(device pointer, bytes) of this rank's symmetric output buffer."""
        p, n = ctypes.c_void_p(), ctypes.c_uint64()
        _check(load().ql_comm_buffer(self._h, ctypes.byref(p), ctypes.byref(n)))
        return p.value, n.value

    def close(self) -> None:
        if getattr(self, "_h", None):
            h, self._h = self._h, None
            _check(load().ql_comm_destroy(h))


def attention_forward_sharded(comm: Comm, kv: KvCache, layer: int, q, k, v, start_pos,
                              num_heads: int, num_kv_heads: int, head_dim: int,
                              rope_theta: float, seq_ids=None, out=None,
                              out_dtype: str | None = None):
    """attention_forward over this rank's heads (num_heads / num_kv_heads are
    the local counts), returning the whole layer's output
    [batch, new_len, num_heads*nranks*head_dim] gathered from every rank.
    Device tensors only; every rank makes the same calls."""
    args, out, single, keep = _attn_call(q, k, v, start_pos, num_heads, num_kv_heads, head_dim,
                                         rope_theta, layer, seq_ids, out, out_dtype,
                                         num_heads * comm.nranks)
    _check(load().ql_attn_forward_sharded(kv.ctx._h, kv._h, comm._h, ctypes.byref(args)))
    return out[0] if single else out
