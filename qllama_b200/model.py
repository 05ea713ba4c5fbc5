"""Python view of include/qllama_model.h: the device Llama model, GGUF loading
and the device sampler.

Mirrors the reference's interface for these pieces:

* ``Llama``            -- Transformer (src/transformer/transformer.rs):
  ``from_gguf`` / ``forward_with_cache`` / the weights by GGUF name;
* ``Llama.generate``   -- generate() of src/main.rs:387-429;
* ``SamplerConfig`` / ``sample`` -- src/sampler/sampler.rs (the uniform draw
  is passed in: the reference draws it from its seeded generator).
"""
from __future__ import annotations

import ctypes

import numpy as np


class LlamaConfig(ctypes.Structure):
    _fields_ = [("vocab_size", ctypes.c_int32), ("hidden_size", ctypes.c_int32),
                ("intermediate_size", ctypes.c_int32), ("num_heads", ctypes.c_int32),
                ("num_kv_heads", ctypes.c_int32), ("num_layers", ctypes.c_int32),
                ("max_position_embeddings", ctypes.c_int32), ("rms_norm_eps", ctypes.c_float),
                ("rope_theta", ctypes.c_float)]

    @property
    def head_dim(self) -> int:
        return self.hidden_size // self.num_heads


class SamplerConfig(ctypes.Structure):
    """SamplerConfig (sampler.rs:15-25); temperature <= 0 is greedy."""
    _fields_ = [("temperature", ctypes.c_float), ("top_k", ctypes.c_int32),
                ("top_p", ctypes.c_float), ("repeat_penalty", ctypes.c_float)]


GREEDY = (0.0, 0, 1.0, 1.0)


def bind(L: ctypes.CDLL) -> None:
    vp, i32, i64 = ctypes.c_void_p, ctypes.c_int32, ctypes.c_int64
    i32p = ctypes.POINTER(i32)
    L.ql_llama_create.argtypes = [vp, ctypes.POINTER(LlamaConfig), ctypes.POINTER(vp)]
    L.ql_llama_destroy.argtypes = [vp]
    L.ql_llama_get_config.argtypes = [vp, ctypes.POINTER(LlamaConfig)]
    L.ql_llama_set_tensor.argtypes = [vp, ctypes.c_char_p, vp, i64]
    L.ql_llama_load_gguf.argtypes = [vp, ctypes.c_char_p, ctypes.POINTER(vp)]
    L.ql_llama_forward.argtypes = [vp, vp, i32, i32p, i32, i64, vp, i32]
    L.ql_sample.argtypes = [vp, vp, i32, vp, i32, ctypes.POINTER(SamplerConfig), ctypes.c_double,
                            vp]
    L.ql_qkv_rope_append.argtypes = [vp, vp, ctypes.c_void_p, vp, i32, vp, vp]
    L.ql_attn_forward_appended.argtypes = [vp, vp, ctypes.c_void_p]
    L.ql_llama_generate.argtypes = [vp, vp, i32, i32p, i32, i32, i32,
                                    ctypes.POINTER(SamplerConfig),
                                    ctypes.POINTER(ctypes.c_double), i32p, i32p]


def _qb():
    import qllama_b200 as qb

    return qb


class Llama:
    """A Llama model on one device (ql_llama)."""

    def __init__(self, ctx, config: LlamaConfig | None = None, handle=None):
        qb = _qb()
        self.ctx = ctx
        if handle is None:
            h = ctypes.c_void_p()
            qb._check(qb.load().ql_llama_create(ctx._h, ctypes.byref(config), ctypes.byref(h)))
            handle = h
        self._h = handle
        cfg = LlamaConfig()
        qb._check(qb.load().ql_llama_get_config(self._h, ctypes.byref(cfg)))
        self.config = cfg

    @classmethod
    def from_gguf(cls, ctx, path: str) -> "Llama":
        """GgufFile::from_path + Transformer::from_gguf."""
        qb = _qb()
        h = ctypes.c_void_p()
        qb._check(qb.load().ql_llama_load_gguf(ctx._h, path.encode(), ctypes.byref(h)))
        return cls(ctx, handle=h)

    def set_tensor(self, name: str, data) -> None:
        """One weight by GGUF name, in the reference's [out, in] layout (f32)."""
        a = np.ascontiguousarray(data, dtype=np.float32)
        qb = _qb()
        qb._check(qb.load().ql_llama_set_tensor(self._h, name.encode(), a.ctypes.data, a.size))

    def kv_cache(self, max_batch: int = 1, dtype: str = "f32"):
        """KvCache::new(num_layers, max_position_embeddings, num_kv_heads, head_dim)."""
        c = self.config
        return _qb().KvCache(self.ctx, c.num_layers, c.max_position_embeddings, c.num_kv_heads,
                             c.head_dim, dtype, 64, max_batch)

    def forward_with_cache(self, ids, start_pos: int, kv, seq: int = 0) -> np.ndarray:
        """Transformer::forward_with_cache: logits [n, vocab] (host f32)."""
        qb = _qb()
        ids = np.ascontiguousarray(ids, dtype=np.int32)
        out = np.empty((ids.size, self.config.vocab_size), np.float32)
        qb._check(qb.load().ql_llama_forward(self._h, kv._h, seq,
                                             ids.ctypes.data_as(ctypes.POINTER(ctypes.c_int32)),
                                             ids.size, start_pos, out.ctypes.data, qb.MEM_HOST))
        return out

    def generate(self, kv, prompt, steps: int, sampler=GREEDY, uniforms=None, eos_id: int = -1,
                 seq: int = 0) -> list[int]:
        """generate() (main.rs:387-429) on the device; `uniforms`: one draw per step."""
        qb = _qb()
        prompt = np.ascontiguousarray(prompt, dtype=np.int32)
        cfg = SamplerConfig(*sampler)
        out = np.zeros(max(1, steps), np.int32)
        n = ctypes.c_int32()
        u = None
        if uniforms is not None:
            uu = np.ascontiguousarray(uniforms, dtype=np.float64)
            u = uu.ctypes.data_as(ctypes.POINTER(ctypes.c_double))
        qb._check(qb.load().ql_llama_generate(
            self._h, kv._h, seq, prompt.ctypes.data_as(ctypes.POINTER(ctypes.c_int32)),
            prompt.size, steps, eos_id, ctypes.byref(cfg), u,
            out.ctypes.data_as(ctypes.POINTER(ctypes.c_int32)), ctypes.byref(n)))
        return out[:n.value].tolist()

    def close(self) -> None:
        if getattr(self, "_h", None):
            _qb().load().ql_llama_destroy(self._h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:  # interpreter shutdown: the library may already be gone
            pass


def sample(ctx, logits, context, sampler, r: float) -> int:
    """Sampler::sample_slice on the device: logits and context are CUDA tensors
    (f32 / int32); returns the token id (synchronises the context)."""
    import torch

    qb = _qb()
    tok = torch.full((1,), -2, dtype=torch.int32, device=logits.device)
    torch.cuda.synchronize(logits.device)  # inputs and tok are written on torch's stream
    cfg = SamplerConfig(*sampler)
    ctxp = context.data_ptr() if context is not None and context.numel() else None
    n = int(context.numel()) if context is not None else 0
    qb._check(qb.load().ql_sample(ctx._h, logits.data_ptr(), int(logits.numel()), ctxp, n,
                                  ctypes.byref(cfg), float(r), tok.data_ptr()))
    ctx.synchronize()
    return int(tok.item())


def qkv_rope_append(kv, layer: int, x, wqkv_t, start_pos, num_heads: int, num_kv_heads: int,
                    head_dim: int, rope_theta: float, seq_ids=None):
    """ql_qkv_rope_append: x [batch, new_len, in_features] and the fused
    transposed weight [in_features, (Hq + 2 Hkv) * hd] as f32 CUDA tensors;
    returns the rotated queries [batch, new_len, Hq, hd] (K/V go to the cache)."""
    import torch

    qb = _qb()
    batch, new_len, K = (int(v) for v in x.shape)
    q_rot = torch.empty(batch, new_len, num_heads, head_dim, dtype=torch.float32, device=x.device)
    starts = np.atleast_1d(np.asarray(start_pos, dtype=np.int64))
    if starts.size == 1 and batch > 1:
        starts = np.repeat(starts, batch)
    seqs = np.arange(batch, dtype=np.int32) if seq_ids is None else np.asarray(seq_ids, np.int32)
    args = qb.AttnArgs(layer, batch, new_len, seqs.ctypes.data_as(ctypes.POINTER(ctypes.c_int32)),
                       starts.ctypes.data_as(ctypes.POINTER(ctypes.c_int64)), num_heads,
                       num_kv_heads, head_dim, rope_theta, qb.F32, qb.F32, qb.MEM_DEVICE,
                       None, None, None, None)
    qb._check(qb.load().ql_qkv_rope_append(kv.ctx._h, kv._h, ctypes.byref(args),
                                           x.contiguous().data_ptr(), K,
                                           wqkv_t.contiguous().data_ptr(), q_rot.data_ptr()))
    return q_rot


def attention_forward_appended(kv, layer: int, q_rot, start_pos, num_heads: int,
                               num_kv_heads: int, head_dim: int, rope_theta: float,
                               seq_ids=None, out_dtype: str = "f32"):
    """ql_attn_forward_appended over the rows qkv_rope_append wrote."""
    import torch

    qb = _qb()
    batch, new_len = int(q_rot.shape[0]), int(q_rot.shape[1])
    out = torch.empty(batch, new_len, num_heads * head_dim,
                      dtype={"f32": torch.float32, "f16": torch.float16,
                             "bf16": torch.bfloat16}[out_dtype], device=q_rot.device)
    starts = np.atleast_1d(np.asarray(start_pos, dtype=np.int64))
    if starts.size == 1 and batch > 1:
        starts = np.repeat(starts, batch)
    seqs = np.arange(batch, dtype=np.int32) if seq_ids is None else np.asarray(seq_ids, np.int32)
    args = qb.AttnArgs(layer, batch, new_len, seqs.ctypes.data_as(ctypes.POINTER(ctypes.c_int32)),
                       starts.ctypes.data_as(ctypes.POINTER(ctypes.c_int64)), num_heads,
                       num_kv_heads, head_dim, rope_theta, qb.F32, qb.DTYPES[out_dtype],
                       qb.MEM_DEVICE, q_rot.data_ptr(), None, None, out.data_ptr())
    qb._check(qb.load().ql_attn_forward_appended(kv.ctx._h, kv._h, ctypes.byref(args)))
    return out
