"""Host-side Llama layers around the attention path, for end-to-end parity tests.

Restates, in numpy f32/f64 as the reference does, the parts of the forward
that sit outside the attention hot path:
  Embedding (src/transformer/layers.rs:57-105), Linear (:112-178, weight
  transposed once, y = x @ W^T via the f32 matmul), RMSNorm (src/tensor/ops.rs:96-136,
  f64 internals), SiLU (ops.rs:222-239), SwiGLU Mlp (layers.rs:538-579),
  residual blocks (layers.rs:598-631) and the model loop
  (src/transformer/transformer.rs:203-266).
The attention core is pluggable: the oracle or the CUDA path.
"""
from __future__ import annotations

import numpy as np

import oracle


def rms_norm(x: np.ndarray, w: np.ndarray, eps: float) -> np.ndarray:
    x64 = x.astype(np.float64)
    out = np.empty_like(x, dtype=np.float32)
    for i in range(x.shape[0]):
        ss = 0.0
        for v in x64[i]:
            ss += v * v
        den = np.sqrt(ss / x.shape[1] + float(np.float32(eps)))
        norm = x64[i] if den == 0.0 else x64[i] / den
        out[i] = (norm * w.astype(np.float64)).astype(np.float32)
    return out


def linear(x: np.ndarray, w_out_in: np.ndarray) -> np.ndarray:
    return oracle.matmul(x, np.ascontiguousarray(w_out_in.T))


def silu(x: np.ndarray) -> np.ndarray:
    """ops.rs:222-239 through the oracle (libm expf, as Rust's f32::exp)."""
    return oracle.silu(np.asarray(x, np.float32))


class TinyModel:
    """Weights from a dict with GGUF names; attention core injected per call."""

    def __init__(self, tensors, prefix, n_embd, n_head, n_kv, n_layers, eps, theta):
        self.t = {k[len(prefix):]: np.asarray(v, dtype=np.float32)
                  for k, v in tensors.items() if k.startswith(prefix)}
        self.n_embd, self.n_head, self.n_kv = n_embd, n_head, n_kv
        self.n_layers, self.eps, self.theta = n_layers, eps, theta
        self.hd = n_embd // n_head

    def _mat(self, name, rows, cols):
        return self.t[name].reshape(rows, cols)

    def vocab(self) -> int:
        return self.t["token_embd.weight"].size // self.n_embd

    def forward(self, ids, start_pos: int, attend) -> np.ndarray:
        """attend(layer, q[n,Hq,hd], k[n,Hkv,hd], v[n,Hkv,hd], start_pos) -> [n, Hq*hd]."""
        E, hd = self.n_embd, self.hd
        emb = self._mat("token_embd.weight", self.vocab(), E)
        x = emb[np.asarray(ids, dtype=np.int64)].astype(np.float32)
        n = x.shape[0]
        kvd = self.n_kv * hd
        for layer in range(self.n_layers):
            p = "blk.%d." % layer
            h = rms_norm(x, self.t[p + "attn_norm.weight"], self.eps)
            q = linear(h, self._mat(p + "attn_q.weight", E, E)).reshape(n, self.n_head, hd)
            k = linear(h, self._mat(p + "attn_k.weight", kvd, E)).reshape(n, self.n_kv, hd)
            v = linear(h, self._mat(p + "attn_v.weight", kvd, E)).reshape(n, self.n_kv, hd)
            a = attend(layer, q, k, v, start_pos)
            a = linear(a, self._mat(p + "attn_output.weight", E, E))
            x = (x + a).astype(np.float32)
            h = rms_norm(x, self.t[p + "ffn_norm.weight"], self.eps)
            ff = self.t[p + "ffn_gate.weight"].size // E
            gate = linear(h, self._mat(p + "ffn_gate.weight", ff, E))
            up = linear(h, self._mat(p + "ffn_up.weight", ff, E))
            hidden = (silu(gate) * up).astype(np.float32)
            x = (x + linear(hidden, self._mat(p + "ffn_down.weight", E, ff))).astype(np.float32)
        x = rms_norm(x, self.t["output_norm.weight"], self.eps)
        lm = self.t.get("output.weight", self.t["token_embd.weight"])
        return linear(x, lm.reshape(-1, E))


def tiny_from_golden(g) -> TinyModel:
    n_embd, _ff, n_head, n_kv, n_layers, _vocab = (int(v) for v in g["tiny/config"])
    tensors = {k: g[k] for k in g.files if k.startswith("tiny/") and "weight" in k}
    return TinyModel(tensors, "tiny/", n_embd, n_head, n_kv, n_layers, float(g["tiny/eps"][0]),
                     float(g["tiny/theta"][0]))


def npref_from_golden(g) -> TinyModel:
    n_layers, _vocab, n_embd, n_head, n_kv, _ffn = (int(v) for v in g["npref/hparams"])
    tensors = {k: g[k] for k in g.files if k.startswith("npref/") and "weight" in k}
    return TinyModel(tensors, "npref/", n_embd, n_head, n_kv, n_layers, 1e-5, 10000.0)


def oracle_full_attend(model: TinyModel):
    def attend(layer, q, k, v, start_pos):
        return oracle.attention_full(q, k, v, start_pos, model.n_head, model.n_kv, model.hd,
                                     model.theta)
    return attend


def oracle_cached_attend(model: TinyModel, cache: "oracle.KvCache"):
    def attend(layer, q, k, v, start_pos):
        return oracle.attention_with_cache(cache, layer, q, k, v, start_pos, model.n_head,
                                           model.n_kv, model.hd, model.theta)
    return attend
