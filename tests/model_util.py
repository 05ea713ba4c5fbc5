"""Shared pieces of the model-host tests: seeded weights of the end-to-end
model configuration, a GGUF writer (the `gguf` package, the format's own
Python implementation) and the oracle's generate loop."""
from __future__ import annotations

import numpy as np

import oracle
from tests import llama_host as lh

# End-to-end model configuration: dim 288, 6 layers, 6/6 heads (head_dim 48),
# SwiGLU hidden 768, vocab 32000, RMSNorm eps 1e-5, RoPE theta 1e4, 256 positions.
C1 = dict(vocab=32000, dim=288, ff=768, heads=6, kv_heads=6, layers=6, max_pos=256, eps=1e-5,
          theta=10000.0)


def c1_weights(seed: int = 1, cfg=C1) -> dict:
    """f32 weights ~ N(0, 0.02) from a seeded PCG64 (numpy default_rng,
    Box-Muller-free ziggurat normals); RMSNorm weights 1.  GGUF names,
    [out, in] layout."""
    rng = np.random.default_rng(seed)
    E, F, V = cfg["dim"], cfg["ff"], cfg["vocab"]
    kvd = cfg["kv_heads"] * (E // cfg["heads"])

    def mat(rows, cols):
        return (rng.standard_normal((rows, cols)) * 0.02).astype(np.float32)

    t = {"token_embd.weight": mat(V, E), "output_norm.weight": np.ones(E, np.float32),
         "output.weight": mat(V, E)}
    for layer in range(cfg["layers"]):
        p = f"blk.{layer}."
        t[p + "attn_norm.weight"] = np.ones(E, np.float32)
        t[p + "ffn_norm.weight"] = np.ones(E, np.float32)
        t[p + "attn_q.weight"] = mat(E, E)
        t[p + "attn_k.weight"] = mat(kvd, E)
        t[p + "attn_v.weight"] = mat(kvd, E)
        t[p + "attn_output.weight"] = mat(E, E)
        t[p + "ffn_gate.weight"] = mat(F, E)
        t[p + "ffn_up.weight"] = mat(F, E)
        t[p + "ffn_down.weight"] = mat(E, F)
    return t


def host_model(tensors: dict, cfg=C1) -> lh.TinyModel:
    return lh.TinyModel(tensors, "", cfg["dim"], cfg["heads"], cfg["kv_heads"], cfg["layers"],
                        cfg["eps"], cfg["theta"])


def oracle_generate(model: lh.TinyModel, prompt, steps: int, max_pos: int, sampler=(0.0, 0, 1.0, 1.0),
                    uniforms=None):
    """generate() (src/main.rs:387-429) on the oracle: the host layers, the
    oracle's cached attention and sampler.  Returns (tokens, top-2 margins of
    each step's logits)."""
    cache = oracle.KvCache(model.n_layers, max_pos, model.n_kv, model.hd)
    attend = lh.oracle_cached_attend(model, cache)
    ids = list(prompt)
    batch, position, out, margins = list(prompt), 0, [], []
    for step in range(steps):
        logits = model.forward(batch, position, attend)[-1]
        top = np.sort(logits)[-2:]
        margins.append(float(top[1] - top[0]))
        r = 0.0 if uniforms is None else float(uniforms[step])
        nxt = oracle.sample(logits, ids, *sampler, r)
        out.append(nxt)
        ids.append(nxt)
        position += len(batch)
        batch = [nxt]
    return out, margins


def write_gguf(path, tensors: dict, n_head: int, n_kv: int, n_layers: int, ff: int, ctx_len: int,
               eps: float, theta: float, f16: bool = False) -> None:
    """A llama-architecture GGUF file of the given weights ([out, in] arrays)."""
    import gguf

    w = gguf.GGUFWriter(str(path), "llama")
    w.add_block_count(n_layers)
    w.add_context_length(ctx_len)
    w.add_embedding_length(int(tensors["token_embd.weight"].shape[1]))
    w.add_feed_forward_length(ff)
    w.add_head_count(n_head)
    w.add_head_count_kv(n_kv)
    w.add_layer_norm_rms_eps(eps)
    w.add_rope_freq_base(theta)
    for name, a in tensors.items():
        a = np.ascontiguousarray(a, np.float32)
        w.add_tensor(name, a.astype(np.float16) if (f16 and a.ndim == 2) else a)
    w.write_header_to_file()
    w.write_kv_data_to_file()
    w.write_tensors_to_file()
    w.close()


def tiny_tensors(g) -> tuple[dict, dict]:
    """The reference's tiny-llama fixture weights from the golden file, shaped
    [out, in], and its configuration."""
    E, F, H, KV, NL, V = (int(v) for v in g["tiny/config"])
    kvd = KV * (E // H)
    shapes = {"token_embd.weight": (V, E), "output.weight": (V, E), "output_norm.weight": (E,)}
    for layer in range(NL):
        p = f"blk.{layer}."
        shapes.update({p + "attn_q.weight": (E, E), p + "attn_k.weight": (kvd, E),
                       p + "attn_v.weight": (kvd, E), p + "attn_output.weight": (E, E),
                       p + "ffn_gate.weight": (F, E), p + "ffn_up.weight": (F, E),
                       p + "ffn_down.weight": (E, F), p + "attn_norm.weight": (E,),
                       p + "ffn_norm.weight": (E,)})
    t = {k: np.asarray(g["tiny/" + k], np.float32).reshape(s) for k, s in shapes.items()}
    cfg = dict(vocab=V, dim=E, ff=F, heads=H, kv_heads=KV, layers=NL, max_pos=128,
               eps=float(g["tiny/eps"][0]), theta=float(g["tiny/theta"][0]))
    return t, cfg
