"""Generate tests/golden/golden.npz from the reference's own Python code.

Run in a checkout that has the reference tree next to it:

    python tests/golden/make_golden.py --reference /path/to/Qllama

It imports, read-only, two Python files of the reference and records their
outputs as fixtures, so that the tests (which run where the reference is
absent) can pin the oracle against them:

* ``tests/fixtures/generate_tiny_llama.py`` -- builds the tiny-llama GGUF in
  memory (16 hidden, 4 heads / 2 KV heads, head_dim 4, 2 layers, vocab 64,
  F16 matrices) and runs its independent Python forward.  The last row for
  tokens [3, 17, 42] is the reference's ``EXPECTED_LOGITS``
  (tests/transformer_from_gguf.rs:148-159).  We store its weights (decoded to
  f32) and the logits of every row for two token sequences.
* ``scripts/numpy_forward_reference.py`` -- the reference's f64 NumPy Llama
  forward (``rope``/``rotate_rows`` :89-114, ``forward`` :117-154).  We run
  ``forward`` on a seeded synthetic GQA model and ``rope``/``rotate_rows`` on
  seeded vectors at the head sizes and thetas of the benchmark shapes.
"""
from __future__ import annotations

import argparse
import importlib.util
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))


def _load(path: str, name: str):
    spec = importlib.util.spec_from_file_location(name, path)
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


def tiny_llama(ref: str, out: dict) -> None:
    gen = _load(os.path.join(ref, "tests", "fixtures", "generate_tiny_llama.py"), "gen_tiny")
    model = gen.TinyLlama(gen.build_gguf())
    for name, values in model.tensors.items():
        out["tiny/" + name] = np.asarray(values, dtype=np.float32)
    out["tiny/config"] = np.array([gen.N_EMBD, gen.N_FF, gen.N_HEAD, gen.N_HEAD_KV,
                                   gen.N_LAYER, gen.N_VOCAB], dtype=np.int64)
    out["tiny/eps"] = np.array([gen.EPS], dtype=np.float64)
    out["tiny/theta"] = np.array([gen.THETA], dtype=np.float64)
    for tag, ids in (("a", [3, 17, 42]), ("b", [5, 9, 1, 60, 33, 7, 21, 42, 0, 18, 3])):
        out[f"tiny/ids_{tag}"] = np.array(ids, dtype=np.int64)
        out[f"tiny/logits_{tag}"] = np.asarray(model.forward(ids), dtype=np.float64)


def numpy_reference(ref: str, out: dict) -> None:
    npref = _load(os.path.join(ref, "scripts", "numpy_forward_reference.py"), "np_ref")
    rng = np.random.default_rng(20261201)
    # f64 forward of a synthetic GQA model: 3 layers, 8 heads / 2 KV heads, head_dim 8.
    n_embd, n_head, n_kv, n_ffn, n_vocab, n_layers = 64, 8, 2, 96, 48, 3
    hd = n_embd // n_head
    hp = {"n_layers": n_layers, "n_vocab": n_vocab, "n_embd": n_embd, "n_head": n_head,
          "n_head_kv": n_kv, "n_ffn": n_ffn, "n_rot": hd, "rms_eps": 1e-5,
          "rope_theta": 10000.0}
    w = {"token_embd.weight": rng.normal(0, 1.0, (n_vocab, n_embd)),
         "output_norm.weight": 1 + 0.1 * rng.normal(size=n_embd),
         "output.weight": rng.normal(0, 0.2, (n_vocab, n_embd))}
    for layer in range(n_layers):
        p = "blk.%d." % layer
        w[p + "attn_norm.weight"] = 1 + 0.1 * rng.normal(size=n_embd)
        w[p + "attn_q.weight"] = rng.normal(0, 0.4, (n_embd, n_embd))
        w[p + "attn_k.weight"] = rng.normal(0, 0.4, (n_kv * hd, n_embd))
        w[p + "attn_v.weight"] = rng.normal(0, 0.4, (n_kv * hd, n_embd))
        w[p + "attn_output.weight"] = rng.normal(0, 0.15, (n_embd, n_embd))
        w[p + "ffn_norm.weight"] = 1 + 0.1 * rng.normal(size=n_embd)
        w[p + "ffn_gate.weight"] = rng.normal(0, 0.15, (n_ffn, n_embd))
        w[p + "ffn_up.weight"] = rng.normal(0, 0.15, (n_ffn, n_embd))
        w[p + "ffn_down.weight"] = rng.normal(0, 0.15, (n_embd, n_ffn))
    # Store the weights in f32 and run the reference on exactly those values.
    w = {k: np.asarray(v, dtype=np.float32).astype(np.float64) for k, v in w.items()}
    ids = rng.integers(0, n_vocab, size=13)
    logits = npref.forward(hp, w, ids)
    for k, v in w.items():
        out["npref/" + k] = v.astype(np.float32)
    out["npref/hparams"] = np.array([n_layers, n_vocab, n_embd, n_head, n_kv, n_ffn],
                                    dtype=np.int64)
    out["npref/ids"] = np.asarray(ids, dtype=np.int64)
    out["npref/logits"] = np.asarray(logits, dtype=np.float64)

    # RoPE golden vectors: [seq, heads, hd] f32 inputs, f64 reference rotation.
    cases = [(4, 3, 8, 10000.0, 0), (5, 2, 48, 10000.0, 17), (3, 4, 64, 10000.0, 700),
             (3, 2, 128, 500000.0, 8190), (2, 2, 128, 10000.0, 32766)]
    for i, (seq, heads, hd_, theta, start) in enumerate(cases):
        x = rng.normal(0, 1, (seq, heads, hd_)).astype(np.float32)
        cos, sin = npref.rope(np.arange(start, start + seq), {"rope_theta": theta}, hd_)
        y = npref.rotate_rows(x.astype(np.float64), cos, sin, hd_)
        out[f"rope/{i}/x"] = x
        out[f"rope/{i}/params"] = np.array([hd_, start], dtype=np.int64)
        out[f"rope/{i}/theta"] = np.array([theta], dtype=np.float64)
        out[f"rope/{i}/y"] = np.asarray(y, dtype=np.float64)


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", required=True, help="root of the reference checkout")
    ap.add_argument("--out", default=os.path.join(HERE, "golden.npz"))
    args = ap.parse_args()
    sys.dont_write_bytecode = True
    out: dict = {}
    tiny_llama(args.reference, out)
    numpy_reference(args.reference, out)
    np.savez_compressed(args.out, **out)
    print("wrote", args.out, "with", len(out), "arrays")


if __name__ == "__main__":
    main()
