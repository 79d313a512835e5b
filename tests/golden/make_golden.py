#!/usr/bin/env python
"""Writes the golden fixtures in this directory from the oracle (the C
restatement of the reference's portable path, itself pinned by the
reference's known-answer tests in test_oracle_golden.py).

Inputs are regenerated deterministically by the library's synthetic
generators (SplitMix64 + Box-Muller, GGML Q4_0 / Q8_0 quantizers), so only
seeds, shapes and expected outputs are stored:

  gemv.npz        - y = project_batch(W, x) for seeded Q4_0 / Q8_0 matrices,
                    M = 1 and M = 3 (repack_cache.rs:715-837);
  tiny_llama.npz  - the tiny Llama (4 layers, dim 512): a 16-token prompt,
                    the prefill logits and the first 32 greedy tokens
                    (recipe.rs:564-608, 807-1163).

Run from the repository root:  python tests/golden/make_golden.py
"""
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.dirname(HERE))

import conftest  # noqa: E402
import gguf_py  # noqa: E402

GEMV_CASES = [("Q4_0", 256, 512, 101), ("Q8_0", 256, 512, 102), ("Q4_0", 1000, 2048, 103)]
TINY_SEED, TINY_PROMPT_SEED, TINY_STEPS = 4242, 11, 32


def gemv_inputs(jal, qname, rows, cols, seed):
    quant = getattr(jal, qname)
    raw = jal.synth_matrix(quant, rows, cols, seed=seed, name=f"golden.gemv.{qname}")
    x = jal.synth_normal(3 * cols, seed=seed, name="golden.gemv.act")
    return quant, raw, x


def tiny_prompt(vocab):
    return np.random.Generator(np.random.PCG64(TINY_PROMPT_SEED)).integers(0, vocab, 16).astype(np.uint32)


def tiny_geom(spec):
    return dict(num_layers=spec.num_layers, hidden_dim=spec.hidden_dim, ffn_dim=spec.ffn_dim,
                n_heads_q=spec.n_heads_q, n_heads_kv=spec.n_heads_kv, head_dim=spec.head_dim,
                vocab_size=spec.vocab_size, rms_eps=spec.rms_eps, rope_theta=spec.rope_theta, neox=False)


def main():
    jal = conftest.load_package()
    conftest._ensure_built()
    import oracle_py as oracle
    out = {}
    for qname, rows, cols, seed in GEMV_CASES:
        quant, raw, x = gemv_inputs(jal, qname, rows, cols, seed)
        w = oracle.RepackedWeight(raw, quant, rows, cols)
        out[f"{qname}_{rows}x{cols}_m1"] = w.project_batch(x[:cols], 1).astype(np.float32)
        out[f"{qname}_{rows}x{cols}_m3"] = w.project_batch(x, 3).astype(np.float32)
    np.savez_compressed(os.path.join(HERE, "gemv.npz"), **out)

    spec = jal.TINY_LLAMA
    buf = jal.synth_gguf(spec, TINY_SEED)
    _, tensors = gguf_py.parse(buf)
    om = oracle.Model(tensors, tiny_geom(spec), nthreads=8)
    cap = 64
    kv = om.new_kv(cap)
    prompt = tiny_prompt(spec.vocab_size)
    logits = om.prefill(kv, cap, prompt, 0)
    tokens, tok = [], int(np.argmax(logits))
    for step in range(TINY_STEPS):
        tokens.append(tok)
        tok = int(np.argmax(om.decode(kv, cap, tok, len(prompt) + step)))
    np.savez_compressed(os.path.join(HERE, "tiny_llama.npz"), prompt=prompt, prefill_logits=logits.astype(np.float32),
                        greedy=np.array(tokens, dtype=np.uint32))
    print("wrote gemv.npz and tiny_llama.npz")


if __name__ == "__main__":
    main()
