"""Committed golden fixtures (tests/golden, written by make_golden.py).

CPU: the oracle reproduces the fixtures bit for bit (so the fixtures and the
oracle pin each other).  GPU: the device reproduces them without the oracle:
the projections within the device-kernel tolerance (max|y - y_ref| /
max|y_ref| <= 1e-3) and, with reference numerics, the tiny Llama's prefill
logits within 1e-4 and its first 32 greedy tokens exactly.
"""
import os
import sys

import numpy as np
import pytest

import gguf_py

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.join(HERE, "golden"))
import make_golden as mg  # noqa: E402

REL_TOL = 1e-3


def rel_err(got, ref):
    got = np.asarray(got, dtype=np.float64)
    ref = np.asarray(ref, dtype=np.float64)
    return float(np.max(np.abs(got - ref)) / max(np.max(np.abs(ref)), 1e-30))


def load(name):
    return np.load(os.path.join(HERE, "golden", name))


def test_oracle_reproduces_gemv_golden(jal, oracle):
    g = load("gemv.npz")
    for qname, rows, cols, seed in mg.GEMV_CASES:
        quant, raw, x = mg.gemv_inputs(jal, qname, rows, cols, seed)
        w = oracle.RepackedWeight(raw, quant, rows, cols)
        assert np.array_equal(w.project_batch(x[:cols], 1).astype(np.float32), g[f"{qname}_{rows}x{cols}_m1"])
        assert np.array_equal(w.project_batch(x, 3).astype(np.float32), g[f"{qname}_{rows}x{cols}_m3"])


def test_oracle_reproduces_tiny_llama_golden(jal, oracle):
    g = load("tiny_llama.npz")
    spec = jal.TINY_LLAMA
    _, tensors = gguf_py.parse(jal.synth_gguf(spec, mg.TINY_SEED))
    om = oracle.Model(tensors, mg.tiny_geom(spec), nthreads=4)
    kv = om.new_kv(64)
    prompt = g["prompt"]
    assert np.array_equal(prompt, mg.tiny_prompt(spec.vocab_size))
    logits = om.prefill(kv, 64, prompt, 0)
    assert np.array_equal(logits.astype(np.float32), g["prefill_logits"])
    tok = int(np.argmax(logits))
    for step in range(8):
        assert tok == int(g["greedy"][step])
        tok = int(np.argmax(om.decode(kv, 64, tok, len(prompt) + step)))


@pytest.mark.gpu
def test_device_gemv_matches_golden(jal, torch_cuda):
    torch = torch_cuda
    g = load("gemv.npz")
    for qname, rows, cols, seed in mg.GEMV_CASES:
        quant, raw, x = mg.gemv_inputs(jal, qname, rows, cols, seed)
        mat = jal.CachedMatrix.repack(raw, quant, rows, cols)
        for m, key in ((1, "m1"), (3, "m3")):
            xd = torch.from_numpy(np.ascontiguousarray(x[:m * cols])).cuda()
            y = torch.zeros(m * rows, dtype=torch.float32, device="cuda")
            mat.gemm(xd, m, y)
            torch.cuda.synchronize()
            want = g[f"{qname}_{rows}x{cols}_{key}"].reshape(m, rows)
            got = y.cpu().numpy().reshape(m, rows)
            for t in range(m):
                assert rel_err(got[t], want[t]) <= REL_TOL


@pytest.mark.gpu
def test_device_reference_numerics_matches_tiny_llama_golden(jal, torch_cuda):
    g = load("tiny_llama.npz")
    spec = jal.TINY_LLAMA
    buf = jal.synth_gguf(spec, mg.TINY_SEED)
    recipe = jal.LlamaRecipe.from_gguf(buf)
    cache = recipe.build_repack_cache(buf)
    ctx = jal.ExecutionContext(recipe, cache, n_ctx=64, kv_dtype=jal.KV_F32, numerics=jal.NUMERICS_REFERENCE)
    logits = ctx.prefill_step(g["prompt"], 0)
    assert np.max(np.abs(logits - g["prefill_logits"])) <= 1e-4
    first = int(np.argmax(logits))
    seq = ctx.decode_greedy(first, mg.TINY_STEPS)
    assert [first] + [int(t) for t in seq[:-1]] == [int(t) for t in g["greedy"]]
