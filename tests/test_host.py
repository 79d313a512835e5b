"""CPU tests of the host side: the C ABI surface, the GGUF writer/reader, the
seeded generator, recipe hydration (recipe.rs) and fail-closed validation.
Each test names the reference test it restates."""
import os
import re

import numpy as np
import pytest

import gguf_py
from conftest import REPO


def header_functions():
    names = []
    for h in ("jal.h", "jal_synth.h", "jal_test.h"):
        src = open(os.path.join(REPO, "include", h)).read()
        src = re.sub(r"/\*.*?\*/", "", src, flags=re.S)
        names += re.findall(r"\b(jal_[a-z0-9_]+)\s*\(", src)
    return sorted(set(names))


def test_library_loads_and_exports_every_declared_symbol(jal):
    lib = jal.lib()
    missing = [n for n in header_functions() if not hasattr(lib, n)]
    assert not missing, missing
    assert "sm_100a" in jal.version()
    assert len(header_functions()) >= 60


def test_synth_gguf_deterministic_and_parseable(jal):
    spec = jal.SynthSpec(num_layers=1, hidden_dim=128, ffn_dim=256, n_heads_q=4, n_heads_kv=2, head_dim=32,
                         vocab_size=64)
    a = jal.synth_gguf(spec, seed=7, nthreads=1)
    b = jal.synth_gguf(spec, seed=7, nthreads=4)
    c = jal.synth_gguf(spec, seed=8, nthreads=4)
    assert np.array_equal(a, b)
    assert not np.array_equal(a, c)
    kv, t = gguf_py.parse(a)
    assert kv["general.architecture"] == "llama" and kv["llama.block_count"] == 1
    assert t["blk.0.attn_q.weight"].dims == [128, 128] and t["blk.0.attn_q.weight"].qtype == jal.Q4_0
    assert t["blk.0.attn_k.weight"].dims == [128, 64]
    assert t["token_embd.weight"].qtype == jal.Q8_0 and t["output.weight"].dims == [128, 64]
    assert np.all(t["blk.0.attn_norm.weight"].data.view(np.float32) == 1.0)


@pytest.mark.parametrize("arch", ["llama", "qwen2"])
def test_oracle_generator_matches_product_gguf_bytes(jal, oracle, arch):
    # The CPU baseline builds its model from the oracle's generator so that
    # it never loads the product library; every tensor (Qwen2's F32 Q/K/V
    # biases included) must be the bytes the product's GGUF holds.
    q = jal.Q8_0 if arch == "qwen2" else jal.Q4_0
    spec = jal.SynthSpec(architecture=arch, num_layers=2, hidden_dim=256, ffn_dim=384, n_heads_q=4, n_heads_kv=2,
                         head_dim=64, vocab_size=96, weight_quant=q, embed_quant=q, head_quant=q,
                         qkv_bias=arch == "qwen2", bias_std=0.5)
    _, t = gguf_py.parse(jal.synth_gguf(spec, seed=5))
    shape = dict(hidden_dim=256, ffn_dim=384, n_heads_q=4, n_heads_kv=2, head_dim=64, vocab_size=96, weight_quant=q,
                 embed_quant=q, head_quant=q, qkv_bias=arch == "qwen2", bias_std=0.5)
    mine = oracle.synth_llama_tensors(shape, 5, 2, nthreads=2)
    assert sorted(mine) == sorted(t)
    for name, tensor in mine.items():
        assert tensor.dims == t[name].dims and tensor.qtype == t[name].qtype, name
        assert np.array_equal(tensor.data, t[name].data), name
    assert ("blk.1.attn_v.bias" in mine) == (arch == "qwen2")


def test_bench_cpu_shapes_match_the_device_workloads(jal):
    # The CPU baseline and the reference arm time the shape the device arm
    # decodes, for every workload the bench offers.
    import importlib.util
    spec = importlib.util.spec_from_file_location("bench_mod", os.path.join(REPO, "bench.py"))
    bench = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(bench)
    device = {"llama3-8b-q4_0": jal.LLAMA3_8B_Q4_0, "qwen2-7b-q8_0": jal.QWEN2_7B_Q8_0,
              "llama3-70b-q4_0": jal.LLAMA3_70B_Q4_0, "tiny": jal.TINY_LLAMA}
    assert sorted(bench.SHAPES) == sorted(device)
    for name, shape in bench.SHAPES.items():
        s = device[name]
        for k in ("num_layers", "hidden_dim", "ffn_dim", "n_heads_q", "n_heads_kv", "head_dim", "vocab_size",
                  "context_length", "weight_quant", "embed_quant", "head_quant"):
            assert shape[k] == getattr(s, k), (name, k)
        for k in ("rms_eps", "rope_theta"):
            assert shape[k] == pytest.approx(getattr(s, k), rel=1e-7), (name, k)
        assert bool(shape.get("qkv_bias")) == s.qkv_bias, name
        assert bool(shape.get("neox")) == (s.architecture == "qwen2"), name


def test_bench_reference_arm_line_without_the_product_library():
    # bench.py --impl reference: one JSON line on the device arm's workload
    # and batch, e2e with no host<->device bytes, and the product library
    # never mapped into the process.
    import json
    import subprocess
    import sys
    code = ("import runpy, sys; sys.argv = ['bench.py', '--impl', 'reference', '--workload', 'tiny', '--steps', '2', "
            "'--warmup', '3', '--batch', '3']; runpy.run_path('bench.py', run_name='__main__'); "
            "print('MAPPED', open('/proc/self/maps').read().count('libjal.so'))")
    out = subprocess.run([sys.executable, "-c", code], cwd=REPO, capture_output=True, text=True, timeout=600)
    assert out.returncode == 0, out.stderr[-2000:]
    lines = out.stdout.strip().splitlines()
    assert lines[-1] == "MAPPED 0"
    d = json.loads(lines[-2])
    assert d["impl"] == "reference" and d["unit"] == "tok/s" and d["higher_is_better"] is True
    assert d["config"]["batch"] == 3 and d["config"]["workload"].startswith("tiny decode bs=3")
    assert d["e2e"] == {"value": d["value"], "unit": "tok/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}
    assert d["cpu_baseline"]["kind"] == "port" and d["cpu_baseline"]["value"] == d["value"] > 0
    assert d["cpu_baseline"]["cores"] >= 1 and "4 layers" in d["cpu_baseline"]["sample"]


def test_synth_weights_are_normal_0_02(jal, oracle):
    raw = jal.synth_matrix(jal.Q8_0, 256, 1024, seed=3, name="probe", std=0.02)
    vals = np.concatenate([oracle.dequantize_block(8, raw[i * 34:(i + 1) * 34]) for i in range(raw.size // 34)])
    assert abs(float(vals.mean())) < 2e-4
    assert abs(float(vals.std()) - 0.02) < 4e-4
    x = jal.synth_normal(1 << 16, seed=1, name="act")
    assert abs(float(x.std()) - 1.0) < 0.02 and abs(float(x.mean())) < 0.02


def test_synth_q5_0_blocks_round_trip_within_half_a_step(jal, oracle):
    # The Q5_0 quantizer (GGML's reference rounding) against the same stream
    # generated as f32: dequantized values within half a quantization step
    # |d| / 2 (plus the f16 rounding of d), except the values clamped at code
    # 31 on the side opposite the block's extreme, which are within one step.
    rows, cols = 64, 1024
    raw = jal.synth_matrix(jal.Q5_0, rows, cols, seed=12, name="q5")
    f32 = jal.synth_matrix(jal.F32, rows, cols, seed=12, name="q5").view(np.float32).reshape(-1, 32)
    blocks = raw.reshape(-1, 22)
    for b in range(blocks.shape[0]):
        deq = oracle.dequantize_block(jal.Q5_0, blocks[b])
        d = abs(float(oracle.f16_to_f32_finite(int(blocks[b, 0]) | (int(blocks[b, 1]) << 8))))
        err = np.abs(deq - f32[b])
        slack = 1e-3 * float(np.max(np.abs(f32[b]))) + 1e-7
        clamped = deq == np.float32(15.0 * -np.sign(f32[b][np.argmax(np.abs(f32[b]))]) * d)
        assert np.all(err[~clamped] <= 0.5 * d + slack)
        assert np.all(err[clamped] <= d + slack)


def test_f16_rounding_is_nearest_even(jal):
    for v in [1.0, 0.5, 1e-3, 65504.0, 7e-8, 3.0517578125e-05, 1.0009765625, 1.00048828125, -2.5]:
        want = int(np.array([v], dtype=np.float32).astype(np.float16).view(np.uint16)[0])
        assert jal.f32_to_f16_bits(v) == want, v


@pytest.mark.parametrize("case", [
    ("qwen2", 896, 4864, 14, 2, 64, 151_936, 24, None, 1),
    ("qwen2", 1536, 8960, 12, 2, 128, 151_936, 28, None, 1),
    ("llama", 3072, 8192, 24, 8, 128, 128_256, 28, 64, 0),
    ("llama4", 5120, 16384, 40, 8, 128, 202_048, 48, 96, 0),
])
def test_recipe_from_metadata_non_8b_scales(jal, case):
    # lib.rs:389-487 test_from_metadata_non_8b_scales_and_rotary_dim
    arch, hidden, ffn, hq, hkv, hd, vocab, layers, rot, rope = case
    kvs = [("general.architecture", arch), (f"{arch}.block_count", layers), (f"{arch}.embedding_length", hidden),
           (f"{arch}.feed_forward_length", ffn), (f"{arch}.attention.head_count", hq),
           (f"{arch}.attention.head_count_kv", hkv), (f"{arch}.attention.key_length", hd),
           (f"{arch}.vocab_size", vocab), (f"{arch}.attention.layer_norm_rms_epsilon", 1e-6),
           (f"{arch}.rope.freq_base", 10000.0)]
    if rot is not None:
        kvs.append((f"{arch}.rope.dimension_count", rot))
    r = jal.LlamaRecipe.from_gguf(gguf_py.write(kvs, []))
    assert r.architecture_id() == arch
    f = r.fields()
    assert (f.hidden_dim, f.ffn_dim, f.n_heads_q, f.n_heads_kv, f.head_dim, f.vocab_size, f.num_layers) == \
        (hidden, ffn, hq, hkv, hd, vocab, layers)
    assert f.rope_type == rope
    assert r.effective_rotary_dim() == (rot if rot is not None else hd)


def test_llama3_smooth_rope_scaling_from_gguf(jal):
    # lib.rs:554-633
    kvs = [("general.architecture", "llama"), ("llama.context_length", 131_072), ("llama.attention.key_length", 128),
           ("llama.rope.freq_base", 500000.0), ("llama.rope.scaling.type", "llama3"),
           ("llama.rope.scaling.factor", 8.0), ("llama.rope.scaling.low_freq_factor", 1.0),
           ("llama.rope.scaling.high_freq_factor", 4.0), ("llama.rope.scaling.original_context_length", 8192)]
    f = jal.LlamaRecipe.from_gguf(gguf_py.write(kvs, [])).fields()
    assert f.rope_scaling_kind == jal.ROPE_SCALING_LLAMA3
    assert (f.rope_factor, f.rope_low_freq_factor, f.rope_high_freq_factor) == (8.0, 1.0, 4.0)
    assert f.rope_original_max_position_embeddings == 8192
    kvs32 = [("general.architecture", "llama"), ("llama.rope.scaling.type", "llama3"),
             ("llama.rope.scaling.factor", 32.0), ("llama.rope.scaling.orig_ctx_len", 4096)]
    f = jal.LlamaRecipe.from_gguf(gguf_py.write(kvs32, [])).fields()
    assert (f.rope_scaling_kind, f.rope_factor, f.rope_low_freq_factor, f.rope_high_freq_factor) == (2, 32.0, 1.0, 4.0)
    assert f.rope_original_max_position_embeddings == 4096
    kvsf = [("general.architecture", "llama"), ("llama.rope.scaling.factors", ("f32[]", [1.5, 2.5]))]
    f = jal.LlamaRecipe.from_gguf(gguf_py.write(kvsf, [])).fields()
    assert f.rope_scaling_kind == jal.ROPE_SCALING_LONGROPE
    bad = [("general.architecture", "llama"), ("llama.rope.scaling.type", "bogus")]
    with pytest.raises(jal.CapabilityMismatch):
        jal.LlamaRecipe.from_gguf(gguf_py.write(bad, []))


def test_recipe_capabilities_and_irope(jal):
    # lib.rs:71-105
    r = jal.LlamaRecipe.new()
    assert r.architecture_id() == "llama"
    for q in (jal.Q4_K, jal.Q5_K, jal.Q5_0, jal.Q8_0, jal.Q4_0, jal.Q6_K, jal.F32, jal.F16, jal.BF16):
        assert r.supports_quant(q)
    assert not r.supports_quant(jal.TQ1_0) and not r.supports_quant(10)
    q = jal.LlamaRecipe.new_qwen2()
    assert q.architecture_id() == "qwen2" and abs(q.rms_eps - 1e-6) < 1e-10 and abs(q.rope_theta - 1e6) < 1.0
    l4 = jal.LlamaRecipe.new_llama4().with_irope_mask([False, True, False, True])
    assert l4.architecture_id() == "llama4"
    assert [l4.should_skip_rope(i) for i in (0, 1, 2, 3, 10)] == [False, True, False, True, False]
    kvs = [("general.architecture", "llama4"), ("llama4.block_count", 8), ("llama4.attention.no_rope_layer_step", 4)]
    r4 = jal.LlamaRecipe.from_gguf(gguf_py.write(kvs, []))
    assert [r4.should_skip_rope(i) for i in range(8)] == [False, False, False, True, False, False, False, True]


def compact_arch_gguf(arch, omit=None, extra=(), fill=None):
    """lib.rs:326-387 build_compact_arch_gguf (hidden 16, ffn 24, 2/1 heads, hd 8, vocab 12, F32)."""
    hidden, ffn, nq, nkv, hd, vocab = 16, 24, 2, 1, 8, 12
    kvs = [("general.architecture", arch), (f"{arch}.block_count", 1), (f"{arch}.embedding_length", 16),
           (f"{arch}.feed_forward_length", 24), (f"{arch}.attention.head_count", 2),
           (f"{arch}.attention.head_count_kv", 1), (f"{arch}.attention.key_length", 8),
           (f"{arch}.attention.layer_norm_rms_epsilon", 1e-5), (f"{arch}.rope.freq_base", 10000.0),
           (f"{arch}.context_length", 16)] + list(extra)
    specs = [("token_embd.weight", [hidden, vocab]), ("blk.0.attn_norm.weight", [hidden]),
             ("blk.0.attn_q.weight", [hidden, nq * hd]), ("blk.0.attn_k.weight", [hidden, nkv * hd]),
             ("blk.0.attn_v.weight", [hidden, nkv * hd]), ("blk.0.attn_output.weight", [nq * hd, hidden]),
             ("blk.0.ffn_norm.weight", [hidden]), ("blk.0.ffn_gate.weight", [hidden, ffn]),
             ("blk.0.ffn_up.weight", [hidden, ffn]), ("blk.0.ffn_down.weight", [ffn, hidden]),
             ("output_norm.weight", [hidden]), ("output.weight", [hidden, vocab])]
    ts = []
    for idx, (n, d) in enumerate(specs):
        if n == omit:
            continue
        payload = fill(idx, n, d) if fill else None
        ts.append((n, 0, d, payload))
    return gguf_py.write(kvs, ts)


@pytest.mark.parametrize("omit", ["blk.0.attn_k.weight", "blk.0.ffn_gate.weight", "output_norm.weight"])
def test_validate_model_rejects_missing_tensors(jal, omit):
    # lib.rs:783-808
    g = compact_arch_gguf("llama", omit=omit)
    r = jal.LlamaRecipe.from_gguf(g)
    with pytest.raises(jal.K3Error):
        r.validate_model(g)


def test_validate_model_arch_rotary_and_quant(jal):
    # lib.rs:810-856
    g = compact_arch_gguf("llama")
    r = jal.LlamaRecipe.from_gguf(g)
    r.validate_model(g)
    with pytest.raises(jal.CapabilityMismatch):
        r.validate_model(compact_arch_gguf("gpt2"))
    r.with_rotary_dim(6).validate_model(g)
    with pytest.raises(jal.CapabilityMismatch):
        jal.LlamaRecipe.from_gguf(g).with_rotary_dim(5).validate_model(g)
    q2k = gguf_py.write([("general.architecture", "llama")], [("blk.0.attn_q.weight", 10, [256, 1], None)])
    with pytest.raises(jal.CapabilityMismatch):
        jal.LlamaRecipe.from_gguf(g).validate_model(q2k)
    with pytest.raises(jal.CapabilityMismatch):
        jal.LlamaRecipe.from_gguf(compact_arch_gguf("gpt2"))


TINY = dict(num_layers=2, hidden_dim=128, ffn_dim=352, n_heads_q=4, n_heads_kv=2, head_dim=32, vocab_size=256,
            rms_eps=1e-5, rope_theta=10000.0)


def tiny_oracle_model(jal, oracle, seed=11, **over):
    spec = jal.SynthSpec(**{**TINY, **{k: v for k, v in over.items() if k in jal.SynthSpec.__dataclass_fields__}})
    buf = jal.synth_gguf(spec, seed)
    _, tensors = gguf_py.parse(buf)
    geom = dict(TINY, neox=over.get("neox", False))
    return oracle.Model(tensors, geom, nthreads=2), buf


def test_oracle_batched_prefill_equals_sequential_decode(jal, oracle):
    # lib.rs:205-324 and tests/batched_prefill_wave3.rs:398-471: batched prefill
    # of [1, 3, 5] == prefill [1] + decode 3 + decode 5 (bit-exact in the oracle).
    m, _ = tiny_oracle_model(jal, oracle)
    cap = 16
    kv_a = m.new_kv(cap)
    la = m.prefill(kv_a, cap, [1, 3, 5], 0)
    kv_b = m.new_kv(cap)
    m.prefill(kv_b, cap, [1], 0)
    m.decode(kv_b, cap, 3, 1)
    lb = m.decode(kv_b, cap, 5, 2)
    assert np.array_equal(la, lb)
    assert np.array_equal(kv_a, kv_b)


def test_oracle_chunked_prefill_equals_single_shot(jal, oracle):
    # tests/batched_prefill_wave3.rs:473-637 / lib.rs:873-961
    m, _ = tiny_oracle_model(jal, oracle, seed=5)
    cap = 16
    prompt = [7, 2, 9, 4, 4, 1, 0, 200]
    kv_a = m.new_kv(cap)
    la = m.prefill(kv_a, cap, prompt, 0)
    kv_b = m.new_kv(cap)
    m.prefill(kv_b, cap, prompt[:3], 0, compute_logits=False)
    lb = m.prefill(kv_b, cap, prompt[3:], 3)
    assert np.array_equal(la, lb) and np.array_equal(kv_a, kv_b)


WAVE3_CASES = [("llama", 0), ("qwen2", 12), ("llama", 13), ("qwen2", 14)]  # F32, Q4_K_M, Q5_K, Q6_K


@pytest.mark.parametrize("arch,quant", WAVE3_CASES)
def test_oracle_mixed_type_model_batched_prefill_equals_sequential(jal, oracle, arch, quant):
    # tests/batched_prefill_wave3.rs:398-471 on its own mixed-type model
    # (dense, K-quant, Q4_0 / Q5_0 / Q8_0 matrices, F16 / BF16 norms and
    # biases): prefill of M = 1, 8, 32 prompt tokens against prefill of the
    # first + sequential decodes, logits and KV within the reference test's
    # bound (|a - b| / max(|b|, 1) < 1e-5 dense, 2e-3 quantized).  In the
    # oracle, as in the reference's portable path, the two are bit-equal.
    import ref_fixtures
    buf = ref_fixtures.wave3_model_gguf(arch, quant)
    recipe = jal.LlamaRecipe.from_gguf(buf)
    recipe.validate_model(buf)
    assert recipe.architecture_id() == arch
    _, tensors = gguf_py.parse(buf)
    geom = dict(num_layers=2, hidden_dim=256, ffn_dim=256, n_heads_q=4, n_heads_kv=2, head_dim=64, vocab_size=64,
                rms_eps=1e-5, rope_theta=10000.0, neox=arch == "qwen2")
    m = oracle.Model(tensors, geom, nthreads=2)
    cap = 64
    tol = 1e-5 if quant == 0 else 2e-3
    for n in (1, 8, 32):
        prompt = [(i * 7 + 3) % 64 for i in range(n)]
        kv_a = m.new_kv(cap)
        la = m.prefill(kv_a, cap, prompt, 0)
        kv_b = m.new_kv(cap)
        lb = m.prefill(kv_b, cap, prompt[:1], 0)
        for i, tok in enumerate(prompt[1:], start=1):
            lb = m.decode(kv_b, cap, tok, i)
        for a, b in ((la, lb), (kv_a, kv_b)):
            assert np.all(np.isfinite(a)) and np.all(np.isfinite(b))
            assert float(np.max(np.abs(a - b) / np.maximum(np.abs(b), 1.0))) < tol
        assert np.array_equal(la, lb) and np.array_equal(kv_a, kv_b)
        assert float(np.max(np.abs(la))) > 0.0


def _wave3_oracle(jal, oracle, arch, quant, sliding_window=0):
    import ref_fixtures
    buf = ref_fixtures.wave3_model_gguf(arch, quant)
    _, tensors = gguf_py.parse(buf)
    geom = dict(num_layers=2, hidden_dim=256, ffn_dim=256, n_heads_q=4, n_heads_kv=2, head_dim=64, vocab_size=64,
                rms_eps=1e-5, rope_theta=10000.0, neox=arch == "qwen2")
    return oracle.Model(tensors, geom, nthreads=2, sliding_window=sliding_window)


@pytest.mark.parametrize("arch,quant,window", [("llama", 0, 0), ("qwen2", 12, 0), ("llama", 6, 8)])
def test_oracle_mixed_type_model_two_chunks_equal_single_shot(jal, oracle, arch, quant, window):
    # tests/batched_prefill_wave3.rs:473-587: a 32-token prompt prefilled at
    # once against chunks [0, 16) without logits and [16, 32) from position
    # 16 (Q5_0 with an 8-token sliding window included), then one decode of
    # token 19 at position 32 on each cache; bit-equal in the oracle.
    m = _wave3_oracle(jal, oracle, arch, quant, window)
    cap = 64
    prompt = [(i * 5 + 1) % 64 for i in range(32)]
    kv_a = m.new_kv(cap)
    la = m.prefill(kv_a, cap, prompt, 0)
    kv_b = m.new_kv(cap)
    m.prefill(kv_b, cap, prompt[:16], 0, compute_logits=False)
    lb = m.prefill(kv_b, cap, prompt[16:], 16)
    assert np.array_equal(la, lb) and np.array_equal(kv_a, kv_b)
    assert np.array_equal(m.decode(kv_a, cap, 19, 32), m.decode(kv_b, cap, 19, 32))
    assert np.array_equal(kv_a, kv_b)


def test_oracle_mixed_type_model_uneven_three_chunks(jal, oracle):
    # tests/batched_prefill_wave3.rs:589-637: chunks [0, 7), [7, 19) without
    # logits and [19, 32) with them equal the single-shot prefill.
    m = _wave3_oracle(jal, oracle, "llama", 0)
    cap = 64
    prompt = [(i * 3 + 9) % 64 for i in range(32)]
    kv_a = m.new_kv(cap)
    la = m.prefill(kv_a, cap, prompt, 0)
    kv_b = m.new_kv(cap)
    for start, end in ((0, 7), (7, 19)):
        m.prefill(kv_b, cap, prompt[start:end], start, compute_logits=False)
    lb = m.prefill(kv_b, cap, prompt[19:], 19)
    assert np.array_equal(la, lb) and np.array_equal(kv_a, kv_b)


WAVE4_CASES = [("llama", 0), ("llama", 1), ("qwen2", 30), ("llama", 2), ("qwen2", 6), ("llama", 8), ("qwen2", 12),
               ("llama", 13), ("qwen2", 14)]  # F32, F16, BF16, Q4_0, Q5_0, Q8_0, Q4_K_M, Q5_K, Q6_K


@pytest.mark.parametrize("arch,quant", WAVE4_CASES)
def test_oracle_single_quant_models_decode(jal, oracle, arch, quant):
    # tests/wave4_zero_alloc_decode_gemv.rs:365-493: a one-layer model with
    # every matrix (embedding and LM head included) in one of the nine
    # admitted types; prefill [1], then decodes of 2, 3, 4, 5 give finite
    # logits, the same with 1 and 4 worker threads (the reference's paths
    # agree bit for bit).  The product's recipe admits and validates each.
    import ref_fixtures
    buf = ref_fixtures.wave4_model_gguf(arch, quant)
    recipe = jal.LlamaRecipe.from_gguf(buf)
    recipe.validate_model(buf)
    _, tensors = gguf_py.parse(buf)
    geom = dict(num_layers=1, hidden_dim=256, ffn_dim=256, n_heads_q=4, n_heads_kv=2, head_dim=64, vocab_size=16,
                rms_eps=1e-5, rope_theta=10000.0, neox=arch == "qwen2")
    runs = []
    for threads in (1, 4):
        m = oracle.Model(tensors, geom, nthreads=threads)
        kv = m.new_kv(16)
        out = [m.prefill(kv, 16, [1], 0)]
        for pos, tok in enumerate((2, 3, 4, 5), start=1):
            out.append(m.decode(kv, 16, tok, pos))
        assert all(np.all(np.isfinite(o)) for o in out)
        runs.append((np.stack(out), kv))
    assert np.array_equal(runs[0][0], runs[1][0]) and np.array_equal(runs[0][1], runs[1][1])
    assert float(np.max(np.abs(runs[0][0]))) > 0.0


def _authentic_oracle(jal, oracle, arch, quant, biases, untied, threads=2):
    import ref_fixtures
    buf = ref_fixtures.authentic_two_layer_gguf(arch, quant, biases, untied)
    recipe = jal.LlamaRecipe.from_gguf(buf)
    recipe.validate_model(buf)
    f = recipe.fields()
    assert (f.num_layers, f.hidden_dim, f.ffn_dim, f.n_heads_q, f.n_heads_kv, f.head_dim, f.vocab_size) == \
        (2, 256, 512, 8, 2, 32, 67)
    _, tensors = gguf_py.parse(buf)
    qwen = arch == "qwen2"
    geom = dict(num_layers=2, hidden_dim=256, ffn_dim=512, n_heads_q=8, n_heads_kv=2, head_dim=32, vocab_size=67,
                rms_eps=1e-6 if qwen else 1e-5, rope_theta=1e6 if qwen else 5e5, neox=qwen)
    return oracle.Model(tensors, geom, nthreads=threads)


def test_oracle_authentic_qwen2_biases_history_and_tied_head(jal, oracle):
    # tests/authentic_gguf_forward.rs:531-628 on the oracle: QKV biases move
    # the logits (sum |diff| > 1e-2), permuting the prefix before the same last
    # token moves them (> 1e-4: causal attention over the whole history with
    # K-RoPE), an untied output.weight differs from the tied embedding
    # (> 1e-2), and an out-of-range token fails.
    cap = 16
    biased = _authentic_oracle(jal, oracle, "qwen2", 8, True, False)
    plain = _authentic_oracle(jal, oracle, "qwen2", 8, False, False)
    untied = _authentic_oracle(jal, oracle, "qwen2", 8, True, True)
    la = biased.prefill(biased.new_kv(cap), cap, [2, 9, 4, 15], 0)
    assert np.all(np.isfinite(la))
    assert float(np.sum(np.abs(la - plain.prefill(plain.new_kv(cap), cap, [2, 9, 4, 15], 0)))) > 1e-2
    assert float(np.sum(np.abs(la - biased.prefill(biased.new_kv(cap), cap, [9, 2, 4, 15], 0)))) > 1e-4
    assert float(np.sum(np.abs(la - untied.prefill(untied.new_kv(cap), cap, [2, 9, 4, 15], 0)))) > 1e-2
    with pytest.raises(oracle.OracleError, match="status 1$"):  # OR_ERR_TENSOR_BOUNDS
        biased.prefill(biased.new_kv(cap), cap, [999], 0)


@pytest.mark.parametrize("quant", [0, 1, 8, 2, 6, 12, 13, 14])
def test_oracle_authentic_batched_prefill_vs_sequential(jal, oracle, quant):
    # tests/authentic_gguf_forward.rs:630-691: prefill [3, 11, 27, 42] then
    # decode 19 against prefill [3] + decodes, logits within 1e-4 (bit-equal
    # in the oracle), untied head, FFN 512 > hidden 256, vocab 67.
    m = _authentic_oracle(jal, oracle, "llama", quant, False, True)
    cap = 16
    kv_a = m.new_kv(cap)
    m.prefill(kv_a, cap, [3, 11, 27, 42], 0)
    la = m.decode(kv_a, cap, 19, 4)
    kv_b = m.new_kv(cap)
    m.prefill(kv_b, cap, [3], 0)
    for pos, tok in enumerate((11, 27, 42), start=1):
        m.decode(kv_b, cap, tok, pos)
    lb = m.decode(kv_b, cap, 19, 4)
    assert np.all(np.isfinite(la)) and np.max(np.abs(la - lb)) < 1e-4
    assert np.array_equal(la, lb) and np.array_equal(kv_a, kv_b)


def test_oracle_authentic_threads_1_vs_4(jal, oracle):
    # tests/authentic_gguf_forward.rs:693-741: the qwen2 Q4_K_M model with
    # biases and an untied head, prefill [1, 5, 9, 13, 17, 21] + decode 8 with
    # 1 and 4 threads: within 1e-5 (bit-equal in the oracle).
    outs = []
    for threads in (1, 4):
        m = _authentic_oracle(jal, oracle, "qwen2", 12, True, True, threads)
        kv = m.new_kv(16)
        m.prefill(kv, 16, [1, 5, 9, 13, 17, 21], 0)
        outs.append(m.decode(kv, 16, 8, 6))
    assert np.all(np.isfinite(outs[0])) and np.array_equal(outs[0], outs[1])


def test_every_entry_point_fails_closed_on_null_arguments(jal):
    # The boundary's error behaviour (K3Error-style status codes,
    # lib.rs:1022-1035): every status-returning entry point called with null
    # handles and zero sizes returns JAL_ERR_INVALID_ARGUMENT with a message
    # (jal_set_device(0) only depends on whether a device exists), the size / count
    # queries return 0 and the frees accept NULL, all without a crash (run in
    # a child process so that a crash fails the test rather than the suite).
    import json
    import subprocess
    import sys
    code = r'''
import ctypes as C, importlib, json, sys
sys.path.insert(0, ".")
jal = importlib.import_module("jero-arch-llama_b200")
lib = jal.lib()
out = {}
for name, (res, args) in jal._SIGS.items():
    if name in ("jal_last_error", "jal_version", "jal_f32_to_f16_bits"):
        continue
    vals = [0.0 if a is C.c_float else (0 if a in (C.c_int, C.c_int32, C.c_uint32, C.c_uint64, C.c_size_t) else None)
            for a in args]
    rc = getattr(lib, name)(*vals)
    out[name] = [rc, (lib.jal_last_error() or b"").decode(errors="replace")]
print(json.dumps(out))
'''
    p = subprocess.run([sys.executable, "-c", code], cwd=REPO, capture_output=True, text=True, timeout=300)
    assert p.returncode == 0, p.stderr[-2000:]
    out = json.loads(p.stdout.strip().splitlines()[-1])
    sigs = jal._SIGS
    import ctypes as C
    for name, (rc, msg) in out.items():
        res = sigs[name][0]
        if res is None:
            assert rc is None, name
        elif res is C.c_size_t or name in ("jal_recipe_should_skip_rope", "jal_recipe_supports_quant"):
            assert rc == 0, name
        elif name == "jal_cached_matrix_quant":
            assert rc == -1
        elif name == "jal_model_cache_matrix":
            assert rc is None
        elif name == "jal_set_device":  # device 0: present on a GPU machine, not here
            assert rc in (jal.OK, jal.ERR_CUDA), name
        else:
            assert rc == jal.ERR_INVALID_ARGUMENT and msg.startswith("null argument"), (name, rc, msg)
    assert len(out) >= 75


def test_gguf_reader_fails_closed_on_corrupt_files(jal):
    # GGUF files are untrusted input: 600 seeded corruptions of a valid file's
    # header region (truncations, random bytes, random 64-bit counts and
    # lengths) through LlamaRecipe.from_gguf + validate_model either parse or
    # raise K3Error; none may crash (a child process runs them).
    import subprocess
    import sys
    code = r'''
import importlib, sys
import numpy as np
sys.path.insert(0, ".")
jal = importlib.import_module("jero-arch-llama_b200")
spec = jal.SynthSpec(num_layers=1, hidden_dim=128, ffn_dim=256, n_heads_q=4, n_heads_kv=2, head_dim=32,
                     vocab_size=64)
buf = jal.synth_gguf(spec, 3)
rng = np.random.default_rng(2024)
hdr = 4096
counts = [0, 0]
for it in range(600):
    b = buf.copy()
    kind = it % 3
    if kind == 0:
        b = b[: int(rng.integers(0, hdr))]
    elif kind == 1:
        for _ in range(int(rng.integers(1, 8))):
            b[int(rng.integers(0, hdr))] = int(rng.integers(0, 256))
    else:
        pos = int(rng.integers(0, hdr - 8))
        b[pos:pos + 8] = np.frombuffer(int(rng.integers(0, 2**63)).to_bytes(8, "little"), dtype=np.uint8)
    try:
        r = jal.LlamaRecipe.from_gguf(b)
        r.validate_model(b)
        counts[0] += 1
    except jal.K3Error:
        counts[1] += 1
print(counts[0], counts[1])
'''
    p = subprocess.run([sys.executable, "-c", code], cwd=REPO, capture_output=True, text=True, timeout=600)
    assert p.returncode == 0, p.stderr[-2000:]
    ok, err = map(int, p.stdout.split()[-2:])
    assert ok + err == 600 and err > 100


def _small_gguf_parts(jal):
    spec = jal.SynthSpec(num_layers=1, hidden_dim=128, ffn_dim=256, n_heads_q=4, n_heads_kv=2, head_dim=32,
                         vocab_size=64)
    kv, t = gguf_py.parse(jal.synth_gguf(spec, 3))
    return kv, [(n, x.qtype, x.dims, x.data) for n, x in t.items()]


@pytest.mark.parametrize("key,value", [("rope.freq_base", float("nan")), ("rope.freq_base", -1.0),
                                       ("rope.freq_base", "x"),
                                       ("attention.layer_norm_rms_epsilon", float("inf")),
                                       ("attention.layer_norm_rms_epsilon", 0.0),
                                       ("feed_forward_length", 0), ("attention.key_length", 1)])
def test_recipe_ignores_invalid_metadata_values(jal, key, value):
    # recipe.rs:311-318, 346-386: a non-finite or non-positive theta / eps, a
    # zero FFN width or a key length below 2 (or a value of the wrong type)
    # is ignored: the field keeps the architecture default, or the value the
    # tensor shapes give.
    kv, tensors = _small_gguf_parts(jal)
    kvs = [(k, value if k == "llama." + key else v) for k, v in kv.items()]
    f = jal.LlamaRecipe.from_gguf(gguf_py.write(kvs, tensors)).fields()
    d = jal.LlamaRecipe.new("llama").fields()
    assert f.rope_theta == (d.rope_theta if key == "rope.freq_base" else 10000.0)
    assert f.rms_eps == d.rms_eps
    assert (f.ffn_dim, f.head_dim, f.hidden_dim, f.vocab_size) == (256, 32, 128, 64)


def test_recipe_metadata_of_wrong_types_fails_closed(jal):
    # Every metadata key of a valid file (plus the optional RoPE-scaling,
    # window and iRoPE keys) replaced by a value of each other type: the
    # recipe parses or raises K3Error, never crashes (child process).
    import subprocess
    import sys
    code = r'''
import importlib, sys
sys.path.insert(0, "."); sys.path.insert(0, "tests")
jal = importlib.import_module("jero-arch-llama_b200")
import gguf_py
spec = jal.SynthSpec(num_layers=1, hidden_dim=128, ffn_dim=256, n_heads_q=4, n_heads_kv=2, head_dim=32, vocab_size=64)
kv, t = gguf_py.parse(jal.synth_gguf(spec, 3))
tensors = [(n, x.qtype, x.dims, x.data) for n, x in t.items()]
keys = list(kv.items())
extra = [("llama.rope.scaling.type", "llama3"), ("llama.rope.scaling.factor", 8.0), ("llama.rope.dimension_count", 16),
         ("llama.attention.sliding_window", 8), ("llama.rope.scaling.original_context_length", 8192),
         ("llama.no_rope_layer_step", 4), ("llama.rope.scaling.low_freq_factor", 1.0)]
bad = ["x", 0.5, -1.0, 0, 1, 2**31, 3, True, ("f32[]", [1.0, 2.0]), ("u32[]", [0]), ("str[]", ["a"]),
       float("nan"), float("inf")]
n = [0, 0]
for i in range(len(keys) + len(extra)):
    for v in bad:
        kvs = list(keys) + ([] if i < len(keys) else [extra[i - len(keys)]])
        j = i if i < len(keys) else len(kvs) - 1
        kvs[j] = (kvs[j][0], v)
        b = gguf_py.write(kvs, tensors)
        try:
            r = jal.LlamaRecipe.from_gguf(b)
            r.validate_model(b)
            n[0] += 1
        except jal.K3Error:
            n[1] += 1
print(n[0], n[1])
'''
    p = subprocess.run([sys.executable, "-c", code], cwd=REPO, capture_output=True, text=True, timeout=600)
    assert p.returncode == 0, p.stderr[-2000:]
    ok, err = map(int, p.stdout.split()[-2:])
    assert ok > 0 and err > 0


def test_integration_rust_stub_matches_the_header():
    # The Rust extern block a maintainer of the reference would add names only
    # functions the C header declares, each with the header's parameter count.
    doc = open(os.path.join(REPO, "INTEGRATION.md")).read()
    block = doc[doc.index('extern "C" {'):doc.index("}\n```")]
    stub = {m.group(1): len([a for a in m.group(2).split(",") if a.strip()])
            for m in re.finditer(r"pub fn (jal_[a-z0-9_]+)\((.*?)\)", block, flags=re.S)}
    src = "".join(open(os.path.join(REPO, "include", h)).read() for h in ("jal.h", "jal_test.h"))
    src = re.sub(r"/\*.*?\*/", "", src, flags=re.S)
    decl = {m.group(1): len([a for a in m.group(2).split(",") if a.strip() and a.strip() != "void"])
            for m in re.finditer(r"\b(jal_[a-z0-9_]+)\s*\(([^;{]*?)\)\s*;", src, flags=re.S)}
    assert len(stub) >= 20
    for name, n in stub.items():
        assert decl.get(name) == n, (name, n, decl.get(name))
