#!/usr/bin/env python
"""Benchmark of the B200 quantized decode/prefill hot path.

Workload (one step = one greedy decode token): Llama-3-8B-shaped model with
random-init N(0, 0.02) weights quantized to Q4_0 (32 layers, dim 4096, 32/8
heads, head_dim 128, FFN 14336, vocab 128256, interleaved RoPE theta 5e5), a
2048-token prefill of uniform-random ids, then batch-1 greedy decode with a
paged fp16 KV cache.  `value` is decode tokens/s over all ranks (each rank
runs an independent replica: weak scaling), timed on the device with CUDA
events around K steps; the weights (4.2 GB) exceed L2 many times, so no
flush is needed between steps.  The JSON line also carries the prefill rate,
the quant-GEMV op sweep (HBM GB/s vs the measured peak), the roofline of the
dominant decode kernel, an end-to-end figure through the C ABI with host
buffers, the CPU baseline (the oracle port on the host cores) and clocks.

`--impl reference` times the reference's portable CPU path (the oracle port,
since the Rust crate cannot be built here) on the host cores.
"""
import argparse
import importlib.util
import json
import os
import statistics
import subprocess
import sys
import time

REPO = os.path.dirname(os.path.abspath(__file__))
PKG_DIR = os.path.join(REPO, "jero-arch-llama_b200")
METRIC = "Q4_0 decode tok/s (bs=1) + quant-GEMV HBM GB/s vs peak; prefill tok/s"
SWEEP = [(4096, 4096), (11008, 4096), (4096, 11008), (14336, 4096), (128256, 4096)]
L2_BYTES = 126 * 1024 * 1024
SEED = 20251201


def load_jal():
    name = "jero_arch_llama_b200"
    if name in sys.modules:
        return sys.modules[name]
    if not os.path.exists(os.path.join(PKG_DIR, "libjal.so")):
        subprocess.run(["make", "-C", PKG_DIR, "-j", "16"], check=True)
    spec = importlib.util.spec_from_file_location(name, os.path.join(PKG_DIR, "__init__.py"))
    mod = importlib.util.module_from_spec(spec)
    sys.modules[name] = mod
    spec.loader.exec_module(mod)
    return mod


def measured_peaks():
    p = os.path.join(REPO, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        with open(p) as f:
            d = json.load(f)
        return float(d["hbm_gbs"]), "measured"
    return 6650.0, "fallback"


def committed_traffic():
    p = os.path.join(REPO, "profiles", "traffic.json")
    if os.path.exists(p):
        with open(p) as f:
            return json.load(f)
    return {}


class ClockSampler:
    """SM clocks and clock-event (throttle) reasons sampled through NVML in a
    background thread during the timed region (reads only; no setting is
    changed).  Falls back to an empty record when NVML is unavailable."""

    REASONS = {"hw_slowdown": 0x8, "hw_thermal_slowdown": 0x40, "sw_thermal_slowdown": 0x20, "sw_power_cap": 0x4}

    def __init__(self, device, period_s=0.01):
        self.device, self.period = device, period_s
        self.samples, self.max_mhz, self.error = [], None, None

    def _run(self):
        import pynvml as nv
        h = nv.nvmlDeviceGetHandleByIndex(self.device)
        self.max_mhz = nv.nvmlDeviceGetMaxClockInfo(h, nv.NVML_CLOCK_SM)
        while not self._stop.is_set():
            try:
                mhz = nv.nvmlDeviceGetClockInfo(h, nv.NVML_CLOCK_SM)
                reasons = nv.nvmlDeviceGetCurrentClocksEventReasons(h)
                self.samples.append((mhz, reasons))
            except nv.NVMLError as e:  # keep the first error for the record
                self.error = self.error or str(e)
            self._stop.wait(self.period)

    def __enter__(self):
        import threading
        self._stop = threading.Event()
        self._thread = None
        try:
            import pynvml as nv
            nv.nvmlInit()
            self._thread = threading.Thread(target=self._run, daemon=True)
            self._thread.start()
        except Exception as e:  # noqa: BLE001 - NVML missing: no clock record
            self.error = f"nvml: {e}"
        return self

    def __exit__(self, *a):
        self._stop.set()
        if self._thread:
            self._thread.join(timeout=5)

    def summary(self):
        sm = [m for m, _ in self.samples]
        reasons = sorted(n for n, bit in self.REASONS.items() if any(r & bit for _, r in self.samples))
        out = {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": self.max_mhz, "reasons": reasons,
               "samples": len(sm), "source": "nvml"}
        if self.error:
            out["error"] = self.error
        return out


def ev_time(torch, fn, stream):
    s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    torch.cuda.synchronize()
    s.record(stream)
    fn()
    e.record(stream)
    e.synchronize()
    return s.elapsed_time(e) / 1e3


def gemv_sweep(jal, torch, peak, quants, iters=200):
    """Op sweep: M x K quant GEMV, rotating weight copies (> 4x L2) so each
    launch streams from HBM.  The launches are captured in a CUDA graph so
    the timing is the kernels', not the host's launch rate."""
    stream = torch.cuda.current_stream()
    res = []
    for qname in quants:
        q = getattr(jal, qname)
        bpb = 18 if q == jal.Q4_0 else 34
        for rows, cols in SWEEP:
            raw = jal.synth_matrix(q, rows, cols, seed=SEED, name=f"sweep.{rows}x{cols}")
            copies = max(2, -(-4 * L2_BYTES // raw.nbytes))
            mats = [jal.CachedMatrix.repack(raw, q, rows, cols) for _ in range(copies)]
            x = torch.from_numpy(jal.synth_normal(cols, seed=SEED, name="sweep.act")).cuda()
            q8 = torch.zeros(cols, dtype=torch.int8, device="cuda")
            sc = torch.zeros(cols // 32, dtype=torch.float32, device="cuda")
            jal.act_quantize_q8(x, 1, cols, q8, sc, stream)
            y = torch.zeros(rows, dtype=torch.float32, device="cuda")
            for i in range(2 * copies):
                mats[i % copies].gemv_q8(q8, sc, y, stream)

            graph = torch.cuda.CUDAGraph()
            with torch.cuda.graph(graph, stream=stream):
                for i in range(iters):
                    mats[i % copies].gemv_q8(q8, sc, y, stream)
            graph.replay()
            t = ev_time(torch, graph.replay, stream) / iters
            del graph
            alg = rows * cols // 32 * bpb + 4 * cols + 4 * rows
            res.append({"quant": qname, "M": rows, "K": cols, "us": round(t * 1e6, 3),
                        "GBps": round(alg / t / 1e9, 1), "frac_of_peak": round(alg / t / 1e9 / peak, 4),
                        "bytes": alg})
            del mats
    return res


def host_cpu():
    try:
        with open("/proc/cpuinfo") as f:
            for line in f:
                if line.startswith("model name"):
                    return line.split(":", 1)[1].strip()
    except OSError:
        pass
    return "unknown"


# The workloads' shapes for the CPU legs (kept here so that the reference arm
# never imports the product package); GGML type ids: Q4_0 = 2, Q8_0 = 8.
SHAPES = {
    "llama3-8b-q4_0": dict(num_layers=32, hidden_dim=4096, ffn_dim=14336, n_heads_q=32, n_heads_kv=8, head_dim=128,
                           vocab_size=128256, context_length=8192, rms_eps=1e-5, rope_theta=500000.0, weight_quant=2,
                           embed_quant=2, head_quant=2),
    "qwen2-7b-q8_0": dict(num_layers=28, hidden_dim=3584, ffn_dim=18944, n_heads_q=28, n_heads_kv=4, head_dim=128,
                          vocab_size=152064, context_length=4096, rms_eps=1e-6, rope_theta=1e6, weight_quant=8,
                          embed_quant=8, head_quant=8, neox=True, qkv_bias=True, bias_std=0.02),
    "llama3-70b-q4_0": dict(num_layers=80, hidden_dim=8192, ffn_dim=28672, n_heads_q=64, n_heads_kv=8, head_dim=128,
                            vocab_size=128256, context_length=8448, rms_eps=1e-5, rope_theta=500000.0,
                            weight_quant=2, embed_quant=2, head_quant=2),
    "tiny": dict(num_layers=4, hidden_dim=512, ffn_dim=1376, n_heads_q=8, n_heads_kv=2, head_dim=64, vocab_size=4096,
                 context_length=256, rms_eps=1e-5, rope_theta=10000.0, weight_quant=2, embed_quant=8, head_quant=8),
}


def prefill_tokens(shape, args):
    """The prompt length the device arm uses for this workload."""
    return min(args.prefill, shape["context_length"] - args.warmup - args.steps - 8)


def cpu_baseline(shape, steps, pos, seed=SEED, batch=1):
    """The oracle port (the reference's portable path restated in C) timed on
    the host cores, without the product library: a 1-layer model with this
    shape (layer 0, embedding and head, generated by the oracle's seeded
    generator) decodes `steps` tokens at positions pos, pos + 1, ...; the KV
    rows of positions [0, pos) hold seeded random values (the step's cost does
    not depend on them).  The LM head projection is timed alone, and
    tok/s = 1 / (L * t_layer + t_head).  The reference decodes one sequence
    per step, so `batch` sequences take batch steps and the aggregate rate is
    the same."""
    sys.path.insert(0, os.path.join(REPO, "tests"))
    import numpy as np  # noqa: E402
    import oracle_py  # noqa: E402

    threads = os.cpu_count() or 1
    geom = dict(shape, num_layers=1)
    t0 = time.perf_counter()
    tensors = oracle_py.synth_llama_tensors(shape, seed, 1, nthreads=threads)
    m = oracle_py.Model(tensors, geom, nthreads=threads, kv_f16=True)
    gen_s = time.perf_counter() - t0
    cap = pos + steps + 1
    kv = m.new_kv(cap)
    kvd = shape["n_heads_kv"] * shape["head_dim"]
    rng = np.random.Generator(np.random.PCG64(seed))
    kv.reshape(2, cap, kvd)[:, :pos, :] = rng.standard_normal((2, pos, kvd), dtype=np.float32)
    head = tensors["output.weight"]
    w = oracle_py.RepackedWeight(head.data, head.qtype, shape["vocab_size"], shape["hidden_dim"])
    x = rng.standard_normal(shape["hidden_dim"], dtype=np.float32)
    t0 = time.perf_counter()
    for i in range(steps):
        m.decode(kv, cap, 5 + i, pos + i)
    t_step = (time.perf_counter() - t0) / steps
    t0 = time.perf_counter()
    for _ in range(steps):
        w.project_batch(x, 1, nthreads=threads)
    t_head = (time.perf_counter() - t0) / steps
    t_layer = max(t_step - t_head, 1e-9)
    t_tok = shape["num_layers"] * t_layer + t_head
    return {"value": round(1.0 / t_tok, 4), "unit": "tok/s", "cores": threads, "kind": "port",
            "cpu": host_cpu(),
            "sample": f"{steps} decode steps at positions {pos}..{pos + steps - 1} of a 1-layer model of the same "
                      f"shape (layer 0 + embedding + LM head, f16-rounded KV) = {t_step * 1e3:.1f} ms/step, LM head "
                      f"alone {t_head * 1e3:.1f} ms; extrapolated to {shape['num_layers']} layers; model build "
                      f"{gen_s:.1f} s (not timed)"
                      + (f"; {batch} sequences decode one after another (the reference has no multi-sequence "
                         "decode), so the aggregate rate equals one sequence's" if batch > 1 else "")}


def reference_arm(args):
    """--impl reference: the reference's portable CPU path (the oracle port,
    since the Rust crate cannot be built here) on the host cores, for the
    device arm's workload, batch and decode position.  It loads only the
    oracle library."""
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    shape = SHAPES[args.workload]
    steps = max(1, args.steps)
    warmup = max(args.warmup, 3)
    n_prefill = prefill_tokens(shape, argparse.Namespace(prefill=args.prefill, warmup=warmup, steps=args.steps))
    base = cpu_baseline(shape, steps, n_prefill + warmup, batch=args.batch)
    wq = "Q8_0" if shape["weight_quant"] == 8 else "Q4_0"
    bs = f"bs={args.batch} (independent sequences)" if args.batch > 1 else "bs=1"
    line = {"impl": "reference", "metric": METRIC, "value": base["value"], "unit": "tok/s", "n_gpus": args.gpus,
            "steps": steps, "warmup": warmup, "ms_per_step": round(1e3 * args.batch / base["value"], 3),
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "int8",
            "data": f"synthetic: seeded N(0,0.02) weights quantized to {wq}, uniform token ids",
            "config": {"workload": f"{args.workload} decode {bs} greedy after a {n_prefill}-token prefill",
                       "batch": args.batch, "layers": shape["num_layers"], "hidden": shape["hidden_dim"],
                       "ffn": shape["ffn_dim"], "vocab": shape["vocab_size"], "kv_cache": "f16-rounded",
                       "impl_detail": "C restatement of the reference's portable path (oracle), OpenMP panels"},
            "cpu_baseline": base,
            "e2e": {"value": base["value"], "unit": "tok/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


def profile_mode(args):
    """Small fixed workloads for ncu (no JSON line):
      gemv   - four launches of the 14336x4096 Q4_0 decode GEMV (M = 1);
      trace  - the bench's Llama-3-8B Q4_0 model after a --prefill prompt:
               the in-graph per-kernel breakdown of the decode step from the
               kernels' own globaltimer stamps (jal_context_trace_decode_step),
               median over 5 traced steps (prints a table, no profiler);
      skinny - four launches of the 3584x18944 Q8_0 GEMM at M = 4 (the
               batched decode's down projection of the Qwen2-7B shape);
      decode - Llama-3-8B Q4_0, 32-token prompt, two decode steps between
               cudaProfilerStart / Stop;
      attn   - the same attention geometry with 2 layers, a --prefill prompt
               and one decode step between cudaProfilerStart / Stop;
      prefill - the 2-layer model, a --prefill-token prompt prefilled once
               to warm up, then again between cudaProfilerStart / Stop."""
    import dataclasses

    import numpy as np
    import torch
    jal = load_jal()
    stream = torch.cuda.Stream()
    torch.cuda.set_stream(stream)
    if args.profile == "trace":
        return trace_mode(args, jal, torch, stream)
    if args.profile == "skinny":
        rows, cols, m = 3584, 18944, 4  # Qwen2-7B down projection at batch 4, Q8_0
        raw = jal.synth_matrix(jal.Q8_0, rows, cols, seed=SEED, name="profile.skinny")
        mat = jal.CachedMatrix.repack(raw, jal.Q8_0, rows, cols)
        x = torch.from_numpy(jal.synth_normal(m * cols, seed=SEED, name="profile.act")).cuda()
        y = torch.zeros(m * rows, dtype=torch.float32, device="cuda")
        for _ in range(4):
            mat.gemm(x, m, y, stream)
        torch.cuda.synchronize()
        print("profile skinny ok", float(y.abs().sum()))
        return 0
    if args.profile == "gemv":
        rows, cols = 14336, 4096
        raw = jal.synth_matrix(jal.Q4_0, rows, cols, seed=SEED, name="profile.gemv")
        mat = jal.CachedMatrix.repack(raw, jal.Q4_0, rows, cols)
        x = torch.from_numpy(jal.synth_normal(cols, seed=SEED, name="profile.act")).cuda()
        q8 = torch.zeros(cols, dtype=torch.int8, device="cuda")
        sc = torch.zeros(cols // 32, dtype=torch.float32, device="cuda")
        jal.act_quantize_q8(x, 1, cols, q8, sc, stream)
        y = torch.zeros(rows, dtype=torch.float32, device="cuda")
        for _ in range(4):
            mat.gemv_q8(q8, sc, y, stream)
        torch.cuda.synchronize()
        print("profile gemv ok", float(y.abs().sum()))
        return 0
    spec = jal.LLAMA3_8B_Q4_0
    n_prompt, n_steps = 32, 2
    if args.profile == "prefill":
        spec = dataclasses.replace(spec, num_layers=2)
        gguf = jal.synth_gguf(spec, SEED)
        recipe = jal.LlamaRecipe.from_gguf(gguf)
        cache = recipe.build_repack_cache(gguf)
        ctx = jal.ExecutionContext(recipe, cache, n_ctx=args.prefill + 64, kv_dtype=jal.KV_F16)
        ctx.set_stream(stream)
        prompt = np.random.Generator(np.random.PCG64(SEED)).integers(0, spec.vocab_size, args.prefill).astype(np.uint32)
        ctx.prefill_step(prompt, 0)
        torch.cuda.synchronize()
        torch.cuda.profiler.start()
        ctx.prefill_step(prompt, 0)
        torch.cuda.synchronize()
        torch.cuda.profiler.stop()
        print("profile prefill ok")
        return 0
    if args.profile == "attn":
        spec = dataclasses.replace(spec, num_layers=2)
        n_prompt, n_steps = args.prefill, 1
    gguf = jal.synth_gguf(spec, SEED)
    recipe = jal.LlamaRecipe.from_gguf(gguf)
    cache = recipe.build_repack_cache(gguf)
    ctx = jal.ExecutionContext(recipe, cache, n_ctx=n_prompt + 64, kv_dtype=jal.KV_F16)
    ctx.set_stream(stream)
    prompt = np.random.Generator(np.random.PCG64(SEED)).integers(0, spec.vocab_size, n_prompt).astype(np.uint32)
    logits = ctx.prefill_step(prompt, 0)
    ctx.decode_greedy(int(np.argmax(logits)), 3)  # captures the decode graph
    torch.cuda.synchronize()
    torch.cuda.profiler.start()
    ctx.decode_greedy(5, n_steps)
    torch.cuda.synchronize()
    torch.cuda.profiler.stop()
    print(f"profile {args.profile} ok")
    return 0


def trace_mode(args, jal, torch, stream):
    import numpy as np
    spec = jal.LLAMA3_8B_Q4_0
    gguf = jal.synth_gguf(spec, SEED)
    recipe = jal.LlamaRecipe.from_gguf(gguf)
    cache = recipe.build_repack_cache(gguf)
    n_prefill = args.prefill
    ctx = jal.ExecutionContext(recipe, cache, n_ctx=n_prefill + 64, kv_dtype=jal.KV_F16)
    ctx.set_stream(stream)
    rng = np.random.Generator(np.random.PCG64(SEED))
    ctx.prefill_step(rng.integers(0, spec.vocab_size, n_prefill).astype(np.uint32), 0)
    ctx.decode_greedy(1, 4)
    L = spec.num_layers
    roles = ["Q/K/V GEMV", "scores k_xattn", "output k_xattn_v", "O GEMV", "gate/up GEMV", "down GEMV"]
    runs = []
    for _ in range(5):
        t = ctx.trace_decode_step(int(rng.integers(0, spec.vocab_size))).astype(np.float64)
        runs.append(t)
    per = {r: {"dur": [], "excl": [], "gap": []} for r in roles + ["LM head"]}
    spans = []
    for t in runs:
        idx = list(range(1, 1 + 6 * L)) + [1 + 6 * L]
        spans.append((t[idx[-1], 1] - t[1, 0]) / 1e3)
        prev_end = None
        for k, i in enumerate(idx):
            role = "LM head" if i == 1 + 6 * L else roles[(i - 1) % 6]
            s, e = t[i, 0], t[i, 1]
            per[role]["dur"].append((e - s) / 1e3)
            if prev_end is not None:
                per[role]["excl"].append((e - prev_end) / 1e3)
                per[role]["gap"].append((s - prev_end) / 1e3)
            prev_end = e
    # Phase marks of the attention kernels, us after the previous launch's end.
    names = {1: ["grid dependency resolved", "scores done", "maxima exchanged", "exp terms in place",
                 "denominator"],
             2: ["grid dependency resolved", "weights in shared memory", "first product stage ready",
                 "chain done"]}
    marks = {1: [[] for _ in range(5)], 2: [[] for _ in range(4)]}
    for t in runs:
        for l in range(L):
            for r in (1, 2):
                i = 1 + 6 * l + r
                for k in range(len(names[r])):
                    if t[i, 2 + k] > 0:
                        marks[r][k].append((t[i, 2 + k] - t[i - 1, 1]) / 1e3)
    print(f"decode step at position ~{n_prefill}: {np.median(spans):.1f} us from the first Q/K/V CTA start to the "
          f"LM head's end (median of 5 traced steps; embedding and argmax not stamped)")
    print("| kernel | launches / step | in-kernel us (median) | critical-path us per launch (end to end) | "
          "critical-path us per step | start - previous end us (median) |")
    print("|---|---|---|---|---|---|")
    for role, d in per.items():
        n = len(d["dur"]) // len(runs)
        ex = float(np.median(d["excl"])) if d["excl"] else float("nan")
        tot = float(np.sum(d["excl"])) / len(runs) if d["excl"] else float("nan")
        gap = float(np.median(d["gap"])) if d["gap"] else float("nan")
        print(f"| {role} | {n} | {np.median(d['dur']):.2f} | {ex:.2f} | {tot:.1f} | {gap:.2f} |")
    for r, kname in ((1, "scores k_xattn"), (2, "output k_xattn_v")):
        print(f"{kname} phases (latest CTA, us after the previous kernel's end, median): " +
              ", ".join(f"{nm} {np.median(v):.2f}" for nm, v in zip(names[r], marks[r]) if v))
    return 0


def batch_arm(args, jal, torch, np, spec, cache, recipe, n_prefill, n_ctx, gen_s, build_s, peak, peak_kind):
    """--batch B: B independent sequences, each prefilled with its own prompt,
    then K steps of jal_decode_batch (the B tokens of a step decoded at once;
    value = B x K / time).  Each step goes through the C ABI and synchronises
    on the device; the e2e line adds the [B, vocab] logits read into one
    page-locked host array."""
    B = args.batch
    stream = torch.cuda.Stream()
    torch.cuda.set_stream(stream)
    ctxs = [jal.ExecutionContext(recipe, cache, n_ctx=n_ctx, kv_dtype=jal.KV_F16) for _ in range(B)]
    for c in ctxs:
        c.set_stream(stream)
    rng = np.random.Generator(np.random.PCG64(SEED))
    prompts = [rng.integers(0, spec.vocab_size, n_prefill).astype(np.uint32) for _ in range(B)]
    t_prefill = 0.0
    for c, p in zip(ctxs, prompts):
        t_prefill += ev_time(torch, lambda: c.prefill_step(p, 0), stream)
    toks = rng.integers(0, spec.vocab_size, B).astype(np.uint32)
    for _ in range(args.warmup):
        jal.decode_batch(ctxs, toks, want_logits=False)
    with ClockSampler(0) as clk:
        t_dec = ev_time(torch, lambda: [jal.decode_batch(ctxs, toks, want_logits=False) for _ in range(args.steps)],
                        stream)
    host = torch.empty((B, spec.vocab_size), dtype=torch.float32).pin_memory().numpy()
    t_e2e = ev_time(torch, lambda: [jal.decode_batch(ctxs, toks, out=host) for _ in range(args.steps)], stream)
    wq = "Q8_0" if spec.weight_quant == jal.Q8_0 else "Q4_0"
    bytes_token = cache.total_aligned_bytes()
    kv_bytes = B * 2 * spec.num_layers * spec.n_heads_kv * spec.head_dim * 2 * (n_prefill + args.warmup + args.steps)
    step_s = t_dec / args.steps
    line = {"metric": METRIC, "value": round(B * args.steps / t_dec, 2), "unit": "tok/s", "n_gpus": 1,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(step_s * 1e3, 4),
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "int8",
            "data": f"synthetic: seeded N(0,0.02) weights quantized to {wq}, uniform-random token ids",
            "config": {"workload": f"{args.workload} decode bs={B} (independent sequences) after {n_prefill}-token "
                                   "prefills", "batch": B,
                       "layers": spec.num_layers, "hidden": spec.hidden_dim, "heads": [spec.n_heads_q, spec.n_heads_kv],
                       "head_dim": spec.head_dim, "ffn": spec.ffn_dim, "vocab": spec.vocab_size,
                       "weights": f"{wq} ({'8.5' if wq == 'Q8_0' else '4.5'} bpw in HBM)", "kv_cache": "paged fp16",
                       "numerics": "reference f32 order (bit-exact with the oracle)", "parallelism": "replicas x1",
                       "l2": f"no flush: each step streams the {bytes_token / 1e9:.1f} GB of weights (> L2)",
                       "gguf_gen_s": round(gen_s, 1), "repack_s": round(build_s, 2)},
            "decode_step": {"bytes_per_step": bytes_token + kv_bytes,
                            "GBps": round((bytes_token + kv_bytes) / step_s / 1e9, 1),
                            "frac_of_peak": round((bytes_token + kv_bytes) / step_s / 1e9 / peak, 4),
                            "peak_GBps": peak, "peak_kind": peak_kind},
            "prefill": {"tokens": int(B * n_prefill), "s": round(t_prefill, 4),
                        "tok_per_s": round(B * n_prefill / t_prefill, 1)},
            "e2e": {"value": round(B * args.steps / t_e2e, 2), "unit": "tok/s", "h2d_bytes_per_step": 4 * B + 8 * B,
                    "d2h_bytes_per_step": 4 * B * spec.vocab_size},
            "gpu_launches": (3 + spec.num_layers * (7 + 2 * B)) * (args.warmup + 2 * args.steps),
            "clocks": clk.summary()}
    if not args.no_cpu:
        line["cpu_baseline"] = cpu_baseline(SHAPES[args.workload], 3, n_prefill + args.warmup, batch=B)
    print(json.dumps(line), flush=True)
    return 0


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=128)
    ap.add_argument("--warmup", type=int, default=8)
    ap.add_argument("--impl", default="jal", choices=["jal", "reference"])
    ap.add_argument("--prefill", type=int, default=2048)
    ap.add_argument("--no-sweep", action="store_true")
    ap.add_argument("--no-cpu", action="store_true")
    ap.add_argument("--workload", default="llama3-8b-q4_0",
                    choices=["llama3-8b-q4_0", "qwen2-7b-q8_0", "llama3-70b-q4_0", "tiny"])
    ap.add_argument("--batch", type=int, default=1,
                    help="decode this many independent sequences per step (jal_decode_batch), one GPU")
    ap.add_argument("--tp", action="store_true",
                    help="with N > 1 ranks: one tensor-parallel model over the N GPUs (strong scaling) "
                         "instead of N independent replicas")
    ap.add_argument("--profile", choices=["gemv", "skinny", "decode", "attn", "prefill", "trace"],
                    help="run a small fixed workload for ncu instead of the benchmark")
    args = ap.parse_args()
    if args.profile:
        return profile_mode(args)
    if args.impl == "reference":
        return reference_arm(args)
    args.warmup = max(args.warmup, 3)

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    import numpy as np
    import torch
    torch.cuda.set_device(local)
    dist = None
    if world > 1:
        import datetime
        import torch.distributed as dist
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=600),
                                device_id=torch.device("cuda", local))
    jal = load_jal()
    jal.set_device(local)
    spec = {"llama3-8b-q4_0": jal.LLAMA3_8B_Q4_0, "qwen2-7b-q8_0": jal.QWEN2_7B_Q8_0,
            "llama3-70b-q4_0": jal.LLAMA3_70B_Q4_0}.get(args.workload, jal.TINY_LLAMA)
    wq = "Q8_0" if spec.weight_quant == jal.Q8_0 else "Q4_0"
    peak, peak_kind = measured_peaks()

    t0 = time.perf_counter()
    gguf = jal.synth_gguf(spec, SEED)
    gen_s = time.perf_counter() - t0
    recipe = jal.LlamaRecipe.from_gguf(gguf)
    t0 = time.perf_counter()
    tp = None
    if dist and args.tp:
        uid = [jal.tp_unique_id() if rank == 0 else None]
        dist.broadcast_object_list(uid, src=0)
        tp = jal.TensorParallel(uid[0], rank, world)
    cache = recipe.build_repack_cache(gguf, device=local, tp=tp)
    build_s = time.perf_counter() - t0
    n_prefill = prefill_tokens(SHAPES[args.workload], args)
    assert SHAPES[args.workload]["context_length"] == spec.context_length
    n_ctx = n_prefill + 2 * (args.warmup + args.steps) + 16
    if args.batch > 1:
        return batch_arm(args, jal, torch, np, spec, cache, recipe, n_prefill, n_ctx, gen_s, build_s, peak, peak_kind)
    ctx = jal.ExecutionContext(recipe, cache, n_ctx=n_ctx, kv_dtype=jal.KV_F16)
    stream = torch.cuda.Stream()  # a capturable stream: decode steps replay a CUDA graph on it
    torch.cuda.set_stream(stream)
    ctx.set_stream(stream)
    rng = np.random.Generator(np.random.PCG64(SEED + (0 if tp else rank)))  # TP ranks feed the same tokens
    prompt = rng.integers(0, spec.vocab_size, n_prefill).astype(np.uint32)

    # Prefill (device-timed; includes the token upload and the logits read).
    logits = None

    def do_prefill():
        nonlocal logits
        logits = ctx.prefill_step(prompt, 0)

    do_prefill()  # warm-up (kernel loads, first-use NCCL connections); the timed pass rewrites the cache
    t_prefill = ev_time(torch, do_prefill, stream)
    tok = int(np.argmax(logits))
    # Decode warm-up, then K timed steps (one CUDA graph launch per token).
    ctx.decode_greedy(tok, args.warmup)
    tok = int(rng.integers(0, spec.vocab_size))
    if dist:
        dist.barrier()
    with ClockSampler(local) as clk:
        t_dec = ev_time(torch, lambda: ctx.decode_greedy(tok, args.steps), stream)
    if dist:
        tt = torch.tensor([t_dec, t_prefill], dtype=torch.float64, device="cuda")
        dist.all_reduce(tt, op=dist.ReduceOp.MAX)
        t_dec, t_prefill = float(tt[0]), float(tt[1])
    # End to end through the C ABI with host buffers: per step the token goes
    # up from pinned memory and the full logits row comes back into a
    # page-locked host array that the caller reuses.
    pos0 = ctx.position()
    host_logits = torch.empty(spec.vocab_size, dtype=torch.float32).pin_memory().numpy()
    t_e2e = ev_time(torch, lambda: [ctx.decode_step(tok, out=host_logits) for _ in range(args.steps)], stream)
    if dist:
        tt = torch.tensor([t_e2e], dtype=torch.float64, device="cuda")
        dist.all_reduce(tt, op=dist.ReduceOp.MAX)
        t_e2e = float(tt[0])
    assert ctx.position() == pos0 + args.steps

    launches = ctx.launches_per_step()
    bytes_token = cache.total_aligned_bytes() - spec.vocab_size * 0  # layer weights + head + norms
    kv_bytes = 2 * spec.num_layers * spec.n_heads_kv * spec.head_dim * 2 * (n_prefill + args.warmup + args.steps // 2)
    if tp:
        kv_bytes //= world  # per GPU: this rank's KV heads (bytes_token is already its shard)
    step_s = t_dec / args.steps
    streams = 1 if tp else world  # token streams: one per replica, one for a tensor-parallel model
    line = {"metric": METRIC, "value": round(streams * args.steps / t_dec, 2), "unit": "tok/s", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(step_s * 1e3, 4),
            "higher_is_better": True, "scaling": "strong" if tp else "weak", "vs_baseline": None, "dtype": "int8",
            "data": f"synthetic: seeded N(0,0.02) weights quantized to {wq}, uniform-random token ids",
            "config": {"workload": f"{args.workload} decode bs=1 greedy after a {n_prefill}-token prefill",
                       "layers": spec.num_layers, "hidden": spec.hidden_dim, "heads": [spec.n_heads_q, spec.n_heads_kv],
                       "head_dim": spec.head_dim, "ffn": spec.ffn_dim, "vocab": spec.vocab_size,
                       "weights": f"{wq} ({'8.5' if wq == 'Q8_0' else '4.5'} bpw in HBM)", "kv_cache": "paged fp16",
                       "numerics": "reference f32 order (bit-exact with the oracle)" if not tp else "relaxed", "parallelism": f"tp{world} ({ctx.tp_exchange()} exchange)" if tp else f"replicas x{world}",
                       "l2": f"no flush: each step streams the {cache.total_aligned_bytes() / 1e9:.1f} GB of weights (> L2)",
                       "gguf_gen_s": round(gen_s, 1), "repack_s": round(build_s, 2)},
            "decode_step": {"bytes_per_token": bytes_token + kv_bytes,
                            "GBps": round((bytes_token + kv_bytes) / step_s / 1e9, 1),
                            "frac_of_peak": round((bytes_token + kv_bytes) / step_s / 1e9 / peak, 4),
                            "peak_GBps": peak, "peak_kind": peak_kind},
            "prefill": {"tokens": int(n_prefill), "s": round(t_prefill, 4),
                        "tok_per_s": round(streams * n_prefill / t_prefill, 1)},
            "e2e": {"value": round(streams * args.steps / t_e2e, 2), "unit": "tok/s", "h2d_bytes_per_step": 4 + 8,
                    "d2h_bytes_per_step": 4 * spec.vocab_size},
            "gpu_launches": launches * (args.steps + args.warmup) + 0,
            "clocks": clk.summary()}
    if rank == 0 and not args.no_sweep:
        sweep = gemv_sweep(jal, torch, peak, ["Q4_0", "Q8_0"])
        line["gemv_sweep"] = sweep
        dom = next(s for s in sweep if s["quant"] == "Q4_0" and s["M"] == 14336)
        traffic = committed_traffic().get("gemv_q4_0_14336x4096")
        line["roofline"] = {"kernel": "k_xgemv<Q4_0,store> 14336x4096 (reference-order decode quant-GEMV, int8 input)",
                            "bound": "hbm",
                            "achieved": dom["GBps"], "peak": peak, "unit": "GB/s",
                            "frac": round(dom["GBps"] / peak, 4), "traffic": traffic,
                            "algorithmic_bytes": dom["bytes"], "peak_kind": peak_kind}
        line["gpu_launches"] += sum(200 + 2 * max(2, -(-4 * L2_BYTES // (s["bytes"]))) for s in sweep)
    if rank == 0 and world == 1 and not args.no_cpu:
        line["cpu_baseline"] = cpu_baseline(SHAPES[args.workload], 3, n_prefill + args.warmup)
    if rank == 0:
        print(json.dumps(line), flush=True)
    del ctx
    del cache
    if dist:
        dist.barrier()
        del tp
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
