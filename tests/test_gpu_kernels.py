"""Device kernels against the oracle (needs a B200).

Bars: repack, activation quantizers, 16-element integer partials and every
projection, RMSNorm, SwiGLU and attention entry point, which all compute in
the reference's f32 order, are equal to the oracle bit for bit.  The RoPE op
(angles computed on the device) is held to max|y - y_ref| / max|y_ref| <= 1e-5,
a normalised max error (rel_err below), not a per-element relative error.
Inputs are seeded synthetic tensors with the shapes of the quant-GEMV op
sweep (M x K in {4096x4096, 11008x4096, 4096x11008, 14336x4096}).
"""
import math

import numpy as np
import pytest

import ref_fixtures as fx

pytestmark = pytest.mark.gpu

REL_TOL = 1e-3
SWEEP = [(4096, 4096), (11008, 4096), (4096, 11008), (14336, 4096)]


def rel_err(got, ref):
    got = np.asarray(got, dtype=np.float64)
    ref = np.asarray(ref, dtype=np.float64)
    return float(np.max(np.abs(got - ref)) / max(np.max(np.abs(ref)), 1e-30))


def dev(torch, a):
    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


@pytest.mark.parametrize("quant_name", ["Q4_0", "Q8_0"])
@pytest.mark.parametrize("rows,cols", SWEEP)
def test_repack_bit_exact_and_gemv_op_sweep(jal, oracle, torch_cuda, quant_name, rows, cols):
    torch = torch_cuda
    quant = getattr(jal, quant_name)
    raw = jal.synth_matrix(quant, rows, cols, seed=1234, name=f"sweep.{rows}x{cols}")
    mat = jal.CachedMatrix.repack(raw, quant, rows, cols)
    assert mat.rows() == rows and mat.cols() == cols
    # 4.5 / 8.5 bits per weight in HBM (GGUF bytes, scales padded per row to 16 B)
    assert mat.aligned_bytes() >= raw.nbytes and mat.aligned_bytes() <= raw.nbytes * 1.01
    ref = oracle.RepackedWeight(raw, quant, rows, cols)
    tiles, scales = mat.export_ref_layout()
    assert np.array_equal(tiles, ref.tiles())
    assert np.array_equal(scales.view(np.uint32), ref.scales().view(np.uint32))
    x = jal.synth_normal(cols, seed=99, name="sweep.act")
    y = torch.zeros(rows, dtype=torch.float32, device="cuda")
    mat.gemm(dev(torch, x), 1, y)
    torch.cuda.synchronize()
    want = ref.project_batch(x, 1)[0]
    assert np.array_equal(y.cpu().numpy(), want)


def test_q5_0_repack_bit_exact_and_projection(jal, oracle, torch_cuda):
    # Q5_0 unpacks to int8 like Q8_0 (unpack_row_i8, repack_cache.rs:840-871)
    # and runs the Q8_0 device layout: reference tiles and scales bit for
    # bit, projections (M = 1 and 5) equal to the oracle's.
    torch = torch_cuda
    rows, cols = 4096, 4096
    raw = jal.synth_matrix(jal.Q5_0, rows, cols, seed=321, name="q5.sweep")
    mat = jal.CachedMatrix.repack(raw, jal.Q5_0, rows, cols)
    assert mat.quant() == jal.Q5_0
    ref = oracle.RepackedWeight(raw, jal.Q5_0, rows, cols)
    tiles, scales = mat.export_ref_layout()
    assert np.array_equal(tiles, ref.tiles())
    assert np.array_equal(scales.view(np.uint32), ref.scales().view(np.uint32))
    for m in (1, 5):
        x = jal.synth_normal(m * cols, seed=322 + m, name="q5.act")
        y = torch.zeros(m * rows, dtype=torch.float32, device="cuda")
        mat.gemm(dev(torch, x), m, y)
        torch.cuda.synchronize()
        want = ref.project_batch(x, m)
        got = y.cpu().numpy().reshape(m, rows)
        assert np.array_equal(got, want)


@pytest.mark.parametrize("quant_name", ["Q4_0", "Q8_0"])
def test_dot16_partials_exact(jal, oracle, torch_cuda, quant_name):
    torch = torch_cuda
    quant = getattr(jal, quant_name)
    rows, cols = 200, 4096
    raw = jal.synth_matrix(quant, rows, cols, seed=5, name="partials")
    mat = jal.CachedMatrix.repack(raw, quant, rows, cols)
    ref = oracle.RepackedWeight(raw, quant, rows, cols)
    x = jal.synth_normal(cols, seed=6, name="partials.act")
    q8, _ = oracle.quantize_act_rows(x, 1, cols)
    out = torch.zeros((rows - 17) * (cols // 16), dtype=torch.int32, device="cuda")
    mat.dot16_partials(dev(torch, q8[0]), 17, rows, out)
    torch.cuda.synchronize()
    assert np.array_equal(out.cpu().numpy().reshape(rows - 17, -1), ref.dot16_partials(q8[0], 17, rows))


def test_act_quantizer_bit_exact(jal, oracle, torch_cuda):
    torch = torch_cuda
    m, k = 5, 4096 + 96
    x = jal.synth_normal(m * k, seed=3, name="act.q").reshape(m, k)
    x[1, 40:72] = 0.0
    x[2, 3] = np.inf
    x[2, 7] = np.nan
    x[3, 100:132] *= 1e-30
    q = torch.zeros(m * k, dtype=torch.int8, device="cuda")
    s = torch.zeros(m * (k // 32), dtype=torch.float32, device="cuda")
    jal.act_quantize_q8(dev(torch, x), m, k, q, s)
    torch.cuda.synchronize()
    rq, rs = oracle.quantize_act_rows(x.ravel(), m, k)
    assert np.array_equal(q.cpu().numpy().reshape(m, k), rq)
    assert np.array_equal(s.cpu().numpy().reshape(m, -1).view(np.uint32), rs.view(np.uint32))


def test_quantize_row_q8_0_bit_exact(jal, oracle, torch_cuda):
    torch = torch_cuda
    n = 4096
    x = jal.synth_normal(n, seed=4, name="q80")
    x[64:96] = 0.0
    x[5] = np.nan
    blocks = torch.zeros(n // 32 * 36, dtype=torch.uint8, device="cuda")
    jal.quantize_row_q8_0(dev(torch, x), n, blocks)
    torch.cuda.synchronize()
    assert np.array_equal(blocks.cpu().numpy(), oracle.quantize_row_q8_0(x))


@pytest.mark.parametrize("m", [2, 3, 4, 8, 37, 200])
@pytest.mark.parametrize("quant_name", ["Q4_0", "Q8_0"])
def test_small_batch_gemv_and_gemm(jal, oracle, torch_cuda, m, quant_name):
    torch = torch_cuda
    quant = getattr(jal, quant_name)
    rows, cols = 1000, 2048
    raw = jal.synth_matrix(quant, rows, cols, seed=8, name="batch")
    mat = jal.CachedMatrix.repack(raw, quant, rows, cols)
    x = jal.synth_normal(m * cols, seed=9, name="batch.act")
    y = torch.zeros(m * rows, dtype=torch.float32, device="cuda")
    mat.gemm(dev(torch, x), m, y)
    torch.cuda.synchronize()
    want = oracle.RepackedWeight(raw, quant, rows, cols).project_batch(x, m)
    assert np.array_equal(y.cpu().numpy().reshape(m, rows), want)


def test_prefill_gemm_llama3_8b_down_projection_2048_tokens(jal, oracle, torch_cuda):
    # The 8B down projection (4096 rows x 14336 columns, Q4_0) over a
    # 2048-token prefill batch, equal to the oracle's gemm_rows bit for bit.
    torch = torch_cuda
    rows, cols, m = 4096, 14336, 2048
    raw = jal.synth_matrix(jal.Q4_0, rows, cols, seed=41, name="down8b")
    mat = jal.CachedMatrix.repack(raw, jal.Q4_0, rows, cols)
    x = jal.synth_normal(m * cols, seed=42, name="down8b.act")
    y = torch.zeros(m * rows, dtype=torch.float32, device="cuda")
    mat.gemm(dev(torch, x), m, y)
    torch.cuda.synchronize()
    import os
    want = oracle.RepackedWeight(raw, jal.Q4_0, rows, cols).project_batch(x, m, nthreads=os.cpu_count() or 1)
    assert np.array_equal(y.cpu().numpy().reshape(m, rows), want)


@pytest.mark.parametrize("quant_name", ["Q4_0", "Q8_0"])
def test_wave2_shapes_vs_compute_row_dot(jal, oracle, torch_cuda, quant_name):
    # tests/repack_wave2_parity.rs:182-236 on the device (rows 73, cols 256, m 3)
    torch = torch_cuda
    quant = getattr(jal, quant_name)
    rows, cols, m = 73, 256, 3
    raw = fx.fill_quant_bytes(rows, cols, quant, 2)
    act = fx.wave2_activation(m, cols)
    mat = jal.CachedMatrix.repack(raw, quant, rows, cols)
    y = torch.zeros(m * rows, dtype=torch.float32, device="cuda")
    mat.gemm(dev(torch, act), m, y)
    torch.cuda.synchronize()
    got = y.cpu().numpy().reshape(m, rows)
    want = oracle.RepackedWeight(raw, quant, rows, cols).project_batch(act, m)
    for t in range(m):
        x = act[t * cols:(t + 1) * cols]
        bound = max(float(np.sqrt(np.sum(x * x))) * math.sqrt(cols), 1.0)
        for r in range(rows):
            exp = oracle.compute_row_dot(r, cols, quant, raw, x)
            assert abs(got[t, r] - exp) / max(bound, abs(exp)) < 1e-2
        assert np.array_equal(got[t], want[t])


@pytest.mark.parametrize("quant_name", ["Q4_0", "Q5_0", "Q8_0"])
def test_streaming_raw_gemv_decode_projection(jal, oracle, torch_cuda, quant_name):
    # gemv_decode_projection (decode_gemv.rs:1289-1388) for a 4096-column head
    torch = torch_cuda
    quant = getattr(jal, quant_name)
    rows, cols = 3000, 4096
    if quant == jal.Q5_0:
        raw = fx.fill_q4_0_or_q5_0(rows, cols, 6, 4)
    else:
        raw = jal.synth_matrix(quant, rows, cols, seed=10, name="head")
    x = jal.synth_normal(cols, seed=11, name="head.act")
    y = torch.zeros(rows, dtype=torch.float32, device="cuda")
    jal.gemv_decode_projection(dev(torch, raw), raw.nbytes, quant, rows, cols, dev(torch, x), y)
    torch.cuda.synchronize()
    # block results are added in the reference's order: bit-exact
    want = oracle.gemv_decode_projection(raw, quant, rows, cols, x)
    assert np.array_equal(y.cpu().numpy().view(np.uint32), want.view(np.uint32))


def _raw_superblock_rows(jal, quant, rows, cols, seed):
    """Random super-block rows (quant bytes uniform) with scale fields drawn
    as f16 / bf16 of small normal values; the first block of row 0 gets an
    Inf scale (sanitised to 0.0625 by the kernels)."""
    rng = np.random.Generator(np.random.PCG64(seed))
    bb = {jal.Q4_K: 144, jal.Q5_K: 176, jal.Q6_K: 210, jal.TQ1_0: 54, jal.TQ2_0: 66}[quant]
    nb = cols // 256
    blk = rng.integers(0, 256, size=(rows, nb, bb), dtype=np.uint8)
    def put16(off, vals):
        blk[:, :, off:off + 2] = vals.astype("<u2").view(np.uint8).reshape(rows, nb, 2)
    f16 = lambda sd: rng.normal(0, sd, (rows, nb)).astype(np.float16).view(np.uint16)
    if quant in (jal.Q4_K, jal.Q5_K):
        put16(0, f16(1e-3)); put16(2, f16(1e-3))
    elif quant == jal.Q6_K:
        put16(208, f16(1e-3))
    elif quant == jal.TQ1_0:
        put16(0, f16(1e-2))
    else:  # TQ2_0: bf16 scale
        put16(64, (rng.normal(0, 1e-2, (rows, nb)).astype(np.float32).view(np.uint32) >> 16).astype(np.uint16))
    off = {jal.Q4_K: 0, jal.Q5_K: 0, jal.Q6_K: 208, jal.TQ1_0: 0, jal.TQ2_0: 64}[quant]
    blk[0, 0, off:off + 2] = (0x00, 0x7C) if quant != jal.TQ2_0 else (0x80, 0x7F)
    return blk.reshape(-1)


def _raw_dense_rows(jal, quant, rows, cols, seed):
    rng = np.random.Generator(np.random.PCG64(seed))
    w = rng.normal(0, 0.02, (rows, cols)).astype(np.float32)
    if quant == jal.F32:
        w[0, 3] = np.inf
        return w.view(np.uint8).reshape(-1)
    if quant == jal.F16:
        h = w.astype(np.float16).view(np.uint16)
        h[0, 3] = 0x7C00
    else:
        h = (w.view(np.uint32) >> 16).astype(np.uint16)
        h[0, 3] = 0x7F80
    return h.view(np.uint8).reshape(-1)


@pytest.mark.parametrize("quant_name", ["Q4_K", "Q5_K", "Q6_K", "TQ1_0", "TQ2_0", "F16", "BF16", "F32"])
def test_streaming_raw_gemv_superblock_and_dense_bit_exact(jal, oracle, torch_cuda, quant_name):
    # gemv_decode_projection for the super-block types (BlockQ8_K activation)
    # and dense rows: the device adds the per-block results in the
    # reference's order, so every output equals the oracle's bit for bit.
    # The second activation carries a NaN and an Inf (zeroed by the
    # quantizer / the dense chunk mask); dense rows use 4000 columns so that
    # the last 256-element chunk is partial.
    torch = torch_cuda
    quant = getattr(jal, quant_name)
    dense = quant in (jal.F16, jal.BF16, jal.F32)
    rows, cols = 1500, (4000 if dense else 4096)
    raw = (_raw_dense_rows if dense else _raw_superblock_rows)(jal, quant, rows, cols, 31)
    for k, x in enumerate([jal.synth_normal(cols, seed=32, name="stream.act"),
                           jal.synth_normal(cols, seed=33, name="stream.act2")]):
        if k == 1:
            x[7], x[300] = np.nan, np.inf
        y = torch.zeros(rows, dtype=torch.float32, device="cuda")
        jal.gemv_decode_projection(dev(torch, raw), raw.nbytes, quant, rows, cols, dev(torch, x), y)
        torch.cuda.synchronize()
        want = oracle.gemv_decode_projection(raw, quant, rows, cols, x)
        got = y.cpu().numpy()
        assert np.all(np.isfinite(want))
        assert np.array_equal(got.view(np.uint32), want.view(np.uint32)), \
            f"{int(np.sum(got != want))} rows differ, max |d| {np.max(np.abs(got - want)):.3e}"


def test_unsupported_quant_fails_closed(jal, torch_cuda):
    with pytest.raises(jal.CapabilityMismatch):
        jal.CachedMatrix.repack(np.zeros(84, np.uint8), 10, 1, 256)
    with pytest.raises(jal.TensorBoundsError):
        jal.CachedMatrix.repack(np.zeros(10, np.uint8), jal.Q4_0, 1, 256)


def test_ops_rmsnorm_rope_swiglu_attention(jal, oracle, torch_cuda):
    torch = torch_cuda
    n = 4096
    x = jal.synth_normal(3 * n, seed=21, name="ops.x")
    w = (1.0 + 0.1 * jal.synth_normal(n, seed=22, name="ops.w")).astype(np.float32)
    out = torch.zeros(3 * n, dtype=torch.float32, device="cuda")
    jal.rmsnorm(dev(torch, x), dev(torch, w), 3, n, 1e-5, out)
    torch.cuda.synchronize()
    got = out.cpu().numpy().reshape(3, n)
    for t in range(3):
        assert np.array_equal(got[t], oracle.rmsnorm_row(x[t * n:(t + 1) * n], w, 1e-5))
    # RoPE: 4 rows, 8 heads of 128 at positions 5..8, Norm and NeoX
    inv = oracle.fill_inv_freq(128, 500000.0, 16)
    for neox in (False, True):
        qk = jal.synth_normal(4 * 1024, seed=23, name="ops.qk")
        d = dev(torch, qk)
        jal.rope(d, 4, 1024, 128, 128, neox, 5, dev(torch, inv))
        torch.cuda.synchronize()
        want = np.concatenate([oracle.apply_rope(qk[t * 1024:(t + 1) * 1024], 128, 128, neox, 5 + t, inv)
                               for t in range(4)])
        assert rel_err(d.cpu().numpy(), want) <= 1e-5
    g = jal.synth_normal(n, seed=24, name="ops.g", std=4.0)
    g[:4] = [25.0, -25.0, 20.0, -20.0]
    u = jal.synth_normal(n, seed=25, name="ops.u")
    o = torch.zeros(n, dtype=torch.float32, device="cuda")
    jal.swiglu(dev(torch, g), dev(torch, u), n, o)
    torch.cuda.synchronize()
    assert np.array_equal(o.cpu().numpy(), oracle.swiglu(g, u))
    # GQA attention: 5 queries at start_pos 11 over 16 positions, 8/2 heads, hd 64, window 0 and 6
    nq, nkv, hd, total, m, sp = 8, 2, 64, 16, 5, 11
    q = jal.synth_normal(m * nq * hd, seed=26, name="att.q")
    k = jal.synth_normal(total * nkv * hd, seed=27, name="att.k")
    v = jal.synth_normal(total * nkv * hd, seed=28, name="att.v")
    for window in (0, 6):
        o = torch.zeros(m * nq * hd, dtype=torch.float32, device="cuda")
        jal.gqa_attention(dev(torch, q), dev(torch, k), dev(torch, v), m, nq, nkv, hd, total, sp, window, 0.125, o)
        torch.cuda.synchronize()
        want = oracle.gqa_attention(q, k, v, m, nq, nkv, hd, total, sp, window, 0.125)
        assert np.array_equal(o.cpu().numpy(), want)


def test_rmsnorm_rows_sequential_sum_stress(jal, oracle, torch_cuda):
    """RMSNorm equals the reference bit for bit on rows built to stress the
    parallel form of its sequential sum of squares (exact::seq_sum_nonneg):
    lengths from 1 to 40000, magnitudes over many binades within a row,
    exact zeros, tiny (subnormal-square) values, values whose squares tie
    against the running sum's rounding grid (small integers and halves), a
    huge leading element, and a row that overflows to inf."""
    torch = torch_cuda
    rng = np.random.Generator(np.random.PCG64(77))
    rows = []
    for n in (1, 2, 3, 5, 31, 32, 33, 100, 255, 512, 1000, 4096, 5000, 8192, 14336, 40000):
        rows.append(rng.standard_normal(n).astype(np.float32))
    n = 4096
    rows.append((rng.standard_normal(n) * np.exp2(rng.integers(-30, 30, n))).astype(np.float32))
    z = rng.standard_normal(n).astype(np.float32)
    z[::3] = 0.0
    rows.append(z)
    rows.append((rng.standard_normal(n) * 1e-23).astype(np.float32))
    rows.append(rng.integers(-8, 9, n).astype(np.float32))
    rows.append((rng.integers(-64, 65, n) * 0.5).astype(np.float32))
    r = rng.standard_normal(n).astype(np.float32)
    r[0] = 3.0e18
    rows.append(r)
    rows.append(np.linspace(1.0, 4096.0, n, dtype=np.float32))
    rows.append(np.full(n, 2.0e19, dtype=np.float32))
    rows.append(np.zeros(n, dtype=np.float32))
    for i, x in enumerate(rows):
        n = x.size
        w = (1.0 + 0.01 * rng.standard_normal(n)).astype(np.float32)
        out = torch.zeros(n, dtype=torch.float32, device="cuda")
        jal.rmsnorm(dev(torch, x), dev(torch, w), 1, n, 1e-5, out)
        torch.cuda.synchronize()
        want = oracle.rmsnorm_row(x, w, 1e-5)
        got = out.cpu().numpy()
        assert np.array_equal(got.view(np.uint32), want.view(np.uint32)), f"row {i} (n={n})"


@pytest.mark.parametrize("quant_name", ["Q4_K", "Q5_K", "Q6_K"])
def test_kquant_repack_export_and_projection_bit_exact(jal, oracle, torch_cuda, quant_name):
    """K-quant matrices in the repacked path (unpack_row_i8, repack_cache.rs:
    890-993; the BlockScaledI8 fold with its min term, :739-783): 300 rows
    (a partial 8-row tile) x 1024 columns of random super-blocks, one with an
    Inf scale; the exported tiles, scales and mins equal the oracle's repack
    bit for bit, and projections at M = 1 and 3 (activations with a NaN and an
    Inf, which the group sums read as zero) equal the oracle's."""
    torch = torch_cuda
    quant = getattr(jal, quant_name)
    rows, cols = 300, 1024
    raw = _raw_superblock_rows(jal, quant, rows, cols, 71)
    mat = jal.CachedMatrix.repack(raw, quant, rows, cols)
    assert mat.quant() == quant and mat.rows() == rows and mat.cols() == cols
    ref = oracle.RepackedWeight(raw, quant, rows, cols)
    tiles, scales = mat.export_ref_layout()
    assert np.array_equal(tiles, ref.tiles())
    assert np.array_equal(scales.view(np.uint32), ref.scales().view(np.uint32))
    if quant != jal.Q6_K:
        assert np.array_equal(mat.export_ref_mins().view(np.uint32), ref.mins().view(np.uint32))
    for m in (1, 3):
        x = jal.synth_normal(m * cols, seed=72 + m, name="kq.act").copy()
        x[5] = np.nan
        x[cols + 7 if m > 1 else 9] = np.inf
        y = torch.zeros(m * rows, dtype=torch.float32, device="cuda")
        mat.gemm(dev(torch, x), m, y)
        torch.cuda.synchronize()
        want = ref.project_batch(x, m)
        got = y.cpu().numpy().reshape(m, rows)
        assert np.array_equal(got.view(np.uint32), want.view(np.uint32))
