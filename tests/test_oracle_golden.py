"""Pins the CPU oracle against the reference crate's own known-answer tests and
structural invariants (CPU only).  Each test names the reference test it
restates."""
import math
import struct

import numpy as np
import pytest

import ref_fixtures as fx


def f16_bits_np(bits):
    return np.array([bits], dtype=np.uint16).view(np.float16).astype(np.float32)[0]


def test_f16_finite_matches_ieee_for_every_finite_half(oracle):
    # f16_to_f32_finite (repack_cache.rs:160-181): exact on finite halves,
    # Inf/NaN -> +-0.0625.
    for bits in range(0, 1 << 16, 7):
        exp = (bits >> 10) & 0x1F
        got = oracle.f16_to_f32_finite(bits)
        if exp == 31:
            assert got == (-0.0625 if bits & 0x8000 else 0.0625)
        else:
            want = f16_bits_np(bits)
            assert struct.pack("<f", got) == struct.pack("<f", want), hex(bits)
    assert oracle.f16_to_f32_finite(0x0001) == 2.0 ** -24
    assert oracle.f16_to_f32_finite(0x3C00) == 1.0


def test_bf16_and_sanitize(oracle):
    # bf16_to_f32_finite (repack_cache.rs:184-191), sanitize_f32_weight (:1028-1036)
    assert oracle.bf16_to_f32_finite(0x3F80) == 1.0
    assert oracle.bf16_to_f32_finite(0x7F80) == 0.0625
    assert oracle.bf16_to_f32_finite(0xFFC0) == -0.0625
    assert oracle.sanitize_f32_weight(2.0e6) == 0.0625
    assert oracle.sanitize_f32_weight(-2.0e6) == -0.0625
    assert oracle.sanitize_f32_weight(float("nan")) == 0.0
    assert oracle.sanitize_f32_weight(5.0) == 5.0


def test_q5_0_known_answer(oracle):
    # lib.rs:653-712 test_q5_0_dequant_repack_and_lm_head
    blk = fx.q5_0_known_block()
    deq = oracle.dequantize_block(6, blk)
    qh = 0xA55A5AA5
    for j in range(16):
        p = int(blk[6 + j])
        e0 = 0.5 * (((p & 0x0F) | (((qh >> j) & 1) << 4)) - 16)
        e1 = 0.5 * (((p >> 4) | (((qh >> (j + 16)) & 1) << 4)) - 16)
        assert abs(deq[j] - e0) < 1e-6 and abs(deq[j + 16] - e1) < 1e-6
    x = (np.arange(32, dtype=np.float32) - np.float32(15.0)) * np.float32(0.1)
    ref_dot = float(np.float32(sum(np.float32(a) * np.float32(b) for a, b in zip(deq, x))))
    assert abs(oracle.compute_row_dot(0, 32, 6, blk, x) - ref_dot) < 1e-5
    out = oracle.gemv_decode_projection(blk, 6, 1, 32, x)
    l2 = float(np.sqrt(np.sum(x * x)))
    bound = max(l2 * math.sqrt(32), abs(ref_dot), 1.0)
    assert abs(out[0] - ref_dot) / bound < 1e-2


def test_q5_k_known_answer(oracle):
    # lib.rs:714-781 test_q5_k_dequant_repack_and_unsupported_quant_rejection
    kb = fx.q5_k_known_block()
    kout = oracle.dequantize_block(13, kb)
    x = ((np.arange(256) % 19).astype(np.float32) - np.float32(9.0)) * np.float32(0.05)
    ref_dot = float(np.dot(kout.astype(np.float64), x.astype(np.float64)))
    assert abs(oracle.compute_row_dot(0, 256, 13, kb, x) - ref_dot) < 1e-4
    w = oracle.RepackedWeight(kb, 13, 1, 256)
    got = w.project_batch(x, 1)[0, 0]
    l2 = float(np.sqrt(np.sum(x * x)))
    bound = max(l2 * 16.0, abs(ref_dot), 1.0)
    assert abs(got - ref_dot) / bound < 1e-2
    lm = oracle.gemv_decode_projection(kb, 13, 1, 256, x)
    assert abs(lm[0] - ref_dot) / bound < 1e-2
    # Q2_K must fail closed (CapabilityMismatch = 2).
    with pytest.raises(oracle.OracleError, match="status 2"):
        oracle.gemv_decode_projection(np.zeros(84, np.uint8), 10, 1, 256, x)


def test_q4_k_m_two_rows(oracle):
    # dispatch.rs:295-359: 6-bit scale/min unpack, repacked vs compute_row_dot < 5e-3
    raw = fx.q4_k_m_two_rows()
    hidden = np.arange(256, dtype=np.float32) * np.float32(0.01) - np.float32(1.2)
    refs = [oracle.compute_row_dot(r, 256, 12, raw, hidden) for r in range(2)]
    lm = oracle.gemv_decode_projection(raw, 12, 2, 256, hidden)
    rep = oracle.RepackedWeight(raw, 12, 2, 256).project_batch(hidden, 1)[0]
    for r in range(2):
        assert abs(lm[r] - refs[r]) / max(abs(refs[r]), 1.0) < 5e-3
        assert abs(rep[r] - refs[r]) / max(abs(refs[r]), 1.0) < 5e-3


def test_rope_norm_vs_neox_partial_rotary(oracle):
    # lib.rs:489-516: partial rotary_dim = 4 on head_dim = 8 at pos 3
    inv = oracle.fill_inv_freq(4, 10000.0, 8)
    orig = np.array([1, 2, 3, 4, 10, 11, 12, 13], dtype=np.float32)
    norm = oracle.apply_rope(orig, 8, 4, False, 3, inv)
    neox = oracle.apply_rope(orig, 8, 4, True, 3, inv)
    assert np.array_equal(norm[4:], orig[4:]) and np.array_equal(neox[4:], orig[4:])
    for i, f in enumerate(inv):
        a = np.float32(3.0) * np.float32(f)
        s, c = math.sin(a), math.cos(a)
        assert abs(norm[2 * i] - (orig[2 * i] * c - orig[2 * i + 1] * s)) < 1e-5
        assert abs(norm[2 * i + 1] - (orig[2 * i] * s + orig[2 * i + 1] * c)) < 1e-5
        assert abs(neox[i] - (orig[i] * c - orig[i + 2] * s)) < 1e-5
        assert abs(neox[i + 2] - (orig[i] * s + orig[i + 2] * c)) < 1e-5


def test_llama3_smooth_inv_freq(oracle):
    # lib.rs:589-614
    inv = oracle.fill_inv_freq(128, 500000.0, 16384, kind=2, factor=8.0, low=1.0, high=4.0, orig=8192)
    orig_ctx = np.float32(8192.0)
    for i, actual in enumerate(inv):
        base = np.float32(1.0) / np.power(np.float32(500000.0), np.float32(2 * i) / np.float32(128.0))
        wl = np.float32(2 * math.pi) / base
        if wl < orig_ctx / 4:
            exp = base
        elif wl > orig_ctx:
            exp = base / 8
        else:
            sm = (orig_ctx / wl - 1) / 3
            exp = (1 - sm) * (base / 8) + sm * base
        assert abs(actual - exp) < 1e-6


def test_per_dimension_factors(oracle):
    # lib.rs:635-650: rope.scaling.factors = [1.5, 2.5] become LongRoPE tables
    inv = oracle.fill_inv_freq(4, 10000.0, 16, kind=3, orig=8192, short=[1.5, 2.5], long=[1.5, 2.5])
    assert abs(inv[0] - 1.0 / 1.5) < 1e-6
    assert abs(inv[1] - (1.0 / 10000.0 ** 0.5) / 2.5) < 1e-6


@pytest.mark.parametrize("rows,last_val,expect_last", [(128_256, 2.0, 32.0), (128_005, 3.0, 48.0)])
def test_lm_head_row_split_closed_forms(oracle, rows, last_val, expect_last):
    # lib.rs:107-158: F32 head, cols 16, hidden = ones
    cols = 16
    w = np.zeros((rows, cols), dtype=np.float32)
    if last_val == 2.0:
        w[0, :] = 1.0
    w[rows - 1, :] = last_val
    out = oracle.gemv_decode_projection(w.view(np.uint8).ravel(), 0, rows, cols, np.ones(cols, np.float32), 4)
    if last_val == 2.0:
        assert abs(out[0] - 16.0) < 1e-4 and abs(out[100]) < 1e-4
    assert abs(out[rows - 1] - expect_last) < 1e-4


ADMITTED = [0, 1, 30, 8, 2, 6, 12, 13, 14]


@pytest.mark.parametrize("quant", ADMITTED)
def test_wave2_repacked_gemm_vs_compute_row_dot(oracle, quant):
    # tests/repack_wave2_parity.rs:182-236 (rows 73, cols 256, m 3)
    rows, cols, m = 73, 256, 3
    act = fx.wave2_activation(m, cols)
    seed = ADMITTED.index(quant) + 1
    raw = fx.fill_quant_bytes(rows, cols, quant, seed)
    w = oracle.RepackedWeight(raw, quant, rows, cols)
    out = w.project_batch(act, m)
    tol = 1e-5 if quant in (0, 1, 30) else 1e-2
    for t in range(m):
        x = act[t * cols:(t + 1) * cols]
        bound = max(float(np.sqrt(np.sum(x * x))) * math.sqrt(cols), 1.0)
        for r in range(rows):
            exp = oracle.compute_row_dot(r, cols, quant, raw, x)
            assert abs(out[t, r] - exp) / max(bound, abs(exp)) < tol


@pytest.mark.parametrize("quant", ADMITTED)
def test_wave3_batched_projection_vs_compute_row_dot(oracle, quant):
    # tests/batched_prefill_wave3.rs:327-396: 192 rows (three 64-row panels)
    # x 256 columns of the wave-3 fill family, M = 1, 8, 32 activation rows
    # ((((23 i + 11 M) % 79) - 39) * 0.025), each output within 1e-5 (dense)
    # or 1.5e-2 (quantized) of compute_row_dot relative to
    # max(|x|_2 sqrt(cols), 1, |expected|).
    rows, cols = 192, 256
    raw = fx.fill_quant_bytes(rows, cols, quant, ADMITTED.index(quant) + 3, fx.WAVE3)
    w = oracle.RepackedWeight(raw, quant, rows, cols)
    tol = 1e-5 if quant in (0, 1, 30) else 1.5e-2
    for m in (1, 8, 32):
        i = np.arange(m * cols, dtype=np.int64)
        act = (((i * 23 + m * 11) % 79).astype(np.float32) - np.float32(39.0)) * np.float32(0.025)
        out = w.project_batch(act, m)
        assert np.array_equal(out, np.stack([w.project_batch(act[t * cols:(t + 1) * cols], 1)[0] for t in range(m)]))
        for t in range(m):
            x = act[t * cols:(t + 1) * cols]
            scale = max(float(np.sqrt(np.sum(x * x))) * math.sqrt(cols), 1.0)
            for r in range(rows):
                exp = oracle.compute_row_dot(r, cols, quant, raw, x)
                assert abs(out[t, r] - exp) / max(scale, abs(exp)) < tol


def test_repack_layout_q4_0_matches_definition(oracle):
    # repack_quantized (repack_cache.rs:639-694): byte (r%8)*16+t of tile
    # (r/8)*k_chunks + ch holds q[r][ch*16+t]; scales[((r/8)*groups+g)*8+r%8].
    rows, cols = 13, 64
    raw = fx.fill_q4_0_or_q5_0(rows, cols, 2, 3)
    w = oracle.RepackedWeight(raw, 2, rows, cols)
    tiles, scales = w.tiles(), w.scales()
    kc, groups = cols // 16, cols // 32
    for r in range(16):
        for g in range(groups):
            blk = raw[(r * groups + g) * 18:(r * groups + g) * 18 + 18] if r < rows else None
            sc = scales[((r // 8) * groups + g) * 8 + r % 8]
            if blk is None:
                assert sc == 0.0
                continue
            assert sc == oracle.f16_to_f32_finite(int(blk[0]) | (int(blk[1]) << 8))
            b = [int(v) for v in blk[2:18]]
            q = [(b[i] & 15) - 8 for i in range(16)] + [(b[i] >> 4) - 8 for i in range(16)]
            for e in range(32):
                ch, t = (g * 32 + e) // 16, (g * 32 + e) % 16
                assert tiles[((r // 8) * kc + ch) * 128 + (r % 8) * 16 + t] == q[e]


def test_projection_is_independent_of_thread_count(oracle):
    # tests/wave4_zero_alloc_decode_gemv.rs:548-623 (bit-identical across workers)
    rows, cols = 300, 512
    raw = fx.fill_q4_0_or_q5_0(rows, cols, 2, 5)
    act = fx.wave2_activation(2, cols)
    w = oracle.RepackedWeight(raw, 2, rows, cols)
    a = w.project_batch(act, 2, nthreads=1)
    b = w.project_batch(act, 2, nthreads=4)
    assert np.array_equal(a, b)
    g1 = oracle.gemv_decode_projection(raw, 2, rows, cols, act[:cols], 1)
    g4 = oracle.gemv_decode_projection(raw, 2, rows, cols, act[:cols], 4)
    assert np.array_equal(g1, g4)


def test_gemv_equals_gemm_row0(oracle):
    # tests/authentic_gguf_forward.rs:435-442 (GEMV == GEMM row 0)
    rows, cols = 133, 256
    raw = fx.fill_q8_0(rows, cols, 2)
    act = fx.wave2_activation(5, cols)
    w = oracle.RepackedWeight(raw, 8, rows, cols)
    gemm = w.project_batch(act, 5)
    gemv = w.project_batch(act[:cols], 1)
    assert np.array_equal(gemm[0], gemv[0])


def test_act_quantizer_semantics(oracle):
    # quantize_single_row_slices (repack_cache.rs:390-422)
    x = np.array([0.5, -1.0, 0.25, float("nan"), float("inf")] + [0.0] * 27 + [3.0] * 10, dtype=np.float32)
    q, s = oracle.quantize_act_rows(x, 1, x.size)
    assert q.shape == (1, 64) and s.shape == (1, 2)
    scale = np.float32(1.0) / np.float32(127.0)
    assert s[0, 0] == scale
    inv = np.float32(1.0) / scale
    assert q[0, 0] == int(np.round(np.float32(0.5) * inv)) and q[0, 1] == -127
    assert q[0, 3] == 0 and q[0, 4] == 0  # non-finite -> 0
    assert s[0, 1] == np.float32(3.0) / np.float32(127.0) and q[0, 32] == 127 and q[0, 42] == 0


@pytest.mark.parametrize("quant", [2, 12, 13, 14, 8])
def test_wave4_streaming_gemv_workers_1_4_8(oracle, quant):
    # tests/wave4_zero_alloc_decode_gemv.rs:548-623: gemv_decode_projection
    # of a 64 x 256 matrix (wave-4 fill, seed 9) with 1, 4 and 8 workers is
    # bit-identical, each row within 0.05 + 1% of compute_row_dot.
    rows, cols = 64, 256
    raw = fx.wave4_fill_tensor(rows, cols, quant, 9)
    i = np.arange(cols, dtype=np.int64)
    x = (((i * 7 + 3) % 19).astype(np.float32) - np.float32(9.0)) * np.float32(0.05)
    outs = [oracle.gemv_decode_projection(raw, quant, rows, cols, x, nthreads=t) for t in (1, 4, 8)]
    assert np.array_equal(outs[0], outs[1]) and np.array_equal(outs[0], outs[2])
    for r in range(rows):
        exp = oracle.compute_row_dot(r, cols, quant, raw, x)
        assert np.isfinite(outs[0][r]) and abs(outs[0][r] - exp) < 0.05 + abs(exp) * 0.01


def test_wave4_152k_vocab_gemv_determinism(oracle):
    # tests/wave4_zero_alloc_decode_gemv.rs:625-683: a 151936 x 256 Q4_0 head,
    # zero except rows 0, 75968 and the last (wave-4 fill, seed row + 1),
    # against a 0.125 activation: the streaming GEMV with 1, 4 and 8 workers
    # agrees bit for bit, and the repacked projection (its own activation
    # quantizer) is zero on exactly the same rows.
    rows, cols, rb = 151_936, 256, 256 // 32 * 18
    raw = np.zeros(rows * rb, dtype=np.uint8)
    for r in (0, 75_968, rows - 1):
        raw[r * rb:(r + 1) * rb] = fx.wave4_fill_tensor(1, cols, 2, r + 1)
    x = np.full(cols, 0.125, dtype=np.float32)
    outs = [oracle.gemv_decode_projection(raw, 2, rows, cols, x, nthreads=t) for t in (1, 4, 8)]
    assert np.array_equal(outs[0], outs[1]) and np.array_equal(outs[0], outs[2])
    rep = oracle.RepackedWeight(raw, 2, rows, cols).project_batch(x, 1, nthreads=8)[0]
    nz = [0, 75_968, rows - 1]
    assert np.all(outs[0][1:75_968] == 0.0) and np.all(outs[0][nz] != 0.0)
    assert np.array_equal(rep == 0.0, outs[0] == 0.0)


def _cos(a, b):
    a, b = np.asarray(a, np.float64), np.asarray(b, np.float64)
    return float(np.dot(a, b) / max(np.linalg.norm(a) * np.linalg.norm(b), 1e-12))


@pytest.mark.parametrize("quant", ADMITTED)
def test_authentic_repacked_gemv_and_gemm_parity(oracle, quant):
    # tests/authentic_gguf_forward.rs:370-468: 133 rows (panels of 64 + 64 + 5,
    # not a multiple of 8) x 256 columns of the realistic fills, M = 1 and 5
    # activation rows ((((23 i + 5) % 101) - 50) * 0.03): each output within
    # 1e-5 (dense) / 1e-2 (quantized) of compute_row_dot relative to
    # max(|x|_2 sqrt(cols), |expected|, 1), cosine > 0.9998 per token, and the
    # M = 1 projection equal to the first row of the M = 5 one within 1e-5.
    rows, cols, m = 133, 256, 5
    raw = fx.authentic_matrix_bytes(rows, cols, quant, ADMITTED.index(quant) + 10)
    w = oracle.RepackedWeight(raw, quant, rows, cols)
    i = np.arange(m * cols, dtype=np.int64)
    act = (((i * 23 + 5) % 101).astype(np.float32) - np.float32(50.0)) * np.float32(0.03)
    tol = 1e-5 if quant in (0, 1, 30) else 1e-2
    single = w.project_batch(act[:cols], 1)[0]
    batched = w.project_batch(act, m)
    assert np.all(np.abs(single - batched[0]) < 1e-5)
    for t in range(m):
        x = act[t * cols:(t + 1) * cols]
        ref = np.array([oracle.compute_row_dot(r, cols, quant, raw, x) for r in range(rows)], dtype=np.float32)
        bound = np.maximum(max(float(np.linalg.norm(x)) * math.sqrt(cols), 1.0), np.abs(ref))
        assert np.all(np.abs(batched[t] - ref) / bound < tol)
        assert _cos(batched[t], ref) > 0.9998


def test_authentic_q4_k_head_rows_identical_across_threads(oracle):
    # tests/authentic_gguf_forward.rs:743-761: a 263 x 256 Q4_K_M head
    # (seed 77) against a 0.25 activation, 1 vs 4 threads, bit-identical.
    raw = fx.authentic_matrix_bytes(263, 256, 12, 77)
    x = np.full(256, 0.25, dtype=np.float32)
    w = oracle.RepackedWeight(raw, 12, 263, 256)
    assert np.array_equal(w.project_batch(x, 1, nthreads=1), w.project_batch(x, 1, nthreads=4))
    assert np.array_equal(oracle.gemv_decode_projection(raw, 12, 263, 256, x, nthreads=1),
                          oracle.gemv_decode_projection(raw, 12, 263, 256, x, nthreads=4))
