"""Deterministic fixtures of the reference crate's own tests, restated.

Each generator follows the reference test helper it names (file:line in the
reference crate) so the known-answer and parity cases run on the same bytes
here.  All f32 arithmetic is done in numpy float32 like the Rust code.
"""
import struct

import numpy as np

f32 = np.float32


def f32_to_f16_bits_trunc(val):
    """tests/repack_wave2_parity.rs:20-41 (truncating f32 -> f16 used by the fixtures)."""
    bits = struct.unpack("<I", struct.pack("<f", float(f32(val))))[0]
    sign = (bits >> 16) & 0x8000
    exp = (bits >> 23) & 0xFF
    mant = bits & 0x7FFFFF
    if exp == 0:
        return sign
    if exp == 0xFF:
        return sign | 0x7C00
    h_exp = exp - 127 + 15
    if h_exp >= 31:
        return sign | 0x7BFF
    if h_exp <= 0:
        return sign
    return sign | (h_exp << 10) | (mant >> 13)


def f32_to_bf16_bits(val):
    """tests/repack_wave2_parity.rs:43-45."""
    return struct.unpack("<I", struct.pack("<f", float(f32(val))))[0] >> 16


# The reference's two families of fill generators differ only in these
# constants: tests/repack_wave2_parity.rs:46-180 (WAVE2) and
# tests/batched_prefill_wave3.rs:45-179 (WAVE3).
WAVE2 = dict(f32_step=0.025, half_step=0.03, q4_d=0.05, q5_d=0.04, k_d=0.02, k_dmin=0.006, q6k_d=0.015)
WAVE3 = dict(f32_step=0.02, half_step=0.025, q4_d=0.04, q5_d=0.03, k_d=0.015, k_dmin=0.004, q6k_d=0.012)


def _f16le(v):
    return np.frombuffer(struct.pack("<H", f32_to_f16_bits_trunc(v)), dtype=np.uint8)


def fill_dense_f32(rows, cols, seed, c=WAVE2):
    """tests/repack_wave2_parity.rs:46-58, batched_prefill_wave3.rs:45-56."""
    idx = np.arange(rows * cols, dtype=np.int64)
    val = (((idx * 19 + seed) % 97).astype(np.float32) - f32(48.0)) * f32(c["f32_step"])
    return val.astype("<f4").view(np.uint8).copy()


def fill_dense_half(rows, cols, quant, seed, c=WAVE2):
    """tests/repack_wave2_parity.rs:60-82, batched_prefill_wave3.rs:58-79
    (quant 1 = F16, 30 = BF16)."""
    mul, mod, off = (17, 67, 33.0) if quant == 1 else (23, 73, 36.0)
    out = np.zeros(rows * cols, dtype=np.uint16)
    for i in range(rows * cols):
        v = (f32((i * mul + seed) % mod) - f32(off)) * f32(c["half_step"])
        out[i] = f32_to_f16_bits_trunc(v) if quant == 1 else f32_to_bf16_bits(v)
    return out.view(np.uint8).copy()


def fill_q8_0(rows, cols, seed, c=WAVE2):
    """tests/repack_wave2_parity.rs:84-98, batched_prefill_wave3.rs:81-95
    (the same in both)."""
    blocks = rows * cols // 32
    out = np.zeros(blocks * 34, dtype=np.uint8)
    for b in range(blocks):
        o = b * 34
        d = f32(0.015) + f32((b + seed) % 7) * f32(0.004)
        out[o:o + 2] = _f16le(d)
        k = np.arange(32)
        signed = ((b * 11 + k * 7 + seed) % 81) - 40
        out[o + 2:o + 34] = signed.astype(np.int8).view(np.uint8)
    return out


def fill_q4_0_or_q5_0(rows, cols, quant, seed, c=WAVE2):
    """tests/repack_wave2_parity.rs:100-123, batched_prefill_wave3.rs:97-120
    (quant 2 = Q4_0, 6 = Q5_0)."""
    blocks = rows * cols // 32
    bb = 18 if quant == 2 else 22
    out = np.zeros(blocks * bb, dtype=np.uint8)
    dh = _f16le(f32(c["q4_d"]) if quant == 2 else f32(c["q5_d"]))
    for b in range(blocks):
        o = b * bb
        out[o:o + 2] = dh
        qs = o + 2
        if quant == 6:
            qh = (0x5A3C96F1 + b * 13) & 0xFFFFFFFF
            out[o + 2:o + 6] = np.frombuffer(struct.pack("<I", qh), dtype=np.uint8)
            qs = o + 6
        i = np.arange(16)
        lo = (b * 5 + i + seed) % 16
        hi = (b * 3 + i * 3 + seed) % 16
        out[qs:qs + 16] = (lo | (hi << 4)).astype(np.uint8)
    return out


def fill_k_quant(rows, cols, quant, seed, c=WAVE2):
    """tests/repack_wave2_parity.rs:125-166, batched_prefill_wave3.rs:122-166
    (12 = Q4_K_M, 13 = Q5_K, 14 = Q6_K)."""
    sblks = rows * cols // 256
    bb = {12: 144, 13: 176, 14: 210}[quant]
    out = np.zeros(sblks * bb, dtype=np.uint8)
    for sb in range(sblks):
        o = sb * bb
        if quant in (12, 13):
            out[o:o + 2] = _f16le(c["k_d"])
            out[o + 2:o + 4] = _f16le(c["k_dmin"])
            for j in range(12):
                out[o + 4 + j] = (sb * 7 + j * 11 + seed) % 64 + 1
            qs = o + 16
            if quant == 13:
                for l_ in range(32):
                    out[o + 16 + l_] = (sb + l_ * 13 + seed) % 256
                qs = o + 48
            for l_ in range(128):
                out[qs + l_] = ((sb * 2 + l_ + seed) % 16) | (((sb * 5 + l_ + seed) % 16) << 4)
        else:
            out[o + 208:o + 210] = _f16le(c["q6k_d"])
            for l_ in range(128):
                out[o + l_] = (sb * 7 + l_ * 3 + seed) % 256
            for l_ in range(64):
                out[o + 128 + l_] = (sb * 11 + l_ * 5 + seed) % 256
            for l_ in range(16):
                out[o + 192 + l_] = np.int8(((sb + l_ * 3 + seed) % 21) - 10).view(np.uint8)
    return out


def fill_quant_bytes(rows, cols, quant, seed, c=WAVE2):
    """tests/repack_wave2_parity.rs:168-180, batched_prefill_wave3.rs:168-179."""
    if quant == 0:
        return fill_dense_f32(rows, cols, seed, c)
    if quant in (1, 30):
        return fill_dense_half(rows, cols, quant, seed, c)
    if quant == 8:
        return fill_q8_0(rows, cols, seed, c)
    if quant in (2, 6):
        return fill_q4_0_or_q5_0(rows, cols, quant, seed, c)
    return fill_k_quant(rows, cols, quant, seed, c)


def wave2_activation(m, cols):
    """tests/repack_wave2_parity.rs:186-195."""
    i = np.arange(m * cols, dtype=np.int64)
    return (((i * 29 + 7) % 89).astype(np.float32) - f32(44.0)) * f32(0.02)


def q5_0_known_block():
    """lib.rs:657-665: d = 0x3800, qh = 0xA55A5AA5, nibbles (j*3+1, j*5+2)."""
    b = np.zeros(22, dtype=np.uint8)
    b[0:2] = np.frombuffer(struct.pack("<H", 0x3800), dtype=np.uint8)
    b[2:6] = np.frombuffer(struct.pack("<I", 0xA55A5AA5), dtype=np.uint8)
    for j in range(16):
        b[6 + j] = ((j * 3 + 1) & 0x0F) | (((j * 5 + 2) & 0x0F) << 4)
    return b


def q5_k_known_block():
    """lib.rs:718-738."""
    k = np.zeros(176, dtype=np.uint8)
    k[0:2] = np.frombuffer(struct.pack("<H", 0x3400), dtype=np.uint8)
    k[2:4] = np.frombuffer(struct.pack("<H", 0x2E00), dtype=np.uint8)
    for i in range(12):
        k[4 + i] = (i * 7 + 3) % 60 + 1
    for i in range(32):
        k[16 + i] = (i * 29 + 11) & 0xFF
    for i in range(128):
        k[48 + i] = ((i * 3 + 1) & 0x0F) | (((i * 7 + 2) & 0x0F) << 4)
    return k


def q4_k_m_two_rows():
    """dispatch.rs:298-327."""
    raw = np.zeros(2 * 144, dtype=np.uint8)
    raw[0:2] = np.frombuffer(struct.pack("<H", 0x3800), dtype=np.uint8)
    raw[2:4] = np.frombuffer(struct.pack("<H", 0x3400), dtype=np.uint8)
    raw[4:16] = [0x95, 0xA6, 0x57, 0x68, 0x83, 0x44, 0xC5, 0x06, 0x37, 0x48, 0x59, 0x6A]
    for i in range(128):
        raw[16 + i] = ((i * 7 + 3) & 0x0F) | (((i * 5 + 9) & 0x0F) << 4)
    raw[144:146] = np.frombuffer(struct.pack("<H", 0x3C00), dtype=np.uint8)
    raw[146:148] = np.frombuffer(struct.pack("<H", 0x3800), dtype=np.uint8)
    raw[148:160] = [3, 5, 7, 9, 2, 4, 6, 8, 0x21, 0x43, 0x65, 0x87]
    for i in range(128):
        raw[160 + i] = ((i * 11 + 1) & 0x0F) | (((i * 3 + 12) & 0x0F) << 4)
    return raw


def wave3_model_gguf(arch, weight_quant, hidden=256):
    """The two-layer mixed-type model of tests/batched_prefill_wave3.rs:215-310
    (build_wave3_test_gguf + write_finite_gguf_payloads, :181-213): hidden =
    ffn, 4 query / 2 KV heads of hidden / 4 dims, vocab 64, context 64.
    Layer 0 holds q / o / gate / up / down in `weight_quant` (k, v Q8_0),
    layer 1 Q8_0 / Q4_0 / Q5_0 projections with `weight_quant` down; norms in
    F16 (llama) or BF16 (qwen2) except ffn_norm of layer 0 and the output
    norm (F32); an F32 LM head; qwen2 adds F16 / F32 / BF16 Q/K/V and O
    biases.  Payloads: tensor i (in file order) of two dims gets
    fill_quant_bytes(rows, cols, quant, i + 1) with the WAVE3 constants; a
    norm gets 0.85 + ((e + i) % 13) * 0.02, a bias
    (((7 e + 11 i) % 29) - 14) * 0.04, in f32 arithmetic."""
    import gguf_py

    n_q, n_kv, vocab = 4, 2, 64
    hd = hidden // n_q
    kvd = n_kv * hd
    norm_q = 30 if arch == "qwen2" else 1
    wq = weight_quant
    specs = [("token_embd.weight", 8, [hidden, vocab]),
             ("blk.0.attn_norm.weight", norm_q, [hidden]),
             ("blk.0.attn_q.weight", wq, [hidden, hidden]),
             ("blk.0.attn_k.weight", 8, [hidden, kvd]),
             ("blk.0.attn_v.weight", 8, [hidden, kvd]),
             ("blk.0.attn_output.weight", wq, [hidden, hidden]),
             ("blk.0.ffn_norm.weight", 0, [hidden]),
             ("blk.0.ffn_gate.weight", wq, [hidden, hidden]),
             ("blk.0.ffn_up.weight", wq, [hidden, hidden]),
             ("blk.0.ffn_down.weight", wq, [hidden, hidden]),
             ("blk.1.attn_norm.weight", norm_q, [hidden]),
             ("blk.1.attn_q.weight", 8, [hidden, hidden]),
             ("blk.1.attn_k.weight", 2, [hidden, kvd]),
             ("blk.1.attn_v.weight", 6, [hidden, kvd]),
             ("blk.1.attn_output.weight", 8, [hidden, hidden]),
             ("blk.1.ffn_norm.weight", norm_q, [hidden]),
             ("blk.1.ffn_gate.weight", 2, [hidden, hidden]),
             ("blk.1.ffn_up.weight", 6, [hidden, hidden]),
             ("blk.1.ffn_down.weight", wq, [hidden, hidden]),
             ("output_norm.weight", 0, [hidden]),
             ("output.weight", 0, [hidden, vocab])]
    if arch == "qwen2":
        specs += [("blk.0.attn_q.bias", 1, [hidden]), ("blk.0.attn_k.bias", 0, [kvd]),
                  ("blk.0.attn_v.bias", 30, [kvd]), ("blk.0.attn_output.bias", 0, [hidden]),
                  ("blk.1.attn_q.bias", 0, [hidden]), ("blk.1.attn_k.bias", 1, [kvd]),
                  ("blk.1.attn_v.bias", 0, [kvd])]
    tensors = []
    for i, (name, q, dims) in enumerate(specs):
        if len(dims) == 2:
            payload = fill_quant_bytes(dims[1], dims[0], q, i + 1, WAVE3)
        else:
            e = np.arange(dims[0], dtype=np.int64)
            if name.endswith("norm.weight"):
                v = f32(0.85) + ((e + i) % 13).astype(np.float32) * f32(0.02)
            else:
                v = (((e * 7 + i * 11) % 29).astype(np.float32) - f32(14.0)) * f32(0.04)
            if q == 0:
                payload = v.astype("<f4").view(np.uint8)
            elif q == 1:
                payload = np.array([f32_to_f16_bits_trunc(x) for x in v], dtype="<u2").view(np.uint8)
            else:
                payload = np.array([f32_to_bf16_bits(x) for x in v], dtype="<u2").view(np.uint8)
        tensors.append((name, q, dims, payload))
    kvs = [("general.architecture", arch), ("general.alignment", 32), (f"{arch}.block_count", 2),
           (f"{arch}.embedding_length", hidden), (f"{arch}.feed_forward_length", hidden),
           (f"{arch}.attention.head_count", n_q), (f"{arch}.attention.head_count_kv", n_kv),
           (f"{arch}.attention.key_length", hd), (f"{arch}.rope.freq_base", 10000.0),
           (f"{arch}.attention.layer_norm_rms_epsilon", 1e-5), (f"{arch}.context_length", 64)]
    return gguf_py.write(kvs, tensors)


def wave4_fill_tensor(rows, cols, quant, seed):
    """tests/wave4_zero_alloc_decode_gemv.rs:123-246 (fill_quantized_row /
    fill_quantized_tensor_bytes): per-row patterns of r, the block index and
    the seed; quantized blocks carry the f16 scale 2^-5 (and min 2^-7)."""
    sc, mn = struct.pack("<H", 0x2800), struct.pack("<H", 0x2000)  # 0.03125, 0.0078125
    rows_out = []
    for r in range(rows):
        c = np.arange(cols, dtype=np.int64)
        if quant == 0:
            v = (((r * 13 + c * 7 + seed) % 23).astype(np.float32) - f32(11.0)) * f32(0.02)
            rows_out.append(v.astype("<f4").view(np.uint8))
            continue
        if quant == 1:
            v = (((r * 11 + c * 5 + seed) % 19).astype(np.float32) - f32(9.0)) * f32(0.025)
            rows_out.append(np.array([f32_to_f16_bits_trunc(x) for x in v], dtype="<u2").view(np.uint8))
            continue
        if quant == 30:
            v = (((r * 17 + c * 3 + seed) % 17).astype(np.float32) - f32(8.0)) * f32(0.025)
            rows_out.append(np.array([f32_to_bf16_bits(x) for x in v], dtype="<u2").view(np.uint8))
            continue
        out = bytearray()
        nb = cols // (256 if quant in (12, 13, 14) else 32)
        for b in range(nb):
            if quant in (2, 6):
                blk = bytearray(sc)
                if quant == 6:
                    blk += struct.pack("<I", 0x55AA55AA)
                blk += bytes((((r + b + j + seed) % 15) | (((r + b + 2 * j + seed) % 15) << 4)) for j in range(16))
            elif quant == 8:
                blk = bytearray(sc) + bytes(np.array([((r + b * 3 + j + seed) % 29) - 14 for j in range(32)],
                                                     dtype=np.int8).view(np.uint8))
            elif quant == 12:
                blk = bytearray(sc) + mn + bytes([0x21] * 12)
                blk += bytes((((r + b + j + seed) % 15) | (((r + 2 * b + 3 * j + seed) % 15) << 4)) for j in range(128))
            elif quant == 13:
                blk = bytearray(sc) + mn + bytes([0x18] * 12) + bytes([0x33] * 32)
                blk += bytes((((r + b + j + seed) % 15) | (((r + b + 3 * j + seed) % 15) << 4)) for j in range(128))
            else:  # 14, Q6_K
                blk = bytearray(((r + b + j * 5 + seed) & 0x77) for j in range(128))
                blk += bytes([0x55] * 64) + bytes([0x03] * 16) + sc
            out += blk
        rows_out.append(np.frombuffer(bytes(out), dtype=np.uint8))
    return np.concatenate(rows_out)


def wave4_model_gguf(arch, quant, hidden=256, ffn=256, n_q=4, n_kv=2, head_dim=64, vocab=16):
    """The one-layer single-quant model of
    tests/wave4_zero_alloc_decode_gemv.rs:248-363 (build_synthetic_quant_gguf):
    every matrix, the embedding and the head in `quant`, F32 norms
    (0.9 + (i % 5) * 0.02) and, for qwen2, F32 Q/K/V biases
    (((i % 7) - 3) * 0.01); matrix i (in file order) filled by
    wave4_fill_tensor(rows, cols, quant, i + 1); context length 16."""
    import gguf_py

    Q, KV = n_q * head_dim, n_kv * head_dim
    specs = [("token_embd.weight", quant, [hidden, vocab]), ("blk.0.attn_norm.weight", 0, [hidden]),
             ("blk.0.attn_q.weight", quant, [hidden, Q]), ("blk.0.attn_k.weight", quant, [hidden, KV]),
             ("blk.0.attn_v.weight", quant, [hidden, KV]), ("blk.0.attn_output.weight", quant, [Q, hidden]),
             ("blk.0.ffn_norm.weight", 0, [hidden]), ("blk.0.ffn_gate.weight", quant, [hidden, ffn]),
             ("blk.0.ffn_up.weight", quant, [hidden, ffn]), ("blk.0.ffn_down.weight", quant, [ffn, hidden]),
             ("output_norm.weight", 0, [hidden]), ("output.weight", quant, [hidden, vocab])]
    if arch == "qwen2":
        specs += [("blk.0.attn_q.bias", 0, [Q]), ("blk.0.attn_k.bias", 0, [KV]), ("blk.0.attn_v.bias", 0, [KV])]
    tensors = []
    for i, (name, q, dims) in enumerate(specs):
        if q == 0 and len(dims) == 1:
            e = np.arange(dims[0], dtype=np.int64)
            if "norm" in name:
                v = f32(0.9) + (e % 5).astype(np.float32) * f32(0.02)
            else:
                v = ((e % 7).astype(np.float32) - f32(3.0)) * f32(0.01)
            payload = v.astype("<f4").view(np.uint8)
        else:
            payload = wave4_fill_tensor(dims[1] if len(dims) > 1 else 1, dims[0], q, i + 1)
        tensors.append((name, q, dims, payload))
    kvs = [("general.architecture", arch), ("general.alignment", 32), (f"{arch}.block_count", 1),
           (f"{arch}.embedding_length", hidden), (f"{arch}.feed_forward_length", ffn),
           (f"{arch}.attention.head_count", n_q), (f"{arch}.attention.head_count_kv", n_kv),
           (f"{arch}.attention.key_length", head_dim), (f"{arch}.attention.layer_norm_rms_epsilon", 1e-5),
           (f"{arch}.rope.freq_base", 10000.0), (f"{arch}.context_length", 16)]
    return gguf_py.write(kvs, tensors)


def authentic_matrix_bytes(rows, cols, quant, seed):
    """tests/authentic_gguf_forward.rs:40-234 (build_realistic_matrix_bytes):
    element or block patterns of the flat index and the seed with fixed f16
    scales per type."""
    n = rows * cols
    i = np.arange(n, dtype=np.int64)
    if quant == 0:
        return ((((i * 13 + seed * 7) % 97).astype(np.float32) - f32(48.0)) * f32(0.015)).astype("<f4").view(np.uint8)
    if quant == 1:
        v = (((i * 11 + seed * 5) % 89).astype(np.float32) - f32(44.0)) * f32(0.02)
        return np.array([f32_to_f16_bits_trunc(x) for x in v], dtype="<u2").view(np.uint8)
    if quant == 30:
        v = (((i * 17 + seed * 3) % 83).astype(np.float32) - f32(41.0)) * f32(0.02)
        return np.array([f32_to_bf16_bits(x) for x in v], dtype="<u2").view(np.uint8)
    out = bytearray()
    if quant in (8, 2, 6):
        d = _f16le({8: 0.025, 2: 0.125, 6: 0.0625}[quant]).tobytes()
        for b in range(n // 32):
            out += d
            if quant == 8:
                out += bytes(np.array([((b * 19 + k * 7 + seed) % 121) - 60 for k in range(32)],
                                      dtype=np.int8).view(np.uint8))
                continue
            if quant == 6:
                out += struct.pack("<I", ((b * 0x9E3779B9) ^ seed) & 0xFFFFFFFF)
            out += bytes((((b * 7 + k * 3 + seed) & 0x0F) | (((b * 11 + k * 5 + seed) & 0x0F) << 4)) for k in range(16))
        return np.frombuffer(bytes(out), dtype=np.uint8)
    for b in range(n // 256):
        if quant in (12, 13):
            out += _f16le(0.05 if quant == 12 else 0.04).tobytes() + _f16le(0.02 if quant == 12 else 0.015).tobytes()
            out += bytes(((b + s * 9 + seed) % 61) + 1 for s in range(12))
            if quant == 13:
                out += bytes(((b * 17 + h * 13 + seed) & 0xFF) for h in range(32))
            out += bytes((((b * 5 + q * 3 + seed) & 0x0F) | (((b * 13 + q * 7 + seed) & 0x0F) << 4)) for q in range(128))
        else:  # 14, Q6_K
            out += bytes(((b * 7 + k * 11 + seed) & 0xFF) for k in range(128))
            out += bytes(((b * 3 + k * 5 + seed) & 0xFF) for k in range(64))
            out += bytes(np.array([((b + s * 3 + seed) % 15) - 7 for s in range(16)], dtype=np.int8).view(np.uint8))
            out += _f16le(0.02).tobytes()
    return np.frombuffer(bytes(out), dtype=np.uint8)


def authentic_two_layer_gguf(arch, quant, with_biases, with_untied_output):
    """tests/authentic_gguf_forward.rs:236-358 (build_two_layer_gguf): two
    layers, hidden 256, FFN 512, 8 / 2 heads of 32 dims, vocab 67, theta 1e6
    and eps 1e-6 for qwen2 (5e5 / 1e-5 for llama), context 64; every matrix
    in `quant` (matrix i in file order filled by
    authentic_matrix_bytes(rows, cols, quant, i + 1)), F32 norms
    0.85 + (e % 13) * 0.02, optional F32 Q/K/V biases
    (((7 e + 11 i) % 29) - 14) * 0.08 and an optional untied output.weight."""
    import gguf_py

    hidden, ffn, n_q, n_kv, hd, vocab = 256, 512, 8, 2, 32, 67
    Q, KV = n_q * hd, n_kv * hd
    specs = [("token_embd.weight", quant, [hidden, vocab])]
    for l_ in range(2):
        b = f"blk.{l_}."
        specs += [(b + "attn_norm.weight", 0, [hidden]), (b + "attn_q.weight", quant, [hidden, Q]),
                  (b + "attn_k.weight", quant, [hidden, KV]), (b + "attn_v.weight", quant, [hidden, KV]),
                  (b + "attn_output.weight", quant, [Q, hidden]), (b + "ffn_norm.weight", 0, [hidden]),
                  (b + "ffn_gate.weight", quant, [hidden, ffn]), (b + "ffn_up.weight", quant, [hidden, ffn]),
                  (b + "ffn_down.weight", quant, [ffn, hidden])]
    specs.append(("output_norm.weight", 0, [hidden]))
    if with_biases:
        for l_ in range(2):
            specs += [(f"blk.{l_}.attn_q.bias", 0, [Q]), (f"blk.{l_}.attn_k.bias", 0, [KV]),
                      (f"blk.{l_}.attn_v.bias", 0, [KV])]
    if with_untied_output:
        specs.append(("output.weight", quant, [hidden, vocab]))
    tensors = []
    for i, (name, q, dims) in enumerate(specs):
        if len(dims) == 1:
            e = np.arange(dims[0], dtype=np.int64)
            if name.endswith("norm.weight"):
                v = f32(0.85) + (e % 13).astype(np.float32) * f32(0.02)
            else:
                v = (((e * 7 + i * 11) % 29).astype(np.float32) - f32(14.0)) * f32(0.08)
            payload = v.astype("<f4").view(np.uint8)
        else:
            payload = authentic_matrix_bytes(dims[1], dims[0], q, i + 1)
        tensors.append((name, q, dims, payload))
    qwen = arch == "qwen2"
    kvs = [("general.architecture", arch), ("general.alignment", 32), (f"{arch}.block_count", 2),
           (f"{arch}.embedding_length", hidden), (f"{arch}.feed_forward_length", ffn),
           (f"{arch}.attention.head_count", n_q), (f"{arch}.attention.head_count_kv", n_kv),
           (f"{arch}.attention.key_length", hd), (f"{arch}.rope.freq_base", 1e6 if qwen else 5e5),
           (f"{arch}.attention.layer_norm_rms_epsilon", 1e-6 if qwen else 1e-5), (f"{arch}.context_length", 64)]
    return gguf_py.write(kvs, tensors)
