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


def fill_dense_f32(rows, cols, seed):
    """tests/repack_wave2_parity.rs:46-58."""
    idx = np.arange(rows * cols, dtype=np.int64)
    val = (((idx * 19 + seed) % 97).astype(np.float32) - f32(48.0)) * f32(0.025)
    return val.astype("<f4").view(np.uint8).copy()


def fill_dense_half(rows, cols, quant, seed):
    """tests/repack_wave2_parity.rs:60-82 (quant 1 = F16, 30 = BF16)."""
    mul, mod, off = (17, 67, 33.0) if quant == 1 else (23, 73, 36.0)
    out = np.zeros(rows * cols, dtype=np.uint16)
    for i in range(rows * cols):
        v = (f32((i * mul + seed) % mod) - f32(off)) * f32(0.03)
        out[i] = f32_to_f16_bits_trunc(v) if quant == 1 else f32_to_bf16_bits(v)
    return out.view(np.uint8).copy()


def fill_q8_0(rows, cols, seed):
    """tests/repack_wave2_parity.rs:84-98."""
    blocks = rows * cols // 32
    out = np.zeros(blocks * 34, dtype=np.uint8)
    for b in range(blocks):
        o = b * 34
        d = f32(0.015) + f32((b + seed) % 7) * f32(0.004)
        out[o:o + 2] = np.frombuffer(struct.pack("<H", f32_to_f16_bits_trunc(d)), dtype=np.uint8)
        k = np.arange(32)
        signed = ((b * 11 + k * 7 + seed) % 81) - 40
        out[o + 2:o + 34] = signed.astype(np.int8).view(np.uint8)
    return out


def fill_q4_0_or_q5_0(rows, cols, quant, seed):
    """tests/repack_wave2_parity.rs:100-123 (quant 2 = Q4_0, 6 = Q5_0)."""
    blocks = rows * cols // 32
    bb = 18 if quant == 2 else 22
    out = np.zeros(blocks * bb, dtype=np.uint8)
    d = f32(0.05) if quant == 2 else f32(0.04)
    dh = struct.pack("<H", f32_to_f16_bits_trunc(d))
    for b in range(blocks):
        o = b * bb
        out[o:o + 2] = np.frombuffer(dh, dtype=np.uint8)
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


def fill_k_quant(rows, cols, quant, seed):
    """tests/repack_wave2_parity.rs:125-166 (12 = Q4_K_M, 13 = Q5_K, 14 = Q6_K)."""
    sblks = rows * cols // 256
    bb = {12: 144, 13: 176, 14: 210}[quant]
    out = np.zeros(sblks * bb, dtype=np.uint8)
    for sb in range(sblks):
        o = sb * bb
        if quant in (12, 13):
            out[o:o + 2] = np.frombuffer(struct.pack("<H", f32_to_f16_bits_trunc(0.02)), dtype=np.uint8)
            out[o + 2:o + 4] = np.frombuffer(struct.pack("<H", f32_to_f16_bits_trunc(0.006)), dtype=np.uint8)
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
            out[o + 208:o + 210] = np.frombuffer(struct.pack("<H", f32_to_f16_bits_trunc(0.015)), dtype=np.uint8)
            for l_ in range(128):
                out[o + l_] = (sb * 7 + l_ * 3 + seed) % 256
            for l_ in range(64):
                out[o + 128 + l_] = (sb * 11 + l_ * 5 + seed) % 256
            for l_ in range(16):
                out[o + 192 + l_] = np.int8(((sb + l_ * 3 + seed) % 21) - 10).view(np.uint8)
    return out


def fill_quant_bytes(rows, cols, quant, seed):
    """tests/repack_wave2_parity.rs:168-180."""
    if quant == 0:
        return fill_dense_f32(rows, cols, seed)
    if quant in (1, 30):
        return fill_dense_half(rows, cols, quant, seed)
    if quant == 8:
        return fill_q8_0(rows, cols, seed)
    if quant in (2, 6):
        return fill_q4_0_or_q5_0(rows, cols, quant, seed)
    return fill_k_quant(rows, cols, quant, seed)


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
