"""ctypes binding of the CPU oracle (oracle/liboracle.so).

Test infrastructure only: the oracle is the checker the device path is
compared against; it is never part of the product path.
"""
import ctypes as C
import os

import numpy as np

_LIB = os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))), "oracle", "liboracle.so")
L = C.CDLL(_LIB)
_P, _SZ, _F, _I = C.c_void_p, C.c_size_t, C.c_float, C.c_int


class Repacked(C.Structure):
    _fields_ = [("rows", _SZ), ("cols", _SZ), ("quant", _I), ("dense", _I), ("blocks_per_row", _SZ),
                ("dense_data", _P), ("k_chunks", _SZ), ("chunks_per_scale", _SZ), ("scale_groups", _SZ),
                ("n_tiles", _SZ), ("tiles", _P), ("scales", _P), ("mins", _P)]


class RopeScaling(C.Structure):
    _fields_ = [("kind", _I), ("factor", _F), ("low_freq_factor", _F), ("high_freq_factor", _F),
                ("original_max_position_embeddings", _SZ), ("short_factor", _P), ("long_factor", _P),
                ("n_factors", _SZ)]


class Tensor(C.Structure):
    _fields_ = [("name", C.c_char_p), ("quant", _I), ("n_dims", _I), ("ne", C.c_uint64 * 4), ("data", _P),
                ("nbytes", _SZ)]


class Geometry(C.Structure):
    _fields_ = [("num_layers", _SZ), ("hidden_dim", _SZ), ("ffn_dim", _SZ), ("n_heads_q", _SZ),
                ("n_heads_kv", _SZ), ("head_dim", _SZ), ("rotary_dim", _SZ), ("vocab_size", _SZ),
                ("rms_eps", _F), ("rope_theta", _F), ("neox", _I), ("skip_rope_layers", _P),
                ("scaling", RopeScaling), ("sliding_window", _SZ), ("kv_f16", _I)]


class BlockQ8_0(C.Structure):
    _fields_ = [("d", _F), ("qs", C.c_int8 * 32)]


_sigs = {
    "or_f16_to_f32_finite": (_F, [C.c_uint16]),
    "or_bf16_to_f32_finite": (_F, [C.c_uint16]),
    "or_sanitize_f32_weight": (_F, [_F]),
    "or_dequantize_q4_0_block": (None, [_P, _P]),
    "or_dequantize_q5_0_block": (None, [_P, _P]),
    "or_dequantize_q8_0_block": (None, [_P, _P]),
    "or_dequantize_q4_k_block": (None, [_P, _P]),
    "or_dequantize_q5_k_block": (None, [_P, _P]),
    "or_dequantize_q6_k_block": (None, [_P, _P]),
    "or_repack": (_I, [_P, _SZ, _I, _SZ, _SZ, C.POINTER(Repacked)]),
    "or_repacked_free": (None, [C.POINTER(Repacked)]),
    "or_quantize_act_rows": (None, [_P, _SZ, _SZ, _P, _P, _P]),
    "or_project_batch": (_I, [C.POINTER(Repacked), _P, _P, _SZ, _I]),
    "or_dot16_partials": (None, [C.POINTER(Repacked), _P, _SZ, _SZ, _P]),
    "or_quantize_row_q8_0": (_I, [_P, _SZ, _P]),
    "or_gemv_decode_projection": (_I, [_P, _SZ, _I, _SZ, _SZ, _P, _P, _I]),
    "or_compute_row_dot": (_F, [_SZ, _SZ, _I, _P, _SZ, _P]),
    "or_rmsnorm_row": (_I, [_P, _P, _P, _SZ, _F]),
    "or_fill_inv_freq": (_I, [_SZ, _F, C.POINTER(RopeScaling), _SZ, _P]),
    "or_apply_rope": (_I, [_P, _SZ, _SZ, _SZ, _I, _SZ, _P]),
    "or_gqa_attention": (_I, [_P, _P, _P, _P, _SZ, _SZ, _SZ, _SZ, _SZ, _SZ, _SZ, _F, _P, _SZ]),
    "or_swiglu": (_I, [_P, _P, _P, _SZ]),
    "or_model_build": (_I, [C.POINTER(Geometry), _P, _SZ, _I, C.POINTER(_P)]),
    "or_model_free": (None, [_P]),
    "or_prefill": (_I, [_P, _P, _SZ, _P, _SZ, _SZ, _I, _P]),
    "or_decode": (_I, [_P, _P, _SZ, C.c_uint32, _SZ, _P]),
    "or_model_vocab": (_SZ, [_P]),
    "or_synth_matrix": (_I, [_I, _SZ, _SZ, C.c_uint64, C.c_char_p, _F, _P, _SZ, _I]),
    "or_f32_to_f16_rne": (C.c_uint16, [_F]),
}
for _n, (_r, _a) in _sigs.items():
    _fn = getattr(L, _n)
    _fn.restype = _r
    _fn.argtypes = _a


def ptr(a):
    return a.ctypes.data if a is not None else None


class OracleError(RuntimeError):
    pass


def check(rc):
    if rc != 0:
        raise OracleError(f"oracle status {rc}")


def f16_to_f32_finite(bits):
    return L.or_f16_to_f32_finite(bits)


def bf16_to_f32_finite(bits):
    return L.or_bf16_to_f32_finite(bits)


def sanitize_f32_weight(v):
    return L.or_sanitize_f32_weight(v)


def dequantize_block(quant, blk):
    blk = np.ascontiguousarray(blk, dtype=np.uint8)
    n = 32 if quant in (2, 6, 8) else 256
    out = np.zeros(n, dtype=np.float32)
    fn = {2: L.or_dequantize_q4_0_block, 6: L.or_dequantize_q5_0_block, 8: L.or_dequantize_q8_0_block,
          12: L.or_dequantize_q4_k_block, 13: L.or_dequantize_q5_k_block, 14: L.or_dequantize_q6_k_block}[quant]
    fn(ptr(blk), ptr(out))
    return out


class RepackedWeight:
    """The reference's portable RepackedWeight (repack_cache.rs:559-838)."""

    def __init__(self, raw, quant, rows, cols):
        self._raw = np.ascontiguousarray(raw, dtype=np.uint8)
        self.s = Repacked()
        check(L.or_repack(ptr(self._raw), self._raw.nbytes, quant, rows, cols, C.byref(self.s)))
        self.rows, self.cols, self.quant = rows, cols, quant

    def __del__(self):
        if hasattr(self, "s"):
            L.or_repacked_free(C.byref(self.s))

    def tiles(self):
        n = self.s.n_tiles * self.s.k_chunks * 128
        return np.ctypeslib.as_array(C.cast(self.s.tiles, C.POINTER(C.c_int8)), shape=(n,)).copy()

    def scales(self):
        n = self.s.n_tiles * self.s.scale_groups * 8
        return np.ctypeslib.as_array(C.cast(self.s.scales, C.POINTER(C.c_float)), shape=(n,)).copy()

    def mins(self):
        n = self.s.n_tiles * self.s.scale_groups * 8
        return np.ctypeslib.as_array(C.cast(self.s.mins, C.POINTER(C.c_float)), shape=(n,)).copy()

    def project_batch(self, act, m, nthreads=1):
        act = np.ascontiguousarray(act, dtype=np.float32)
        out = np.zeros(m * self.rows, dtype=np.float32)
        check(L.or_project_batch(C.byref(self.s), ptr(out), ptr(act), m, nthreads))
        return out.reshape(m, self.rows)

    def dot16_partials(self, q8, r0, r1):
        q8 = np.ascontiguousarray(q8, dtype=np.int8)
        out = np.zeros((r1 - r0) * (self.cols // 16), dtype=np.int32)
        L.or_dot16_partials(C.byref(self.s), ptr(q8), r0, r1, ptr(out))
        return out.reshape(r1 - r0, self.cols // 16)


def quantize_act_rows(act, m, k):
    act = np.ascontiguousarray(act, dtype=np.float32)
    nb = (k + 31) // 32
    f = np.zeros(m * nb * 32, dtype=np.float32)
    q = np.zeros(m * nb * 32, dtype=np.int8)
    s = np.zeros(m * nb, dtype=np.float32)
    L.or_quantize_act_rows(ptr(act), m, k, ptr(f), ptr(q), ptr(s))
    return q.reshape(m, nb * 32), s.reshape(m, nb)


def quantize_row_q8_0(x):
    x = np.ascontiguousarray(x, dtype=np.float32)
    out = (BlockQ8_0 * (x.size // 32))()
    check(L.or_quantize_row_q8_0(ptr(x), x.size, C.addressof(out)))
    return np.frombuffer(bytes(out), dtype=np.uint8)


def gemv_decode_projection(raw, quant, rows, cols, x, nthreads=1):
    raw = np.ascontiguousarray(raw, dtype=np.uint8)
    x = np.ascontiguousarray(x, dtype=np.float32)
    out = np.zeros(rows, dtype=np.float32)
    check(L.or_gemv_decode_projection(ptr(raw), raw.nbytes, quant, rows, cols, ptr(x), ptr(out), nthreads))
    return out


def compute_row_dot(row, cols, quant, raw, hidden):
    raw = np.ascontiguousarray(raw, dtype=np.uint8)
    hidden = np.ascontiguousarray(hidden, dtype=np.float32)
    return L.or_compute_row_dot(row, cols, quant, ptr(raw), raw.nbytes, ptr(hidden))


def rmsnorm_row(x, w, eps):
    x = np.ascontiguousarray(x, dtype=np.float32)
    w = np.ascontiguousarray(w, dtype=np.float32)
    out = np.zeros_like(x)
    check(L.or_rmsnorm_row(ptr(out), ptr(x), ptr(w), x.size, eps))
    return out


def _scaling(kind=0, factor=1.0, low=1.0, high=4.0, orig=8192, short=None, long=None):
    sc = RopeScaling()
    sc.kind, sc.factor, sc.low_freq_factor, sc.high_freq_factor = kind, factor, low, high
    sc.original_max_position_embeddings = orig
    keep = []
    if short is not None:
        s = np.ascontiguousarray(short, dtype=np.float32)
        l_ = np.ascontiguousarray(long, dtype=np.float32)
        keep = [s, l_]
        sc.short_factor, sc.long_factor, sc.n_factors = ptr(s), ptr(l_), s.size
    return sc, keep


def fill_inv_freq(head_dim, theta, seq_len, **scaling):
    sc, keep = _scaling(**scaling)
    out = np.zeros(head_dim // 2, dtype=np.float32)
    check(L.or_fill_inv_freq(head_dim, theta, C.byref(sc), seq_len, ptr(out)))
    return out


def apply_rope(qk, head_dim, rotary_dim, neox, pos, inv_freq):
    qk = np.array(qk, dtype=np.float32)
    inv = np.ascontiguousarray(inv_freq, dtype=np.float32)
    check(L.or_apply_rope(ptr(qk), qk.size, head_dim, rotary_dim, 1 if neox else 0, pos, ptr(inv)))
    return qk


def gqa_attention(q, k, v, m, nq, nkv, hd, total_seq, start_pos, window, scale):
    q, k, v = (np.ascontiguousarray(a, dtype=np.float32) for a in (q, k, v))
    out = np.zeros(m * nq * hd, dtype=np.float32)
    scratch = np.zeros(total_seq + 1, dtype=np.float32)
    check(L.or_gqa_attention(ptr(out), ptr(q), ptr(k), ptr(v), m, nq, nkv, hd, total_seq, start_pos, window, scale,
                             ptr(scratch), scratch.size))
    return out


def swiglu(g, u):
    g = np.ascontiguousarray(g, dtype=np.float32)
    u = np.ascontiguousarray(u, dtype=np.float32)
    out = np.zeros_like(g)
    check(L.or_swiglu(ptr(out), ptr(g), ptr(u), g.size))
    return out


class Model:
    """The cached recipe forward (prefill_step_with_cache / decode_step_with_cache)."""

    def __init__(self, tensors, geom: dict, nthreads=1, skip_rope=None, scaling=None, sliding_window=0,
                 kv_f16=False):
        self._keep = []
        arr = (Tensor * len(tensors))()
        for i, t in enumerate(tensors.values()):
            arr[i].name = t.name.encode()
            arr[i].quant = t.qtype
            arr[i].n_dims = len(t.dims)
            for d, v in enumerate(t.dims):
                arr[i].ne[d] = v
            arr[i].data = ptr(t.data)
            arr[i].nbytes = t.nbytes
            self._keep.append(t.data)
        g = Geometry()
        for k in ("num_layers", "hidden_dim", "ffn_dim", "n_heads_q", "n_heads_kv", "head_dim", "vocab_size"):
            setattr(g, k, geom[k])
        g.rotary_dim = geom.get("rotary_dim", geom["head_dim"])
        g.rms_eps, g.rope_theta, g.neox = geom["rms_eps"], geom["rope_theta"], 1 if geom.get("neox") else 0
        if skip_rope is not None:
            sk = np.ascontiguousarray(skip_rope, dtype=np.uint8)
            self._keep.append(sk)
            g.skip_rope_layers = ptr(sk)
        sc, keep = _scaling(**(scaling or {}))
        self._keep += keep
        g.scaling = sc
        g.sliding_window = sliding_window
        g.kv_f16 = 1 if kv_f16 else 0
        h = _P()
        check(L.or_model_build(C.byref(g), C.addressof(arr), len(tensors), nthreads, C.byref(h)))
        self.h = h.value
        self.geom = geom
        self.vocab = L.or_model_vocab(self.h)
        self.kv_dim = geom["n_heads_kv"] * geom["head_dim"]

    def __del__(self):
        if getattr(self, "h", None):
            L.or_model_free(self.h)

    def new_kv(self, seq_cap):
        return np.zeros(self.geom["num_layers"] * 2 * seq_cap * self.kv_dim, dtype=np.float32)

    def prefill(self, kv, seq_cap, tokens, start_pos, compute_logits=True):
        toks = np.ascontiguousarray(tokens, dtype=np.uint32)
        logits = np.zeros(self.vocab, dtype=np.float32)
        check(L.or_prefill(self.h, ptr(kv), seq_cap, ptr(toks), toks.size, start_pos, 1 if compute_logits else 0,
                           ptr(logits)))
        return logits

    def decode(self, kv, seq_cap, token, pos):
        logits = np.zeros(self.vocab, dtype=np.float32)
        check(L.or_decode(self.h, ptr(kv), seq_cap, token, pos, ptr(logits)))
        return logits


_ROW = {0: (1, 4), 2: (32, 18), 8: (32, 34)}


def synth_matrix(quant, rows, cols, seed, name, std=0.02, nthreads=1):
    """Seeded synthetic rows x cols tensor in raw GGUF block order (the same
    bytes as the product library's generator for the same arguments)."""
    e, b = _ROW[quant]
    out = np.empty(rows * (cols // e) * b, dtype=np.uint8)
    check(L.or_synth_matrix(quant, rows, cols, seed, name.encode(), std, ptr(out), out.nbytes, nthreads))
    return out


class SynthTensor:
    def __init__(self, name, dims, qtype, data):
        self.name, self.dims, self.qtype, self.data = name, dims, qtype, data

    @property
    def nbytes(self):
        return self.data.nbytes


def synth_llama_tensors(shape, seed, layers, nthreads=1):
    """Tensors of a seeded synthetic Llama-layout model with only the first
    `layers` blocks (names, shapes and values as in the GGUF generator):
    shape = dict(hidden_dim, ffn_dim, n_heads_q, n_heads_kv, head_dim,
    vocab_size, weight_quant, embed_quant, head_quant), optionally qkv_bias
    (F32 Q/K/V biases, as Qwen2 has) with bias_std."""
    H, F = shape["hidden_dim"], shape["ffn_dim"]
    Q, KV = shape["n_heads_q"] * shape["head_dim"], shape["n_heads_kv"] * shape["head_dim"]
    wq, ws = shape["weight_quant"], 0.02
    ones = np.ones(H, dtype=np.float32).view(np.uint8)
    t = {}

    def add(name, q, cols, rows, ones_vec=False):
        data = ones if ones_vec else synth_matrix(q, rows, cols, seed, name, ws, nthreads)
        t[name] = SynthTensor(name, [cols] if ones_vec else [cols, rows], q, data)

    add("token_embd.weight", shape["embed_quant"], H, shape["vocab_size"])
    for layer in range(layers):
        b = f"blk.{layer}."
        add(b + "attn_norm.weight", 0, H, 1, True)
        add(b + "attn_q.weight", wq, H, Q)
        add(b + "attn_k.weight", wq, H, KV)
        add(b + "attn_v.weight", wq, H, KV)
        add(b + "attn_output.weight", wq, Q, H)
        if shape.get("qkv_bias"):
            for nm, n in (("attn_q.bias", Q), ("attn_k.bias", KV), ("attn_v.bias", KV)):
                t[b + nm] = SynthTensor(b + nm, [n], 0,
                                        synth_matrix(0, 1, n, seed, b + nm, shape.get("bias_std", 0.02), nthreads))
        add(b + "ffn_norm.weight", 0, H, 1, True)
        add(b + "ffn_gate.weight", wq, H, F)
        add(b + "ffn_up.weight", wq, H, F)
        add(b + "ffn_down.weight", wq, F, H)
    add("output_norm.weight", 0, H, 1, True)
    add("output.weight", shape["head_quant"], H, shape["vocab_size"])
    return t
