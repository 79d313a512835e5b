"""Host-side binding of the B200 hot path of jero-arch-llama.

A ctypes mirror of the C ABI in include/jal.h (the drop-in boundary).  The
class and method names follow the reference crate: ``LlamaRecipe``
(recipe.rs:110), ``ModelRepackCache`` (repack_cache.rs:2129), ``CachedMatrix``
(repack_cache.rs:1502), ``gemv_decode_projection`` (decode_gemv.rs:1395) and
an ``ExecutionContext`` with ``prefill_step`` / ``decode_step``.  Errors are
raised as :class:`K3Error` subclasses carrying the C status code, mirroring
jero_core::K3Error.

Device buffers are passed as integer device pointers (for example
``torch.Tensor.data_ptr()``); nothing here computes on the CPU.  The CUDA
library ``libjal.so`` must be built in-tree (``make`` in this directory);
importing this module fails loudly when it is missing.
"""
from __future__ import annotations

import ctypes as C
import os
from dataclasses import dataclass, field

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_HERE, "libjal.so")

# ---- constants (include/jal.h) ---------------------------------------------
OK = 0
ERR_TENSOR_BOUNDS = 1
ERR_CAPABILITY_MISMATCH = 2
ERR_CONTEXT_LENGTH_EXCEEDED = 3
ERR_CUDA = 4
ERR_INVALID_ARGUMENT = 5
ERR_NCCL = 6
ERR_TIMEOUT = 7

F32, F16, Q4_0, Q5_0, Q8_0, Q4_K, Q5_K, Q6_K, BF16, TQ1_0, TQ2_0 = 0, 1, 2, 6, 8, 12, 13, 14, 30, 34, 35
ROPE_NORM, ROPE_NEOX = 0, 1
ROPE_SCALING_NONE, ROPE_SCALING_LINEAR, ROPE_SCALING_LLAMA3, ROPE_SCALING_LONGROPE = 0, 1, 2, 3
KV_F32, KV_F16 = 0, 1
NUMERICS_FAST, NUMERICS_REFERENCE, NUMERICS_RELAXED = 0, 1, 2  # jal_context_config.numerics

BLOCK_GEOMETRY = {F32: (1, 4), F16: (1, 2), BF16: (1, 2), Q4_0: (32, 18), Q5_0: (32, 22), Q8_0: (32, 34),
                  Q4_K: (256, 144), Q5_K: (256, 176), Q6_K: (256, 210), TQ1_0: (256, 54), TQ2_0: (256, 66)}


def row_bytes(quant: int, cols: int) -> int:
    e, b = BLOCK_GEOMETRY[quant]
    if cols <= 0 or cols % e:
        raise TensorBoundsError(f"cols {cols} incompatible with quant {quant}")
    return cols // e * b


class K3Error(RuntimeError):
    """A non-zero status from the C ABI (jero_core::K3Error)."""

    code = -1

    def __init__(self, msg: str, code: int | None = None):
        super().__init__(msg)
        if code is not None:
            self.code = code


class TensorBoundsError(K3Error):
    code = ERR_TENSOR_BOUNDS


class CapabilityMismatch(K3Error):
    code = ERR_CAPABILITY_MISMATCH


class ContextLengthExceeded(K3Error):
    code = ERR_CONTEXT_LENGTH_EXCEEDED


class CudaError(K3Error):
    code = ERR_CUDA


class NcclError(K3Error):
    code = ERR_NCCL


class DeviceTimeout(K3Error):
    """A bounded device wait (a copy, a peer's exchange words) gave up."""
    code = ERR_TIMEOUT


_ERRORS = {ERR_TENSOR_BOUNDS: TensorBoundsError, ERR_CAPABILITY_MISMATCH: CapabilityMismatch,
           ERR_CONTEXT_LENGTH_EXCEEDED: ContextLengthExceeded, ERR_CUDA: CudaError, ERR_NCCL: NcclError,
           ERR_TIMEOUT: DeviceTimeout}


class RecipeFields(C.Structure):
    _fields_ = [("architecture", C.c_char * 16),
                ("num_layers", C.c_uint64), ("hidden_dim", C.c_uint64), ("ffn_dim", C.c_uint64),
                ("n_heads_q", C.c_uint64), ("n_heads_kv", C.c_uint64), ("head_dim", C.c_uint64),
                ("vocab_size", C.c_uint64), ("rms_eps", C.c_float), ("rope_theta", C.c_float),
                ("rope_type", C.c_int32), ("rotary_dim", C.c_int64), ("rope_scaling_kind", C.c_int32),
                ("rope_factor", C.c_float), ("rope_low_freq_factor", C.c_float),
                ("rope_high_freq_factor", C.c_float), ("rope_original_max_position_embeddings", C.c_uint64)]


class ContextConfig(C.Structure):
    _fields_ = [("n_ctx", C.c_uint64), ("kv_dtype", C.c_int32), ("page_size", C.c_uint32),
                ("sliding_window", C.c_uint64), ("use_graphs", C.c_int32), ("numerics", C.c_int32)]


class SynthConfig(C.Structure):
    _fields_ = [("architecture", C.c_char * 16),
                ("num_layers", C.c_uint64), ("hidden_dim", C.c_uint64), ("ffn_dim", C.c_uint64),
                ("n_heads_q", C.c_uint64), ("n_heads_kv", C.c_uint64), ("head_dim", C.c_uint64),
                ("vocab_size", C.c_uint64), ("context_length", C.c_uint64),
                ("rms_eps", C.c_float), ("rope_theta", C.c_float),
                ("weight_quant", C.c_int32), ("embed_quant", C.c_int32), ("head_quant", C.c_int32),
                ("qkv_bias", C.c_int32), ("weight_std", C.c_float), ("bias_std", C.c_float)]


_P = C.c_void_p
_SZ = C.c_size_t


class TpPlanFields(C.Structure):
    _fields_ = [(n, C.c_uint64) for n in ("rank", "world", "q_lo", "q_n", "kv_lo", "kv_n", "f_lo", "f_n",
                                          "v_lo", "v_n", "v_pad")]


# name -> (restype, argtypes)
_SIGS = {
    "jal_last_error": (C.c_char_p, []),
    "jal_version": (C.c_char_p, []),
    "jal_set_device": (C.c_int, [C.c_int]),
    "jal_device_sm_count": (C.c_int, [C.POINTER(C.c_int)]),
    "jal_cached_matrix_repack": (C.c_int, [_P, _SZ, C.c_int, C.c_int, _SZ, _SZ, _P, C.POINTER(_P)]),
    "jal_cached_matrix_free": (None, [_P]),
    "jal_cached_matrix_rows": (_SZ, [_P]),
    "jal_cached_matrix_cols": (_SZ, [_P]),
    "jal_cached_matrix_quant": (C.c_int, [_P]),
    "jal_cached_matrix_aligned_bytes": (_SZ, [_P]),
    "jal_cached_matrix_export_ref_layout": (C.c_int, [_P, _P, _SZ, _P, _SZ]),
    "jal_cached_matrix_gemm": (C.c_int, [_P, _P, _SZ, _P, _P]),
    "jal_cached_matrix_gemm_noalloc": (C.c_int, [_P, _P, _SZ, _P, _P]),
    "jal_cached_matrix_gemv_q8": (C.c_int, [_P, _P, _P, _P, _P]),
    "jal_cached_matrix_dot16_partials": (C.c_int, [_P, _P, _SZ, _SZ, _P, _P]),
    "jal_act_quantize_q8": (C.c_int, [_P, _SZ, _SZ, _P, _P, _P]),
    "jal_quantize_row_q8_0": (C.c_int, [_P, _SZ, _P, _P]),
    "jal_gemv_decode_projection": (C.c_int, [_P, _SZ, C.c_int, _SZ, _SZ, _P, _P, _P]),
    "jal_op_rmsnorm": (C.c_int, [_P, _P, _SZ, _SZ, C.c_float, _P, _P]),
    "jal_op_rope": (C.c_int, [_P, _SZ, _SZ, _SZ, _SZ, C.c_int, _SZ, _P, _P]),
    "jal_op_swiglu": (C.c_int, [_P, _P, _SZ, _P, _P]),
    "jal_op_gqa_attention": (C.c_int, [_P, _P, _P, _SZ, _SZ, _SZ, _SZ, _SZ, _SZ, _SZ, C.c_float, _P, _P]),
    "jal_recipe_new": (C.c_int, [C.c_char_p, C.POINTER(_P)]),
    "jal_recipe_from_gguf": (C.c_int, [_P, _SZ, C.POINTER(_P)]),
    "jal_recipe_free": (None, [_P]),
    "jal_recipe_get_fields": (C.c_int, [_P, C.POINTER(RecipeFields)]),
    "jal_recipe_set_fields": (C.c_int, [_P, C.POINTER(RecipeFields)]),
    "jal_recipe_set_irope_mask": (C.c_int, [_P, _P, _SZ]),
    "jal_recipe_should_skip_rope": (C.c_int, [_P, _SZ]),
    "jal_recipe_set_longrope": (C.c_int, [_P, _P, _P, _SZ, C.c_uint64]),
    "jal_recipe_supports_quant": (C.c_int, [_P, C.c_int]),
    "jal_recipe_validate_model": (C.c_int, [_P, _P, _SZ]),
    "jal_recipe_decode_scratch_bytes": (_SZ, [_P, _SZ]),
    "jal_model_repack_cache_build": (C.c_int, [_P, _P, _SZ, C.c_int, C.POINTER(_P)]),
    "jal_model_repack_cache_build_tp": (C.c_int, [_P, _P, _SZ, C.c_int, _P, C.POINTER(_P)]),
    "jal_tp_plan": (C.c_int, [_SZ, _SZ, _SZ, _SZ, C.c_int, C.c_int, C.POINTER(TpPlanFields)]),
    "jal_tp_unique_id": (C.c_int, [_P]),
    "jal_tp_init": (C.c_int, [_P, C.c_int, C.c_int, C.POINTER(_P)]),
    "jal_tp_free": (None, [_P]),
    "jal_model_repack_cache_free": (None, [_P]),
    "jal_model_cache_num_layers": (_SZ, [_P]),
    "jal_model_cache_hidden_dim": (_SZ, [_P]),
    "jal_model_cache_ffn_dim": (_SZ, [_P]),
    "jal_model_cache_total_q": (_SZ, [_P]),
    "jal_model_cache_total_kv": (_SZ, [_P]),
    "jal_model_cache_vocab_size": (_SZ, [_P]),
    "jal_model_cache_norm_count": (_SZ, [_P]),
    "jal_model_cache_bias_count": (_SZ, [_P]),
    "jal_model_cache_repacked_matrix_count": (_SZ, [_P]),
    "jal_model_cache_total_aligned_bytes": (_SZ, [_P]),
    "jal_model_cache_matrix": (_P, [_P, _SZ, C.c_int]),
    "jal_context_new": (C.c_int, [_P, _P, C.POINTER(ContextConfig), C.POINTER(_P)]),
    "jal_kv_cache_alloc": (C.c_int, [_P, C.c_uint64, C.c_int32, C.c_uint32, C.POINTER(_P)]),
    "jal_kv_cache_free": (None, [_P]),
    "jal_kv_cache_bytes": (_SZ, [_P]),
    "jal_context_new_with_kv": (C.c_int, [_P, _P, C.POINTER(ContextConfig), _P, C.POINTER(_P)]),
    "jal_context_set_position": (C.c_int, [_P, _SZ]),
    "jal_context_test_stall_kv_copy": (C.c_int, [_P, C.c_uint32, C.c_uint64]),
    "jal_test_peer_exchange_timeout": (C.c_int, [_P, C.c_uint64, C.POINTER(C.c_double)]),
    "jal_context_free": (None, [_P]),
    "jal_context_position": (_SZ, [_P]),
    "jal_context_reset": (C.c_int, [_P]),
    "jal_prefill_step": (C.c_int, [_P, _P, _SZ, _SZ, C.c_int, _P, _SZ]),
    "jal_decode_step": (C.c_int, [_P, C.c_uint32, _P, _SZ]),
    "jal_decode_greedy": (C.c_int, [_P, C.c_uint32, _SZ, _P]),
    "jal_cached_matrix_export_ref_mins": (C.c_int, [_P, _P, _SZ]),
    "jal_decode_batch": (C.c_int, [_P, _SZ, _P, _P, _SZ]),
    "jal_context_trace_decode_step": (C.c_int, [_P, C.c_uint32, _P, _SZ, C.POINTER(_SZ)]),
    "jal_context_batch_logits_device": (C.c_int, [_P, C.POINTER(_P)]),
    "jal_context_export_kv": (C.c_int, [_P, _SZ, _P, _SZ]),
    "jal_context_logits_device": (C.c_int, [_P, C.POINTER(_P)]),
    "jal_context_last_step_launches": (C.c_int, [_P, C.POINTER(_SZ)]),
    "jal_context_tp_exchange": (C.c_int, [_P, C.POINTER(C.c_int)]),
    "jal_context_set_stream": (C.c_int, [_P, _P]),
    "jal_synth_gguf_size": (C.c_int, [C.POINTER(SynthConfig), C.POINTER(_SZ)]),
    "jal_synth_gguf_write": (C.c_int, [C.POINTER(SynthConfig), C.c_uint64, _P, _SZ, C.c_int]),
    "jal_synth_matrix": (C.c_int, [C.c_int, _SZ, _SZ, C.c_uint64, C.c_char_p, C.c_float, _P, _SZ, C.c_int]),
    "jal_synth_normal_f32": (C.c_int, [C.c_uint64, C.c_char_p, _SZ, C.c_float, _P, C.c_int]),
    "jal_f32_to_f16_bits": (C.c_uint16, [C.c_float]),
}

_lib = None


def lib() -> C.CDLL:
    """Load libjal.so once; raise if it has not been built."""
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise ImportError(f"{LIB_PATH} is missing: build it with `make -C {_HERE}` (nvcc, sm_100a)")
        l = C.CDLL(LIB_PATH)
        for name, (res, args) in _SIGS.items():
            fn = getattr(l, name)
            fn.restype = res
            fn.argtypes = args
        _lib = l
    return _lib


def _check(rc: int) -> None:
    if rc != OK:
        msg = lib().jal_last_error().decode(errors="replace")
        raise _ERRORS.get(rc, K3Error)(msg, rc)


def _ptr(x) -> int | None:
    """Device pointer of a torch tensor, an int, or None."""
    if x is None:
        return None
    if isinstance(x, int):
        return x
    if hasattr(x, "data_ptr"):
        return x.data_ptr()
    if hasattr(x, "ctypes"):
        return x.ctypes.data
    raise TypeError(f"cannot take a pointer of {type(x)}")


def _stream(s) -> int | None:
    if s is None:
        return None
    return getattr(s, "cuda_stream", s)


def nthreads_default() -> int:
    return os.cpu_count() or 1


def set_device(device: int) -> None:
    _check(lib().jal_set_device(device))


def sm_count() -> int:
    n = C.c_int(0)
    _check(lib().jal_device_sm_count(C.byref(n)))
    return n.value


# ---- CachedMatrix (repack_cache.rs:1502-1788) -------------------------------
class CachedMatrix:
    def __init__(self, handle: int, owned: bool = True, keepalive=None):
        self._h = handle
        self._owned = owned
        self._keep = keepalive

    @classmethod
    def repack(cls, raw, quant: int, rows: int, cols: int, on_device: bool = False, stream=None) -> "CachedMatrix":
        """CachedMatrix::repack (repack_cache.rs:1516): raw GGUF rows (numpy
        bytes on the host, or a device pointer with on_device=True)."""
        n = raw.nbytes if hasattr(raw, "nbytes") else len(raw)
        if not on_device and isinstance(raw, (bytes, bytearray)):
            raw = (C.c_uint8 * n).from_buffer_copy(raw)
            p = C.addressof(raw)
        else:
            p = _ptr(raw)
        out = _P()
        _check(lib().jal_cached_matrix_repack(p, n, 1 if on_device else 0, quant, rows, cols, _stream(stream),
                                              C.byref(out)))
        return cls(out.value)

    def __del__(self):
        if getattr(self, "_owned", False) and self._h and _lib is not None:
            _lib.jal_cached_matrix_free(self._h)
            self._h = None

    @property
    def handle(self) -> int:
        return self._h

    def rows(self) -> int:
        return lib().jal_cached_matrix_rows(self._h)

    def cols(self) -> int:
        return lib().jal_cached_matrix_cols(self._h)

    def quant(self) -> int:
        return lib().jal_cached_matrix_quant(self._h)

    def aligned_bytes(self) -> int:
        return lib().jal_cached_matrix_aligned_bytes(self._h)

    def export_ref_layout(self):
        """(tiles int8, scales f32) numpy arrays in the reference's portable
        layout (repack_cache.rs:639-694)."""
        import numpy as np
        rows, cols = self.rows(), self.cols()
        nt = (rows + 7) // 8
        group = 16 if self.quant() == Q6_K else 32
        tiles = np.zeros(nt * (cols // 16) * 128, dtype=np.int8)
        scales = np.zeros(nt * (cols // group) * 8, dtype=np.float32)
        _check(lib().jal_cached_matrix_export_ref_layout(self._h, tiles.ctypes.data, tiles.size,
                                                         scales.ctypes.data, scales.size))
        return tiles, scales

    def export_ref_mins(self):
        """Group mins (f32, Q4_K / Q5_K) in the reference's portable layout."""
        import numpy as np
        mins = np.zeros(((self.rows() + 7) // 8) * (self.cols() // 32) * 8, dtype=np.float32)
        _check(lib().jal_cached_matrix_export_ref_mins(self._h, mins.ctypes.data, mins.size))
        return mins

    def gemm(self, x, m: int, y, stream=None) -> None:
        """project_batch (repack_cache.rs:1724): y[m, rows] = quant(x[m, cols]) . W^T."""
        _check(lib().jal_cached_matrix_gemm(self._h, _ptr(x), m, _ptr(y), _stream(stream)))

    def gemm_noalloc(self, x, m: int, y, stream=None) -> None:
        """Like gemm, but allocates no device memory: the activation scratch is a
        fixed 2 MiB device array shared by every call (calls that overlap on the
        GPU race); the work is only enqueued on the stream."""
        _check(lib().jal_cached_matrix_gemm_noalloc(self._h, _ptr(x), m, _ptr(y), _stream(stream)))

    def gemv_q8(self, q8, scales, y, stream=None) -> None:
        """gemv_with_act_view (repack_cache.rs:1636) with a quantized activation."""
        _check(lib().jal_cached_matrix_gemv_q8(self._h, _ptr(q8), _ptr(scales), _ptr(y), _stream(stream)))

    def dot16_partials(self, q8, r0: int, r1: int, out, stream=None) -> None:
        _check(lib().jal_cached_matrix_dot16_partials(self._h, _ptr(q8), r0, r1, _ptr(out), _stream(stream)))


def act_quantize_q8(x, m: int, k: int, q8, scales, stream=None) -> None:
    """QuantizedActQ8::quantize_into (repack_cache.rs:491-531)."""
    _check(lib().jal_act_quantize_q8(_ptr(x), m, k, _ptr(q8), _ptr(scales), _stream(stream)))


def quantize_row_q8_0(x, n: int, blocks, stream=None) -> None:
    """quantize_row_q8_0 (decode_gemv.rs:294-313); blocks: n/32 x 36 bytes."""
    _check(lib().jal_quantize_row_q8_0(_ptr(x), n, _ptr(blocks), _stream(stream)))


def gemv_decode_projection(raw, raw_len: int, quant: int, rows: int, cols: int, x, y, stream=None) -> None:
    """gemv_decode_projection (decode_gemv.rs:1395) over raw GGUF rows on the device."""
    _check(lib().jal_gemv_decode_projection(_ptr(raw), raw_len, quant, rows, cols, _ptr(x), _ptr(y),
                                            _stream(stream)))


def rmsnorm(x, w, m: int, n: int, eps: float, out, stream=None) -> None:
    _check(lib().jal_op_rmsnorm(_ptr(x), _ptr(w), m, n, eps, _ptr(out), _stream(stream)))


def rope(qk, m: int, row_len: int, head_dim: int, rotary_dim: int, neox: bool, pos0: int, inv_freq,
         stream=None) -> None:
    _check(lib().jal_op_rope(_ptr(qk), m, row_len, head_dim, rotary_dim, 1 if neox else 0, pos0, _ptr(inv_freq),
                             _stream(stream)))


def swiglu(gate, up, n: int, out, stream=None) -> None:
    _check(lib().jal_op_swiglu(_ptr(gate), _ptr(up), n, _ptr(out), _stream(stream)))


def gqa_attention(q, k, v, m, n_heads_q, n_heads_kv, head_dim, total_seq, start_pos, sliding_window, scale, out,
                  stream=None) -> None:
    _check(lib().jal_op_gqa_attention(_ptr(q), _ptr(k), _ptr(v), m, n_heads_q, n_heads_kv, head_dim, total_seq,
                                      start_pos, sliding_window, scale, _ptr(out), _stream(stream)))


# ---- LlamaRecipe (recipe.rs:110-547) ----------------------------------------
class LlamaRecipe:
    def __init__(self, handle: int):
        self._h = handle

    @classmethod
    def new(cls, architecture: str = "llama") -> "LlamaRecipe":
        out = _P()
        _check(lib().jal_recipe_new(architecture.encode(), C.byref(out)))
        return cls(out.value)

    @classmethod
    def new_llama4(cls) -> "LlamaRecipe":
        return cls.new("llama4")

    @classmethod
    def new_qwen2(cls) -> "LlamaRecipe":
        return cls.new("qwen2")

    @classmethod
    def from_gguf(cls, gguf) -> "LlamaRecipe":
        buf = _as_buffer(gguf)
        out = _P()
        _check(lib().jal_recipe_from_gguf(buf[0], buf[1], C.byref(out)))
        return cls(out.value)

    def __del__(self):
        if getattr(self, "_h", None) and _lib is not None:
            _lib.jal_recipe_free(self._h)
            self._h = None

    @property
    def handle(self) -> int:
        return self._h

    def fields(self) -> RecipeFields:
        f = RecipeFields()
        _check(lib().jal_recipe_get_fields(self._h, C.byref(f)))
        return f

    def set_fields(self, f: RecipeFields) -> None:
        _check(lib().jal_recipe_set_fields(self._h, C.byref(f)))

    def __getattr__(self, name):
        if name.startswith("_"):
            raise AttributeError(name)
        f = self.fields()
        if name == "architecture":
            return f.architecture.decode()
        if name == "rotary_dim":
            return None if f.rotary_dim < 0 else f.rotary_dim
        if hasattr(f, name):
            return getattr(f, name)
        raise AttributeError(name)

    def architecture_id(self) -> str:
        return self.fields().architecture.decode()

    def effective_rotary_dim(self) -> int:
        f = self.fields()
        return f.head_dim if f.rotary_dim < 0 else f.rotary_dim

    def with_rotary_dim(self, rd: int) -> "LlamaRecipe":
        f = self.fields()
        f.rotary_dim = rd
        self.set_fields(f)
        return self

    def with_rope_type(self, rope_type: int) -> "LlamaRecipe":
        f = self.fields()
        f.rope_type = rope_type
        self.set_fields(f)
        return self

    def with_irope_mask(self, mask) -> "LlamaRecipe":
        arr = (C.c_uint8 * len(mask))(*[1 if m else 0 for m in mask])
        _check(lib().jal_recipe_set_irope_mask(self._h, C.addressof(arr), len(mask)))
        return self

    def with_rope_scaling_longrope(self, short, long, orig_ctx: int) -> "LlamaRecipe":
        n = len(short)
        s = (C.c_float * n)(*short)
        l_ = (C.c_float * n)(*long)
        _check(lib().jal_recipe_set_longrope(self._h, C.addressof(s), C.addressof(l_), n, orig_ctx))
        return self

    def should_skip_rope(self, layer: int) -> bool:
        return bool(lib().jal_recipe_should_skip_rope(self._h, layer))

    def supports_quant(self, quant: int) -> bool:
        return bool(lib().jal_recipe_supports_quant(self._h, quant))

    def validate_model(self, gguf) -> None:
        buf = _as_buffer(gguf)
        _check(lib().jal_recipe_validate_model(self._h, buf[0], buf[1]))

    def decode_scratch_bytes(self, seq_len_upper_bound: int) -> int:
        return lib().jal_recipe_decode_scratch_bytes(self._h, seq_len_upper_bound)

    def build_repack_cache(self, gguf, device: int = 0, tp: "TensorParallel" = None) -> "ModelRepackCache":
        """build_repack_cache (recipe.rs:481-509); with `tp`, this rank's shard."""
        buf = _as_buffer(gguf)
        out = _P()
        if tp is None:
            _check(lib().jal_model_repack_cache_build(self._h, buf[0], buf[1], device, C.byref(out)))
        else:
            _check(lib().jal_model_repack_cache_build_tp(self._h, buf[0], buf[1], device, tp._h, C.byref(out)))
        cache = ModelRepackCache(out.value)
        cache._tp = tp  # the communicator outlives the cache
        return cache


# ---- tensor parallelism (one process per GPU, NCCL) -----------------------------
def tp_plan(n_heads_q: int, n_heads_kv: int, ffn_dim: int, vocab: int, rank: int, world: int) -> dict:
    """Shard plan of one rank (no GPU needed): head, FFN and vocabulary ranges."""
    f = TpPlanFields()
    _check(lib().jal_tp_plan(n_heads_q, n_heads_kv, ffn_dim, vocab, rank, world, C.byref(f)))
    return {n: getattr(f, n) for n, _ in TpPlanFields._fields_}


def tp_unique_id() -> bytes:
    """128-byte NCCL unique id; rank 0 creates it and shares it with the other ranks."""
    buf = (C.c_uint8 * 128)()
    _check(lib().jal_tp_unique_id(C.addressof(buf)))
    return bytes(buf)


class TensorParallel:
    """NCCL communicator of one rank on the current device (collective: every
    rank constructs it with the same id)."""

    def __init__(self, unique_id: bytes, rank: int, world: int):
        if len(unique_id) != 128:
            raise ValueError("the NCCL unique id is 128 bytes")
        buf = (C.c_uint8 * 128).from_buffer_copy(unique_id)
        out = _P()
        _check(lib().jal_tp_init(C.addressof(buf), rank, world, C.byref(out)))
        self._h = out.value
        self.rank, self.world = rank, world

    def __del__(self):
        if getattr(self, "_h", None) and _lib is not None:
            _lib.jal_tp_free(self._h)
            self._h = None


def _as_buffer(b):
    """(pointer, length) of a bytes-like / numpy uint8 object (kept alive by the caller)."""
    if hasattr(b, "ctypes"):
        return b.ctypes.data, b.nbytes
    if isinstance(b, bytes):
        return C.cast(C.c_char_p(b), C.c_void_p).value, len(b)
    if isinstance(b, bytearray):
        arr = (C.c_uint8 * len(b)).from_buffer(b)
        return C.addressof(arr), len(b)
    raise TypeError(f"unsupported buffer {type(b)}")


# ---- ModelRepackCache (repack_cache.rs:2129-2380) ---------------------------
class ModelRepackCache:
    MATRICES = ("q", "k", "v", "output", "gate", "up", "down")

    def __init__(self, handle: int):
        self._h = handle

    def __del__(self):
        if getattr(self, "_h", None) and _lib is not None:
            _lib.jal_model_repack_cache_free(self._h)
            self._h = None

    @property
    def handle(self) -> int:
        return self._h

    def num_layers(self) -> int: return lib().jal_model_cache_num_layers(self._h)
    def hidden_dim(self) -> int: return lib().jal_model_cache_hidden_dim(self._h)
    def ffn_dim(self) -> int: return lib().jal_model_cache_ffn_dim(self._h)
    def total_q(self) -> int: return lib().jal_model_cache_total_q(self._h)
    def total_kv(self) -> int: return lib().jal_model_cache_total_kv(self._h)
    def vocab_size(self) -> int: return lib().jal_model_cache_vocab_size(self._h)
    def norm_count(self) -> int: return lib().jal_model_cache_norm_count(self._h)
    def bias_count(self) -> int: return lib().jal_model_cache_bias_count(self._h)
    def repacked_matrix_count(self) -> int: return lib().jal_model_cache_repacked_matrix_count(self._h)
    def total_aligned_bytes(self) -> int: return lib().jal_model_cache_total_aligned_bytes(self._h)

    def matrix(self, layer: int, which: str) -> CachedMatrix:
        """A borrowed CachedMatrix of layer `layer` (layer == num_layers: LM head)."""
        idx = 0 if layer == self.num_layers() else self.MATRICES.index(which)
        h = lib().jal_model_cache_matrix(self._h, layer, idx)
        if not h:
            raise TensorBoundsError(f"no matrix {which} in layer {layer}")
        return CachedMatrix(h, owned=False, keepalive=self)


# ---- ExecutionContext + prefill_step / decode_step --------------------------
class KvCache:
    """Caller-owned KV storage for a model (the reference's KvCacheView): it
    outlives the contexts made over it and keeps its contents."""

    def __init__(self, cache: "ModelRepackCache", n_ctx: int, kv_dtype: int = KV_F16, page_size: int = 64):
        out = _P()
        _check(lib().jal_kv_cache_alloc(cache.handle, n_ctx, kv_dtype, page_size, C.byref(out)))
        self._h = out.value
        self._cache = cache
        self.n_ctx, self.kv_dtype, self.page_size = n_ctx, kv_dtype, page_size

    def __del__(self):
        if getattr(self, "_h", None) and _lib is not None:
            _lib.jal_kv_cache_free(self._h)
            self._h = None

    @property
    def handle(self) -> int:
        return self._h

    def nbytes(self) -> int:
        return lib().jal_kv_cache_bytes(self._h)


class ExecutionContext:
    def __init__(self, recipe: LlamaRecipe, cache: ModelRepackCache, n_ctx: int, kv_dtype: int = KV_F16,
                 page_size: int = 64, sliding_window: int = 0, use_graphs: bool = True,
                 numerics: int = None, kv: KvCache = None):
        if numerics is None:
            numerics = NUMERICS_FAST
        cfg = ContextConfig(n_ctx, kv_dtype, page_size, sliding_window, 1 if use_graphs else 0, numerics)
        out = _P()
        if kv is None:
            _check(lib().jal_context_new(recipe.handle, cache.handle, C.byref(cfg), C.byref(out)))
        else:
            _check(lib().jal_context_new_with_kv(recipe.handle, cache.handle, C.byref(cfg), kv.handle, C.byref(out)))
        self._h = out.value
        self._recipe, self._cache, self._kv = recipe, cache, kv
        self.vocab = cache.vocab_size()

    def set_position(self, pos: int) -> None:
        """Resume at `pos` over a KV cache whose positions [0, pos) are filled."""
        _check(lib().jal_context_set_position(self._h, pos))

    def __del__(self):
        if getattr(self, "_h", None) and _lib is not None:
            _lib.jal_context_free(self._h)
            self._h = None

    @property
    def handle(self) -> int:
        return self._h

    def position(self) -> int:
        return lib().jal_context_position(self._h)

    def reset(self) -> None:
        _check(lib().jal_context_reset(self._h))

    def prefill_step(self, tokens, start_pos: int | None = None, compute_logits: bool = True):
        """prefill_step_with_cache (recipe.rs:517): returns the last token's logits (numpy) or None."""
        import numpy as np
        toks = np.ascontiguousarray(np.asarray(tokens, dtype=np.uint32))
        sp = self.position() if start_pos is None else start_pos
        logits = np.zeros(self.vocab, dtype=np.float32) if compute_logits else None
        _check(lib().jal_prefill_step(self._h, toks.ctypes.data if toks.size else None, toks.size, sp,
                                      1 if compute_logits else 0,
                                      logits.ctypes.data if logits is not None else None,
                                      self.vocab if logits is not None else 0))
        return logits

    def decode_step(self, token: int, want_logits: bool = True, out=None):
        """decode_step_with_cache (recipe.rs:555): logits of the new position (numpy) or None.

        `out`: a C-contiguous float32 numpy array of vocab length to receive
        the logits (returned); a caller that reuses one page-locked array
        (e.g. ``torch.empty(vocab).pin_memory().numpy()``) avoids a pageable
        copy and a fresh allocation per step."""
        import numpy as np
        if out is not None:
            if out.dtype != np.float32 or out.shape != (self.vocab,) or not out.flags["C_CONTIGUOUS"]:
                raise ValueError("out must be a contiguous float32 array of vocab length")
            logits = out
        else:
            logits = np.zeros(self.vocab, dtype=np.float32) if want_logits else None
        _check(lib().jal_decode_step(self._h, token, logits.ctypes.data if logits is not None else None,
                                     self.vocab if logits is not None else 0))
        return logits

    def decode_greedy(self, token: int, n_steps: int):
        import numpy as np
        out = np.zeros(n_steps, dtype=np.uint32)
        _check(lib().jal_decode_greedy(self._h, token, n_steps, out.ctypes.data))
        return out

    def export_kv(self, n_pos: int, num_layers: int, kv_dim: int):
        import numpy as np
        out = np.zeros(num_layers * 2 * n_pos * kv_dim, dtype=np.float32)
        _check(lib().jal_context_export_kv(self._h, n_pos, out.ctypes.data, out.size))
        return out

    def logits_device_ptr(self) -> int:
        p = _P()
        _check(lib().jal_context_logits_device(self._h, C.byref(p)))
        return p.value

    def trace_decode_step(self, token: int):
        """Two greedy decode steps; the second's per-launch globaltimer stamps
        in ns as a [launches, 8] uint64 array: start, end, then the phase
        marks (0 where none).  jal_test.h."""
        import numpy as np
        cap = 4096
        out = np.zeros(8 * cap, dtype=np.uint64)
        n = _SZ()
        _check(lib().jal_context_trace_decode_step(self._h, token, out.ctypes.data, out.size, C.byref(n)))
        return out[: 8 * min(n.value, cap)].reshape(-1, 8)

    def set_stream(self, stream) -> None:
        """Issue this context's work on `stream` (torch stream or cudaStream_t); None = own stream."""
        _check(lib().jal_context_set_stream(self._h, _stream(stream)))

    def launches_per_step(self) -> int:
        n = _SZ()
        _check(lib().jal_context_last_step_launches(self._h, C.byref(n)))
        return n.value

    def tp_exchange(self) -> str:
        """'none' (one rank), 'nccl' (all-reduce) or 'peer' (partial sums
        exchanged over peer memory inside the GEMVs) for the decode step."""
        v = C.c_int()
        _check(lib().jal_context_tp_exchange(self._h, C.byref(v)))
        return {0: "none", 1: "nccl", 2: "peer"}[v.value]


def decode_batch(contexts, tokens, want_logits: bool = True, out=None):
    """One decode step for several independent sequences (jal_decode_batch):
    token i at contexts[i]'s position.  The contexts share one model cache and
    own distinct KV caches; each advances by one.  Returns the logits as a
    [n, vocab] float32 array (or `out`, filled), or None."""
    import numpy as np
    n = len(contexts)
    toks = np.ascontiguousarray(np.asarray(tokens, dtype=np.uint32))
    if toks.shape != (n,):
        raise ValueError("one token per context")
    hs = (_P * n)(*[c._h for c in contexts])
    vocab = contexts[0].vocab
    logits = None
    if out is not None:
        if out.dtype != np.float32 or out.shape != (n, vocab) or not out.flags["C_CONTIGUOUS"]:
            raise ValueError("out must be a contiguous float32 [n, vocab] array")
        logits = out
    elif want_logits:
        logits = np.empty((n, vocab), dtype=np.float32)
    _check(lib().jal_decode_batch(hs, n, toks.ctypes.data, logits.ctypes.data if logits is not None else None,
                                  logits.size if logits is not None else 0))
    return logits


# ---- synthetic GGUF models (include/jal_synth.h) -----------------------------
@dataclass
class SynthSpec:
    architecture: str = "llama"
    num_layers: int = 4
    hidden_dim: int = 512
    ffn_dim: int = 1376
    n_heads_q: int = 8
    n_heads_kv: int = 2
    head_dim: int = 64
    vocab_size: int = 4096
    context_length: int = 256
    rms_eps: float = 1e-5
    rope_theta: float = 10000.0
    weight_quant: int = Q4_0
    embed_quant: int = Q8_0
    head_quant: int = Q8_0
    qkv_bias: bool = False
    weight_std: float = 0.02
    bias_std: float = 0.02

    def to_c(self) -> SynthConfig:
        c = SynthConfig()
        c.architecture = self.architecture.encode()
        for k in ("num_layers", "hidden_dim", "ffn_dim", "n_heads_q", "n_heads_kv", "head_dim", "vocab_size",
                  "context_length", "rms_eps", "rope_theta", "weight_quant", "embed_quant", "head_quant",
                  "weight_std", "bias_std"):
            setattr(c, k, getattr(self, k))
        c.qkv_bias = 1 if self.qkv_bias else 0
        return c


# Workloads named by the benchmark and the parity tests.
TINY_LLAMA = SynthSpec()
LLAMA3_8B_Q4_0 = SynthSpec(num_layers=32, hidden_dim=4096, ffn_dim=14336, n_heads_q=32, n_heads_kv=8, head_dim=128,
                           vocab_size=128256, context_length=8192, rope_theta=500000.0, weight_quant=Q4_0,
                           embed_quant=Q4_0, head_quant=Q4_0)
QWEN2_7B_Q8_0 = SynthSpec(architecture="qwen2", num_layers=28, hidden_dim=3584, ffn_dim=18944, n_heads_q=28,
                          n_heads_kv=4, head_dim=128, vocab_size=152064, context_length=4096, rms_eps=1e-6,
                          rope_theta=1e6, weight_quant=Q8_0, embed_quant=Q8_0, head_quant=Q8_0, qkv_bias=True)
LLAMA3_70B_Q4_0 = SynthSpec(num_layers=80, hidden_dim=8192, ffn_dim=28672, n_heads_q=64, n_heads_kv=8, head_dim=128,
                            vocab_size=128256, context_length=8448, rope_theta=500000.0, weight_quant=Q4_0,
                            embed_quant=Q4_0, head_quant=Q4_0)


def synth_gguf(spec: SynthSpec, seed: int, nthreads: int | None = None):
    """Seeded synthetic GGUF v3 bytes (numpy uint8)."""
    import numpy as np
    cfg = spec.to_c()
    n = _SZ()
    _check(lib().jal_synth_gguf_size(C.byref(cfg), C.byref(n)))
    buf = np.empty(n.value, dtype=np.uint8)
    _check(lib().jal_synth_gguf_write(C.byref(cfg), seed, buf.ctypes.data, buf.nbytes,
                                      nthreads or nthreads_default()))
    return buf


def synth_matrix(quant: int, rows: int, cols: int, seed: int, name: str, std: float = 0.02,
                 nthreads: int | None = None):
    import numpy as np
    buf = np.empty(rows * row_bytes(quant, cols), dtype=np.uint8)
    _check(lib().jal_synth_matrix(quant, rows, cols, seed, name.encode(), std, buf.ctypes.data, buf.nbytes,
                                  nthreads or nthreads_default()))
    return buf


def synth_normal(n: int, seed: int, name: str, std: float = 1.0, nthreads: int | None = None):
    import numpy as np
    out = np.empty(n, dtype=np.float32)
    _check(lib().jal_synth_normal_f32(seed, name.encode(), n, std, out.ctypes.data, nthreads or nthreads_default()))
    return out


def f32_to_f16_bits(v: float) -> int:
    return lib().jal_f32_to_f16_bits(v)


def version() -> str:
    return lib().jal_version().decode()
