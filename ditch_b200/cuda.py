"""Host-side mirror of ditch's compute seam over the C ABI of libditch_cuda.so.

`Device` mirrors `compute.Device` with the per-op VTable entries
(src/compute.zig:90-117); `Model` is the resident model with the coarse
entries that replace `model.forward`, `Engine.getResidualMeanObserved`,
`abliterate.apply` and `KlDivergence` when the device is CUDA
(include/ditch_cuda.h documents each entry and the reference it mirrors).

There is no CPU fallback here: if the library is missing the import fails,
and a status other than OK raises. `Unsupported` is the seam's
`error.Unsupported` (ditch would run its CPU kernel; this package does not).
"""
import ctypes as C
import os
import weakref

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_HERE, "libditch_cuda.so")

OK, UNSUPPORTED, DEVICE_FAILED, OUT_OF_MEMORY, INVALID = 0, 1, 2, 3, 4

# tensor.DType codes (src/tensor.zig:11-32)
DTYPE = {"f32": 0, "f16": 1, "bf16": 2, "q8_0": 5, "q4_0": 6, "q4_1": 7, "q5_0": 8, "q5_1": 9, "q4_k": 10,
         "q6_k": 11, "q8_k": 12}
# resident storage formats
FMT = {"f32": 0, "bf16": 1, "f16": 2, "fp8": 3, "int": 4, "mxfp4": 5, "q8_0": 6, "q4_k": 7}
SCALE_F32, SCALE_BF16 = 0, 1


class DitchCudaError(RuntimeError):
    def __init__(self, code, msg):
        super().__init__(f"ditch_cuda status {code}: {msg}")
        self.code = code


class Unsupported(DitchCudaError):
    pass


class ModelConfig(C.Structure):
    _fields_ = [
        ("n_layers", C.c_int), ("hidden", C.c_int), ("heads", C.c_int), ("kv_heads", C.c_int),
        ("head_dim", C.c_int), ("inter", C.c_int), ("vocab", C.c_int), ("eps", C.c_float),
        ("rope_theta", C.c_double), ("rope_scaling", C.c_int), ("rope_factor", C.c_double),
        ("rope_low_ff", C.c_double), ("rope_high_ff", C.c_double), ("rope_orig_max", C.c_double),
        ("qk_norm", C.c_int), ("n_experts", C.c_int), ("top_k", C.c_int), ("moe_inter", C.c_int),
        ("norm_topk", C.c_int), ("moe_layers", C.POINTER(C.c_uint8)), ("max_seq", C.c_int),
        ("ep_rank", C.c_int), ("ep_world", C.c_int), ("tp_rank", C.c_int), ("tp_world", C.c_int),
        ("rope_factors", C.POINTER(C.c_float)), ("n_rope_factors", C.c_size_t),
        ("rope_attention_factor", C.c_double), ("rope_beta_fast", C.c_double), ("rope_beta_slow", C.c_double),
        ("rope_truncate", C.c_int),
    ]


# spec keys of the RoPE scaling fields beyond the llama3 ones, with their defaults
ROPE_EXTRA = dict(rope_attention_factor=1.0, rope_beta_fast=32.0, rope_beta_slow=1.0, rope_truncate=1)


class TensorDesc(C.Structure):
    _fields_ = [
        ("name", C.c_char_p), ("format", C.c_int), ("slabs", C.c_size_t), ("rows", C.c_size_t),
        ("cols", C.c_size_t), ("data", C.c_void_p), ("data_bytes", C.c_size_t), ("scales", C.c_void_p),
        ("scales_bytes", C.c_size_t), ("scales_dtype", C.c_int), ("zeros", C.c_void_p),
        ("zeros_bytes", C.c_size_t), ("block_rows", C.c_int), ("block_cols", C.c_int), ("bits", C.c_int),
        ("on_device", C.c_int),
    ]


class Params(C.Structure):
    """abliterate.Params (src/abliterate.zig:40-45)."""
    _fields_ = [("max_weight", C.c_float), ("max_weight_position", C.c_float), ("min_weight", C.c_float),
                ("min_weight_distance", C.c_float)]


_lib = None
vp, sz, f32p, f64p, u8p, u16p, u32p, u64p = (C.c_void_p, C.c_size_t, C.POINTER(C.c_float), C.POINTER(C.c_double),
                                             C.POINTER(C.c_uint8), C.POINTER(C.c_uint16), C.POINTER(C.c_uint32),
                                             C.POINTER(C.c_uint64))

# exported entry -> (restype, argtypes); include/ditch_cuda.h declares each
SIGNATURES = {
    "ditch_cuda_last_error": (C.c_char_p, []),
    "ditch_cuda_version": (C.c_char_p, []),
    "ditch_cuda_device_count": (C.c_int, []),
    "ditch_cuda_open": (C.c_int, [C.c_int, C.c_uint64, C.POINTER(vp)]),
    "ditch_cuda_close": (None, [vp]),
    "ditch_cuda_forget_weights": (None, [vp]),
    "ditch_cuda_served": (C.c_uint64, [vp]),
    "ditch_cuda_set_weights_stable": (None, [vp, C.c_int]),
    "ditch_cuda_matmul_t": (C.c_int, [vp, f32p, f32p, sz, u8p, sz, C.c_int, sz, sz]),
    "ditch_cuda_matvec_t_multi": (C.c_int, [vp, f32p, u8p, sz, C.c_int, sz, sz, f32p, sz]),
    "ditch_cuda_row_norms": (C.c_int, [vp, f32p, u8p, sz, C.c_int, sz, sz]),
    "ditch_cuda_attention_scores": (C.c_int, [vp, f32p, sz, f32p, sz, f32p, sz, sz, C.c_float]),
    "ditch_cuda_attention_values": (C.c_int, [vp, f32p, sz, f32p, sz, f32p, sz, sz]),
    "ditch_cuda_gated_activation": (C.c_int, [vp, C.c_uint32, f32p, f32p, f32p, sz, sz, sz, sz]),
    "ditch_cuda_rmsnorm_rows": (C.c_int, [vp, f32p, f32p, f32p, sz, sz, sz, C.c_float, C.c_int]),
    "ditch_cuda_layernorm_rows": (C.c_int, [vp, f32p, f32p, f32p, sz, f32p, sz, sz, C.c_float, C.c_int]),
    "ditch_cuda_softmax_rows": (C.c_int, [vp, f32p, sz, sz]),
    "ditch_cuda_rope_rows": (C.c_int, [vp, f32p, sz, sz, f32p, f32p, sz, sz, u32p, C.c_int]),
    "ditch_cuda_dequant_fp8": (C.c_int, [vp, u8p, f32p, sz, sz, sz, sz, u16p]),
    "ditch_cuda_dequant_int": (C.c_int, [vp, u32p, sz, f32p, sz, u32p, u32p, sz, sz, C.c_int, sz, u16p]),
    "ditch_cuda_dequant_mxfp4": (C.c_int, [vp, u8p, u8p, sz, sz, C.c_int, u16p]),
    "ditch_cuda_dequant_ggml": (C.c_int, [vp, C.c_int, u8p, sz, sz, f32p]),
    "ditch_cuda_model_load": (C.c_int, [vp, C.POINTER(ModelConfig), C.POINTER(TensorDesc), sz, C.POINTER(vp)]),
    "ditch_cuda_model_free": (None, [vp]),
    "ditch_cuda_model_load_checkpoint": (C.c_int, [vp, C.c_char_p, C.c_int, C.POINTER(vp)]),
    "ditch_cuda_checkpoint_inspect": (C.c_int, [C.c_char_p, C.POINTER(ModelConfig), C.POINTER(sz),
                                                C.POINTER(C.c_uint8), sz, f32p, sz]),
    "ditch_cuda_model_bytes": (C.c_uint64, [vp]),
    "ditch_cuda_export_checkpoint": (C.c_int, [vp, C.c_char_p, C.c_char_p, C.c_int, C.c_uint64]),
    "ditch_cuda_export_config": (C.c_int, [C.c_char_p, sz, C.c_int, C.c_int, C.c_char_p, sz, C.POINTER(sz)]),
    "ditch_cuda_model_delta": (C.c_int, [vp, sz, C.c_int, sz, f32p, f32p, sz, C.POINTER(sz)]),
    "ditch_cuda_round_f32": (C.c_int, [vp, f32p, sz, C.c_int, u16p]),
    "ditch_cuda_forward": (C.c_int, [vp, u32p, u32p, u32p, sz, C.POINTER(sz), sz, f32p, C.POINTER(sz), sz, f32p]),
    "ditch_cuda_generate": (C.c_int, [vp, u32p, C.POINTER(sz), sz, sz, u32p, sz, u32p, C.POINTER(sz)]),
    "ditch_cuda_set_row_normalization": (C.c_int, [vp, C.c_int, sz, C.c_uint64]),
    "ditch_cuda_residual_sums": (C.c_int, [vp, u32p, C.POINTER(sz), sz, sz, sz, f64p, u64p]),
    "ditch_cuda_directions": (C.c_int, [vp, f64p, C.c_uint64, f64p, C.c_uint64, C.c_int, f32p]),
    "ditch_cuda_set_directions": (C.c_int, [vp, f32p, sz]),
    "ditch_cuda_apply_edit": (C.c_int, [vp, C.POINTER(Params), C.POINTER(Params), C.c_float, C.c_int]),
    "ditch_cuda_apply_expert_edit": (C.c_int, [vp, C.POINTER(Params), C.POINTER(Params), C.c_float, C.c_int, sz,
                                               C.c_float]),
    "ditch_cuda_reset_edits": (C.c_int, [vp]),
    "ditch_cuda_rank_experts": (C.c_int, [vp, sz, f32p, u32p, f32p]),
    "ditch_cuda_kl_init": (C.c_int, [vp, u32p, C.POINTER(sz), sz]),
    "ditch_cuda_kl_score": (C.c_int, [vp, f64p]),
    "ditch_cuda_kl_score_prompts": (C.c_int, [vp, u32p, C.POINTER(sz), sz, f64p]),
    "ditch_cuda_edit_weight_bf16": (C.c_int, [vp, vp, sz, sz, vp, C.c_float]),
    "ditch_cuda_edit_weight_bf16_noalloc": (C.c_int, [vp, sz, sz, vp, C.c_float, vp]),
    "ditch_cuda_weight_load": (C.c_int, [vp, C.POINTER(TensorDesc), C.POINTER(vp)]),
    "ditch_cuda_weight_free": (None, [vp]),
    "ditch_cuda_weight_format": (C.c_int, [vp]),
    "ditch_cuda_weight_gemm": (C.c_int, [vp, vp, sz, vp, C.c_int]),
    "ditch_cuda_weight_decode": (C.c_int, [vp, vp]),
    "ditch_cuda_set_decode_staging": (C.c_int, [vp, C.c_int]),
    "ditch_cuda_set_deterministic": (C.c_int, [vp, C.c_int]),
    "ditch_cuda_set_f32_split": (C.c_int, [vp, C.c_int]),
    "ditch_cuda_set_cta_pairs": (C.c_int, [vp, C.c_int]),
    "ditch_cuda_set_attention_tc": (C.c_int, [vp, C.c_int]),
    "ditch_cuda_set_decode_cache": (C.c_int, [vp, C.c_int]),
    "ditch_cuda_peer_handle_bytes": (sz, []),
    "ditch_cuda_group_create": (C.c_int, [vp, C.c_int, C.c_int, sz, C.POINTER(vp), vp]),
    "ditch_cuda_group_open": (C.c_int, [vp, vp]),
    "ditch_cuda_group_free": (None, [vp]),
    "ditch_cuda_group_barrier": (C.c_int, [vp]),
    "ditch_cuda_group_set_wait_budget": (C.c_int, [vp, C.c_double]),
    "ditch_cuda_model_group_bytes": (sz, [vp, sz]),
    "ditch_cuda_model_set_group": (C.c_int, [vp, vp, sz]),
    "ditch_cuda_model_dp_group_bytes": (sz, [vp, sz]),
    "ditch_cuda_model_set_dp_group": (C.c_int, [vp, vp]),
    "ditch_cuda_group_allreduce_f64": (C.c_int, [vp, f64p, sz]),
    "ditch_cuda_set_profiling": (C.c_int, [vp, C.c_int]),
    "ditch_cuda_gemm_stats": (C.c_int, [vp, f64p, u64p, f64p]),
    "ditch_cuda_reset_stats": (C.c_int, [vp]),
    "ditch_cuda_launches": (C.c_uint64, [vp]),
    "ditch_cuda_timer_start": (C.c_int, [vp]),
    "ditch_cuda_timer_stop": (C.c_int, [vp, f32p]),
    "ditch_cuda_synchronize": (C.c_int, [vp]),
}


def lib():
    """Loads libditch_cuda.so (built by `make -C ditch_b200`); raises if absent."""
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise ImportError(f"{LIB_PATH} is missing: build it with `make -C ditch_b200`")
        L = C.CDLL(LIB_PATH)
        for name, (res, args) in SIGNATURES.items():
            fn = getattr(L, name)
            fn.restype = res
            fn.argtypes = args
        _lib = L
    return _lib


def check(status):
    if status == OK:
        return
    msg = lib().ditch_cuda_last_error().decode(errors="replace")
    if status == UNSUPPORTED:
        raise Unsupported(status, msg)
    raise DitchCudaError(status, msg)


def _p(a, t):
    if a is None:
        return None
    assert a.flags["C_CONTIGUOUS"]
    return a.ctypes.data_as(t)


def _f32(a):
    return np.ascontiguousarray(a, np.float32)


def _u8(a):
    return np.ascontiguousarray(a).view(np.uint8).reshape(-1)


class Device:
    """A CUDA device behind the compute seam (compute.Device)."""

    def __init__(self, ordinal=0, memory_budget=0):
        h = vp()
        check(lib().ditch_cuda_open(ordinal, memory_budget, C.byref(h)))
        self.h = h
        self.ordinal = ordinal
        self._children = weakref.WeakSet()  # models, weights and groups living on this device

    def _adopt(self, child):
        self._children.add(child)

    def close(self):
        """Closes the models, weights and groups still open on this device
        (their handles point into it), then the device."""
        if self.h:
            for child in list(self._children):
                child.close()
            lib().ditch_cuda_close(self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def __enter__(self):
        return self

    def __exit__(self, *a):
        self.close()

    # ---- VTable entries ----
    def matmul_t(self, x, w_raw, dtype, rows, cols):
        x = _f32(x).reshape(-1, cols)
        w = _u8(w_raw)
        out = np.zeros((x.shape[0], rows), np.float32)
        check(lib().ditch_cuda_matmul_t(self.h, _p(out, f32p), _p(x, f32p), x.shape[0], _p(w, u8p), w.size,
                                        DTYPE[dtype], rows, cols))
        return out

    def matvec_t_multi(self, w_raw, dtype, rows, cols, y):
        y = _f32(y).reshape(-1, rows)
        w = _u8(w_raw)
        out = np.zeros((y.shape[0], cols), np.float32)
        check(lib().ditch_cuda_matvec_t_multi(self.h, _p(out, f32p), _p(w, u8p), w.size, DTYPE[dtype], rows, cols,
                                              _p(y, f32p), y.shape[0]))
        return out

    def row_norms(self, w_raw, dtype, rows, cols):
        w = _u8(w_raw)
        out = np.zeros(rows, np.float32)
        check(lib().ditch_cuda_row_norms(self.h, _p(out, f32p), _p(w, u8p), w.size, DTYPE[dtype], rows, cols))
        return out

    def attention_scores(self, q, k, stride, scale, n_keys):
        q, k = _f32(q), _f32(k).reshape(-1)
        out = np.zeros(n_keys, np.float32)
        check(lib().ditch_cuda_attention_scores(self.h, _p(out, f32p), n_keys, _p(q, f32p), q.size, _p(k, f32p),
                                                k.size, stride, scale))
        return out

    def attention_values(self, scores, v, stride, vd):
        s, v = _f32(scores), _f32(v).reshape(-1)
        out = np.zeros(vd, np.float32)
        check(lib().ditch_cuda_attention_values(self.h, _p(out, f32p), vd, _p(s, f32p), s.size, _p(v, f32p),
                                                v.size, stride))
        return out

    def gated_activation(self, gate, up, n, length, in_stride, out_stride, act=0):
        g = _f32(gate).reshape(-1)
        u = None if up is None else _f32(up).reshape(-1)
        out = np.zeros((n - 1) * out_stride + length, np.float32)
        check(lib().ditch_cuda_gated_activation(self.h, act, _p(out, f32p), _p(g, f32p), _p(u, f32p), n, length,
                                                in_stride, out_stride))
        return out

    def rmsnorm_rows(self, x, weight, eps, gemma_style=False):
        x = _f32(x)
        n, length = x.shape
        w = None if weight is None else _f32(weight)
        out = np.zeros_like(x)
        check(lib().ditch_cuda_rmsnorm_rows(self.h, _p(out, f32p), _p(x, f32p), _p(w, f32p),
                                            0 if w is None else w.size, n, length, eps, int(gemma_style)))
        return out

    def layernorm_rows(self, x, weight, bias, eps, one_plus=False):
        x = _f32(x)
        n, length = x.shape
        w = None if weight is None else _f32(weight)
        b = None if bias is None else _f32(bias)
        out = np.zeros_like(x)
        check(lib().ditch_cuda_layernorm_rows(self.h, _p(out, f32p), _p(x, f32p), _p(w, f32p),
                                              0 if w is None else w.size, _p(b, f32p), n, length, eps,
                                              int(one_plus)))
        return out

    def softmax_rows(self, x):
        x = _f32(x).copy()
        check(lib().ditch_cuda_softmax_rows(self.h, _p(x, f32p), x.shape[0], x.shape[1]))
        return x

    def rope_rows(self, x, cos_t, sin_t, pos, style=0):
        x = _f32(x).copy()
        n, dim = x.shape
        c, s = _f32(cos_t), _f32(sin_t)
        pos = np.ascontiguousarray(pos, np.uint32)
        check(lib().ditch_cuda_rope_rows(self.h, _p(x, f32p), n, dim, _p(c, f32p), _p(s, f32p), c.shape[0],
                                         c.shape[1], _p(pos, u32p), style))
        return x

    # ---- decoders ----
    def dequant_fp8(self, codes, scales, br, bc):
        codes, scales = np.ascontiguousarray(codes, np.uint8), _f32(scales)
        rows, cols = codes.shape
        out = np.zeros((rows, cols), np.uint16)
        check(lib().ditch_cuda_dequant_fp8(self.h, _p(codes, u8p), _p(scales, f32p), rows, cols, br, bc,
                                           _p(out, u16p)))
        return out

    def dequant_int(self, packed, scales, zeros, rows, cols, bits, group, g_idx=None):
        packed = np.ascontiguousarray(packed).view(np.uint32)
        scales = _f32(scales)
        zeros = None if zeros is None else np.ascontiguousarray(zeros).view(np.uint32)
        g_idx = None if g_idx is None else np.ascontiguousarray(g_idx).astype(np.uint32)
        out = np.zeros((rows, cols), np.uint16)
        check(lib().ditch_cuda_dequant_int(self.h, _p(packed, u32p), packed.shape[-1], _p(scales, f32p),
                                           scales.shape[-1], _p(zeros, u32p), _p(g_idx, u32p), rows, cols, bits,
                                           group, _p(out, u16p)))
        return out

    def dequant_mxfp4(self, blocks, scales, rows, cols, transposed=False):
        b = np.ascontiguousarray(blocks, np.uint8)
        s = np.ascontiguousarray(scales, np.uint8)
        out = np.zeros((cols, rows) if transposed else (rows, cols), np.uint16)
        check(lib().ditch_cuda_dequant_mxfp4(self.h, _p(b, u8p), _p(s, u8p), rows, cols, int(transposed),
                                             _p(out, u16p)))
        return out

    def dequant_ggml(self, dtype, raw, n):
        raw = _u8(raw)
        out = np.zeros(n, np.float32)
        check(lib().ditch_cuda_dequant_ggml(self.h, DTYPE[dtype], _p(raw, u8p), raw.size, n, _p(out, f32p)))
        return out

    def edit_weight_bf16(self, w_ptr, rows, cols, r_ptr, alpha):
        """W <- W - alpha r (r^T W) on device memory (pointers as ints)."""
        check(lib().ditch_cuda_edit_weight_bf16(self.h, w_ptr, rows, cols, r_ptr, alpha))

    # ---- timing ----
    def set_decode_staging(self, min_tokens):
        """Dense GEMMs over quantised weights with at least `min_tokens` tokens
        decode the weight once to bf16 scratch; 0 keeps every decode in the GEMM."""
        check(lib().ditch_cuda_set_decode_staging(self.h, int(min_tokens)))

    def set_cta_pairs(self, level):
        """Wide dense bf16 GEMMs on CTA pairs (cta_group::2): 0 never, 1
        single-accumulator products, 2 the SwiGLU products too."""
        check(lib().ditch_cuda_set_cta_pairs(self.h, int(level)))

    def set_attention_tc(self, level):
        """Prefill attention of prompts up to 128 tokens on tcgen05: 0 never
        (the mma.sync kernel), 1 one CTA per (prompt, kv head), 2 (default)
        two CTAs per SM for prompts of at most 64 tokens."""
        check(lib().ditch_cuda_set_attention_tc(self.h, int(level)))

    def set_f32_split(self, on):
        """Models loaded afterwards run f32-level split-bf16 products for their
        f32 / f16 weights (three times the tensor-core work)."""
        check(lib().ditch_cuda_set_f32_split(self.h, int(bool(on))))

    def set_decode_cache(self, on):
        """Staged GEMMs keep their weight's decoded bf16 copy (default on)."""
        check(lib().ditch_cuda_set_decode_cache(self.h, int(bool(on))))

    def round_f32(self, values, dtype):
        """The export's rounding of f32 values to "bf16" or "f16" bits."""
        v = np.ascontiguousarray(values, np.float32).reshape(-1)
        out = np.zeros(v.size, np.uint16)
        check(lib().ditch_cuda_round_f32(self.h, _p(v, f32p), v.size, DTYPE[dtype], _p(out, u16p)))
        return out.reshape(np.shape(values))

    def set_deterministic(self, on):
        """K splits summed in a fixed order instead of atomically (default off)."""
        check(lib().ditch_cuda_set_deterministic(self.h, int(bool(on))))

    def set_profiling(self, on):
        check(lib().ditch_cuda_set_profiling(self.h, int(on)))

    def gemm_stats(self):
        ms, n, fl = C.c_double(), C.c_uint64(), C.c_double()
        check(lib().ditch_cuda_gemm_stats(self.h, C.byref(ms), C.byref(n), C.byref(fl)))
        return ms.value, n.value, fl.value

    def reset_stats(self):
        check(lib().ditch_cuda_reset_stats(self.h))

    def launches(self):
        return int(lib().ditch_cuda_launches(self.h))

    def served(self):
        return int(lib().ditch_cuda_served(self.h))

    def timer_start(self):
        check(lib().ditch_cuda_timer_start(self.h))

    def timer_stop(self):
        ms = C.c_float()
        check(lib().ditch_cuda_timer_stop(self.h, C.byref(ms)))
        return ms.value

    def synchronize(self):
        check(lib().ditch_cuda_synchronize(self.h))


class Tensor:
    """One entry of the model's tensor table (ditch_cuda_tensor)."""

    def __init__(self, name, fmt, rows, cols, data, slabs=1, scales=None, scales_dtype=SCALE_F32, zeros=None,
                 block_rows=0, block_cols=0, bits=0):
        self.name, self.fmt, self.rows, self.cols, self.slabs = name, fmt, rows, cols, slabs
        self.data, self.scales, self.zeros = data, scales, zeros
        self.scales_dtype, self.block_rows, self.block_cols, self.bits = scales_dtype, block_rows, block_cols, bits

    @staticmethod
    def _ref(a, keep):
        """(pointer, bytes, on_device) of a numpy array or a CUDA torch tensor;
        the array whose memory the pointer names (a contiguous copy when `a`
        is not contiguous) goes into `keep`, which outlives the C call."""
        if a is None:
            return None, 0, 0
        if hasattr(a, "data_ptr"):  # torch tensor on the device
            keep.append(a)
            return a.data_ptr(), a.numel() * a.element_size(), 1 if a.is_cuda else 0
        a = np.ascontiguousarray(a)
        keep.append(a)
        return a.ctypes.data, a.nbytes, 0

    def desc(self, keep):
        d, db, dev = self._ref(self.data, keep)
        s, sb, _ = self._ref(self.scales, keep)
        z, zb, _ = self._ref(self.zeros, keep)
        name = self.name.encode()
        keep.append(name)
        return TensorDesc(name, FMT[self.fmt], self.slabs, self.rows, self.cols, d, db, s, sb, self.scales_dtype, z,
                          zb, self.block_rows, self.block_cols, self.bits, dev)


class Weight:
    """One resident weight and its dequant-fused GEMM (device pointers in/out)."""

    FORMATS = {0: "bf16", 1: "fp8", 2: "mxfp4", 3: "int4", 4: "q8_0", 5: "q4_k"}

    def __init__(self, device, tensor):
        self.dev = device
        keep = []
        d = tensor.desc(keep)
        h = vp()
        check(lib().ditch_cuda_weight_load(device.h, C.byref(d), C.byref(h)))
        self.h = h
        self.rows, self.cols = tensor.rows, tensor.cols
        device._adopt(self)

    def format(self):
        return self.FORMATS.get(lib().ditch_cuda_weight_format(self.h), "?")

    def gemm(self, x_ptr, m, out_ptr, k_splits=1):
        """out[m][rows] (f32) = x[m][cols] (bf16) . W^T, asynchronous on the device stream."""
        check(lib().ditch_cuda_weight_gemm(self.h, x_ptr, m, out_ptr, k_splits))

    def decode(self, out_ptr):
        check(lib().ditch_cuda_weight_decode(self.h, out_ptr))

    def close(self):
        if self.h:
            lib().ditch_cuda_weight_free(self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


class Group:
    """One rank's share of a peer group (GPUs of one node over NVLink).

    `exchange(handle_bytes) -> list of every rank's handle bytes` is the host
    transport (e.g. torch.distributed.all_gather_object)."""

    def __init__(self, device, rank, world, nbytes, exchange):
        self.dev = device
        n = int(lib().ditch_cuda_peer_handle_bytes())
        buf = (C.c_uint8 * n)()
        h = vp()
        check(lib().ditch_cuda_group_create(device.h, rank, world, nbytes, C.byref(h), C.cast(buf, vp)))
        self.h = h
        handles = exchange(bytes(buf))
        allh = (C.c_uint8 * (n * world)).from_buffer_copy(b"".join(handles))
        check(lib().ditch_cuda_group_open(self.h, C.cast(allh, vp)))
        device._adopt(self)

    def barrier(self):
        check(lib().ditch_cuda_group_barrier(self.h))

    def set_wait_budget(self, seconds):
        """Budget of every wait of the group's exchanges (30 s by default)."""
        check(lib().ditch_cuda_group_set_wait_budget(self.h, float(seconds)))

    def allreduce_f64(self, values):
        """Every rank's f64 array summed over the group (rank order, the same
        bits on every rank); returns a new array."""
        out = np.array(values, np.float64, copy=True).reshape(-1)
        check(lib().ditch_cuda_group_allreduce_f64(self.h, _p(out, f64p), out.size))
        return out.reshape(np.shape(values))

    def close(self):
        if self.h:
            lib().ditch_cuda_group_free(self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


def inspect_checkpoint(path):
    """The model spec and tensor count ditch_cuda_model_load_checkpoint would
    use for a Hugging Face directory or a GGUF file (no device needed)."""
    cfg = ModelConfig()
    n = sz(0)
    flags = (C.c_uint8 * 4096)()
    factors = np.zeros(4096, np.float32)
    check(lib().ditch_cuda_checkpoint_inspect(str(path).encode(), C.byref(cfg), C.byref(n), flags, 4096,
                                              _p(factors, f32p), factors.size))
    spec = dict(n_layers=cfg.n_layers, hidden=cfg.hidden, heads=cfg.heads, kv_heads=cfg.kv_heads,
                head_dim=cfg.head_dim, inter=cfg.inter, vocab=cfg.vocab, eps=cfg.eps, rope_theta=cfg.rope_theta,
                rope_scaling=cfg.rope_scaling, rope_factor=cfg.rope_factor, rope_low_ff=cfg.rope_low_ff,
                rope_high_ff=cfg.rope_high_ff, rope_orig_max=cfg.rope_orig_max, qk_norm=cfg.qk_norm)
    if cfg.rope_scaling in (3, 4):
        spec.update({k: getattr(cfg, k) for k in ROPE_EXTRA})
    if cfg.n_rope_factors:
        spec["rope_factors"] = factors[: cfg.n_rope_factors].copy()
    if cfg.n_experts:
        spec.update(n_experts=cfg.n_experts, top_k=cfg.top_k, moe_inter=cfg.moe_inter, norm_topk=cfg.norm_topk,
                    moe_layers=[bool(flags[i]) for i in range(cfg.n_layers)])
    return spec, n.value


def export_config(text, dtype=None, strip_quantization_config=False):
    """The config.json text an export writes (ditch_cuda_export_config)."""
    raw = text.encode()
    n = sz(0)
    code = -1 if dtype is None else DTYPE[dtype]
    check(lib().ditch_cuda_export_config(raw, len(raw), code, int(strip_quantization_config), None, 0, C.byref(n)))
    buf = C.create_string_buffer(n.value + 1)
    check(lib().ditch_cuda_export_config(raw, len(raw), code, int(strip_quantization_config), buf, n.value, C.byref(n)))
    return buf.raw[: n.value].decode()


COMPONENTS = {"attn_o_proj": 0, "mlp_down_proj": 1, "expert_down_proj": 2}


class Model:
    """A model resident in HBM (the coarse C-ABI entries)."""

    @classmethod
    def from_checkpoint(cls, device, path, max_seq=4096):
        """Loads a Hugging Face directory or a GGUF file
        (ditch_cuda_model_load_checkpoint)."""
        spec, _ = inspect_checkpoint(path)
        self = cls.__new__(cls)
        self.dev, self.spec, self._moe = device, spec, None
        h = vp()
        check(lib().ditch_cuda_model_load_checkpoint(device.h, str(path).encode(), int(max_seq), C.byref(h)))
        self.h = h
        self.source = str(path)
        device._adopt(self)
        return self

    def export(self, out_dir, source=None, dtype=None, max_shard_bytes=0):
        """Writes the checkpoint with this model's deltas merged
        (ditch_cuda_export_checkpoint); `source` defaults to the directory
        the model was loaded from, `dtype` ("f32", "f16", "bf16") to each
        tensor's own."""
        src = source or getattr(self, "source", None)
        if src is None:
            raise ValueError("no source checkpoint: pass source=")
        check(lib().ditch_cuda_export_checkpoint(self.h, str(src).encode(), str(out_dir).encode(),
                                                 -1 if dtype is None else DTYPE[dtype], int(max_shard_bytes)))

    def delta(self, layer, component, expert=0):
        """(a [rank][cols], b [rows][rank]) of an edited weight, or None."""
        s = self.spec
        comp = COMPONENTS[component]
        cols = {0: s["heads"] * s["head_dim"], 1: s.get("inter", 0), 2: s.get("moe_inter", 0)}[comp]
        a = np.zeros((4, max(cols, 1)), np.float32)
        b = np.zeros((s["hidden"], 4), np.float32)
        r = sz(0)
        check(lib().ditch_cuda_model_delta(self.h, layer, comp, expert, _p(a, f32p), _p(b, f32p), 4, C.byref(r)))
        if r.value == 0:
            return None
        k = r.value
        a = np.ascontiguousarray(a.reshape(-1)[: k * cols].reshape(k, cols))
        b = np.ascontiguousarray(b.reshape(-1)[: s["hidden"] * k].reshape(s["hidden"], k))
        return a, b

    def __init__(self, device, spec, tensors, max_seq=4096, ep_rank=0, ep_world=1, tp_rank=0, tp_world=1):
        self.dev = device
        self.spec = spec
        cfg = ModelConfig(
            n_layers=spec["n_layers"], hidden=spec["hidden"], heads=spec["heads"], kv_heads=spec["kv_heads"],
            head_dim=spec["head_dim"], inter=spec.get("inter", 0), vocab=spec["vocab"], eps=spec["eps"],
            rope_theta=spec["rope_theta"], rope_scaling=int(spec.get("rope_scaling", 0)),
            rope_factor=spec.get("rope_factor", 1.0), rope_low_ff=spec.get("rope_low_ff", 1.0),
            rope_high_ff=spec.get("rope_high_ff", 1.0), rope_orig_max=spec.get("rope_orig_max", 1.0),
            qk_norm=int(spec.get("qk_norm", 0)), n_experts=spec.get("n_experts", 0), top_k=spec.get("top_k", 0),
            moe_inter=spec.get("moe_inter", 0), norm_topk=int(spec.get("norm_topk", 1)), max_seq=max_seq,
            ep_rank=ep_rank, ep_world=ep_world, tp_rank=tp_rank, tp_world=tp_world,
            **{k: spec.get(k, v) for k, v in ROPE_EXTRA.items()})
        self._rope = None
        if spec.get("rope_factors") is not None:
            self._rope = np.ascontiguousarray(spec["rope_factors"], np.float32)
            cfg.rope_factors = _p(self._rope, f32p)
            cfg.n_rope_factors = self._rope.size
        self._moe = None
        if spec.get("moe_layers"):
            self._moe = np.array([1 if x else 0 for x in spec["moe_layers"]], np.uint8)
            cfg.moe_layers = self._moe.ctypes.data_as(C.POINTER(C.c_uint8))
        keep = []
        descs = (TensorDesc * len(tensors))(*[t.desc(keep) for t in tensors])
        h = vp()
        check(lib().ditch_cuda_model_load(device.h, C.byref(cfg), descs, len(tensors), C.byref(h)))
        self.h = h
        device._adopt(self)

    def close(self):
        if self.h:
            lib().ditch_cuda_model_free(self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def bytes(self):
        return int(lib().ditch_cuda_model_bytes(self.h))

    def group_bytes(self, max_tokens):
        """Peer-group region bytes this expert- or tensor-parallel model needs."""
        return int(lib().ditch_cuda_model_group_bytes(self.h, max_tokens))

    def set_group(self, group, max_tokens):
        """Runs the model expert- or tensor-parallel (as loaded) over `group`."""
        check(lib().ditch_cuda_model_set_group(self.h, group.h, max_tokens))
        self._group = group  # the group outlives the model's use of it

    def dp_group_bytes(self, max_prompts):
        """Peer-group region bytes the data-parallel reductions need."""
        return int(lib().ditch_cuda_model_dp_group_bytes(self.h, max_prompts))

    def set_dp_group(self, group):
        """Residual sums and KL combined over `group`'s ranks (None detaches)."""
        check(lib().ditch_cuda_model_set_dp_group(self.h, group.h if group else None))
        self._dp_group = group

    def forward(self, tokens, row_b, row_pos, capture_rows=(), logit_rows=()):
        s = self.spec
        tokens = np.ascontiguousarray(tokens, np.uint32)
        rb = np.ascontiguousarray(row_b, np.uint32)
        rp = np.ascontiguousarray(row_pos, np.uint32)
        cap = np.ascontiguousarray(capture_rows, np.uintp)
        lr = np.ascontiguousarray(logit_rows, np.uintp)
        res = np.zeros((s["n_layers"] + 1, len(cap), s["hidden"]), np.float32)
        logits = np.zeros((len(lr), s["vocab"]), np.float32)
        check(lib().ditch_cuda_forward(self.h, _p(tokens, u32p), _p(rb, u32p), _p(rp, u32p), len(tokens),
                                       _p(cap, C.POINTER(sz)) if len(cap) else None, len(cap),
                                       _p(res, f32p) if len(cap) else None,
                                       _p(lr, C.POINTER(sz)) if len(lr) else None, len(lr),
                                       _p(logits, f32p) if len(lr) else None))
        return res, logits

    @staticmethod
    def _flat(prompts):
        tokens = np.ascontiguousarray(np.concatenate([np.asarray(p, np.uint32) for p in prompts]), np.uint32)
        offs = np.zeros(len(prompts) + 1, np.uintp)
        offs[1:] = np.cumsum([len(p) for p in prompts])
        return tokens, offs

    def set_row_normalization(self, mode, lora_rank=3, seed=0):
        """Options.row_normalization of the following edits: "none", "pre" or
        "full" (a rank-`lora_rank` delta from a randomised SVD seeded with
        `seed` + the matrix's index)."""
        code = {"none": 0, "pre": 1, "full": 2}[mode]
        check(lib().ditch_cuda_set_row_normalization(self.h, code, int(lora_rank), int(seed)))

    def generate(self, prompts, max_new_tokens, eos_ids=()):
        """Greedy generation (model.generate, src/model.zig:5359-5444): a list
        of token lists, one per prompt, each ending at its first EOS token
        (kept) or after max_new_tokens tokens (at least one)."""
        tokens, offs = self._flat(prompts)
        eos = np.ascontiguousarray(eos_ids, np.uint32)
        stride = max(int(max_new_tokens), 1)
        out = np.zeros((len(prompts), stride), np.uint32)
        counts = np.zeros(len(prompts), np.uintp)
        check(lib().ditch_cuda_generate(self.h, _p(tokens, u32p), _p(offs, C.POINTER(sz)), len(prompts),
                                        int(max_new_tokens), _p(eos, u32p) if len(eos) else None, len(eos),
                                        _p(out, u32p), _p(counts, C.POINTER(sz))))
        return [out[i, :counts[i]].tolist() for i in range(len(prompts))]

    def residual_sums(self, prompts, window=1, batch_size=0):
        s = self.spec
        tokens, offs = self._flat(prompts)
        sums = np.zeros((s["n_layers"] + 1, s["hidden"]), np.float64)
        count = C.c_uint64(0)
        check(lib().ditch_cuda_residual_sums(self.h, _p(tokens, u32p), _p(offs, C.POINTER(sz)), len(prompts), window,
                                             batch_size, _p(sums, f64p), C.byref(count)))
        return sums, count.value

    def directions(self, good_sums, good_count, bad_sums, bad_count, orthogonalize=True):
        s = self.spec
        g = np.ascontiguousarray(good_sums, np.float64)
        b = np.ascontiguousarray(bad_sums, np.float64)
        dirs = np.zeros((s["n_layers"] + 1, s["hidden"]), np.float32)
        check(lib().ditch_cuda_directions(self.h, _p(g, f64p), good_count, _p(b, f64p), bad_count,
                                          int(orthogonalize), _p(dirs, f32p)))
        return dirs

    def set_directions(self, dirs):
        d = _f32(dirs)
        check(lib().ditch_cuda_set_directions(self.h, _p(d, f32p), d.shape[0]))

    @staticmethod
    def _params(p):
        return None if p is None else C.byref(Params(*p))

    def apply_edit(self, attn_o=None, mlp_down=None, direction_index=None):
        di = -1.0 if direction_index is None else float(direction_index)
        check(lib().ditch_cuda_apply_edit(self.h, self._params(attn_o), self._params(mlp_down), di,
                                          int(direction_index is not None)))

    def apply_expert_edit(self, attn_o=None, mlp_down=None, direction_index=None, n_experts=0, strength=1.0):
        di = -1.0 if direction_index is None else float(direction_index)
        check(lib().ditch_cuda_apply_expert_edit(self.h, self._params(attn_o), self._params(mlp_down), di,
                                                 int(direction_index is not None), n_experts, strength))

    def reset_edits(self):
        check(lib().ditch_cuda_reset_edits(self.h))

    def rank_experts(self, layer, v):
        E = self.spec["n_experts"]
        v = _f32(v)
        order = np.zeros(E, np.uint32)
        scores = np.zeros(E, np.float32)
        check(lib().ditch_cuda_rank_experts(self.h, layer, _p(v, f32p), _p(order, u32p), _p(scores, f32p)))
        return order, scores

    def kl_init(self, prompts):
        tokens, offs = self._flat(prompts)
        check(lib().ditch_cuda_kl_init(self.h, _p(tokens, u32p), _p(offs, C.POINTER(sz)), len(prompts)))

    def kl_score(self):
        v = C.c_double()
        check(lib().ditch_cuda_kl_score(self.h, C.byref(v)))
        return v.value

    def kl_score_prompts(self, tokens, offs, n_prompts):
        """KL with the prompts uploaded from host memory (flattened form)."""
        v = C.c_double()
        check(lib().ditch_cuda_kl_score_prompts(self.h, _p(tokens, u32p), _p(offs, C.POINTER(sz)), n_prompts,
                                                C.byref(v)))
        return v.value
