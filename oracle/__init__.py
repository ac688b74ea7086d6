"""ctypes bindings of the CPU oracle (``libditch_oracle.so``).

TEST INFRASTRUCTURE ONLY: the oracle is the parity checker for the CUDA
product and the timed CPU baseline. Only ``tests/``, ``__graft_entry__.smoke()``
and ``bench.py``'s CPU-baseline leg import this package.
"""
import ctypes as C
import os

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))
_LIB = None

f32p = C.POINTER(C.c_float)
u16p = C.POINTER(C.c_uint16)
u8p = C.POINTER(C.c_uint8)
u32p = C.POINTER(C.c_uint32)
f64p = C.POINTER(C.c_double)
szp = C.POINTER(C.c_size_t)


class Config(C.Structure):
    _fields_ = [
        ("n_layers", C.c_int), ("hidden", C.c_int), ("heads", C.c_int), ("kv_heads", C.c_int),
        ("head_dim", C.c_int), ("inter", C.c_int), ("vocab", C.c_int), ("eps", C.c_float),
        ("rope_theta", C.c_double), ("qk_norm", C.c_int), ("rope_scaling", C.c_int),
        ("rope_factor", C.c_double), ("rope_low_ff", C.c_double), ("rope_high_ff", C.c_double),
        ("rope_orig_max", C.c_double), ("n_experts", C.c_int), ("top_k", C.c_int),
        ("moe_inter", C.c_int), ("norm_topk", C.c_int),
        ("rope_factors", f32p), ("n_rope_factors", C.c_size_t), ("rope_attention_factor", C.c_double),
        ("rope_beta_fast", C.c_double), ("rope_beta_slow", C.c_double), ("rope_truncate", C.c_int),
    ]


class Layer(C.Structure):
    _fields_ = [
        ("input_norm", f32p), ("post_norm", f32p),
        ("q", f32p), ("k", f32p), ("v", f32p), ("o", f32p),
        ("qb", f32p), ("kb", f32p), ("vb", f32p),
        ("q_norm", f32p), ("k_norm", f32p),
        ("gate", f32p), ("up", f32p), ("down", f32p),
        ("router", f32p), ("e_gate", f32p), ("e_up", f32p), ("e_down", f32p),
        ("o_da", f32p), ("o_db", f32p), ("o_rank", C.c_size_t),
        ("down_da", f32p), ("down_db", f32p), ("down_rank", C.c_size_t),
        ("e_down_da", C.POINTER(f32p)), ("e_down_db", C.POINTER(f32p)),
        ("e_down_rank", szp),
    ]


class Model(C.Structure):
    _fields_ = [("c", Config), ("embed", f32p), ("final_norm", f32p), ("lm_head", f32p),
                ("layers", C.POINTER(Layer)), ("w_bf16", C.c_int)]


class Params(C.Structure):
    _fields_ = [("max_weight", C.c_float), ("max_weight_position", C.c_float),
                ("min_weight", C.c_float), ("min_weight_distance", C.c_float)]


def lib():
    """Loads the oracle library (built by ``make -C oracle``)."""
    global _LIB
    if _LIB is None:
        path = os.path.join(_HERE, "libditch_oracle.so")
        if not os.path.exists(path):
            raise RuntimeError("oracle not built: run `make -C oracle`")
        L = C.CDLL(path)
        L.or_f32_to_bf16.restype = C.c_uint16
        L.or_f32_to_bf16.argtypes = [C.c_float]
        L.or_bf16_to_f32.restype = C.c_float
        L.or_bf16_to_f32.argtypes = [C.c_uint16]
        L.or_f16_to_f32.restype = C.c_float
        L.or_f16_to_f32.argtypes = [C.c_uint16]
        L.or_dot.restype = C.c_float
        L.or_dot.argtypes = [f32p, f32p, C.c_size_t]
        L.or_matmul_t.argtypes = [f32p, f32p, C.c_size_t, f32p, C.c_size_t, C.c_size_t, f32p, f32p, C.c_size_t]
        L.or_matvec_t_multi.argtypes = [f32p, f32p, C.c_size_t, C.c_size_t, f32p, C.c_size_t]
        L.or_row_norms.argtypes = [f32p, f32p, C.c_size_t, C.c_size_t]
        L.or_rmsnorm.argtypes = [f32p, f32p, f32p, C.c_size_t, C.c_float]
        L.or_softmax_inplace.argtypes = [f32p, C.c_size_t]
        L.or_log_softmax.argtypes = [f32p, f32p, C.c_size_t]
        L.or_gated_silu.argtypes = [f32p, f32p, f32p, C.c_size_t, C.c_size_t, C.c_size_t, C.c_size_t]
        L.or_rope_table.argtypes = [f32p, f32p, C.c_size_t, C.c_size_t, C.c_double, C.c_int,
                                    C.c_double, C.c_double, C.c_double, C.c_double]
        L.or_dequant_ggml.restype = C.c_int
        L.or_dequant_ggml.argtypes = [C.c_int, u8p, f32p, C.c_size_t]
        L.or_ggml_block_size.restype = C.c_size_t
        L.or_ggml_block_size.argtypes = [C.c_int]
        L.or_ggml_block_bytes.restype = C.c_size_t
        L.or_ggml_block_bytes.argtypes = [C.c_int]
        L.or_quant_q8_0.argtypes = [f32p, u8p, C.c_size_t]
        L.or_quant_q4_k.argtypes = [f32p, u8p, C.c_size_t]
        L.or_e4m3_value.restype = C.c_float
        L.or_e4m3_value.argtypes = [C.c_uint8]
        L.or_e8m0_scale.restype = C.c_float
        L.or_e8m0_scale.argtypes = [C.c_uint8]
        L.or_dequant_fp8.argtypes = [u8p, f32p, C.c_size_t, C.c_size_t, C.c_size_t, C.c_size_t, u16p]
        L.or_dequant_int_packed.argtypes = [u32p, C.c_size_t, f32p, u32p, u32p, C.c_size_t,
                                            C.c_size_t, C.c_int, C.c_size_t, u16p]
        L.or_dequant_mxfp4_packed.argtypes = [u8p, u8p, C.c_size_t, C.c_size_t, u16p]
        L.or_dequant_mxfp4_transposed.argtypes = [u8p, u8p, C.c_size_t, C.c_size_t, u16p]
        L.or_unpack_field.restype = C.c_uint32
        L.or_unpack_field.argtypes = [u32p, C.c_size_t, C.c_int]
        L.or_quant_fp8_block.argtypes = [f32p, C.c_size_t, C.c_size_t, C.c_size_t, C.c_size_t, u8p, f32p]
        L.or_quant_mxfp4_packed.argtypes = [f32p, C.c_size_t, C.c_size_t, u8p, u8p]
        L.or_quant_int_packed.argtypes = [f32p, C.c_size_t, C.c_size_t, C.c_int, C.c_size_t, u32p, f32p, u32p]
        L.or_forward.restype = C.c_int
        L.or_forward.argtypes = [C.POINTER(Model), u32p, u32p, u32p, C.c_size_t, szp, C.c_size_t,
                                 f32p, szp, C.c_size_t, f32p]
        L.or_kernel_weight.restype = C.c_int
        L.or_kernel_weight.argtypes = [Params, C.c_size_t, f32p]
        L.or_compute_directions.argtypes = [f32p, f32p, C.c_size_t, C.c_size_t, C.c_int, f32p]
        L.or_compute_delta_none.argtypes = [f32p, C.c_size_t, C.c_size_t, f32p, C.c_float, f32p, f32p]
        L.or_materialize.argtypes = [f32p, C.c_size_t, C.c_size_t, f32p, f32p, C.c_size_t, f32p]
        L.or_score_down.restype = C.c_float
        L.or_score_down.argtypes = [f32p, C.c_size_t, C.c_size_t, f32p]
        L.or_rank_scores.argtypes = [f32p, C.c_size_t, u32p]
        L.or_residual_sums.argtypes = [f32p, C.c_size_t, C.c_size_t, C.c_size_t, szp, szp, C.c_size_t, f64p]
        L.or_kl_first_token.restype = C.c_double
        L.or_kl_first_token.argtypes = [f32p, f32p, C.c_size_t, C.c_size_t, f64p]
        L.or_f32_to_bf16_array.argtypes = [f32p, C.c_size_t, u16p]
        L.or_matmul_t_bf16.argtypes = [f32p, f32p, C.c_size_t, u16p, C.c_size_t, C.c_size_t, f32p, f32p,
                                       C.c_size_t]
        L.or_set_threads.argtypes = [C.c_int]
        L.or_get_threads.restype = C.c_int
        _LIB = L
    return _LIB


def ptr(a, t=f32p):
    """Pointer to a C-contiguous numpy array (None stays NULL)."""
    if a is None:
        return None
    assert a.flags["C_CONTIGUOUS"], "array must be C-contiguous"
    return a.ctypes.data_as(t)


def f32(a):
    return np.ascontiguousarray(a, dtype=np.float32)


# ---- thin numpy wrappers --------------------------------------------------

def bf16_bits_to_f32(bits):
    return (np.asarray(bits, np.uint16).astype(np.uint32) << 16).view(np.float32)


def f32_to_bf16_bits(x):
    """src/tensor.zig:423-430 (round to nearest even, NaN kept quiet): in C
    over all threads for large arrays, in numpy otherwise."""
    x = np.ascontiguousarray(x, np.float32)
    if x.size >= (1 << 20):
        out = np.empty(x.shape, np.uint16)
        lib().or_f32_to_bf16_array(ptr(x), x.size, ptr(out, u16p))
        return out
    b = x.view(np.uint32)
    nan = (b & 0x7FFFFFFF) > 0x7F800000
    r = ((b + np.uint32(0x7FFF) + ((b >> 16) & 1)) >> 16).astype(np.uint16)
    return np.where(nan, ((b >> 16) | 0x40).astype(np.uint16), r)


def matmul_t(x, w, da=None, db=None):
    x, w = f32(x), f32(w)
    n, cols = x.shape
    rows = w.shape[0]
    out = np.zeros((n, rows), np.float32)
    rank = 0 if da is None else da.reshape(-1, cols).shape[0]
    da = None if da is None else f32(da)
    db = None if db is None else f32(db)
    lib().or_matmul_t(ptr(out), ptr(x), n, ptr(w), rows, cols, ptr(da), ptr(db), rank)
    return out


def matmul_t_bf16(x, w_bits):
    """matmulT over bf16 weights (bit array [rows][cols]) through ditch's
    half-precision path (src/tensor.zig:827-883, 449-486)."""
    x = f32(x)
    w_bits = np.ascontiguousarray(w_bits, np.uint16)
    n, rows = x.shape[0], w_bits.shape[0]
    out = np.zeros((n, rows), np.float32)
    lib().or_matmul_t_bf16(ptr(out), ptr(x), n, ptr(w_bits, u16p), rows, w_bits.shape[1], None, None, 0)
    return out


def matvec_t_multi(w, y):
    w, y = f32(w), f32(y).reshape(-1, w.shape[0])
    out = np.zeros((y.shape[0], w.shape[1]), np.float32)
    lib().or_matvec_t_multi(ptr(out), ptr(w), w.shape[0], w.shape[1], ptr(y), y.shape[0])
    return out


def row_norms(w):
    w = f32(w)
    out = np.zeros(w.shape[0], np.float32)
    lib().or_row_norms(ptr(out), ptr(w), w.shape[0], w.shape[1])
    return out


def dequant_ggml(dtype, raw, n):
    raw = np.ascontiguousarray(raw, np.uint8)
    out = np.zeros(n, np.float32)
    if lib().or_dequant_ggml(dtype, ptr(raw, u8p), ptr(out), n) != 0:
        raise ValueError("bad ggml dtype or size")
    return out


def quant_q8_0(x):
    x = f32(x).ravel()
    out = np.zeros(x.size // 32 * 34, np.uint8)
    lib().or_quant_q8_0(ptr(x), ptr(out, u8p), x.size)
    return out


def quant_q4_k(x):
    x = f32(x).ravel()
    out = np.zeros(x.size // 256 * 144, np.uint8)
    lib().or_quant_q4_k(ptr(x), ptr(out, u8p), x.size)
    return out


def dequant_fp8(codes, scales, br, bc):
    codes = np.ascontiguousarray(codes, np.uint8)
    scales = f32(scales)
    rows, cols = codes.shape
    out = np.zeros((rows, cols), np.uint16)
    lib().or_dequant_fp8(ptr(codes, u8p), ptr(scales), rows, cols, br, bc, ptr(out, u16p))
    return out


def dequant_int_packed(packed, scales, zeros, rows, cols, bits, group, g_idx=None):
    packed = np.ascontiguousarray(packed).view(np.uint32)
    scales = f32(scales)
    zeros = None if zeros is None else np.ascontiguousarray(zeros).view(np.uint32)
    g_idx = None if g_idx is None else np.ascontiguousarray(g_idx).astype(np.uint32)
    out = np.zeros((rows, cols), np.uint16)
    lib().or_dequant_int_packed(ptr(packed, u32p), packed.shape[-1], ptr(scales), ptr(zeros, u32p),
                                ptr(g_idx, u32p), rows, cols, bits, group, ptr(out, u16p))
    return out


def dequant_mxfp4_packed(blocks, scales, rows, cols):
    blocks = np.ascontiguousarray(blocks, np.uint8)
    scales = np.ascontiguousarray(scales, np.uint8)
    out = np.zeros((rows, cols), np.uint16)
    lib().or_dequant_mxfp4_packed(ptr(blocks, u8p), ptr(scales, u8p), rows, cols, ptr(out, u16p))
    return out


def quant_fp8_block(w, br=128, bc=128):
    w = f32(w)
    rows, cols = w.shape
    codes = np.zeros((rows, cols), np.uint8)
    scales = np.zeros((-(-rows // br), -(-cols // bc)), np.float32)
    lib().or_quant_fp8_block(ptr(w), rows, cols, br, bc, ptr(codes, u8p), ptr(scales))
    return codes, scales


def quant_mxfp4_packed(w):
    w = f32(w)
    rows, cols = w.shape
    blocks = np.zeros((rows, cols // 2), np.uint8)
    scales = np.zeros((rows, cols // 32), np.uint8)
    lib().or_quant_mxfp4_packed(ptr(w), rows, cols, ptr(blocks, u8p), ptr(scales, u8p))
    return blocks, scales


def quant_int_packed(w, bits=4, group=128):
    w = f32(w)
    rows, cols = w.shape
    wpr = -(-cols * bits // 32)
    packed = np.zeros((rows, wpr), np.uint32)
    scales = np.zeros((rows, cols // group), np.float32)
    zeros = np.zeros((-(-rows * bits // 32), cols // group), np.uint32)
    lib().or_quant_int_packed(ptr(w), rows, cols, bits, group, ptr(packed, u32p), ptr(scales), ptr(zeros, u32p))
    return packed, scales, zeros


def kernel_weight(p, layer):
    out = C.c_float(0)
    ok = lib().or_kernel_weight(Params(*p), layer, C.byref(out))
    return float(out.value) if ok else None


def compute_directions(good, bad, orthogonalize=True):
    good, bad = f32(good), f32(bad)
    entries, hidden = good.shape
    out = np.zeros_like(good)
    lib().or_compute_directions(ptr(good), ptr(bad), entries, hidden, int(orthogonalize), ptr(out))
    return out


def compute_delta_none(w, v, lam):
    w, v = f32(w), f32(v)
    a = np.zeros(w.shape[1], np.float32)
    b = np.zeros(w.shape[0], np.float32)
    lib().or_compute_delta_none(ptr(w), w.shape[0], w.shape[1], ptr(v), lam, ptr(a), ptr(b))
    return a, b


def compute_delta_pre(w, v, lam):
    """computeOutputDelta with row_normalization = pre, K = 1
    (src/abliterate.zig:305-323): n = rowNorms(W), vn = v / n (0 where n is
    0), a = vn^T W, b = -lam v n, in ditch's f32 order."""
    w, v = f32(w), f32(v)
    n = row_norms(w)
    with np.errstate(divide="ignore", invalid="ignore"):
        vn = np.where(n > 0, v / n, np.float32(0)).astype(np.float32)
    a = matvec_t_multi(w, vn[None, :])[0].astype(np.float32)
    b = ((np.float32(-lam) * v) * n).astype(np.float32)
    return a, b


def materialize(w, a, b):
    w = f32(w)
    a, b = f32(a).reshape(-1, w.shape[1]), f32(b).reshape(w.shape[0], -1)
    out = np.zeros_like(w)
    lib().or_materialize(ptr(w), w.shape[0], w.shape[1], ptr(a), ptr(b), a.shape[0], ptr(out))
    return out


def score_down(w, v):
    w, v = f32(w), f32(v)
    return float(lib().or_score_down(ptr(w), w.shape[0], w.shape[1], ptr(v)))


def rank_scores(scores):
    s = f32(scores)
    out = np.zeros(s.size, np.uint32)
    lib().or_rank_scores(ptr(s), s.size, ptr(out, u32p))
    return out


def kl_first_token(baseline_logp, logits):
    b, l = f32(baseline_logp), f32(logits)
    per = np.zeros(b.shape[0], np.float64)
    v = lib().or_kl_first_token(ptr(b), ptr(l), b.shape[0], b.shape[1], ptr(per, f64p))
    return v, per


def log_softmax(x):
    x = f32(x)
    out = np.zeros_like(x)
    for i in range(x.shape[0]):
        lib().or_log_softmax(ptr(out[i]), ptr(x[i]), x.shape[1])
    return out


def residual_sums(res, first_capture, take):
    res = f32(res)
    entries, nc, hidden = res.shape
    fc = np.ascontiguousarray(first_capture, np.uintp)
    tk = np.ascontiguousarray(take, np.uintp)
    sums = np.zeros((entries, hidden), np.float64)
    lib().or_residual_sums(ptr(res), entries, nc, hidden, ptr(fc, szp), ptr(tk, szp), len(tk), ptr(sums, f64p))
    return sums


# ---- row_normalization = full (src/abliterate.zig:324-350, 409-538) -------

def orthonormalize_rows(vecs):
    """abliterate.orthonormalize (src/abliterate.zig:409-423): modified
    Gram-Schmidt, two passes, zero for a vanishing vector."""
    v = f32(vecs).copy()
    for i in range(v.shape[0]):
        for _ in range(2):
            for j in range(i):
                v[i] -= np.float32(np.dot(v[i], v[j])) * v[j]
        nrm = np.float32(np.sqrt(np.dot(v[i], v[i])))
        v[i] = v[i] / nrm if nrm > 1e-20 else 0.0
    return v


def jacobi_eigen(m):
    """abliterate.jacobiEigen (src/abliterate.zig:427-470): cyclic Jacobi in
    f32; returns (matrix with the eigenvalues on its diagonal, vectors in
    columns)."""
    m = f32(m).copy()
    n = m.shape[0]
    vecs = np.eye(n, dtype=np.float32)
    for _ in range(50):
        off = float(np.sum(m.astype(np.float64) ** 2) - np.sum(np.diag(m).astype(np.float64) ** 2))
        if off < 1e-18:
            break
        for p in range(n):
            for q in range(p + 1, n):
                apq = m[p, q]
                if abs(apq) < 1e-20:
                    continue
                theta = np.float32((m[q, q] - m[p, p]) / (np.float32(2) * apq))
                with np.errstate(over="ignore"):  # theta^2 may overflow to inf, then t = 0, as in f32
                    t = np.float32(np.sign(theta) / (abs(theta) + np.sqrt(theta * theta + np.float32(1))))
                t = np.float32(1) if theta == 0 else t
                cs = np.float32(1) / np.float32(np.sqrt(t * t + np.float32(1)))
                sn = t * cs
                cp, cq = m[:, p].copy(), m[:, q].copy()
                m[:, p], m[:, q] = cs * cp - sn * cq, sn * cp + cs * cq
                rp, rq = m[p, :].copy(), m[q, :].copy()
                m[p, :], m[q, :] = cs * rp - sn * rq, sn * rp + cs * rq
                vp, vq = vecs[:, p].copy(), vecs[:, q].copy()
                vecs[:, p], vecs[:, q] = cs * vp - sn * vq, sn * vp + cs * vq
    return m, vecs


def sketch_normals(seed, count):
    """The sketch of ditch_b200's full-mode edit: SplitMix64 then Box-Muller
    (the library's generator, not ditch's; both only seed the randomised
    SVD's test matrix)."""
    mask = (1 << 64) - 1
    s = seed & mask
    out = np.zeros(count, np.float32)
    i = 0

    def nxt():
        nonlocal s
        s = (s + 0x9E3779B97F4A7C15) & mask
        z = s
        z = ((z ^ (z >> 30)) * 0xBF58476D1CE4E5B9) & mask
        z = ((z ^ (z >> 27)) * 0x94D049BB133111EB) & mask
        return z ^ (z >> 31)

    while i < count:
        u1 = ((nxt() >> 11) + 1.0) * 2.0 ** -53
        u2 = (nxt() >> 11) * 2.0 ** -53
        r, th = np.sqrt(-2.0 * np.log(u1)), 6.283185307179586 * u2
        out[i] = np.float32(r * np.cos(th))
        if i + 1 < count:
            out[i + 1] = np.float32(r * np.sin(th))
        i += 2
    return out


def compute_delta_full(w, v, lam, lora_rank=3, seed=0, omega=None):
    """computeOutputDelta with row_normalization = full, K = 1
    (src/abliterate.zig:324-350) and randomizedSvd (473-538): the rank-r
    delta (a [r][cols], b [rows][r]) of W' = diag(n) rownorm(Wn + B A^T), from
    the implicit operator D = diag(c) W + d a^T, 2 r + 4 sketch vectors and 6
    power iterations. `omega` overrides the seeded sketch [q][cols]."""
    w, v = f32(w), f32(v)
    rows, cols = w.shape
    lam = np.float32(lam)
    n = row_norms(w)
    with np.errstate(divide="ignore", invalid="ignore"):
        vn = np.where(n > 0, v / n, np.float32(0)).astype(np.float32)
    a = matvec_t_multi(w, vn[None, :])[0]
    wa = matmul_t(a[None, :], w)[0]
    gram = np.float32(np.dot(a, a))
    bij = -lam * v
    with np.errstate(divide="ignore", invalid="ignore"):
        wn_dot_a = np.where(n > 0, wa / n, np.float32(0)).astype(np.float32)
    s2 = np.float32(1) + np.float32(2) * bij * wn_dot_a + bij * (-lam * v) * gram
    s = np.sqrt(np.maximum(s2, np.float32(1e-12))).astype(np.float32)
    c = (np.float32(1) / s - np.float32(1)).astype(np.float32)
    d = (n * (-lam * v) / s).astype(np.float32)

    def apply(x):  # (D X^T)^T for x [q][cols]
        y = matmul_t(x, w) * c
        return (y + np.outer(x @ a, d)).astype(np.float32)

    def apply_t(y):  # (D^T Y^T)^T for y [q][rows]
        x = matvec_t_multi(w, y * c)
        return (x + np.outer(y @ d, a)).astype(np.float32)

    r = max(int(lora_rank), 1)
    q = min(2 * r + 4, min(rows, cols))
    if omega is None:
        omega = sketch_normals(seed, q * cols).reshape(q, cols)
    qy = orthonormalize_rows(apply(omega))
    for _ in range(6):
        qx = orthonormalize_rows(apply_t(qy))
        qy = orthonormalize_rows(apply(qx))
    bt = apply_t(qy)
    m, vecs = jacobi_eigen(bt @ bt.T)
    order = sorted(range(q), key=lambda i: -float(m[i, i]))
    rank = min(r, q)
    la = np.zeros((rank, cols), np.float32)
    lb = np.zeros((rows, rank), np.float32)
    for k in range(rank):
        src = order[k]
        sk = np.float32(np.sqrt(max(float(m[src, src]), 0.0)))
        uk = (vecs[:, src] @ qy).astype(np.float32)
        vk = (vecs[:, src] @ bt).astype(np.float32)
        vk = vk / sk if sk > 1e-12 else np.zeros(cols, np.float32)
        sq = np.float32(np.sqrt(max(float(sk), 0.0)))
        la[k] = sq * vk
        lb[:, k] = uk * sq
    return la, lb


def materialize_rank(w, a, b):
    """W + b a (a [r][cols], b [rows][r]) in f32."""
    return (f32(w) + f32(b) @ f32(a)).astype(np.float32)


def export_merge_rows(w, a, b):
    """src/export.zig:108-112 (tensor.axpy per rank term, src/tensor.zig:561-570):
    every row of W (f32 [rows][cols]) gets b[row][k] * a[k] added for k in
    order, each product rounded to f32 before the add."""
    y = np.array(w, np.float32, copy=True)
    a, b = f32(a).reshape(-1, y.shape[1]), f32(b).reshape(y.shape[0], -1)
    for k in range(a.shape[0]):
        y = y + b[:, k:k + 1] * a[k][None, :]
    return y


def export_merge_cols(w, a, b):
    """The transposed merge (src/export.zig:114-122, src/moe.zig:380-387):
    W [in][out] gets, at (j, i), the rank terms b[i][k] * a[k][j] summed
    first (in k order, rounded per step) and then added."""
    y = np.array(w, np.float32, copy=True)
    a, b = f32(a).reshape(-1, y.shape[0]), f32(b).reshape(y.shape[1], -1)
    acc = np.zeros_like(y)
    for k in range(a.shape[0]):
        acc = acc + a[k][:, None] * b[:, k][None, :]
    return y + acc


def f32_to_f16_bits(x):
    """IEEE binary16 round to nearest even (Zig's @floatCast, src/tensor.zig:437-440)."""
    with np.errstate(over="ignore"):  # overflow to infinity is the rule
        return np.ascontiguousarray(x, np.float32).astype(np.float16).view(np.uint16)
