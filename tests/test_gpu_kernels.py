"""CUDA kernels against the oracle, through the C ABI.

Decoders are bit-exact (src/dequant.zig / src/quant.zig rules). The per-op
seam entries follow ditch's selftest contract (src/selftest.zig:34-41):
matmul 1e-4 abs / 1e-3 rel, element-wise 1e-5 / 1e-4, reductions 1e-4 / 1e-4,
over a shape sweep with 1x1, odd sizes and non-multiples of the tile sizes
(src/selftest.zig:124-135).
"""
import numpy as np
import pytest

import oracle

pytestmark = pytest.mark.gpu

rng = np.random.default_rng(20261201)


def close(got, want, atol, rtol, extra=0.0):
    err = np.abs(got.astype(np.float64) - want.astype(np.float64)).ravel()
    bound = (atol + rtol * np.abs(want.astype(np.float64)) + extra).ravel()
    worst = int(np.argmax(err - bound))
    assert np.all(err <= bound), f"max err {err.max():.3g}; worst {err[worst]:.3g} vs bound {bound[worst]:.3g}"


def same_bits(a, b):
    np.testing.assert_array_equal(np.asarray(a).view(np.uint16), np.asarray(b).view(np.uint16))


# ---- decoders ----
@pytest.mark.parametrize("rows,cols,br,bc", [(128, 256, 128, 128), (37, 40, 16, 8), (1, 16, 1, 16), (300, 128, 128, 128),
                                         (3, 8240, 128, 128), (5, 4128, 2, 32)])
def test_dequant_fp8_bit_exact(device, rows, cols, br, bc):
    codes = rng.integers(0, 256, (rows, cols), dtype=np.uint8)
    codes.flat[:256 if codes.size >= 256 else codes.size] = np.arange(min(256, codes.size), dtype=np.uint8)
    scales = (rng.random((-(-rows // br), -(-cols // bc))) * 0.01 + 1e-4).astype(np.float32)
    same_bits(device.dequant_fp8(codes, scales, br, bc), oracle.dequant_fp8(codes, scales, br, bc))


@pytest.mark.parametrize("bits,group,actorder,cols", [(4, 128, False, 128), (4, 16, False, 128), (8, 32, False, 128),
                                                      (3, 32, False, 128), (4, 16, True, 128), (4, 32, False, 8224)])
def test_dequant_int_bit_exact(device, bits, group, actorder, cols):
    rows = 24
    wpr = -(-cols * bits // 32)
    packed = rng.integers(0, 2 ** 32, (rows, wpr), dtype=np.uint64).astype(np.uint32)
    groups = cols // group
    scales = oracle.bf16_bits_to_f32(oracle.f32_to_bf16_bits(rng.random((rows, groups)).astype(np.float32) * 0.01))
    zeros = rng.integers(0, 2 ** 32, (-(-rows * bits // 32), groups), dtype=np.uint64).astype(np.uint32)
    g_idx = rng.permutation(np.arange(cols) // group).astype(np.uint32) if actorder else None
    got = device.dequant_int(packed, scales, zeros, rows, cols, bits, group, g_idx)
    want = oracle.dequant_int_packed(packed, scales, zeros, rows, cols, bits, group, g_idx)
    same_bits(got, want)
    same_bits(device.dequant_int(packed, scales, None, rows, cols, bits, group, g_idx),
              oracle.dequant_int_packed(packed, scales, None, rows, cols, bits, group, g_idx))


@pytest.mark.parametrize("transposed,rows,cols", [(False, 40, 96), (True, 40, 96), (False, 3, 8320)])
def test_dequant_mxfp4_bit_exact(device, transposed, rows, cols):
    blocks = rng.integers(0, 256, (rows, cols // 2), dtype=np.uint8)
    scales = rng.integers(100, 140, (rows, cols // 32), dtype=np.uint8)
    scales[0, 0], scales[1, 1], scales[2, 2] = 0, 255, 254  # subnormal, infinite and largest scales
    got = device.dequant_mxfp4(blocks, scales, rows, cols, transposed)
    L = oracle.lib()
    want = np.zeros(got.shape, np.uint16)
    fn = L.or_dequant_mxfp4_transposed if transposed else L.or_dequant_mxfp4_packed
    fn(oracle.ptr(blocks, oracle.u8p), oracle.ptr(scales, oracle.u8p), rows, cols, oracle.ptr(want, oracle.u16p))
    same_bits(got, want)


def ggml_blocks(dtype, nblocks):
    bb = oracle.lib().or_ggml_block_bytes(dtype)
    raw = rng.integers(0, 256, (nblocks, bb), dtype=np.uint8)
    d = (rng.random(nblocks) * 0.01 + 1e-3).astype(np.float16).view(np.uint8).reshape(nblocks, 2)
    if dtype == 11:  # q6_k: d at the end
        raw[:, 208:210] = d
    elif dtype == 12:  # q8_k: f32 d first
        raw[:, 0:4] = (rng.random(nblocks).astype(np.float32) * 0.01).view(np.uint8).reshape(nblocks, 4)
    else:
        raw[:, 0:2] = d
        if dtype in (7, 9, 10):  # second f16 (min / dmin)
            raw[:, 2:4] = d[::-1]
    return raw


@pytest.mark.parametrize("dtype", [5, 6, 7, 8, 9, 10, 11, 12])
def test_dequant_ggml_bit_exact(device, dtype):
    names = {5: "q8_0", 6: "q4_0", 7: "q4_1", 8: "q5_0", 9: "q5_1", 10: "q4_k", 11: "q6_k", 12: "q8_k"}
    bs = oracle.lib().or_ggml_block_size(dtype)
    raw = ggml_blocks(dtype, 12)
    n = 12 * bs
    np.testing.assert_array_equal(device.dequant_ggml(names[dtype], raw, n).view(np.uint32),
                                  oracle.dequant_ggml(dtype, raw, n).view(np.uint32))


# ---- the per-op seam ----
SHAPES = [(1, 1, 1), (3, 5, 7), (17, 33, 65), (64, 128, 256), (130, 300, 200), (256, 1024, 1024), (5, 2000, 96)]


@pytest.mark.parametrize("n,rows,cols", SHAPES)
@pytest.mark.parametrize("dtype", ["f32", "bf16", "f16"])
def test_matmul_t_matches_oracle(device, n, rows, cols, dtype):
    x = rng.standard_normal((n, cols)).astype(np.float32)
    w32 = rng.standard_normal((rows, cols)).astype(np.float32)
    if dtype == "f32":
        raw, wref = w32, w32
    elif dtype == "bf16":
        raw = oracle.f32_to_bf16_bits(w32)
        wref = oracle.bf16_bits_to_f32(raw)
    else:
        raw = w32.astype(np.float16)
        wref = raw.astype(np.float32)
    got = device.matmul_t(x, raw, dtype, rows, cols)
    # Split-bf16 drops x_lo * W_lo (|x_lo| <= 2^-9 |x|, |W_lo| <= 2^-9 |W|) and
    # accumulates in f32 on the tensor cores: on top of the selftest bound, an
    # error of at most 8e-6 * sum_k |x_k| |W_k| (the dot's condition) is allowed.
    cond = np.abs(x).astype(np.float64) @ np.abs(wref).astype(np.float64).T
    close(got, oracle.matmul_t(x, wref), 1e-4, 1e-3, 8e-6 * cond)


@pytest.mark.parametrize("dtype", ["q8_0", "q4_k"])
def test_matmul_t_gguf(device, dtype):
    n, rows, cols = 9, 70, 512
    w = (rng.standard_normal((rows, cols)) * 0.02).astype(np.float32)
    raw = oracle.quant_q8_0(w) if dtype == "q8_0" else oracle.quant_q4_k(w)
    wref = oracle.dequant_ggml(5 if dtype == "q8_0" else 10, raw, rows * cols).reshape(rows, cols)
    x = rng.standard_normal((n, cols)).astype(np.float32)
    close(device.matmul_t(x, raw, dtype, rows, cols), oracle.matmul_t(x, wref), 1e-4, 1e-3)


@pytest.mark.parametrize("rows,cols,q", [(1, 1, 1), (33, 65, 2), (512, 300, 1), (1000, 2048, 3)])
def test_matvec_and_row_norms(device, rows, cols, q):
    w = rng.standard_normal((rows, cols)).astype(np.float32)
    y = rng.standard_normal((q, rows)).astype(np.float32)
    y[0, 0] = 0  # rows with y == 0 are skipped
    close(device.matvec_t_multi(w, "f32", rows, cols, y), oracle.matvec_t_multi(w, y), 1e-4 * np.sqrt(rows), 1e-4)
    close(device.row_norms(w, "f32", rows, cols), oracle.row_norms(w), 1e-4, 1e-4)


def test_elementwise_entries(device):
    n, length = 7, 200
    x = rng.standard_normal((n, length)).astype(np.float32)
    w = rng.standard_normal(length).astype(np.float32)
    L = oracle.lib()
    want = np.zeros_like(x)
    for i in range(n):
        L.or_rmsnorm(oracle.ptr(want[i]), oracle.ptr(x[i]), oracle.ptr(w), length, 1e-6)
    close(device.rmsnorm_rows(x, w, 1e-6), want, 1e-5, 1e-4)
    sm = x.copy()
    for i in range(n):
        L.or_softmax_inplace(oracle.ptr(sm[i]), length)
    close(device.softmax_rows(x), sm, 1e-5, 1e-4)
    up = rng.standard_normal((n, length)).astype(np.float32)
    g = np.zeros_like(x)
    L.or_gated_silu(oracle.ptr(g), oracle.ptr(x), oracle.ptr(up), n, length, length, length)
    close(device.gated_activation(x, up, n, length, length, length).reshape(n, length), g, 1e-5, 1e-4)
    # rope (neox) against applyRope on rows at mixed positions
    half, table = 32, 50
    cos_t = np.zeros((table, half), np.float32)
    sin_t = np.zeros((table, half), np.float32)
    L.or_rope_table(oracle.ptr(cos_t), oracle.ptr(sin_t), table, 2 * half, 1e4, 0, 1.0, 1.0, 1.0, 1.0)
    r = rng.standard_normal((n, 2 * half)).astype(np.float32)
    pos = rng.integers(0, table, n).astype(np.uint32)
    want = r.copy()
    for i in range(n):
        L.or_apply_rope(oracle.ptr(want[i]), oracle.ptr(cos_t[pos[i]]), oracle.ptr(sin_t[pos[i]]), 2 * half)
    close(device.rope_rows(r, cos_t, sin_t, pos), want, 1e-5, 1e-4)
    # attention scores / values
    hd, keys, stride = 64, 9, 80
    q = rng.standard_normal(hd).astype(np.float32)
    k = rng.standard_normal(keys * stride).astype(np.float32)
    s = device.attention_scores(q, k, stride, 0.125, keys)
    want = np.array([oracle.lib().or_dot(oracle.ptr(q), oracle.ptr(k[p * stride:]), hd) * 0.125 for p in range(keys)])
    close(s, want, 1e-4, 1e-4)
    p = rng.random(keys).astype(np.float32)
    close(device.attention_values(p, k, stride, hd),
          np.array([sum(p[j] * k[j * stride + i] for j in range(keys)) for i in range(hd)], np.float32), 1e-4, 1e-4)


def test_edit_weight_bf16(device):
    """W <- W - alpha r (r^T W) on device memory, against the oracle's f32 edit rounded to bf16."""
    torch = pytest.importorskip("torch")
    rows, cols, alpha = 256, 384, 0.7
    w32 = (rng.standard_normal((rows, cols)) * 0.02).astype(np.float32)
    wb = oracle.f32_to_bf16_bits(w32)
    r = rng.standard_normal(rows).astype(np.float32)
    r /= np.linalg.norm(r)
    wt = torch.from_numpy(wb.view(np.int16).copy()).cuda()
    rt = torch.from_numpy(r).cuda()
    device.edit_weight_bf16(wt.data_ptr(), rows, cols, rt.data_ptr(), alpha)
    got = oracle.bf16_bits_to_f32(wt.cpu().numpy().view(np.uint16))
    wf = oracle.bf16_bits_to_f32(wb)
    a, b = oracle.compute_delta_none(wf, r, alpha)
    want = oracle.materialize(wf, a, b)
    close(got, want, 2e-5, 8e-3)  # one bf16 rounding of the result
    assert np.abs(r @ got).max() < np.abs(r @ wf).max() * (1 - alpha) + 1e-3


@pytest.mark.parametrize("rows,cols", [(37, 264), (130, 8), (1000, 4104), (4099, 520)])
def test_edit_weight_bf16_shapes(device, rows, cols):
    """The piece-wise GEMV-T and the rank-1 update at ragged shapes: rows not a
    multiple of the 8 row lanes or of a 64-row run, columns that leave the
    last 256-column block part empty."""
    torch = pytest.importorskip("torch")
    w32 = (rng.standard_normal((rows, cols)) * 0.02).astype(np.float32)
    wb = oracle.f32_to_bf16_bits(w32)
    r = rng.standard_normal(rows).astype(np.float32)
    r /= np.linalg.norm(r)
    wt = torch.from_numpy(wb.view(np.int16).copy()).cuda()
    device.edit_weight_bf16(wt.data_ptr(), rows, cols, torch.from_numpy(r).cuda().data_ptr(), 0.5)
    got = oracle.bf16_bits_to_f32(wt.cpu().numpy().view(np.uint16))
    wf = oracle.bf16_bits_to_f32(wb)
    a, b = oracle.compute_delta_none(wf, r, 0.5)
    close(got, oracle.materialize(wf, a, b), 2e-5, 8e-3)


@pytest.mark.parametrize("hidden,inter,block", [(256, 1040, (128, 16)), (200, 520, (64, 128)), (512, 4608, (128, 128)),
                                                (264, 4128, (16, 32))])
def test_edit_delta_fp8_matches_oracle(device, hidden, inter, block):
    """A = v^T W over FP8 block-scaled weights (the decoded bf16 operand) at
    shapes that take the piece kernel (columns a multiple of 16) and the
    byte-wise one (520 columns), against the oracle's matvecTMulti."""
    from synth import make_model
    import ditch_b200
    spec, w, tensors = make_model(970 + hidden, n_layers=1, hidden=hidden, heads=4, kv_heads=2,
                                  head_dim=hidden // 4, inter=inter, fmt="fp8", block=block)
    m = ditch_b200.Model(device, spec, tensors, max_seq=16)
    dirs = rng.standard_normal((2, hidden)).astype(np.float32)
    dirs /= np.linalg.norm(dirs, axis=1, keepdims=True)
    m.set_directions(dirs)
    p = (1.0, 0.0, 1.0, 1.0)
    lam = oracle.kernel_weight(p, 0)
    assert lam is not None
    m.apply_edit(p, p)
    for comp, name in (("o", "attn_o_proj"), ("down", "mlp_down_proj")):
        a, _ = oracle.compute_delta_none(w[f"L0.{comp}"], dirs[1], lam)
        da, _ = m.delta(0, name)
        got = np.asarray(da[0][: a.size])
        assert np.abs(got - a).max() <= 1e-5 * np.abs(a).max() + 1e-8, comp
    m.close()


def test_edit_weight_bf16_rejects_odd_pointers(device):
    """w must start on a 2-byte boundary and r on a 4-byte one; the check comes
    before any launch (these dummy pointers are never dereferenced)."""
    from ditch_b200 import DitchCudaError

    with pytest.raises(DitchCudaError, match="aligned"):
        device.edit_weight_bf16(17, 8, 8, 16, 1.0)
    with pytest.raises(DitchCudaError, match="aligned"):
        device.edit_weight_bf16(16, 8, 8, 18, 1.0)
