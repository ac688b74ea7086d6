"""The two plans of the quantised-weight GEMM: decode inside the GEMM (each
128 x 64 weight tile decoded into shared memory per token tile) and staged
decode (the weight decoded once to bf16 scratch, then the bf16 GEMM).

Both build the operand with the reference's arithmetic (FP8 block
src/dequant.zig:477-514, INT4 pack-quantized 518-597, MXFP4 natural layout
643-673: the f32 product rounded to bf16), so each equals x . W^T over the
standalone decoder's bf16 weight up to f32 accumulation order, and the two are
bit-identical where neither splits K (no atomics, same order of k-steps)."""
import pytest
import torch

from bench_configs import make_weight

pytestmark = pytest.mark.gpu

SHAPES = [
    (3200, 1024, 1500),  # 25 x 6 tiles of 256 tokens: no split-K in either plan
    (384, 512, 1100),    # few tiles: split-K with atomics
    (640, 2048, 100),    # a narrow token tile
]


def _bound(x, w):
    # |sum - ref| <= 2^-18 * sum_k |x_k| |w_k| + tiny: f32 accumulation over K
    return (x.float().abs() @ w.float().abs().T) * 2.0 ** -18 + 1e-6


@pytest.mark.parametrize("fmt", ["fp8", "mxfp4", "int4", "q8_0", "q4_k"])
@pytest.mark.parametrize("shape", range(len(SHAPES)))
def test_staged_and_fused_plans(device, fmt, shape):
    rows, cols, m = SHAPES[shape]
    torch.backends.cuda.matmul.allow_tf32 = False
    gen = torch.Generator(device="cuda").manual_seed(17 + shape)
    W, _ = make_weight(device, fmt, rows, cols, gen)
    x = torch.randn(m, cols, device="cuda", generator=gen).to(torch.bfloat16)
    dec = torch.empty(rows, cols, device="cuda", dtype=torch.bfloat16)
    torch.cuda.synchronize()  # the library's stream does not wait for torch's
    W.decode(dec.data_ptr())
    device.synchronize()
    ref = x.float() @ dec.float().T
    bound = _bound(x, dec)
    outs = []
    try:
        for plan in (0, 1):  # 0: always in the GEMM; 1: staged from one token on
            device.set_decode_staging(plan)
            out = torch.full((m, rows), float("nan"), device="cuda", dtype=torch.float32)
            torch.cuda.synchronize()
            W.gemm(x.data_ptr(), m, out.data_ptr())
            device.synchronize()
            err = (out - ref).abs()
            assert bool((err <= bound).all()), (plan, float(err.max()), float(bound.min()))
            outs.append(out)
    finally:
        device.set_decode_staging(1024)
        W.close()
    if shape == 0:
        assert torch.equal(outs[0], outs[1])


@pytest.mark.parametrize("fmt", ["bf16", "fp8", "mxfp4"])
@pytest.mark.parametrize("rows,cols,m", [(1408, 2048, 128), (1408, 2048, 5), (384, 512, 1100), (640, 4096, 300)])
def test_split_products_are_deterministic(device, fmt, rows, cols, m):
    """In deterministic mode, stream-K tiles (split between CTAs) and the
    split weight-streaming product are summed in a fixed order: repeated
    calls give the same bits, within the f32 bound of the decoded operand's
    product. The default (atomic) splits stay within the same bound."""
    torch.backends.cuda.matmul.allow_tf32 = False
    gen = torch.Generator(device="cuda").manual_seed(rows + m)
    W, _ = make_weight(device, fmt, rows, cols, gen)
    x = torch.randn(m, cols, device="cuda", generator=gen).to(torch.bfloat16)
    dec = torch.empty(rows, cols, device="cuda", dtype=torch.bfloat16)
    torch.cuda.synchronize()
    W.decode(dec.data_ptr())
    device.synchronize()
    ref = x.float() @ dec.float().T
    bound = _bound(x, dec)
    outs = []
    try:
        for det in (0, 1, 1, 1):
            device.set_deterministic(det)
            out = torch.full((m, rows), float("nan"), device="cuda", dtype=torch.float32)
            torch.cuda.synchronize()
            W.gemm(x.data_ptr(), m, out.data_ptr())
            device.synchronize()
            assert bool(((out - ref).abs() <= bound).all()), (det, float((out - ref).abs().max()))
            outs.append(out)
    finally:
        device.set_deterministic(0)
        W.close()
    assert torch.equal(outs[1], outs[2]) and torch.equal(outs[1], outs[3])


def test_q8_0_operand_is_ditchs_decode(device):
    """The Q8_0 GEMM operand (repacked codes and f32 scales, decoded in the
    GEMM or staged) equals ditch's f32 decode d * q (src/quant.zig:81-85)
    rounded to bf16, bit for bit, across mixed-sign and zero blocks."""
    import numpy as np

    import oracle
    from ditch_b200 import Tensor, Weight

    rng = np.random.default_rng(8)
    rows, cols = 96, 256
    w = (rng.standard_normal((rows, cols)) * 0.05).astype(np.float32)
    w[3, :32] = 0.0  # an all-zero block (d = 0)
    raw = oracle.quant_q8_0(w).reshape(rows, -1)
    W = Weight(device, Tensor("w", "q8_0", rows, cols, raw))
    assert W.format() == "q8_0"
    got = torch.empty(rows, cols, device="cuda", dtype=torch.int16)
    W.decode(got.data_ptr())
    device.synchronize()
    want = oracle.f32_to_bf16_bits(oracle.dequant_ggml(5, raw, rows * cols).reshape(rows, cols))
    assert np.array_equal(got.cpu().numpy().view(np.uint16), want)
    W.close()


def test_q4_k_operand_is_ditchs_decode(device):
    """The Q4_K GEMM operand (codes in element order and (d * scale, dmin *
    min) pairs, decoded in the GEMM, in the weight-streaming product or
    staged) equals ditch's f32 decode d1 * q - m1 (src/quant.zig:148-173)
    rounded to bf16, bit for bit: sub-scales and mins from 0 to 63 (the
    high-bit packing of sub-blocks 4-7), zero and negative super-block
    scales; the fused and staged GEMMs give the same bits."""
    import numpy as np

    import oracle
    from ditch_b200 import Tensor, Weight

    rng = np.random.default_rng(12)
    rows, cols = 256, 1024
    n_blk = rows * cols // 256
    raw = rng.integers(0, 256, (n_blk, 144), dtype=np.uint8)  # every scale / min / nibble pattern
    d = (rng.standard_normal(n_blk) * 0.01).astype(np.float16)
    dmin = (rng.standard_normal(n_blk) * 0.01).astype(np.float16)
    d[::17] = 0
    dmin[::13] = 0
    raw[:, 0:2] = d.view(np.uint8).reshape(-1, 2)
    raw[:, 2:4] = dmin.view(np.uint8).reshape(-1, 2)
    raw = np.ascontiguousarray(raw.reshape(rows, -1))
    W = Weight(device, Tensor("w", "q4_k", rows, cols, raw))
    assert W.format() == "q4_k"
    got = torch.empty(rows, cols, device="cuda", dtype=torch.int16)
    W.decode(got.data_ptr())
    device.synchronize()
    want = oracle.f32_to_bf16_bits(oracle.dequant_ggml(10, raw, rows * cols).reshape(rows, cols))
    assert np.array_equal(got.cpu().numpy().view(np.uint16), want)
    x = (torch.randn(600, cols, device="cuda") * 0.1).to(torch.bfloat16)
    dec = torch.from_numpy(want.view(np.int16)).cuda().view(torch.bfloat16)
    outs = []
    device.set_deterministic(True)
    try:
        for plan in (0, 1):
            device.set_decode_staging(plan)
            out = torch.empty(600, rows, device="cuda", dtype=torch.float32)
            torch.cuda.synchronize()
            W.gemm(x.data_ptr(), 600, out.data_ptr())
            device.synchronize()
            outs.append(out)
        for m in (1, 7, 16):  # the weight-streaming product decodes the same operand
            out = torch.empty(m, rows, device="cuda", dtype=torch.float32)
            torch.cuda.synchronize()
            W.gemm(x.data_ptr(), m, out.data_ptr())
            device.synchronize()
            ref = x[:m].float() @ dec.float().T
            assert bool(((out - ref).abs() <= _bound(x[:m], dec)).all()), m
    finally:
        device.set_decode_staging(1024)
        device.set_deterministic(False)
        W.close()
    assert torch.equal(outs[0], outs[1])
    ref = x.float() @ dec.float().T
    assert bool(((outs[0] - ref).abs() <= _bound(x, dec)).all())


def test_fp8_operand_is_ditchs_decode(device):
    """Every E4M3 code (subnormals, both zeros, NaN) under block scales from
    1e-30 to 300 (past 2^8 the decoders take their conversion path): the
    staged operand equals ditch's bf16(f32(code) * scale) bit for bit (NaN as
    NaN), and the GEMM decoding in the tile and the staged GEMM give the same
    bits."""
    import numpy as np

    import oracle
    from ditch_b200 import Tensor, Weight

    rows, cols = 256, 512
    codes = np.tile(np.arange(256, dtype=np.uint8), rows * cols // 256).reshape(rows, cols)
    codes = np.ascontiguousarray(np.roll(codes, 37, axis=1))
    scales = np.array([[1e-30, 0.5, 3e-4, 300.0], [2.0 ** -7, 1.0, 255.9, 7e-3]], np.float32)
    W = Weight(device, Tensor("w", "fp8", rows, cols, codes, scales=scales, block_rows=128, block_cols=128))
    got = torch.empty(rows, cols, device="cuda", dtype=torch.int16)
    W.decode(got.data_ptr())
    device.synchronize()
    got = got.cpu().numpy().view(np.uint16)
    want = oracle.dequant_fp8(codes, scales, 128, 128)
    nan_g = ((got & 0x7F80) == 0x7F80) & ((got & 0x7F) != 0)
    nan_w = ((want & 0x7F80) == 0x7F80) & ((want & 0x7F) != 0)
    assert np.array_equal(nan_g, nan_w)
    assert np.array_equal(got[~nan_g], want[~nan_w])
    # the fused and staged GEMMs over the same operand (rows without NaN codes)
    finite = codes.copy()
    finite[(finite & 0x7F) == 0x7F] = 0x01
    W2 = Weight(device, Tensor("w", "fp8", rows, cols, finite, scales=scales, block_rows=128, block_cols=128))
    x = (torch.randn(600, cols, device="cuda") * 0.01).to(torch.bfloat16)
    outs = []
    device.set_deterministic(True)  # both plans split K the same way, summed in order
    try:
        for plan in (0, 1):
            device.set_decode_staging(plan)
            out = torch.empty(600, rows, device="cuda", dtype=torch.float32)
            torch.cuda.synchronize()
            W2.gemm(x.data_ptr(), 600, out.data_ptr())
            device.synchronize()
            outs.append(out)
    finally:
        device.set_decode_staging(1024)
        device.set_deterministic(False)
        W.close()
        W2.close()
    assert torch.equal(outs[0], outs[1])


@pytest.mark.parametrize("fmt", ["bf16", "fp8", "mxfp4", "int4", "q8_0", "q4_k"])
@pytest.mark.parametrize("m", [1, 5, 16])
@pytest.mark.parametrize("rows,cols", [(1000, 1024), (4160, 4096), (264, 14336)])
def test_weight_streaming_small_m(device, fmt, m, rows, cols):
    """1..16 tokens take the weight-streaming product (mma.sync over the
    decoded stored format, K split across the grid): equal to x . W^T over
    the decoded weight up to f32 accumulation order. Shapes: a partial last
    16-row block, many row blocks, and few rows over a long K (many
    splits, a partial last one)."""
    torch.backends.cuda.matmul.allow_tf32 = False
    gen = torch.Generator(device="cuda").manual_seed(31 + m)
    W, _ = make_weight(device, fmt, rows, cols, gen)
    x = torch.randn(m, cols, device="cuda", generator=gen).to(torch.bfloat16)
    dec = torch.empty(rows, cols, device="cuda", dtype=torch.bfloat16)
    torch.cuda.synchronize()
    W.decode(dec.data_ptr())
    device.synchronize()
    ref = x.float() @ dec.float().T
    out = torch.full((m, rows), float("nan"), device="cuda", dtype=torch.float32)
    torch.cuda.synchronize()
    W.gemm(x.data_ptr(), m, out.data_ptr())
    device.synchronize()
    err = (out - ref).abs()
    assert bool((err <= _bound(x, dec)).all()), float(err.max())
    W.close()
