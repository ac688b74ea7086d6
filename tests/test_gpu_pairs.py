"""The CTA-pair GEMM (tcgen05 cta_group::2, ditch_cuda_set_cta_pairs) against
the one-CTA kernel and torch's f32 product.

Both kernels multiply the same bf16 operands with f32 accumulation in k
order, so a product's outputs must agree to the last bits of f32 rounding
(bound 1e-6 relative to max |out|); against torch's f32 product of the bf16
values the bound is 1e-5 relative. Through a forward, the one-CTA kernel's K
splits of small products can flip bf16 roundings of later inputs, so the two
forwards are compared within the forward bound of the other tests. Shapes cover one pair tile, weight rows that
leave the odd CTA of the last pair tile empty, ragged token tiles and K not
a multiple of the 64-wide k-stage. The forward check runs every epilogue the
pairs take (bias, SwiGLU, residual add, rank-1 delta) through a model.
"""
import numpy as np
import pytest

import ditch_b200
import oracle
from oracle.model import OracleModel, flatten_batch
from synth import make_model, prompts

pytestmark = pytest.mark.gpu


@pytest.fixture
def pairs(device):
    yield device
    device.set_cta_pairs(2)  # the library's default


@pytest.mark.parametrize("rows,cols,m", [(256, 256, 512), (4096 + 128, 1024 + 64, 1000), (6144, 4096, 2048),
                                         (384, 512, 777)])
def test_pair_gemm_matches_one_cta(pairs, rows, cols, m):
    torch = pytest.importorskip("torch")
    g = torch.Generator(device="cuda").manual_seed(rows + cols + m)
    w = (torch.randn(rows, cols, generator=g, device="cuda") * 0.02).to(torch.bfloat16)
    x = torch.randn(m, cols, generator=g, device="cuda").to(torch.bfloat16)
    W = ditch_b200.Weight(pairs, ditch_b200.Tensor("w", "bf16", rows, cols, w))
    outs = []
    for level in (0, 1):
        pairs.set_cta_pairs(level)
        out = torch.full((m, rows), float("nan"), device="cuda")
        torch.cuda.synchronize()
        W.gemm(x.data_ptr(), m, out.data_ptr())
        pairs.synchronize()
        outs.append(out.cpu().numpy())
    ref = (x.float() @ w.float().T).cpu().numpy()
    scale = float(np.abs(ref).max())
    assert np.isfinite(outs[1]).all()
    assert np.abs(outs[1] - outs[0]).max() <= 1e-6 * scale
    assert np.abs(outs[1] - ref).max() <= 1e-5 * scale
    W.close()


def test_pair_forward_matches_one_cta_and_oracle(pairs):
    spec, w, tensors = make_model(950, n_layers=2, hidden=512, heads=8, kv_heads=2, head_dim=64, inter=1024,
                                  qkv_bias=True)
    ps = prompts(951, [128] * 5 + [40], spec["vocab"])  # 680 tokens: the pairs take every dense GEMM
    toks, rb, rp, cap, first, take, last = flatten_batch(ps, 10 ** 6)
    rng = np.random.default_rng(952)
    dirs = rng.standard_normal((spec["n_layers"] + 1, spec["hidden"])).astype(np.float32)
    dirs /= np.linalg.norm(dirs, axis=1, keepdims=True)
    got = []
    for level in (0, 2):  # one CTA per tile; every dense product on pairs, SwiGLU included
        pairs.set_cta_pairs(level)
        m = ditch_b200.Model(pairs, spec, tensors, max_seq=128)
        m.set_directions(dirs)
        m.apply_edit((1.2, 1.0, 0.5, 2.0), (0.9, 0.0, 0.3, 2.0))  # rank-1 deltas in the o / down epilogues
        got.append(m.forward(toks, rb, rp, cap, last))
        m.close()
    (r0, l0), (r1, l1) = got
    # the one-CTA kernel splits K of these small products (atomic partial sums),
    # so bf16 roundings of later GEMM inputs can differ: the forward bound
    for a, b in ((r0, r1), (l0, l1)):
        assert np.abs(b - a).max() <= 2e-3 + 2e-2 * np.abs(a).max()
    om = OracleModel(spec, w)
    for li in range(spec["n_layers"]):
        for comp, p in (("o", (1.2, 1.0, 0.5, 2.0)), ("down", (0.9, 0.0, 0.3, 2.0))):
            lam = oracle.kernel_weight(p, li)
            if lam is not None:
                a, b = oracle.compute_delta_none(w[f"L{li}.{comp}"], dirs[li + 1], lam)
                om.set_delta(li, comp, a, b)
    _, ol = om.forward(toks, rb, rp, cap, last)
    for i in range(len(ps)):
        assert np.abs(l1[i] - ol[i]).max() <= 2e-3 + 2e-2 * np.abs(ol[i]).max(), i
