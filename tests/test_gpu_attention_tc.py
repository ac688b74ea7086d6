"""The tcgen05 prefill attention (attention_tc.cu, used when every prompt of
the batch is at most 128 tokens) against the oracle and the mma.sync kernel.

Both kernels split Q, K, V and the softmax weights into bf16 hi + lo and sum
hi*hi + hi*lo + lo*hi in f32; they differ in the order of the f32 sums, so
their attention outputs agree to f32 rounding, and the bf16 rounding of
those outputs (the o_proj GEMM's input) can flip. Through a forward the two
are compared within the forward bound of the other tests, and each against
the oracle: max |err| <= 2e-3 + 2e-2 * max |ref| per logit row and per
captured residual row.

Levels 2 (two CTAs per SM, Q staged by 64-dim halves, for prompts of at
most 64 tokens) and 1 (one CTA per SM, the whole Q tile staged) are each
checked. The cases cover both
key widths (prompts up to 64 and up to 128 tokens), head sizes 64 and 128,
query groups of 1, 2, 3, 4 and 8 heads per kv head (tiles of two 64-row
heads with an empty half, one 128-row head per tile), q/k norms, ragged
prompts, one-token prompts, and more (prompt, kv head) items than the SMs
hold at once."""
import numpy as np
import pytest

import ditch_b200
from oracle.model import OracleModel, flatten_batch
from synth import make_model, prompts

pytestmark = pytest.mark.gpu

_RAGGED = [int(n) for n in np.random.default_rng(320).integers(1, 65, 40)]

CASES = [
    (dict(head_dim=128, heads=8, kv_heads=2, hidden=512), [64, 1, 37, 64, 5]),
    (dict(head_dim=128, heads=4, kv_heads=1, hidden=512, qk_norm=True), [100, 128, 3, 65]),
    (dict(head_dim=64, heads=6, kv_heads=2, hidden=384), [64, 17, 2]),
    (dict(head_dim=64, heads=8, kv_heads=1, hidden=512, qkv_bias=True), [90, 128, 1]),
    (dict(head_dim=128, heads=4, kv_heads=4, hidden=512), [64, 9]),
    # 160 (prompt, kv head) CTAs, more than one wave at one CTA per SM
    (dict(head_dim=128, heads=8, kv_heads=4, hidden=512, n_layers=1), _RAGGED),
    (dict(head_dim=64, heads=16, kv_heads=4, hidden=512, n_layers=1, qk_norm=True), _RAGGED),
]


@pytest.fixture
def tc_device(device):
    yield device
    device.set_attention_tc(2)  # the library's default


def bound(ref):
    return 2e-3 + 2e-2 * float(np.abs(ref).max())


@pytest.mark.parametrize("case", range(len(CASES)))
def test_tc_attention_matches_oracle_and_mma(tc_device, case):
    kw, lens = CASES[case]
    spec, f32, tensors = make_model(300 + case, **kw)
    ps = prompts(310 + case, lens, spec["vocab"])
    toks, rb, rp, cap, first, take, last = flatten_batch(ps, 2)
    got = {}
    for level in (2, 1, 0):  # two CTAs per SM, one CTA per SM, the mma.sync kernel
        tc_device.set_attention_tc(level)
        m = ditch_b200.Model(tc_device, spec, tensors, max_seq=256)
        got[level] = m.forward(toks, rb, rp, cap, last)
        m.close()
    ores, ologits = OracleModel(spec, f32).forward(toks, rb, rp, cap, last)
    res_mma, log_mma = got[0]
    for level in (2, 1):
        res_tc, log_tc = got[level]
        worst = 0.0
        for i in range(len(ps)):
            err = float(np.abs(log_tc[i] - ologits[i]).max())
            worst = max(worst, err / bound(ologits[i]))
            assert err <= bound(ologits[i]), (level, i)
            assert np.abs(log_tc[i] - log_mma[i]).max() <= bound(log_mma[i]), (level, i)
        for l in range(spec["n_layers"] + 1):
            err = float(np.abs(res_tc[l] - ores[l]).max())
            worst = max(worst, err / bound(ores[l]))
            assert err <= bound(ores[l]), (level, l)
            assert np.abs(res_tc[l] - res_mma[l]).max() <= bound(res_mma[l]), (level, l)
        print(f"case {case} level {level}: worst error {worst:.3f} of the bound")
