"""f32-level products (ditch_cuda_set_f32_split) against the oracle.

With the mode on, a model's f32 weights are kept as [hi | lo | hi] bf16
segments and every GEMM input as [hi | hi | lo], so the bf16 tensor cores add
hi.hi + hi.lo + lo.hi with f32 accumulation: about 2^-16 relative per
product against ditch's f32 engine (src/tensor.zig:1023-1045), instead of
the default mode's bf16 rounding of weights and activations (about 2^-9).

The weights here are genuinely f32 (bf16 values plus a small perturbation,
so every lo segment is non-zero). Bounds, per compared vector (every residual
entry of every row, the last-token logits): max |err| <= 1e-5 + 2e-4 * max
|ref|, a hundredth of the default mode's 2e-3 + 2e-2 * max |ref|; the edit's
KL within 1e-3 relative; greedy generation equal to the oracle's where the
oracle's top two logits differ by more than that bound.
"""
import numpy as np
import pytest

import ditch_b200
import oracle
from oracle.model import OracleModel, argmax_first, flatten_batch
from parity_report import record, record_value
from synth import make_model, prompts

pytestmark = pytest.mark.gpu

ATOL, RTOL = 1e-5, 2e-4


def bound(want):
    return ATOL + RTOL * float(np.abs(want).max())


def f32_model(seed, **kw):
    """make_model's weights perturbed off the bf16 grid, given as f32 tensors."""
    spec, w, _ = make_model(seed, **kw)
    rng = np.random.default_rng(seed + 1)
    out, tensors = {}, []
    for name, a in w.items():
        a = np.asarray(a, np.float32)
        if a.ndim == 2:
            a = (a + rng.standard_normal(a.shape).astype(np.float32) * np.float32(3e-5)).astype(np.float32)
        out[name] = a
        rows, cols = (a.shape[0], 1) if a.ndim == 1 else a.shape
        tensors.append(ditch_b200.Tensor(name, "f32", rows, cols, a))
    return spec, out, tensors


@pytest.fixture
def split(device):
    device.set_f32_split(True)
    yield device
    device.set_f32_split(False)


CASES = [dict(head_dim=64, heads=4, kv_heads=2, hidden=256, qkv_bias=True),
         dict(head_dim=128, heads=4, kv_heads=1, hidden=512, qk_norm=True, inter=520),
         dict(head_dim=32, heads=6, kv_heads=3, hidden=200, inter=300)]


@pytest.mark.parametrize("case", range(len(CASES)))
def test_split_forward_matches_oracle(split, case):
    spec, w, tensors = f32_model(700 + case, **CASES[case])
    ps = prompts(710 + case, [1, 5, 64, 65, 33], spec["vocab"])
    m = ditch_b200.Model(split, spec, tensors, max_seq=128)
    toks, rb, rp, cap, first, take, last = flatten_batch(ps, 10 ** 6)
    res, logits = m.forward(toks, rb, rp, cap, last)
    ores, ologits = OracleModel(spec, w).forward(toks, rb, rp, cap, last)
    for l in range(res.shape[0]):
        e = record(f"split case {case}", f"residual entry {l}", res[l], ores[l], bound=bound(ores[l]))
        for r in range(res.shape[1]):
            assert np.abs(res[l, r] - ores[l, r]).max() <= bound(ores[l, r]), (l, r)
    record(f"split case {case}", "last-token logits", logits, ologits, bound=bound(ologits))
    for i in range(len(ps)):
        assert np.abs(logits[i] - ologits[i]).max() <= bound(ologits[i]), i
    m.close()


def test_split_edit_and_kl(split):
    spec, w, tensors = f32_model(720, **CASES[0])
    ps = prompts(721, [12, 30, 7, 40], spec["vocab"])
    m = ditch_b200.Model(split, spec, tensors, max_seq=64)
    rng = np.random.default_rng(722)
    dirs = rng.standard_normal((spec["n_layers"] + 1, spec["hidden"])).astype(np.float32)
    dirs /= np.linalg.norm(dirs, axis=1, keepdims=True)
    m.set_directions(dirs)
    m.kl_init(ps)
    po, pd = (1.2, 0.0, 0.5, 3.0), (0.8, 1.0, 0.3, 2.0)
    m.apply_edit(po, pd)
    kl = m.kl_score()
    om = OracleModel(spec, w)
    for li in range(spec["n_layers"]):
        for comp, p in (("o", po), ("down", pd)):
            lam = oracle.kernel_weight(p, li)
            if lam is None:
                continue
            a, b = oracle.compute_delta_none(w[f"L{li}.{comp}"], dirs[li + 1], lam)
            om.set_delta(li, comp, a, b)
            da, _ = m.delta(li, "attn_o_proj" if comp == "o" else "mlp_down_proj")
            e = record("split edit", f"A = v^T W (layer {li} {comp})", da[0][: a.size], a)
            assert e["max_abs"] <= 1e-5 * e["ref_max_abs"] + 1e-8
    toks, rb, rp, cap, first, take, last = flatten_batch(ps)
    _, base = OracleModel(spec, w).forward(toks, rb, rp, (), last)
    _, edited = om.forward(toks, rb, rp, (), last)
    okl, _ = oracle.kl_first_token(oracle.log_softmax(base), edited)
    record_value("split edit", "first-token KL", kl, okl, bound="1e-3 relative")
    assert okl > 0 and abs(kl - okl) <= 1e-3 * okl, (kl, okl)
    m.close()


def test_split_generate_matches_oracle(split):
    spec, w, tensors = f32_model(730, **CASES[1])
    ps = prompts(731, [9, 20, 3], spec["vocab"])
    m = ditch_b200.Model(split, spec, tensors, max_seq=64)
    got = m.generate(ps, 8)
    om = OracleModel(spec, w)
    for i, p in enumerate(ps):
        seq = np.concatenate([np.asarray(p, np.uint32), np.asarray(got[i][:-1], np.uint32)])
        toks, rb, rp, cap, _, _, _ = flatten_batch([seq], 10 ** 6)
        rows = np.arange(len(p) - 1, len(seq), dtype=np.uintp)
        _, logits = om.forward(toks, rb, rp, logit_rows=rows)
        for j, t in enumerate(got[i]):
            best, gap = argmax_first(logits[j])
            if gap > bound(logits[j]):
                assert t == best, (i, j, t, best)
            else:
                assert logits[j][t] >= logits[j][best] - bound(logits[j]), (i, j)
    m.close()


def test_split_refuses_routed_experts(split):
    spec, w, tensors = make_model(740, hidden=128, head_dim=32, heads=4, kv_heads=2,
                                  moe=dict(experts=4, top_k=2, inter=64))
    with pytest.raises(ditch_b200.Unsupported, match="dense"):
        ditch_b200.Model(split, spec, tensors, max_seq=32)
