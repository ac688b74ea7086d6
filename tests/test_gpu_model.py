"""The resident model (forward, capture, edit, KL, directions) on the GPU
against the reference fixtures and the oracle.

Tolerance: the device forward runs its weight products as bf16 tensor-core
MMAs with f32 accumulation (activations rounded to bf16 at every GEMM input,
the residual stream kept in f32), against ditch's all-f32 CPU engine. The
bound used here is max abs error <= FWD_ATOL + FWD_RTOL * max|reference| per
compared vector; the reference's own fixture check is 2e-3 max abs on f32
(src/model_test.zig:62, 70).
"""
import numpy as np
import pytest

import ditch_b200
import oracle
from golden_loader import Golden
from oracle.model import OracleModel, flatten_batch

pytestmark = pytest.mark.gpu

FWD_ATOL, FWD_RTOL = 2e-3, 2e-2
DENSE = ["qwen2", "llama", "qwen3", "qwen2_fp8", "qwen2_int4", "qwen3_moe", "qwen3_moe_big", "qwen3_moe_fused",
         "qwen3_moe_fused_t", "mixtral", "qwen2_gguf", "llama_gguf"]


def bound(want):
    return FWD_ATOL + FWD_RTOL * float(np.abs(want).max())


ROUTER_TIE = 2e-2  # router logit gap below which bf16 activations may pick the other expert


def near_tied_tokens(g, toks, rb, rp, cap, last):
    """Token rows whose top-k boundary in some routed layer is a near-tie in
    the oracle: the gap between the k-th and (k+1)-th router logit is below
    ROUTER_TIE. ditch picks the first maximum of f32 scores
    (src/moe.zig:971-985); the device computes the router input from
    activations rounded to bf16 at every GEMM, so such a token can take the
    other expert, which changes its row and, through attention, the later rows
    of its prompt. The router input of layer l is x + attn(x): the oracle's
    layer-l output with that layer's experts set to zero."""
    s = g.spec
    if not s.get("moe_layers"):
        return set()
    w = g.f32_weights()
    k = s["top_k"]
    tied = set()
    for li in range(s["n_layers"]):
        if not s["moe_layers"][li]:
            continue
        w0 = dict(w)
        for a in ("gate", "up", "down"):
            w0[f"L{li}.e_{a}"] = np.zeros_like(w[f"L{li}.e_{a}"])
        res, _ = OracleModel(s, w0).forward(toks, rb, rp, cap, last)
        x = res[li + 1]
        h = x / np.sqrt((x * x).mean(axis=1, keepdims=True) + s["eps"]) * w[f"L{li}.post_norm"]
        top = np.sort(h @ w[f"L{li}.router"].T, axis=1)[:, ::-1]
        tied |= set(np.nonzero(top[:, k - 1] - top[:, k] < ROUTER_TIE)[0].tolist())
    return tied


def load(device, family):
    g = Golden(family)
    return g, ditch_b200.Model(device, g.spec, g.cuda_tensors(), max_seq=64)


@pytest.mark.parametrize("family", DENSE)
def test_fixture_forward(device, family):
    """Every prompt's last logits and last-token residual entries against the
    reference and the oracle (the reference's own check). With routed
    experts, a prompt with a near-tied routing choice (see near_tied_tokens)
    is checked on its rows before that token instead, every entry: causal
    attention keeps them independent of the choice."""
    g, m = load(device, family)
    toks, rb, rp, cap, first, take, last = flatten_batch(g.prompts(), 10 ** 6)  # capture every row
    res, logits = m.forward(toks, rb, rp, cap, last)
    om = OracleModel(g.spec, g.f32_weights())
    ores, ologits = om.forward(toks, rb, rp, cap, last)
    tied = near_tied_tokens(g, toks, rb, rp, cap, last)
    checked = 0
    start = 0
    for i, c in enumerate(g.cases):
        n = len(c["ids"])
        assert np.isfinite(logits[i]).all()
        stop = min([t - start for t in tied if start <= t < start + n] + [n])
        if stop < n:  # near-tied routing: the rows before the tie, every entry
            for pos in range(stop):
                for l in range(res.shape[0]):
                    got, want = res[l, start + pos], ores[l, start + pos]
                    assert np.abs(got - want).max() <= bound(want), (i, pos, l)
                checked += 1
            start += n
            continue
        start += n
        checked += 1
        assert np.abs(logits[i] - c["last_logits"]).max() <= bound(c["last_logits"])
        assert np.abs(res[:, start - 1] - c["last_hidden"]).max() <= bound(c["last_hidden"])
        assert np.abs(logits[i] - ologits[i]).max() <= bound(ologits[i])
        assert int(np.argmax(logits[i])) == c["argmax"]
    assert checked > 0
    m.close()


def test_forward_rejects_bad_rows_and_tokens(device):
    g, m = load(device, "qwen2")
    with pytest.raises(ditch_b200.Unsupported):
        m.forward([1, 2, 3], [0, 0, 0], [0, 2, 3], [], [2])  # positions not contiguous
    with pytest.raises(ditch_b200.DitchCudaError):
        m.forward([1, 2, 99999], [0, 0, 0], [0, 1, 2], [], [2])  # token outside the table
    res, logits = m.forward([1, 2, 3], [0, 0, 0], [0, 1, 2], [], [2])  # the context is still usable
    assert np.isfinite(logits).all()
    m.close()


@pytest.mark.parametrize("family", ["qwen2", "qwen2_fp8"])
def test_edit_and_kl(device, family):
    """abliterate.apply (none mode) + KlDivergence on device vs the oracle with the same deltas."""
    g, m = load(device, family)
    s = g.spec
    prompts = g.prompts()
    rng = np.random.default_rng(5)
    dirs = rng.standard_normal((s["n_layers"] + 1, s["hidden"])).astype(np.float32)
    dirs /= np.linalg.norm(dirs, axis=1, keepdims=True)
    m.set_directions(dirs)
    m.kl_init(prompts)
    assert abs(m.kl_score()) < 1e-6  # base model: KL 0 (src/scorers.zig:839-926)
    po = (1.2, 0.0, 0.5, 3.0)
    pd = (0.8, 1.0, 0.3, 2.0)
    m.apply_edit(po, pd)
    kl = m.kl_score()
    assert kl > 0
    # the oracle with deltas from its own GEMV of the f32 weights
    w = g.f32_weights()
    om = OracleModel(s, w)
    for li in range(s["n_layers"]):
        v = dirs[li + 1]
        for comp, p, name in (("o", po, "o"), ("down", pd, "down")):
            lam = oracle.kernel_weight(p, li)
            if lam is None:
                continue
            a, b = oracle.compute_delta_none(w[f"L{li}.{name}"], v, lam)
            om.set_delta(li, comp, a, b)
    toks, rb, rp, cap, first, take, last = flatten_batch(prompts)
    _, base_logits = OracleModel(s, w).forward(toks, rb, rp, (), last)
    _, ed_logits = om.forward(toks, rb, rp, (), last)
    okl, _ = oracle.kl_first_token(oracle.log_softmax(base_logits), ed_logits)
    assert abs(kl - okl) <= 2e-3 + 0.05 * abs(okl), (kl, okl)
    # the e2e entry (prompts uploaded in the call) gives the same value
    tokens = np.concatenate(prompts).astype(np.uint32)
    offs = np.zeros(len(prompts) + 1, np.uintp)
    offs[1:] = np.cumsum([len(p) for p in prompts])
    assert m.kl_score_prompts(tokens, offs, len(prompts)) == kl
    m.reset_edits()
    assert abs(m.kl_score()) < 1e-6
    # interpolated global direction (direction_index)
    m.apply_edit(po, pd, direction_index=0.6)
    assert m.kl_score() > 0
    m.close()


def test_moe_expert_ranking_and_edits(device):
    """moe.rankScores / scoreDown and the broad and selective expert edits vs the oracle."""
    g, m = load(device, "qwen3_moe")
    s = g.spec
    w = g.f32_weights()
    rng = np.random.default_rng(9)
    dirs = rng.standard_normal((s["n_layers"] + 1, s["hidden"])).astype(np.float32)
    dirs /= np.linalg.norm(dirs, axis=1, keepdims=True)
    m.set_directions(dirs)
    moe_layers = [i for i in range(s["n_layers"]) if s["moe_layers"][i]]
    for li in moe_layers:
        v = dirs[li + 1]
        order, scores = m.rank_experts(li, v)
        osc = np.array([oracle.score_down(w[f"L{li}.e_down"][e], v) for e in range(s["n_experts"])], np.float32)
        np.testing.assert_allclose(scores, osc, rtol=1e-4, atol=1e-6)
        np.testing.assert_array_equal(order, oracle.rank_scores(osc))
    prompts = g.prompts()
    toks, rb, rp, cap, first, take, last = flatten_batch(prompts)
    m.kl_init(prompts)
    po, pd = (1.0, 1.0, 0.5, 2.0), (1.1, 1.0, 0.4, 2.0)

    def oracle_kl(selected):
        om = OracleModel(s, w)
        for li in range(s["n_layers"]):
            v = dirs[li + 1]
            lam = oracle.kernel_weight(po, li)
            if lam is not None:
                a, b = oracle.compute_delta_none(w[f"L{li}.o"], v, lam)
                om.set_delta(li, "o", a, b)
            lam = oracle.kernel_weight(pd, li)
            if lam is None:
                continue
            if not s["moe_layers"][li]:
                a, b = oracle.compute_delta_none(w[f"L{li}.down"], v, lam)
                om.set_delta(li, "down", a, b)
                continue
            for e, weight in selected(li, v, lam):
                a, b = oracle.compute_delta_none(w[f"L{li}.e_down"][e], v, weight)
                om.set_delta(li, ("e", e), a, b)
        _, base = OracleModel(s, w).forward(toks, rb, rp, (), last)
        _, ed = om.forward(toks, rb, rp, (), last)
        return oracle.kl_first_token(oracle.log_softmax(base), ed)[0]

    # broad: every expert's down projection gets the layer's lambda
    m.apply_edit(po, pd)
    want = oracle_kl(lambda li, v, lam: [(e, lam) for e in range(s["n_experts"])])
    got = m.kl_score()
    assert abs(got - want) <= 2e-3 + 0.05 * abs(want), (got, want)
    # selective: the top-2 ranked experts get lambda * strength
    m.apply_expert_edit(po, pd, n_experts=2, strength=0.7)

    def top2(li, v, lam):
        sc = np.array([oracle.score_down(w[f"L{li}.e_down"][e], v) for e in range(s["n_experts"])], np.float32)
        return [(int(e), lam * 0.7) for e in oracle.rank_scores(sc)[:2]]

    want = oracle_kl(top2)
    got = m.kl_score()
    assert abs(got - want) <= 2e-3 + 0.05 * abs(want), (got, want)
    m.close()


def test_residual_sums_and_directions(device):
    """engine.getResidualMeanObserved + computeDirections vs the oracle."""
    g, m = load(device, "qwen2")
    s = g.spec
    rng = np.random.default_rng(11)
    good = [rng.integers(0, s["vocab"], rng.integers(3, 12)).astype(np.uint32) for _ in range(5)]
    bad = [rng.integers(0, s["vocab"], rng.integers(3, 12)).astype(np.uint32) for _ in range(6)]
    om = OracleModel(s, g.f32_weights())
    for window in (1, 3):
        sums = {}
        for name, ps in (("good", good), ("bad", bad)):
            dsum, count = m.residual_sums(ps, window=window, batch_size=4)
            assert count == len(ps)
            toks, rb, rp, cap, first, take, last = flatten_batch(ps, window)
            res, _ = om.forward(toks, rb, rp, cap, ())
            osum = oracle.residual_sums(res, first, take)
            assert np.abs(dsum - osum).max() <= bound(osum)
            sums[name] = (dsum, count, osum)
        dirs = m.directions(sums["good"][0], sums["good"][1], sums["bad"][0], sums["bad"][1], True)
        gm = (sums["good"][2] / len(good)).astype(np.float32)
        bm = (sums["bad"][2] / len(bad)).astype(np.float32)
        odirs = oracle.compute_directions(gm, bm, True)
        cos = np.sum(dirs * odirs, axis=1)
        assert cos.min() > 0.99, cos
    m.close()


@pytest.mark.parametrize("family", ["qwen2", "qwen2_fp8", "qwen2_int4", "qwen3_moe"])
def test_pre_normalised_edit(device, family):
    """row_normalization = pre (src/abliterate.zig:295-323): the device's
    edited KL against the oracle with a = (v / n)^T W, b = -lambda v n (n the
    row norms of the decoded weights), for o_proj, down_proj and (MoE) every
    expert's down projection; then the selective expert edit in the same
    mode."""
    g, m = load(device, family)
    s = g.spec
    w = g.f32_weights()
    rng = np.random.default_rng(11)
    dirs = rng.standard_normal((s["n_layers"] + 1, s["hidden"])).astype(np.float32)
    dirs /= np.linalg.norm(dirs, axis=1, keepdims=True)
    m.set_directions(dirs)
    prompts = g.prompts()
    toks, rb, rp, cap, first, take, last = flatten_batch(prompts)
    m.kl_init(prompts)
    po, pd = (1.1, 0.0, 0.5, 3.0), (0.9, 1.0, 0.3, 2.0)
    moe = s.get("moe_layers") or [False] * s["n_layers"]

    def oracle_kl(expert_weights):
        om = OracleModel(s, w)
        for li in range(s["n_layers"]):
            v = dirs[li + 1]
            lam = oracle.kernel_weight(po, li)
            if lam is not None:
                om.set_delta(li, "o", *oracle.compute_delta_pre(w[f"L{li}.o"], v, lam))
            lam = oracle.kernel_weight(pd, li)
            if lam is None:
                continue
            if not moe[li]:
                om.set_delta(li, "down", *oracle.compute_delta_pre(w[f"L{li}.down"], v, lam))
                continue
            for e, weight in expert_weights(li, v, lam):
                om.set_delta(li, ("e", e), *oracle.compute_delta_pre(w[f"L{li}.e_down"][e], v, weight))
        _, base = OracleModel(s, w).forward(toks, rb, rp, (), last)
        _, ed = om.forward(toks, rb, rp, (), last)
        return oracle.kl_first_token(oracle.log_softmax(base), ed)[0]

    m.set_row_normalization("pre")
    m.apply_edit(po, pd)
    got = m.kl_score()
    want = oracle_kl(lambda li, v, lam: [(e, lam) for e in range(s["n_experts"])])
    assert got > 0 and abs(got - want) <= 2e-3 + 0.05 * abs(want), (got, want)
    if s.get("moe_layers"):
        m.apply_expert_edit(po, pd, n_experts=2, strength=0.7)

        def top2(li, v, lam):
            sc = np.array([oracle.score_down(w[f"L{li}.e_down"][e], v) for e in range(s["n_experts"])], np.float32)
            return [(int(e), lam * 0.7) for e in oracle.rank_scores(sc)[:2]]

        got, want = m.kl_score(), oracle_kl(top2)
        assert abs(got - want) <= 2e-3 + 0.05 * abs(want), (got, want)
    m.set_row_normalization("none")
    m.close()


@pytest.mark.parametrize("family", ["qwen2", "qwen2_fp8", "llama"])
def test_full_normalised_edit(device, family):
    """row_normalization = full (src/abliterate.zig:324-350, randomized SVD
    473-538): the device's rank-3 deltas against the oracle's restatement
    run with the same seeded sketch (matrix k of the edit takes seed + k, in
    the order layer by layer, o_proj then down_proj), compared through the
    edited KL."""
    g, m = load(device, family)
    s = g.spec
    w = g.f32_weights()
    rng = np.random.default_rng(13)
    dirs = rng.standard_normal((s["n_layers"] + 1, s["hidden"])).astype(np.float32)
    dirs /= np.linalg.norm(dirs, axis=1, keepdims=True)
    m.set_directions(dirs)
    prompts = g.prompts()
    toks, rb, rp, cap, first, take, last = flatten_batch(prompts)
    m.kl_init(prompts)
    po, pd = (1.1, 0.0, 0.5, 3.0), (0.9, 1.0, 0.3, 2.0)
    seed = 77
    m.set_row_normalization("full", lora_rank=3, seed=seed)
    m.apply_edit(po, pd)
    got = m.kl_score()
    om = OracleModel(s, w)
    k = 0
    for li in range(s["n_layers"]):
        v = dirs[li + 1]
        for comp, p in (("o", po), ("down", pd)):
            lam = oracle.kernel_weight(p, li)
            if lam is None:
                continue
            a, b = oracle.compute_delta_full(w[f"L{li}.{comp}"], v, lam, lora_rank=3, seed=seed + k)
            k += 1
            om.set_delta(li, comp, a, b)
    _, base = OracleModel(s, w).forward(toks, rb, rp, (), last)
    _, ed = om.forward(toks, rb, rp, (), last)
    want = oracle.kl_first_token(oracle.log_softmax(base), ed)[0]
    assert got > 0 and abs(got - want) <= 2e-3 + 0.05 * abs(want), (got, want)
    m.set_row_normalization("none")
    m.close()


@pytest.mark.parametrize("selective", [False, True])
def test_full_normalised_expert_edit(device, selective):
    """row_normalization = full on routed experts (src/moe.zig:1648, 1751: the
    reference's own full-mode expert tests): every edited expert's down
    projection gets a rank-3 delta from the randomised SVD, seeded in the
    device's order (layer by layer: o_proj, then the experts in the order they
    are edited, or the dense down_proj), against the oracle through the
    edited KL; broad (every expert) and selective (top 2 by alignment)."""
    g, m = load(device, "qwen3_moe")
    s = g.spec
    w = g.f32_weights()
    rng = np.random.default_rng(21)
    dirs = rng.standard_normal((s["n_layers"] + 1, s["hidden"])).astype(np.float32)
    dirs /= np.linalg.norm(dirs, axis=1, keepdims=True)
    m.set_directions(dirs)
    prompts = g.prompts()
    toks, rb, rp, cap, first, take, last = flatten_batch(prompts)
    m.kl_init(prompts)
    po, pd = (1.1, 0.0, 0.5, 3.0), (0.9, 1.0, 0.3, 2.0)
    seed = 41
    m.set_row_normalization("full", lora_rank=3, seed=seed)
    if selective:
        m.apply_expert_edit(po, pd, n_experts=2, strength=0.8)
    else:
        m.apply_edit(po, pd)
    got = m.kl_score()
    om = OracleModel(s, w)
    k = 0
    for li in range(s["n_layers"]):
        v = dirs[li + 1]
        lam = oracle.kernel_weight(po, li)
        if lam is not None:
            om.set_delta(li, "o", *oracle.compute_delta_full(w[f"L{li}.o"], v, lam, lora_rank=3, seed=seed + k))
            k += 1
        lam = oracle.kernel_weight(pd, li)
        if lam is None:
            continue
        if not s["moe_layers"][li]:
            om.set_delta(li, "down", *oracle.compute_delta_full(w[f"L{li}.down"], v, lam, lora_rank=3, seed=seed + k))
            k += 1
            continue
        if selective:
            sc = np.array([oracle.score_down(w[f"L{li}.e_down"][e], v) for e in range(s["n_experts"])], np.float32)
            chosen = [(int(e), lam * 0.8) for e in oracle.rank_scores(sc)[:2]]
        else:
            chosen = [(e, lam) for e in range(s["n_experts"])]
        for e, weight in chosen:
            a, b = oracle.compute_delta_full(w[f"L{li}.e_down"][e], v, weight, lora_rank=3, seed=seed + k)
            k += 1
            om.set_delta(li, ("e", e), a, b)
            got_d = m.delta(li, "expert_down_proj", e)
            assert got_d is not None and got_d[0].shape[0] == 3
    _, base = OracleModel(s, w).forward(toks, rb, rp, (), last)
    _, ed = om.forward(toks, rb, rp, (), last)
    want = oracle.kl_first_token(oracle.log_softmax(base), ed)[0]
    assert got > 0 and abs(got - want) <= 2e-3 + 0.05 * abs(want), (got, want)
    m.set_row_normalization("none")
    m.close()
