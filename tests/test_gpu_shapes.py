"""One decoder layer at each BASELINE configuration's shapes, on the GPU
through the C ABI, against the oracle (ditch's f32 CPU engine restated),
with the max abs and max rel errors of every compared quantity reported
(tests/parity_report.py; DITCH_PARITY_REPORT=<file> keeps them).

* C2 (Llama-3-8B: hidden 4096, 32 / 8 heads of 128, SwiGLU 14336, vocab
  128256, FP8 E4M3 with 128 x 128 f32 block scales, RoPE theta 5e5): the
  residual stream at both capture entries of every row and the last-token
  logits (src/model.zig:4619-4853), the residual sums and the directions
  (src/engine.zig:314-438, src/abliterate.zig:88-109), the none-mode edit
  deltas A = v^T W of o_proj and down_proj (src/abliterate.zig:264-280) and
  the first-token KL after that edit (src/scorers.zig:378-402).
* C4 (Qwen3-MoE: hidden 2048, 32 / 4 heads of 128 with q / k norms, 128
  MXFP4 experts of 768 with top-8 softmax routing, vocab 151936): the forward
  (src/moe.zig:998-1228) with near-tied routing rows left out as in
  test_gpu_model.py, and every expert's alignment score and their ranking
  (src/moe.zig:1239-1306).
* C5 (Llama-3-70B: hidden 8192, 64 / 8 heads of 128, SwiGLU 28672, vocab
  128256, bf16): the forward, the edit deltas and the KL.

Bounds: the forward as everywhere in these tests, max |err| <= 2e-3 + 2e-2 *
max |ref| per compared vector (bf16 tensor-core products with f32
accumulation against an all-f32 engine); the deltas A within 1e-4 of max |A|
(f32 GEMV-T sums in another order); residual sums within 2e-2 * max |ref|
(they are sums of the forward's residuals); direction cosine >= 0.999; KL
within 2e-3 + 5 %; expert scores within 1e-4 relative and the same order
where neighbouring scores differ by more than that.
"""
import numpy as np
import pytest

import ditch_b200
import oracle
from oracle.model import OracleModel, flatten_batch
from parity_report import record, record_value
from synth import make_model, prompts

pytestmark = pytest.mark.gpu

FWD_ATOL, FWD_RTOL = 2e-3, 2e-2
ROUTER_TIE = 2e-2


def bound(want):
    return FWD_ATOL + FWD_RTOL * float(np.abs(want).max())


C2 = dict(n_layers=1, hidden=4096, heads=32, kv_heads=8, head_dim=128, inter=14336, vocab=128256, eps=1e-5,
          rope_theta=5e5, fmt="fp8", block=(128, 128), share_embed_data=True, device_normals=True)
C4 = dict(n_layers=1, hidden=2048, heads=32, kv_heads=4, head_dim=128, inter=768, vocab=151936, eps=1e-6,
          rope_theta=1e6, qk_norm=True, fmt="mxfp4", moe=dict(experts=128, top_k=8, inter=768),
          share_embed_data=True, device_normals=True)
C5 = dict(n_layers=1, hidden=8192, heads=64, kv_heads=8, head_dim=128, inter=28672, vocab=128256, eps=1e-5,
          rope_theta=5e5, fmt="bf16", share_embed_data=True, device_normals=True)

# one layer: kernel_weight(p, 0) = p.max_weight when max_weight_position = 0
PO, PD = (1.2, 0.0, 0.5, 3.0), (0.8, 0.0, 0.3, 2.0)


def check_forward(case, m, om, ps, skip_rows=()):
    """Every captured residual row (both entries) and every last-token logit
    row within the bound. Rows in `skip_rows` (near-tied routing) are left
    out: in a one-layer model the routed experts come after the layer's
    attention, so a row's expert choice changes that row alone."""
    toks, rb, rp, cap, first, take, last = flatten_batch(ps, 10 ** 6)  # capture every row
    res, logits = m.forward(toks, rb, rp, cap, last)
    ores, ologits = om.forward(toks, rb, rp, cap, last)
    keep = np.ones(len(toks), bool)
    keep[list(skip_rows)] = False
    keep_prompt = keep[np.asarray(last, np.int64)]
    assert keep.sum() > 0.5 * len(toks)
    for l in range(res.shape[0]):
        rows = keep if l == res.shape[0] - 1 else np.ones(len(toks), bool)
        got, want = res[l][rows], ores[l][rows]
        worst = max(float(np.abs(got[r] - want[r]).max() - bound(want[r])) for r in range(len(got)))
        record(case, f"residual entry {l} ({int(rows.sum())} rows)", got, want, bound=bound(want))
        assert worst <= 0.0, (l, worst)
    got, want = logits[keep_prompt], ologits[keep_prompt]
    record(case, f"last-token logits ({int(keep_prompt.sum())} prompts)", got, want, bound=bound(want))
    for i in np.nonzero(keep_prompt)[0]:
        assert np.abs(logits[i] - ologits[i]).max() <= bound(ologits[i]), i
        assert int(np.argmax(logits[i])) == int(np.argmax(ologits[i])), i
    return toks, rb, rp, last


def check_edit_and_kl(case, m, om_spec, w, ps, dirs):
    """The none-mode deltas of o_proj / down_proj and the KL after the edit."""
    m.set_directions(dirs)
    m.kl_init(ps)
    assert abs(m.kl_score()) < 1e-6  # base model (src/scorers.zig:839-926)
    m.apply_edit(PO, PD)
    kl = m.kl_score()
    om = OracleModel(om_spec, w)
    v = dirs[1]
    for comp, p, name in (("attn_o_proj", PO, "o"), ("mlp_down_proj", PD, "down")):
        lam = oracle.kernel_weight(p, 0)
        a, b = oracle.compute_delta_none(w[f"L0.{name}"], v, lam)
        om.set_delta(0, "o" if name == "o" else "down", a, b)
        da, db = m.delta(0, comp)
        e = record(case, f"edit delta A = v^T W ({name})", da[0], a, bound=1e-4 * float(np.abs(a).max()))
        assert e["max_abs"] <= 1e-4 * e["ref_max_abs"] + 1e-7
        record(case, f"edit delta b = -lambda v ({name})", db[:, 0], b)
        np.testing.assert_allclose(db[:, 0], b, rtol=1e-6, atol=1e-9)
    toks, rb, rp, cap, first, take, last = flatten_batch(ps)
    _, base = OracleModel(om_spec, w).forward(toks, rb, rp, (), last)
    _, edited = om.forward(toks, rb, rp, (), last)
    okl, _ = oracle.kl_first_token(oracle.log_softmax(base), edited)
    record_value(case, "first-token KL after the edit", kl, okl, bound="2e-3 + 5%")
    assert kl > 0
    assert abs(kl - okl) <= 2e-3 + 0.05 * abs(okl), (kl, okl)


def unit_dirs(seed, n, hidden):
    rng = np.random.default_rng(seed)
    d = rng.standard_normal((n, hidden)).astype(np.float32)
    return d / np.linalg.norm(d, axis=1, keepdims=True)


def test_c2_layer(device):
    spec, w, tensors = make_model(2002, **C2)
    ps = prompts(2003, [64] * 8, spec["vocab"])
    m = ditch_b200.Model(device, spec, tensors, max_seq=64)
    del tensors
    om = OracleModel(spec, w)
    check_forward("C2 layer", m, om, ps)
    # residual sums (window 1) and directions from a good and a bad half
    good, bad = ps[:4], ps[4:]
    gs, gc = m.residual_sums(good, window=1)
    bs, bc = m.residual_sums(bad, window=1)
    osums = []
    for half in (good, bad):
        toks, rb, rp, cap, first, take, last = flatten_batch(half)
        ores, _ = om.forward(toks, rb, rp, cap, ())
        osums.append(oracle.residual_sums(ores, first, take))
    for name, got, want in (("good", gs, osums[0]), ("bad", bs, osums[1])):
        e = record("C2 layer", f"residual sums ({name}, f64)", got, want, bound=2e-2 * float(np.abs(want).max()))
        assert e["max_rel"] <= 2e-2
    assert gc == bc == 4
    dirs = m.directions(gs, gc, bs, bc, True)
    odirs = oracle.compute_directions((osums[0] / 4).astype(np.float32), (osums[1] / 4).astype(np.float32), True)
    for l in range(dirs.shape[0]):
        cos = float(np.dot(dirs[l], odirs[l]) / (np.linalg.norm(dirs[l]) * np.linalg.norm(odirs[l])))
        record_value("C2 layer", f"direction cosine (entry {l})", cos, 1.0, bound=">= 0.999")
        assert cos >= 0.999, (l, cos)
    check_edit_and_kl("C2 layer", m, spec, w, ps, unit_dirs(2004, 2, spec["hidden"]))
    m.close()


def near_tied_rows(spec, w, toks, rb, rp):
    """Rows whose top-k boundary is a near-tie in the oracle's router (gap
    between the k-th and (k+1)-th router logit below ROUTER_TIE): bf16
    activations may pick the other expert there (src/moe.zig:971-985 takes
    the first maximum of f32 scores)."""
    k = spec["top_k"]
    w0 = dict(w)
    for a in ("gate", "up", "down"):
        w0[f"L0.e_{a}"] = np.zeros_like(w[f"L0.e_{a}"])
    cap = np.arange(len(toks), dtype=np.uintp)
    res, _ = OracleModel(spec, w0).forward(toks, rb, rp, cap, ())
    x = res[1]
    h = x / np.sqrt((x * x).mean(axis=1, keepdims=True) + spec["eps"]) * w["L0.post_norm"]
    top = np.sort(h @ w["L0.router"].T, axis=1)[:, ::-1]
    return set(np.nonzero(top[:, k - 1] - top[:, k] < ROUTER_TIE)[0].tolist())


def test_c4_layer(device):
    spec, w, tensors = make_model(4004, **C4)
    ps = prompts(4005, [64] * 8, spec["vocab"])
    m = ditch_b200.Model(device, spec, tensors, max_seq=64)
    del tensors
    toks, rb, rp, cap, first, take, last = flatten_batch(ps, 10 ** 6)
    tied = near_tied_rows(spec, w, toks, rb, rp)
    record_value("C4 layer", "near-tied routing rows left out", len(tied), 0, rows=len(toks))
    check_forward("C4 layer", m, OracleModel(spec, w), ps, skip_rows=tied)
    v = unit_dirs(4006, 1, spec["hidden"])[0]
    order, scores = m.rank_experts(0, v)
    osc = np.array([oracle.score_down(w["L0.e_down"][e], v) for e in range(spec["n_experts"])], np.float32)
    e = record("C4 layer", "expert alignment scores ||v^T W_down|| / ||W_down||_F (128 experts)", scores, osc)
    assert e["max_elem_rel"] <= 1e-4
    oorder = oracle.rank_scores(osc)
    ranked = osc[oorder]
    gap = np.abs(np.diff(ranked)) > 1e-4 * np.abs(ranked[:-1])  # gap[i]: ranks i and i + 1 do not nearly tie
    for i in range(len(ranked)):  # a rank clear of both neighbours holds the oracle's expert
        if (i == 0 or gap[i - 1]) and (i == len(ranked) - 1 or gap[i]):
            assert order[i] == oorder[i], i
    record_value("C4 layer", "expert ranking agreement", float(np.mean(order == oorder)), 1.0)
    m.close()


def test_c5_layer(device):
    spec, w, tensors = make_model(5005, **C5)
    ps = prompts(5006, [32] * 4, spec["vocab"])
    m = ditch_b200.Model(device, spec, tensors, max_seq=32)
    del tensors
    check_forward("C5 layer", m, OracleModel(spec, w), ps)
    check_edit_and_kl("C5 layer", m, spec, w, ps, unit_dirs(5007, 2, spec["hidden"]))
    m.close()
