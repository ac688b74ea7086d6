"""Greedy generation on the device (ditch_cuda_generate: prefill into a KV
cache, then one-row decode steps) against the oracle.

Every generated token is checked teacher-forced: the oracle runs the
forward over the prompt plus the device's tokens and the device's token at
step j must be the oracle's first maximum of row j, or, where the oracle's
top two logits are closer than the forward tolerance (FWD_ATOL + FWD_RTOL *
max |row|, the bound of test_gpu_model.py), a logit within that tolerance of
the maximum. The stop rule (EOS kept, max_new_tokens, at least one token) is
checked exactly. The fixture families also pin the first token to the
reference's argmax, as src/model_test.zig:76-83 does with its own generate.
"""
import numpy as np
import pytest

import ditch_b200
from golden_loader import Golden
from oracle.model import OracleModel, argmax_first, flatten_batch
from synth import make_model, prompts
from test_gpu_model import near_tied_tokens

pytestmark = pytest.mark.gpu

FWD_ATOL, FWD_RTOL = 2e-3, 2e-2


class _Weights:
    """The two members near_tied_tokens reads."""

    def __init__(self, spec, f32):
        self.spec, self._w = spec, f32

    def f32_weights(self):
        return self._w


def check_generation(om, ps, got, max_new, eos=(), routed=None):
    """Teacher-forced check of the device's tokens; returns (tokens, exact)
    counts: all checked tokens and those with a clear oracle maximum. With
    routed experts (`routed` = (spec, f32 weights)) a prompt whose sequence
    has a near-tied routing choice (test_gpu_model.near_tied_tokens) at or
    before a failing row is not checked past that row: the device may take
    the other expert there."""
    eos = set(int(e) for e in eos)
    n_tok = n_exact = 0
    for i, p in enumerate(ps):
        g = got[i]
        assert 1 <= len(g) <= max(max_new, 1), (i, len(g))
        stopped = g[-1] in eos
        assert stopped or len(g) == max(max_new, 1), (i, g)
        assert not any(t in eos for t in g[:-1]), (i, g)
        seq = np.concatenate([np.asarray(p, np.uint32), np.asarray(g[:-1], np.uint32)])
        toks, rb, rp, cap, _, _, last = flatten_batch([seq], 10 ** 6)
        rows = np.arange(len(p) - 1, len(seq), dtype=np.uintp)
        _, logits = om.forward(toks, rb, rp, logit_rows=rows)
        tied = None
        for j, t in enumerate(g):
            row = logits[j]
            best, gap = argmax_first(row)
            tol = FWD_ATOL + FWD_RTOL * float(np.abs(row).max())
            ok = t == best if gap > tol else row[t] >= row[best] - tol
            if not ok and routed is not None:
                if tied is None:
                    tied = near_tied_tokens(_Weights(*routed), toks, rb, rp, cap, last)
                if tied and min(tied) <= len(p) - 1 + j:
                    break
            assert ok, (i, j, t, best, gap, float(row[best] - row[t]))
            n_exact += int(gap > tol)
            n_tok += 1
    return n_tok, n_exact


CASES = {
    # head size 64: the tensor-core prefill ropes keys in place and the cache copies them
    "dense_hd64_bias": dict(n_layers=3, hidden=256, heads=4, kv_heads=2, head_dim=64, inter=512, qkv_bias=True),
    # head size 32 with q/k norms: the generic prefill, keys normed and roped while stored
    "qknorm_hd32_gqa4": dict(n_layers=2, hidden=256, heads=8, kv_heads=2, head_dim=32, inter=384, qk_norm=True),
    "fp8_hd128": dict(n_layers=2, hidden=256, heads=2, kv_heads=1, head_dim=128, inter=512, fmt="fp8",
                      block=(128, 128)),
    # 7 query heads per kv head (padded to 8 in the register decode path), and plain multi-head attention
    "gqa7_hd64": dict(n_layers=2, hidden=256, heads=14, kv_heads=2, head_dim=64, inter=512, qkv_bias=True),
    "mha_hd128": dict(n_layers=2, hidden=256, heads=2, kv_heads=2, head_dim=128, inter=512),
    "moe_mxfp4": dict(n_layers=2, hidden=256, heads=4, kv_heads=2, head_dim=64, inter=256, fmt="mxfp4",
                      moe=dict(experts=8, top_k=2, inter=128)),
}


@pytest.mark.parametrize("case", sorted(CASES))
def test_generate_matches_oracle(device, case):
    spec, f32, tensors = make_model(900 + sorted(CASES).index(case), **CASES[case])
    ps = prompts(31, [5, 17, 1, 33, 9], spec["vocab"])
    m = ditch_b200.Model(device, spec, tensors, max_seq=64)
    om = OracleModel(spec, f32)
    got = m.generate(ps, 12)
    routed = (spec, f32) if spec.get("moe_layers") else None
    n_tok, n_exact = check_generation(om, ps, got, 12, routed=routed)
    assert n_tok >= 12 * (len(ps) - 1), n_tok
    assert n_exact >= n_tok // 2, (n_exact, n_tok)  # most tokens have a clear maximum
    # where no step is a near-tie the whole continuation equals the oracle's own greedy run
    want, gaps = om.generate(ps, 12)
    for i in range(len(ps)):
        tol = 2 * FWD_ATOL + 0.05
        if min(gaps[i]) > tol and routed is None:
            assert got[i] == want[i], (i, got[i], want[i])
    m.close()


def test_generate_stops_at_eos_and_length(device):
    spec, f32, tensors = make_model(950, n_layers=2, hidden=256, heads=4, kv_heads=2, head_dim=64, inter=512)
    ps = prompts(32, [8, 3, 21], spec["vocab"])
    m = ditch_b200.Model(device, spec, tensors, max_seq=64)
    om = OracleModel(spec, f32)
    free = m.generate(ps, 10)
    eos = [free[0][3], free[2][6]]
    got = m.generate(ps, 10, eos)
    check_generation(om, ps, got, 10, eos)
    if not any(free[0][3] in free[i][:3] for i in (1, 2)):
        # the decode batches match the free run's until prompt 0 stops at its 4th token
        assert got[0] == free[0][:len(got[0])] and len(got[0]) <= 4 and got[0][-1] in eos
    # at least one token, whatever max_new_tokens says (src/model.zig:5406-5410)
    for max_new in (0, 1):
        one = m.generate(ps, max_new)
        assert [len(g) for g in one] == [1] * len(ps)
        assert [g[0] for g in one] == [f[0] for f in free]
    # the first token is the prefill's argmax
    toks, rb, rp, _, _, _, last = flatten_batch(ps)
    _, logits = m.forward(toks, rb, rp, logit_rows=last)
    assert [f[0] for f in free] == [argmax_first(r)[0] for r in logits]
    m.close()


def test_generate_rejects_too_long(device):
    spec, f32, tensors = make_model(951, n_layers=1, hidden=128, heads=2, kv_heads=1, head_dim=64, inter=256)
    m = ditch_b200.Model(device, spec, tensors, max_seq=32)
    with pytest.raises(ditch_b200.DitchCudaError):
        m.generate(prompts(1, [20], spec["vocab"]), 20)
    assert len(m.generate(prompts(1, [20], spec["vocab"]), 12)[0]) == 12  # still usable
    m.close()


FAMILIES = ["qwen2", "llama", "qwen3", "qwen2_fp8", "qwen2_int4", "qwen3_moe", "mixtral", "qwen2_gguf"]


@pytest.mark.parametrize("family", FAMILIES)
def test_fixture_generation(device, family):
    """src/model_test.zig:76-83: generate 4 tokens; the first is the
    reference's argmax. All 4 are checked teacher-forced against the oracle."""
    g = Golden(family)
    m = ditch_b200.Model(device, g.spec, g.cuda_tensors(), max_seq=64)
    ps = g.prompts()
    got = m.generate(ps, 4)
    for i, c in enumerate(g.cases):
        assert got[i][0] == c["argmax"], (family, i)
    routed = (g.spec, g.f32_weights()) if g.spec.get("moe_layers") else None
    check_generation(OracleModel(g.spec, g.f32_weights()), ps, got, 4, routed=routed)
    m.close()


def test_keyword_rate_on_device(device):
    """KeywordRate (src/scorers.zig:97-155) with the device generating and a
    toy tokenizer on the host: the rate is the share of responses with a
    marker, batch by batch; deterministic mode makes the repeated generation
    bit-identical so the two counts must agree exactly."""
    from ditch_b200.scorers import is_match, keyword_rate

    spec, f32, tensors = make_model(960, n_layers=2, hidden=256, heads=4, kv_heads=2, head_dim=64, inter=512)
    ps = prompts(33, [6, 9, 12, 4, 20, 7], spec["vocab"])
    m = ditch_b200.Model(device, spec, tensors, max_seq=64)
    words = ["sorry", "a", "b", "c", "d", "e", "f"]

    def detok(toks):
        return " ".join(words[t % 7] for t in toks)

    device.set_deterministic(True)
    try:
        first = []
        r = keyword_rate(m, ps, detok, max_new_tokens=8, batch_size=4, first_tokens=first)
        outs = m.generate(ps[:4], 8) + m.generate(ps[4:], 8)
    finally:
        device.set_deterministic(False)
    want = [is_match(detok(o)) for o in outs]
    assert r["value"] == sum(want) / len(ps) and r["pruned"] is None
    assert first == [(o[0], w) for o, w in zip(outs, want)]
    check_generation(OracleModel(spec, f32), ps, outs, 8)
    m.close()
