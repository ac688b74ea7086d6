"""The CPU oracle against the reference's golden fixtures and known answers.

These pin the oracle before it is trusted as the parity checker of the CUDA
product: the fixture models and their reference outputs come from ditch's own
tests/fixtures (src/model_test.zig:58-84, 2e-3 max abs), the known answers
from its inline tests (file:line on each test).
"""
import math

import numpy as np
import pytest

import oracle
from golden_loader import Golden
from oracle.model import OracleModel, flatten_batch

FAMILIES = ["qwen2", "llama", "qwen3", "qwen3_moe", "qwen2_fp8", "qwen2_int4", "qwen3_moe_big", "qwen3_moe_fused",
            "qwen3_moe_fused_t", "mixtral", "qwen2_gguf", "llama_gguf"]


@pytest.mark.parametrize("family", FAMILIES)
def test_fixture_forward(family):
    """src/model_test.zig:58-84: last logits and every residual entry within 2e-3."""
    g = Golden(family)
    m = OracleModel(g.spec, g.f32_weights())
    toks, rb, rp, cap, first, take, last = flatten_batch(g.prompts())
    res, logits = m.forward(toks, rb, rp, cap, last)
    for i, c in enumerate(g.cases):
        assert np.abs(logits[i] - c["last_logits"]).max() < 2e-3
        assert np.abs(res[:, i, :] - c["last_hidden"]).max() < 2e-3
        assert int(np.argmax(logits[i])) == c["argmax"]


@pytest.mark.parametrize("family", FAMILIES)
def test_fixture_generation(family):
    """src/model_test.zig:76-83: greedy generation of 4 tokens starts with
    the reference's argmax; each step's token is the first maximum of that
    step's logits over the extended sequence (src/model.zig:5378-5444)."""
    g = Golden(family)
    m = OracleModel(g.spec, g.f32_weights())
    toks, gaps = m.generate(g.prompts(), 4)
    assert [t[0] for t in toks] == [c["argmax"] for c in g.cases]
    assert all(len(t) == 4 for t in toks)
    seq = [np.concatenate([p, np.asarray(t[:3], np.uint32)]) for p, t in zip(g.prompts(), toks)]
    ft, rb, rp, cap, first, take, last = flatten_batch(seq)
    _, logits = m.forward(ft, rb, rp, cap, last)
    assert [int(np.argmax(r)) for r in logits] == [t[3] for t in toks]


def test_generation_stop_rules():
    """EOS is kept and ends the prompt; max_new_tokens 0 and 1 give one
    token (src/model.zig:5404-5440)."""
    g = Golden("qwen2")
    m = OracleModel(g.spec, g.f32_weights())
    free, _ = m.generate(g.prompts(), 6)
    stop, _ = m.generate(g.prompts(), 6, eos_ids=[free[0][2]])
    assert stop[0] == free[0][:free[0].index(free[0][2]) + 1]
    for n in (0, 1):
        one, _ = m.generate(g.prompts(), n)
        assert [len(t) for t in one] == [1] * len(free)


def test_pre_normalised_edit_removes_direction():
    """src/abliterate.zig:554-592, row_normalization = pre, K = 1: the
    direction vanishes from the row-normalised edited matrix,
    sum_i (v_i / n_i) W'_ij ~ 0, and the delta stays rank 1."""
    rng = np.random.default_rng(7)
    w = rng.standard_normal((6, 5)).astype(np.float32)
    v = rng.standard_normal(6).astype(np.float32)
    v /= np.linalg.norm(v)
    a, b = oracle.compute_delta_pre(w, v, 1.0)
    assert a.shape == (5,) and b.shape == (6,)
    wp = oracle.materialize(w, a, b)
    n = oracle.row_norms(w)
    assert np.abs((v / n) @ wp).max() < 1e-4
    # a zero row keeps its zero norm out of the division (vn = 0 there)
    w[2] = 0.0
    a, b = oracle.compute_delta_pre(w, v, 0.5)
    assert np.isfinite(a).all() and b[2] == 0.0


def test_full_normalised_edit_reconstructs_the_renormalised_matrix():
    """src/abliterate.zig:554-620, row_normalization = full, K = 1, lora_rank
    5 on a 6 x 5 matrix: the rank-5 randomised SVD reproduces
    W' = diag(n) rownorm(Wn - v a^T), a = v^T Wn, within 1e-3."""
    rng = np.random.default_rng(7)
    w = rng.standard_normal((6, 5)).astype(np.float32)
    v = rng.standard_normal(6).astype(np.float32)
    v /= np.linalg.norm(v)
    la, lb = oracle.compute_delta_full(w, v, 1.0, lora_rank=5, seed=1)
    assert la.shape == (5, 5) and lb.shape == (6, 5)
    wp = oracle.materialize_rank(w, la, lb)
    n = np.linalg.norm(w, axis=1)
    wn = w / n[:, None]
    a = v @ wn
    rows = wn - np.outer(v, a)
    want = rows / np.linalg.norm(rows, axis=1, keepdims=True) * n[:, None]
    assert np.abs(wp - want).max() < 1e-3
    # rank 3 (ditch's default) of the same: close, not exact
    la3, lb3 = oracle.compute_delta_full(w, v, 1.0, lora_rank=3, seed=1)
    assert la3.shape == (3, 5)
    assert np.abs(oracle.materialize_rank(w, la3, lb3) - want).max() < 0.5


def test_argmax_first_rule():
    """src/model.zig:5194-5204: the first maximum wins, NaN never does, a row
    with nothing above -inf gives 0."""
    from oracle.model import argmax_first
    assert argmax_first(np.array([1, 3, 3], np.float32))[0] == 1
    assert argmax_first(np.array([np.nan, 2, np.nan, 2], np.float32))[0] == 1
    assert argmax_first(np.array([-np.inf, -np.inf], np.float32))[0] == 0
    assert argmax_first(np.array([np.nan, -np.inf], np.float32))[0] == 0


def test_fixture_forward_unbatched_matches_batched():
    """One prompt per call gives the same rows as the batched call (engine batching)."""
    g = Golden("qwen2")
    m = OracleModel(g.spec, g.f32_weights())
    toks, rb, rp, cap, first, take, last = flatten_batch(g.prompts())
    res, logits = m.forward(toks, rb, rp, cap, last)
    for i, p in enumerate(g.prompts()):
        t1, b1, p1, c1, _, _, l1 = flatten_batch([p])
        r1, lg1 = m.forward(t1, b1, p1, c1, l1)
        np.testing.assert_array_equal(lg1[0], logits[i])
        np.testing.assert_array_equal(r1[:, 0], res[:, i])


def test_matmul_delta_known_answer():
    """src/tensor.zig:1400-1421: W=[[1,2],[3,4],[5,6]], delta a=[1,0], b=[1,1,1]."""
    w = np.array([[1, 2], [3, 4], [5, 6]], np.float32)
    out = oracle.matmul_t(np.ones((1, 2)), w, np.array([1, 0], np.float32), np.ones(3, np.float32))
    np.testing.assert_array_equal(out[0], [4, 8, 12])
    np.testing.assert_array_equal(oracle.matvec_t_multi(w, np.ones(3))[0], [9, 12])


def _f16_bytes(v):
    return np.array([v], np.float16).view(np.uint8)


def test_q8_0_known_block():
    """src/quant.zig:367-388: d = 2.5/127 and q[5] = 127 for the block's maximum."""
    rng = np.random.default_rng(1)
    x = ((rng.random(64) * 2 - 1) * 2).astype(np.float32)
    x[0], x[5], x[17] = 0, 2.5, -2.5
    q = oracle.quant_q8_0(x)
    assert q[2 + 5] == 127
    y = oracle.dequant_ggml(5, q, 64)
    for blk in range(2):
        amax = np.abs(x[blk * 32:(blk + 1) * 32]).max()
        d = float(np.float16(amax / 127))
        assert np.all(np.abs(x[blk * 32:(blk + 1) * 32] - y[blk * 32:(blk + 1) * 32]) <= d * 0.5 + amax * 1e-3)
    assert abs(y[5] - 2.5) <= 2.5e-3


def test_q4_k_hand_built_block():
    """src/quant.zig:426-448."""
    b = np.zeros(144, np.uint8)
    b[0:2] = _f16_bytes(0.5)
    b[2:4] = _f16_bytes(0.25)
    b[4 + 0], b[4 + 4], b[4 + 1], b[4 + 5] = 4, 2, 8, 1
    b[4 + 8] = 0x35
    b[4 + 0] |= 0x40
    b[16 + 0] = 0x3 | (0x9 << 4)
    b[16 + 64] = 0x7
    y = oracle.dequant_ggml(10, b, 256)
    assert abs(y[0] - (0.5 * 4 * 3 - 0.25 * 2)) < 1e-6
    assert abs(y[32] - (0.5 * 8 * 9 - 0.25 * 1)) < 1e-6
    assert abs(y[1] - (-0.25 * 2)) < 1e-6
    assert abs(y[128] - (0.5 * 21 * 7 - 0.25 * 3)) < 1e-6


def test_q6_k_and_q8_k_hand_built():
    """src/quant.zig:450-482."""
    b = np.zeros(210, np.uint8)
    b[208:210] = _f16_bytes(0.125)
    b[192] = np.uint8(3)
    b[194] = np.int8(-2).view(np.uint8)
    b[0] = 0xA
    b[128] = 0x2
    b[32] = 0x1
    b[128] |= 0x1 << 2
    y = oracle.dequant_ggml(11, b, 256)
    assert abs(y[0] - 0.125 * 3 * 10) < 1e-6
    assert abs(y[32] - 0.125 * -2 * -15) < 1e-6
    assert abs(y[1] - 0.125 * 3 * -32) < 1e-6
    b = np.zeros(292, np.uint8)
    b[0:4] = np.array([0.75], np.float32).view(np.uint8)
    b[4 + 3] = np.int8(-100).view(np.uint8)
    b[4 + 255] = 64
    y = oracle.dequant_ggml(12, b, 256)
    assert y[3] == -75 and y[255] == 48 and y[0] == 0


def test_fp8_table():
    """src/dequant.zig:1290-1310: 0x7e -> 448, 0x01 -> 2^-9, 0x7f NaN."""
    L = oracle.lib()
    assert L.or_e4m3_value(0x7E) == 448.0
    assert L.or_e4m3_value(0x01) == 2.0 ** -9
    assert math.isnan(L.or_e4m3_value(0x7F))
    assert L.or_e4m3_value(0xFE) == -448.0


def test_e8m0_times_e2m1_exact():
    """src/dequant.zig:263-268."""
    L = oracle.lib()
    e2m1 = [0, 0.5, 1, 1.5, 2, 3, 4, 6, -0.0, -0.5, -1, -1.5, -2, -3, -4, -6]
    for b in range(255):
        s = L.or_e8m0_scale(b)
        for v in e2m1:
            assert np.float32(v * 2.0 ** (b - 127)) == np.float32(v) * np.float32(s)


def test_unpack_field_straddles_words():
    """src/dequant.zig unpackField: a 5-bit field across a word boundary."""
    vals = [3, 17, 31, 0, 9, 22, 5, 30]
    words = np.zeros(2, np.uint32)
    for i, v in enumerate(vals):
        s = i * 5
        words[s // 32] |= np.uint32((v << (s % 32)) & 0xFFFFFFFF)
        if s % 32 + 5 > 32:
            words[s // 32 + 1] |= np.uint32(v >> (32 - s % 32))
    got = [oracle.lib().or_unpack_field(words.ctypes.data_as(oracle.u32p), i, 5) for i in range(len(vals))]
    assert got == vals


def test_kernel_weight_shape():
    """src/abliterate.zig:736-742."""
    p = (1.0, 10.0, 0.2, 4.0)
    assert abs(oracle.kernel_weight(p, 10) - 1.0) < 1e-6
    assert abs(oracle.kernel_weight(p, 8) - 0.6) < 1e-6
    assert abs(oracle.kernel_weight(p, 14) - 0.2) < 1e-6
    assert oracle.kernel_weight(p, 15) is None


def test_edit_removes_direction():
    """src/abliterate.zig:554-624 (none mode): v^T W' = (1 - lambda) v^T W, so lambda = 1 removes it."""
    rng = np.random.default_rng(7)
    w = rng.standard_normal((6, 5)).astype(np.float32)
    v = rng.standard_normal(6).astype(np.float32)
    v /= np.linalg.norm(v)
    a, b = oracle.compute_delta_none(w, v, 1.0)
    w2 = oracle.materialize(w, a, b)
    assert np.abs(v @ w2).max() < 1e-4


def test_directions_recover_planted_direction():
    """Difference of means recovers a planted unit direction (src/directions.zig:514-699)."""
    rng = np.random.default_rng(3)
    d = rng.standard_normal(64).astype(np.float32)
    d /= np.linalg.norm(d)
    good = rng.standard_normal((3, 64)).astype(np.float32) * 0.01
    bad = good + 2.0 * d
    dirs = oracle.compute_directions(good, bad, orthogonalize=False)
    for e in range(3):
        assert abs(float(dirs[e] @ d)) > 0.999


def test_kl_zero_on_identical_logits():
    """src/scorers.zig:839-926: KL is 0 on the base model."""
    rng = np.random.default_rng(0)
    logits = rng.standard_normal((4, 271)).astype(np.float32)
    base = oracle.log_softmax(logits)
    kl, per = oracle.kl_first_token(base, logits)
    assert abs(kl) < 1e-6
    kl2, _ = oracle.kl_first_token(base, logits + rng.standard_normal(logits.shape).astype(np.float32))
    assert kl2 > 0


def test_rank_scores_ties_by_index():
    """src/moe.zig:1296-1306: descending, ties keep index order."""
    np.testing.assert_array_equal(oracle.rank_scores([0.5, 0.9, 0.5, 0.9, 0.1]), [1, 3, 0, 2, 4])
