"""The resident forward on seeded synthetic models against the oracle, at the
shapes the reference fixtures do not reach: head sizes 64 and 128 (the tiled
attention kernel), prompts longer than one 64-row chunk, GQA, q/k norms, FP8
block weights, MXFP4 routed experts, and every RoPE scaling type.

Tolerance as in test_gpu_model.py: max |err| <= 2e-3 + 2e-2 * max |ref|."""
import numpy as np
import pytest

import ditch_b200
from oracle.model import OracleModel, flatten_batch
from synth import make_model, prompts

pytestmark = pytest.mark.gpu

CASES = [
    dict(head_dim=64, heads=4, kv_heads=2, hidden=256),
    dict(head_dim=128, heads=4, kv_heads=1, hidden=512, qk_norm=True),
    dict(head_dim=128, heads=8, kv_heads=2, hidden=512, fmt="fp8"),
    dict(head_dim=64, heads=4, kv_heads=4, hidden=256, qkv_bias=True, fmt="fp8", block=(32, 64)),
]


def check_forward(device, spec, f32, tensors, ps, max_bad_rows=0.0):
    """Every logit row and every captured residual row within the bound, or
    (routed experts) all but a fraction `max_bad_rows` of them: top-k routing
    is a discrete function of router logits computed from a residual stream
    that carries bf16 rounding, so near-tied experts can swap on either side
    (src/moe.zig:971-985 picks the first maximum of f32 scores)."""
    m = ditch_b200.Model(device, spec, tensors, max_seq=256)
    toks, rb, rp, cap, first, take, last = flatten_batch(ps, 2)
    res, logits = m.forward(toks, rb, rp, cap, last)
    ores, ologits = OracleModel(spec, f32).forward(toks, rb, rp, cap, last)
    rows_bad = rows = 0
    for i in range(len(ps)):
        tol = 2e-3 + 2e-2 * float(np.abs(ologits[i]).max())
        rows += 1
        rows_bad += int(np.abs(logits[i] - ologits[i]).max() > tol)
    for l in range(spec["n_layers"] + 1):
        tol = 2e-3 + 2e-2 * float(np.abs(ores[l]).max())
        err = np.abs(res[l] - ores[l]).max(axis=1)
        rows += err.size
        rows_bad += int((err > tol).sum())
        assert err.max() <= 10 * tol, l  # a swapped expert changes a row, not the scale
    assert rows_bad <= max_bad_rows * rows, f"{rows_bad} of {rows} rows outside the bound"
    m.close()


@pytest.mark.parametrize("case", range(len(CASES)))
def test_synthetic_dense_forward(device, case):
    kw = dict(CASES[case])
    spec, f32, tensors = make_model(100 + case, **kw)
    ps = prompts(7 + case, [1, 5, 64, 65, 150, 33], spec["vocab"])
    check_forward(device, spec, f32, tensors, ps)


ROPES = [
    dict(rope_scaling=2, rope_factor=2.5),
    dict(rope_scaling=3, rope_factor=4.0, rope_orig_max=32.0, rope_beta_fast=32.0, rope_beta_slow=1.0,
         rope_truncate=1, rope_attention_factor=float(np.float32(0.1 * np.log(4.0) + 1.0))),
    dict(rope_scaling=3, rope_factor=8.0, rope_orig_max=64.0, rope_beta_fast=16.0, rope_beta_slow=2.0,
         rope_truncate=0, rope_attention_factor=1.2),
    dict(rope_scaling=4, rope_factors=32, rope_attention_factor=1.0),
    dict(rope_scaling=4, rope_factors=27, rope_attention_factor=1.15),  # fewer divisors than frequencies
]


@pytest.mark.parametrize("case", range(len(ROPES)))
def test_rope_scalings_match_oracle(device, case):
    """Linear, YaRN (truncated and not) and per-frequency divisors (GGUF
    rope_freqs, LongRoPE) against the oracle's fillRope (src/model.zig:
    2200-2282); plain RoPE is outside the bound at these positions, so the
    scaling is what the check measures."""
    spec, f32, tensors = make_model(200 + case, head_dim=64, heads=4, kv_heads=2, hidden=256)
    r = dict(ROPES[case])
    if "rope_factors" in r:
        r["rope_factors"] = np.random.default_rng(210 + case).uniform(1.0, 8.0, r["rope_factors"]).astype(np.float32)
    scaled = dict(spec, **r)
    ps = prompts(220 + case, [1, 40, 150], spec["vocab"])
    check_forward(device, scaled, f32, tensors, ps)
    toks, rb, rp, cap, first, take, last = flatten_batch(ps, 2)
    _, a = OracleModel(scaled, f32).forward(toks, rb, rp, cap, last)
    _, b = OracleModel(spec, f32).forward(toks, rb, rp, cap, last)
    assert max(np.abs(a[i] - b[i]).max() - (2e-3 + 2e-2 * np.abs(a[i]).max()) for i in range(len(ps))) > 0


@pytest.mark.parametrize("fmt,staging", [("bf16", 1024), ("mxfp4", 1024), ("mxfp4", 0)])
def test_synthetic_moe_forward(device, fmt, staging):
    """MXFP4 experts with the default plan (each expert stack decoded once to
    bf16 and kept, the grouped GEMM over the copy) and with staging off (the
    grouped GEMM decoding MXFP4 tile by tile)."""
    spec, f32, tensors = make_model(300, hidden=256, head_dim=64, heads=4, kv_heads=2, fmt=fmt,
                                    moe=dict(experts=16, top_k=4, inter=128))
    ps = prompts(31, [40, 17, 64, 3, 70], spec["vocab"])
    device.set_decode_staging(staging)
    try:
        check_forward(device, spec, f32, tensors, ps, max_bad_rows=0.2)
    finally:
        device.set_decode_staging(1024)


def test_moe_expert_copy_equals_in_gemm_decode(device):
    """The grouped GEMM over the kept bf16 copy of an MXFP4 expert stack and
    the grouped GEMM decoding tile by tile see the same bf16 operand: the
    forwards agree bit for bit."""
    spec, f32, tensors = make_model(301, hidden=256, head_dim=64, heads=4, kv_heads=2, fmt="mxfp4",
                                    moe=dict(experts=16, top_k=4, inter=128))
    ps = prompts(32, [40, 17, 64, 3, 70], spec["vocab"])
    from oracle.model import flatten_batch as fb
    toks, rb, rp, cap, first, take, last = fb(ps, 2)
    outs = []
    device.set_deterministic(True)
    try:
        for staging in (1024, 0):
            device.set_decode_staging(staging)
            m = ditch_b200.Model(device, spec, tensors, max_seq=128)
            outs.append(m.forward(toks, rb, rp, cap, last))
            m.close()
    finally:
        device.set_decode_staging(1024)
        device.set_deterministic(False)
    assert np.array_equal(outs[0][0], outs[1][0]) and np.array_equal(outs[0][1], outs[1][1])


@pytest.mark.parametrize("case", [2, 3])
def test_synthetic_dense_forward_staged(device, case):
    """The staged-decode plan (weights decoded once to bf16, then the bf16
    GEMM, SwiGLU pair included) forced on for every GEMM of the FP8 models."""
    kw = dict(CASES[case])
    spec, f32, tensors = make_model(100 + case, **kw)
    ps = prompts(7 + case, [1, 5, 64, 65, 150, 33], spec["vocab"])
    device.set_decode_staging(1)
    try:
        check_forward(device, spec, f32, tensors, ps)
    finally:
        device.set_decode_staging(1024)
