"""BASELINE config 1 at full size on the GPU against the oracle.

A Qwen2-0.5B-shaped decoder (24 layers, hidden 896, 14 / 2 heads of 64,
SwiGLU 4864, vocab 151936, q/k/v biases, tied embedding) with seeded
N(0, 0.02) f32 weights. Two batches of 64 prompts x 48 uniform token ids.
Pipeline: capture the last-token residual of every layer entry (good and bad
batch), difference-of-means directions (orthogonalised), the none-mode rank-1
edit of o_proj and down_proj with a seeded kernel weight, and the first-token
KL over the full vocabulary on the first batch against the unedited model.
The oracle (ditch's f32 engine) runs its own full pipeline once; the device
runs it in both precision modes:

* default: the f32 weights as bf16 tensor-core products with f32
  accumulation (weights and activations rounded to bf16 at each GEMM input).
  Bounds: residual means max abs error <= 2e-2 * max |mean| per layer entry;
  directions cosine >= 0.99 per entry; KL relative error <= 5 %.
* f32 split (ditch_cuda_set_f32_split): hi / lo bf16 segments, f32-level
  products. Bounds: residual means within ditch's own fixture tolerance,
  2e-3 max abs (src/model_test.zig:62, 70), per entry; directions cosine >=
  0.9999; KL relative error <= 1 %.
The errors are recorded (tests/parity_report.py).
"""
import numpy as np
import pytest

import ditch_b200
import oracle
from oracle.model import OracleModel, flatten_batch
from parity_report import record, record_value

pytestmark = pytest.mark.gpu

C1 = dict(n_layers=24, hidden=896, heads=14, kv_heads=2, head_dim=64, inter=4864, vocab=151936, eps=1e-6,
          rope_theta=1e6, tied=True)
PARAMS_O = (1.3, 17.0, 0.5, 8.0)
PARAMS_DOWN = (1.0, 16.0, 0.4, 9.0)


def c1_weights(seed):
    rng = np.random.default_rng(seed)
    s = C1
    H, I, qd, kvd = s["hidden"], s["inter"], s["heads"] * s["head_dim"], s["kv_heads"] * s["head_dim"]

    def w(*shape):
        return rng.standard_normal(shape, dtype=np.float32) * np.float32(0.02)

    out = {"embed": w(s["vocab"], H), "final_norm": np.ones(H, np.float32)}
    out["lm_head"] = out["embed"]
    for i in range(s["n_layers"]):
        out.update({f"L{i}.input_norm": np.ones(H, np.float32), f"L{i}.post_norm": np.ones(H, np.float32),
                    f"L{i}.q": w(qd, H), f"L{i}.k": w(kvd, H), f"L{i}.v": w(kvd, H), f"L{i}.o": w(H, qd),
                    f"L{i}.qb": w(qd), f"L{i}.kb": w(kvd), f"L{i}.vb": w(kvd), f"L{i}.gate": w(I, H),
                    f"L{i}.up": w(I, H), f"L{i}.down": w(H, I)})
    return out


def c1_prompts():
    rng = np.random.default_rng(7)
    good = [rng.integers(0, C1["vocab"], 48).astype(np.uint32) for _ in range(64)]
    bad = [rng.integers(0, C1["vocab"], 48).astype(np.uint32) for _ in range(64)]
    return good, bad


@pytest.fixture(scope="module")
def c1_oracle():
    """The oracle's pipeline on the C1 inputs: residual sums, directions, KL."""
    s = C1
    w = c1_weights(2026)
    good, bad = c1_prompts()
    om = OracleModel(s, w)
    osums = {}
    for name, ps in (("good", good), ("bad", bad)):
        toks, rb, rp, cap, first, take, last = flatten_batch(ps, 1)
        res, _ = om.forward(toks, rb, rp, cap, ())
        osums[name] = oracle.residual_sums(res, first, take)
    gmean, bmean = (osums["good"] / 64).astype(np.float32), (osums["bad"] / 64).astype(np.float32)
    odirs = oracle.compute_directions(gmean, bmean, True)
    toks, rb, rp, cap, first, take, last = flatten_batch(good, 1)
    _, base = om.forward(toks, rb, rp, (), last)
    for li in range(s["n_layers"]):
        for comp, p in (("o", PARAMS_O), ("down", PARAMS_DOWN)):
            lam = oracle.kernel_weight(p, li)
            if lam is not None:
                a, b = oracle.compute_delta_none(w[f"L{li}.{comp}"], odirs[li + 1], lam)
                om.set_delta(li, comp, a, b)
    _, edited = om.forward(toks, rb, rp, (), last)
    okl, _ = oracle.kl_first_token(oracle.log_softmax(base), edited)
    return w, osums, odirs, okl


@pytest.mark.parametrize("mode", ["bf16", "split"])
def test_c1_pipeline_matches_oracle(device, c1_oracle, mode):
    s = C1
    w, osums, odirs, okl = c1_oracle
    tensors = []
    for name, a in w.items():
        rows, cols = (a.shape[0], 1) if a.ndim == 1 else a.shape
        tensors.append(ditch_b200.Tensor(name, "f32", rows, cols, a))
    device.set_f32_split(mode == "split")
    try:
        m = ditch_b200.Model(device, s, tensors, max_seq=64)
    finally:
        device.set_f32_split(False)
    good, bad = c1_prompts()
    gs, gc = m.residual_sums(good, window=1)
    bs, bc = m.residual_sums(bad, window=1)
    dirs = m.directions(gs, gc, bs, bc, True)
    m.kl_init(good)
    m.apply_edit(PARAMS_O, PARAMS_DOWN)
    kl = m.kl_score()

    case = f"C1 ({mode})"
    mean_err = np.abs(gs / gc - osums["good"] / 64).max(axis=1)
    mean_scale = np.abs(osums["good"] / 64).max(axis=1)
    record(case, "residual means, good batch (25 entries)", gs / gc, osums["good"] / 64,
           bound=2e-3 if mode == "split" else None)
    record(case, "residual means, bad batch (25 entries)", bs / bc, osums["bad"] / 64)
    cos = np.sum(dirs * odirs, axis=1)
    record_value(case, "direction cosine (min over 25 entries)", float(cos.min()), 1.0)
    record_value(case, "first-token KL after the edit", kl, okl)
    if mode == "split":
        assert mean_err.max() <= 2e-3, mean_err.max()
        assert np.abs(bs / bc - osums["bad"] / 64).max() <= 2e-3
        assert cos.min() >= 0.9999
        assert okl > 0 and abs(kl - okl) <= 0.01 * abs(okl)
    else:
        assert np.all(mean_err <= 2e-2 * mean_scale)
        assert cos.min() >= 0.99
        assert okl > 0 and abs(kl - okl) <= 0.05 * abs(okl)
    m.close()
