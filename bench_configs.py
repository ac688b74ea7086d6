"""The other BASELINE configurations of `bench.py` (`--config ...`).

* `gemm`: one resident-weight GEMM (a profiling target): `--fmt`, `--rows`, `--cols`, `--m`.
* `c3`: the standalone dequant + GEMM sweep of BASELINE config 3. Weights of
  [4096 x 4096], [14336 x 4096] and [4096 x 14336] are stored as GGUF Q8_0,
  GGUF Q4_K, INT4 (group 128, packed zero points) and MXFP4, with bf16
  activations for M in {1, 16, 128, 1024, 8192}. Per case: `ms` per call of
  back-to-back calls (host launch costs included), `kernel_ms` the device
  time of the product's kernels, and from it TFLOP/s (M >= 128) or GB/s over
  weight + activation + output bytes (M < 128).
* `c5`: on one GPU, the in-place rank-1 edit W <- W - alpha_l r_l (r_l^T W)
  on all 80 o_proj [8192 x 8192] and down_proj [8192 x 28672] bf16 matrices
  of a Llama-3-70B shape (HBM GB/s over the algorithmic 3 x 48.32 GB). Under
  torchrun with 2 or more GPUs, the C5 trial tensor-parallel: the 141 GB
  model split by heads and MLP columns, 64 prompts x 32 tokens, the none-mode
  edit of every o_proj / down_proj shard, the forward with the o / down
  partial sums all-reduced over NVLink peer memory, and the first-token KL.
* `c1`: BASELINE config 1, the Qwen2-0.5B-shaped fp32 model (24 layers,
  hidden 896, 14/2 heads of 64, SwiGLU 4864, vocab 151936, q/k/v biases, tied
  embedding, seeded N(0, 0.02) f32 weights) with two batches of 64 prompts x
  48 tokens: capture, directions, then per trial the none-mode edit of
  o_proj / down_proj and the KL forward of the first batch. The CPU baseline
  is ditch's engine restated in C (the oracle) timed on one whole trial of
  the same workload (the edit GEMVs, the forward with the deltas, the KL).
* `c4`: the Qwen3-MoE-shaped trial loop of BASELINE config 4 on one GPU: 48
  layers, hidden 2048, 32/4 heads of 128 with q/k norms, 128 routed experts
  (top-8 softmax, renormalised) of intermediate 768 stored as MXFP4, bf16
  attention, vocab 151936; 256 prompts x 64 tokens. A trial is the
  expert-selective edit (o_proj plus the down projections of the 8 experts per
  layer best aligned with the direction, src/moe.zig:1373-1477), the edited
  forward and the first-token KL.

* `gen`: greedy generation (the device half of ditch's KeywordRate scorer,
  src/scorers.zig:95-155) on the C2 model: `--prompts` (default 128) prompts
  x `--seq` tokens, `--max-new` (default 100, ditch's max_response_length)
  tokens each, no EOS so every prompt runs to the limit. A step is one
  ditch_cuda_generate call: the prefill into the KV cache and the decode
  steps, with the per-step host round trip of the tokens included.

All weights are seeded synthetic N(0, 0.02), generated and quantised on the
GPU with torch (device-memory plumbing; the kernels under test are the
library's).
"""
import json
import math
import os
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))


def _peaks():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        d = json.load(open(p))
        return d["hbm_gbs"], d["bf16_tflops"], "measured"
    return 6650.0, 1590.0, "fallback"


# ---- quantisers on the GPU (synthetic data; formats as ditch stores them) ----
def q8_0_blocks(w):
    """GGUF Q8_0 (src/quant.zig:245-255): per 32: d = amax / 127 (f16), q = round(x / d)."""
    import torch

    rows, cols = w.shape
    x = w.float().view(rows, cols // 32, 32)
    d = x.abs().amax(-1) / 127.0
    inv = torch.where(d != 0, 1.0 / d, torch.zeros_like(d))
    q = torch.round(x * inv[..., None]).clamp(-127, 127).to(torch.int8)
    d16 = d.half().view(torch.uint8).view(rows, cols // 32, 2)
    return torch.cat([d16, q.view(torch.uint8)], -1).reshape(rows, cols // 32 * 34).contiguous()


def q4_k_blocks(w):
    """A valid GGUF Q4_K encoding (d, dmin, 6-bit sub-scales / mins, nibbles)."""
    import torch

    rows, cols = w.shape
    nb = cols // 256
    x = w.float().view(rows, nb, 8, 32)
    lo = x.amin(-1).clamp(max=0)
    hi = x.amax(-1).clamp(min=0)
    sc, mn = (hi - lo) / 15.0, -lo
    d = (sc.amax(-1) / 63.0).half()
    dmin = (mn.amax(-1) / 63.0).half()
    df, dmf = d.float()[..., None], dmin.float()[..., None]
    ls = torch.where(df > 0, torch.round(sc / df), torch.zeros_like(sc)).clamp(0, 63).to(torch.int32)
    lm = torch.where(dmf > 0, torch.round(mn / dmf), torch.zeros_like(mn)).clamp(0, 63).to(torch.int32)
    ds, ms = (df * ls)[..., None], (dmf * lm)[..., None]
    q = torch.where(ds > 0, torch.round((x + ms) / ds), torch.zeros_like(x)).clamp(0, 15).to(torch.int32)
    s12 = torch.zeros(rows, nb, 12, dtype=torch.int32, device=w.device)
    for j in range(4):  # get_scale_min_k4 layout (src/quant.zig:140-146)
        s12[..., j] = ls[..., j] | ((ls[..., j + 4] >> 4) << 6)
        s12[..., j + 4] = lm[..., j] | ((lm[..., j + 4] >> 4) << 6)
        s12[..., j + 8] = (ls[..., j + 4] & 0xF) | ((lm[..., j + 4] & 0xF) << 4)
    nib = (q[:, :, 0::2, :] | (q[:, :, 1::2, :] << 4)).reshape(rows, nb, 128)
    head = torch.cat([d.view(torch.uint8).view(rows, nb, 2), dmin.view(torch.uint8).view(rows, nb, 2)], -1)
    out = torch.cat([head, s12.to(torch.uint8), nib.to(torch.uint8)], -1)
    return out.reshape(rows, nb * 144).contiguous()


def int4_packed(w, group=128):
    """compressed-tensors pack-quantized INT4, asymmetric (tools/make_fixture.py:156-194 rule)."""
    import torch

    rows, cols = w.shape
    g = cols // group
    x = w.float().view(rows, g, group)
    mn = x.amin(-1).clamp(max=0)
    mx = x.amax(-1).clamp(min=0)
    scale = ((mx - mn).clamp(min=1e-8) / 15.0).to(torch.bfloat16).float()
    zp = torch.round(-8 - mn / scale).clamp(-8, 7)
    q = (torch.round(x / scale[..., None]) + zp[..., None]).clamp(-8, 7).to(torch.int64) + 8
    q = q.view(rows, cols // 8, 8)
    words = torch.zeros(rows, cols // 8, dtype=torch.int64, device=w.device)
    for i in range(8):
        words |= q[..., i] << (4 * i)
    z = (zp.to(torch.int64) + 8).view(rows // 8, 8, g)
    zw = torch.zeros(rows // 8, g, dtype=torch.int64, device=w.device)
    for i in range(8):
        zw |= z[:, i, :] << (4 * i)
    as_u32 = lambda t: t.to(torch.int64).bitwise_and(0xFFFFFFFF).to(torch.int32)  # noqa: E731
    return as_u32(words).contiguous(), scale.contiguous(), as_u32(zw).contiguous()


E2M1 = [0.0, 0.5, 1.0, 1.5, 2.0, 3.0, 4.0, 6.0]


def mxfp4_packed(w):
    """MXFP4, natural layout (tools/make_fixture.py:210-224): e = floor(log2(amax / 6))."""
    import torch

    rows, cols = w.shape
    x = w.float().view(rows, cols // 32, 32)
    amax = x.abs().amax(-1)
    e = torch.where(amax > 0, torch.floor(torch.log2(amax.clamp(min=1e-30) / 6.0)), torch.zeros_like(amax))
    e = e.clamp(-127, 127)
    y = (x / torch.exp2(e)[..., None]).clamp(-6, 6)
    grid = torch.tensor(E2M1, device=w.device)
    mag = (y.abs()[..., None] - grid).abs().argmin(-1)
    code = (mag | ((y < 0).to(torch.int64) << 3)).to(torch.uint8)
    packed = (code[..., 0::2] | (code[..., 1::2] << 4)).reshape(rows, cols // 2).contiguous()
    return packed, (e + 127).to(torch.uint8).contiguous()


def make_weight(dev, fmt, rows, cols, gen):
    import torch

    from ditch_b200 import Tensor, Weight
    from ditch_b200.cuda import SCALE_F32

    w = (torch.randn(rows, cols, generator=gen, device="cuda") * 0.02).to(torch.bfloat16)
    if fmt == "bf16":
        t = Tensor("w", "bf16", rows, cols, w)
        wbytes = rows * cols * 2
    elif fmt == "fp8":
        from bench import fp8_block_quant

        codes, sc = fp8_block_quant(w)
        t = Tensor("w", "fp8", rows, cols, codes, scales=sc, block_rows=128, block_cols=128)
        wbytes = rows * cols + sc.numel() * 4
    elif fmt == "q8_0":
        raw = q8_0_blocks(w)
        t = Tensor("w", "q8_0", rows, cols, raw)
        wbytes = raw.numel()
    elif fmt == "q4_k":
        raw = q4_k_blocks(w)
        t = Tensor("w", "q4_k", rows, cols, raw)
        wbytes = raw.numel()
    elif fmt == "int4":
        words, scale, zeros = int4_packed(w)
        t = Tensor("w", "int", rows, cols, words, scales=scale, scales_dtype=SCALE_F32, zeros=zeros, block_cols=128,
                   bits=4)
        wbytes = words.numel() * 4 + scale.numel() * 2 + zeros.numel() * 4  # scales bf16 on disk
    elif fmt == "mxfp4":
        packed, scales = mxfp4_packed(w)
        t = Tensor("w", "mxfp4", rows, cols, packed, scales=scales)
        wbytes = packed.numel() + scales.numel()
    else:
        raise ValueError(fmt)
    W = Weight(dev, t)
    del w, t
    return W, wbytes


def time_gemm(dev, W, m, cols, rows, steps, warmup, k_splits=1, kernel_time=False):
    """ms per call of back-to-back calls (CUDA events around the loop: host
    launch costs included when the device outruns the host); with
    `kernel_time`, also the device time of the product's own kernels (CUDA
    events around each launch, summed by the library)."""
    import torch

    x = torch.randn(m, cols, device="cuda").to(torch.bfloat16)
    out = torch.empty(m, rows, device="cuda", dtype=torch.float32)
    torch.cuda.synchronize()
    for _ in range(warmup):
        W.gemm(x.data_ptr(), m, out.data_ptr(), k_splits)
    dev.synchronize()
    dev.timer_start()
    for _ in range(steps):
        W.gemm(x.data_ptr(), m, out.data_ptr(), k_splits)
    ms = dev.timer_stop() / steps
    if not kernel_time:
        return ms, x, out
    dev.set_profiling(True)
    dev.reset_stats()
    for _ in range(steps):
        W.gemm(x.data_ptr(), m, out.data_ptr(), k_splits)
    kms, n, _ = dev.gemm_stats()
    dev.set_profiling(False)
    return ms, kms / max(n, 1), x, out


def run_gemm(args, dev):
    import torch

    gen = torch.Generator(device="cuda").manual_seed(args.seed)
    W, wbytes = make_weight(dev, args.fmt, args.rows, args.cols, gen)
    ms, kms, _, _ = time_gemm(dev, W, args.m, args.cols, args.rows, args.steps, args.warmup, kernel_time=True)
    hbm, tf, src = _peaks()
    tflops = 2.0 * args.m * args.rows * args.cols / ms / 1e9
    stage = 1024 if args.stage_min_tokens is None else args.stage_min_tokens
    plan = ("streaming" if args.m <= 16 else "staged" if W.format() != "bf16" and 0 < stage <= args.m
            else "in-gemm")
    bytes_ = wbytes + 2 * args.m * args.cols + 4 * args.m * args.rows
    print(json.dumps({"config": "gemm", "fmt": args.fmt, "gemm_format": W.format(), "decode_plan": plan,
                      "rows": args.rows, "cols": args.cols, "m": args.m, "ms": round(ms, 4),
                      "kernel_ms": round(kms, 4), "tflops": round(tflops, 1),
                      "kernel_gbs": round(bytes_ / kms / 1e6, 1), "frac_of_burst_bf16": round(tflops / tf, 4),
                      "kernel_frac_of_hbm": round(bytes_ / kms / 1e6 / hbm, 4), "peak_source": src}), flush=True)
    W.close()


def run_c3(args, dev):
    import torch

    hbm, tf, src = _peaks()
    gen = torch.Generator(device="cuda").manual_seed(args.seed)
    results = []
    # every timed call decodes its weight (in the GEMM, or staged for >= 1024
    # tokens): no bf16 copy is kept between calls, so the sweep measures the
    # dequant and the GEMM together
    dev.set_decode_cache(False)
    for fmt in ("q8_0", "q4_k", "int4", "mxfp4"):
        for rows, cols in ((4096, 4096), (14336, 4096), (4096, 14336)):
            W, wbytes = make_weight(dev, fmt, rows, cols, gen)
            for m in (1, 16, 128, 1024, 8192):
                # the library picks the plan: weight streaming (m <= 16),
                # decode in the GEMM with one-wave split-K, or staged decode
                ms, kms, _, _ = time_gemm(dev, W, m, cols, rows, args.steps, args.warmup, kernel_time=True)
                flops = 2.0 * m * rows * cols
                bytes_ = wbytes + 2 * m * cols + 4 * m * rows
                r = {"fmt": fmt, "gemm_format": W.format(), "shape": [rows, cols], "m": m, "ms": round(ms, 4),
                     "kernel_ms": round(kms, 4), "tflops": round(flops / kms / 1e9, 2),
                     "gbs": round(bytes_ / kms / 1e6, 1), "bound": "hbm" if m < 128 else "tensor"}
                r["frac"] = round(r["gbs"] / hbm if m < 128 else r["tflops"] / tf, 4)
                results.append(r)
                print(json.dumps(r), flush=True)
            W.close()
            torch.cuda.empty_cache()
    dev.set_decode_cache(True)
    print(json.dumps({"config": "c3", "cases": len(results), "peak_source": src, "hbm_gbs": hbm,
                      "bf16_tflops_burst": tf, "decode_cache": False}), flush=True)


def run_c5(args, dev):
    """In-place edit of 80 o_proj + 80 down_proj bf16 matrices (48.3 GB)."""
    import torch

    import ditch_b200

    hbm, tf, src = _peaks()
    L, H, I = args.layers or 80, 8192, 28672
    gen = torch.Generator(device="cuda").manual_seed(args.seed)
    mats = []
    for _ in range(L):
        for rows, cols in ((H, H), (H, I)):
            w = torch.empty(rows, cols, dtype=torch.bfloat16, device="cuda")
            w.normal_(0.0, 0.02, generator=gen)
            mats.append(w)
    rs = torch.randn(L, H, generator=gen, device="cuda")
    rs = (rs / rs.norm(dim=1, keepdim=True)).contiguous()
    rng = np.random.default_rng(args.seed)
    p = (float(rng.uniform(0.8, 1.5)), float(rng.uniform(0.6 * (L - 1), L - 1)), 0.0, float(rng.uniform(1, 0.6 * L)))
    p = (p[0], p[1], float(rng.uniform(0, 1)) * p[0], p[3])

    def kernel_weight(layer):
        dist = abs(float(layer) - p[1])
        if dist > p[3]:
            return 0.0
        return p[0] + (dist / p[3]) * (p[2] - p[0])

    alphas = [kernel_weight(l) for l in range(L)]
    lib = ditch_b200.lib()
    stream = torch.cuda.current_stream()

    def sweep():
        for l in range(L):
            for k in range(2):
                w = mats[2 * l + k]
                st = lib.ditch_cuda_edit_weight_bf16_noalloc(w.data_ptr(), w.shape[0], w.shape[1],
                                                             rs[l].data_ptr(), alphas[l], stream.cuda_stream)
                if st != 0:
                    raise RuntimeError(lib.ditch_cuda_last_error())

    for _ in range(args.warmup):
        sweep()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for _ in range(args.steps):
        sweep()
    e1.record(stream)
    torch.cuda.synchronize()
    ms = e0.elapsed_time(e1) / args.steps
    elems = sum(w.numel() for w in mats)
    algo = 3 * 2 * elems
    print(json.dumps({"config": "c5", "metric": "edit-kernel HBM GB/s", "layers": L, "elements": elems,
                      "algorithmic_bytes": algo, "ms_per_edit": round(ms, 3), "gbs": round(algo / ms / 1e6, 1),
                      "frac": round(algo / ms / 1e6 / hbm, 4), "peak": hbm, "peak_source": src,
                      "note": "all 80 o_proj + down_proj edited per step (GEMV-T read + rank-1 read/write)"}),
          flush=True)


def stored_bytes(fmt, rows, cols):
    """Bytes of a weight as the library keeps it in HBM (the decoders' input):
    FP8 codes + f32 128x128 block scales; MXFP4 nibbles + E8M0 per 32; INT4
    words + f32 group scales + packed zero points (groups of 128); Q8_0
    repacked to int8 codes + an f32 scale per 32; Q4_K repacked to nibbles +
    an f32 (d*scale, dmin*min) pair per 32."""
    n = rows * cols
    if fmt == "fp8":
        return n + (-(-rows // 128)) * (-(-cols // 128)) * 4
    if fmt == "mxfp4":
        return n // 2 + n // 32
    if fmt == "int4":
        g = cols // 128
        return n // 2 + rows * g * 4 + (rows // 8) * g * 4
    if fmt == "q8_0":
        return n + n // 32 * 4
    if fmt == "q4_k":
        return n // 2 + n // 32 * 8
    if fmt == "bf16":
        return 2 * n
    raise ValueError(fmt)


def run_hbm(args, dev):
    """The HBM-bound kernels one at a time, at sizes well above L2 (126 MB),
    timed with CUDA events on the stream they run on:
    * the standalone decoders (ditch_cuda_weight_decode: k_dequant_fp8_bf16,
      k_dequant_mxfp4_bf16, k_dequant_int_bf16, k_stage_decode for the
      repacked Q8_0 / Q4_K) of a 28672 x 8192 weight (C5's down_proj shape):
      algorithmic bytes = stored bytes in + 2 B per element out;
    * the in-place rank-1 edit of the same shape in bf16 (k_gemv_t_bf16 then
      k_rank1_bf16): 3 x 2 B per element (GEMV-T read, update read + write).
    One line per kernel family, GB/s against the measured HBM copy bandwidth."""
    import torch

    hbm, tf, src = _peaks()
    rows, cols = args.rows if args.rows != 4096 else 28672, args.cols if args.cols != 4096 else 8192
    gen = torch.Generator(device="cuda").manual_seed(args.seed)
    out = torch.empty(rows, cols, dtype=torch.bfloat16, device="cuda")
    results = []
    for fmt in ("fp8", "mxfp4", "int4", "q8_0", "q4_k"):
        W, _ = make_weight(dev, fmt, rows, cols, gen)
        torch.cuda.synchronize()
        for _ in range(args.warmup):
            W.decode(out.data_ptr())
        dev.synchronize()
        dev.timer_start()
        for _ in range(args.steps):
            W.decode(out.data_ptr())
        ms = dev.timer_stop() / args.steps
        algo = stored_bytes(fmt, rows, cols) + 2 * rows * cols
        r = {"kernel": f"decode {fmt} -> bf16", "shape": [rows, cols], "ms": round(ms, 4),
             "algorithmic_bytes": algo, "gbs": round(algo / ms / 1e6, 1), "frac": round(algo / ms / 1e6 / hbm, 4)}
        results.append(r)
        print(json.dumps(r), flush=True)
        W.close()
        torch.cuda.empty_cache()
    w = out
    w.normal_(0.0, 0.02, generator=gen)
    r_vec = torch.randn(rows, generator=gen, device="cuda")
    r_vec /= r_vec.norm()
    for _ in range(args.warmup):
        dev.edit_weight_bf16(w.data_ptr(), rows, cols, r_vec.data_ptr(), 0.5)
    dev.synchronize()
    dev.timer_start()
    for _ in range(args.steps):
        dev.edit_weight_bf16(w.data_ptr(), rows, cols, r_vec.data_ptr(), 0.5)
    ms = dev.timer_stop() / args.steps
    algo = 3 * 2 * rows * cols
    r = {"kernel": "edit bf16 (GEMV-T + rank-1 update)", "shape": [rows, cols], "ms": round(ms, 4),
         "algorithmic_bytes": algo, "gbs": round(algo / ms / 1e6, 1), "frac": round(algo / ms / 1e6 / hbm, 4)}
    results.append(r)
    print(json.dumps(r), flush=True)
    print(json.dumps({"config": "hbm", "kernels": len(results), "peak_gbs": hbm, "peak_source": src,
                      "l2": "every input larger than L2 (126 MB)"}), flush=True)


C1 = dict(n_layers=24, hidden=896, heads=14, kv_heads=2, head_dim=64, inter=4864, vocab=151936, eps=1e-6,
          rope_theta=1e6, tied=True)


def c1_weights(seed, n_layers):
    rng = np.random.default_rng(seed)
    s = C1
    H, I, qd, kvd = s["hidden"], s["inter"], s["heads"] * s["head_dim"], s["kv_heads"] * s["head_dim"]

    def w(*shape):
        return rng.standard_normal(shape, dtype=np.float32) * np.float32(0.02)

    out = {"embed": w(s["vocab"], H), "final_norm": np.ones(H, np.float32)}
    out["lm_head"] = out["embed"]
    for i in range(n_layers):
        out.update({f"L{i}.input_norm": np.ones(H, np.float32), f"L{i}.post_norm": np.ones(H, np.float32),
                    f"L{i}.q": w(qd, H), f"L{i}.k": w(kvd, H), f"L{i}.v": w(kvd, H), f"L{i}.o": w(H, qd),
                    f"L{i}.qb": w(qd), f"L{i}.kb": w(kvd), f"L{i}.vb": w(kvd), f"L{i}.gate": w(I, H),
                    f"L{i}.up": w(I, H), f"L{i}.down": w(H, I)})
    return out


def c1_cpu_trial(spec, w, dirs, good, po, pd, reps):
    """One C1 trial on ditch's CPU engine restated (oracle): the none-mode
    delta of every o_proj / down_proj with a kernel weight (A = v^T W on the
    CPU), the forward of the KL batch with the deltas, log-softmax and KL."""
    import oracle
    from bench import host_threads
    from oracle.model import OracleModel, flatten_batch

    oracle.lib().or_set_threads(host_threads())
    m = OracleModel(spec, w)
    toks, rb, rp, cap, first, take, last = flatten_batch(good, 1)
    _, base = m.forward(toks, rb, rp, (), last)
    lb = oracle.log_softmax(base)
    t0 = time.perf_counter()
    for _ in range(reps):
        m.reset_deltas()
        for li in range(spec["n_layers"]):
            for comp, p, name in (("o", po, f"L{li}.o"), ("down", pd, f"L{li}.down")):
                lam = oracle.kernel_weight(p, li)
                if lam is not None:
                    a, b = oracle.compute_delta_none(w[name], dirs[li + 1], lam)
                    m.set_delta(li, comp, a, b)
        _, logits = m.forward(toks, rb, rp, (), last)
        kl, _ = oracle.kl_first_token(lb, logits)
    return (time.perf_counter() - t0) / reps, kl, oracle.lib().or_get_threads()


def run_c1(args, dev):
    import torch

    import ditch_b200
    from bench import Clocks, measured_peaks, trial_params

    L = args.layers or C1["n_layers"]
    spec = dict(C1, n_layers=L)
    P, S = args.prompts or 64, 48
    t0 = time.time()
    w = c1_weights(args.seed, L)
    tensors = []
    for name, a in w.items():
        rows, cols = (a.shape[0], 1) if a.ndim == 1 else a.shape
        tensors.append(ditch_b200.Tensor(name, "f32", rows, cols, a))
    model = ditch_b200.Model(dev, spec, tensors, max_seq=S)
    load_s = time.time() - t0
    rng = np.random.default_rng(args.seed + 1)
    good = [rng.integers(0, spec["vocab"], S).astype(np.uint32) for _ in range(P)]
    bad = [rng.integers(0, spec["vocab"], S).astype(np.uint32) for _ in range(P)]
    dev.synchronize()
    dev.timer_start()
    gs, gc = model.residual_sums(good, window=1, batch_size=P)
    bs, bc = model.residual_sums(bad, window=1, batch_size=P)
    dirs = model.directions(gs, gc, bs, bc, True)
    capture_ms = dev.timer_stop()
    model.kl_init(good)
    tokens_flat = np.concatenate(good).astype(np.uint32)
    offs = np.zeros(P + 1, np.uintp)
    offs[1:] = np.cumsum([len(p) for p in good])
    trial_rng = np.random.default_rng(args.seed + 7)
    kls, trials = [], []

    def step(e2e):
        po, pd, di = trial_params(trial_rng, L)
        trials.append((po, pd))
        model.apply_edit(po, pd, None)
        kls.append(model.kl_score_prompts(tokens_flat, offs, P) if e2e else model.kl_score())

    def timed(e2e, steps):
        torch.cuda.synchronize()
        dev.synchronize()
        dev.timer_start()
        for _ in range(steps):
            step(e2e)
        return dev.timer_stop()

    for _ in range(args.warmup):
        step(False)
    dev.set_profiling(True)
    dev.reset_stats()
    clocks = Clocks(torch.cuda.current_device())
    ms = timed(False, args.steps)
    clk = clocks.stop()
    gemm_ms, gemm_launches, gemm_flops = dev.gemm_stats()
    launches = dev.launches()
    dev.set_profiling(False)
    for _ in range(max(1, args.warmup // 2)):
        step(True)
    ms_e2e = timed(True, args.steps)
    hbm, tf_burst, tf_sust, src = measured_peaks()
    tokens = P * S
    achieved = gemm_flops / (gemm_ms / 1000.0) / 1e12 if gemm_ms > 0 else 0.0
    line = {
        "metric": "trial-eval forward tokens/s", "value": round(tokens * args.steps / (ms / 1000.0), 1),
        "unit": "tokens/s", "n_gpus": 1, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": round(ms / args.steps, 3), "s_per_trial": round(ms / args.steps / 1000.0, 5),
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
        "dtype": "f32 weights run as bf16 MMA with f32 accumulate", "data": "synthetic",
        "config": {"workload": "C1: Qwen2-0.5B-shaped fp32, trial = none-mode rank-1 edit of o_proj/down_proj + "
                               "edited forward + first-token KL over 151936 logits",
                   "layers": L, "prompts_per_gpu": P, "seq_len": S, "vocab": spec["vocab"], "parallelism": "dp1",
                   "l2": "weights 0.7 GB bf16 + logits; the working set exceeds L2"},
        "e2e": {"value": round(tokens * args.steps / (ms_e2e / 1000.0), 1), "unit": "tokens/s",
                "h2d_bytes_per_step": int(tokens * 4 + (P + 1) * 8), "d2h_bytes_per_step": 8,
                "ms_per_step": round(ms_e2e / args.steps, 3)},
        "roofline": {"bound": "tensor", "kernel": "gemm_kernel: tcgen05 bf16 MMA", "achieved": round(achieved, 1),
                     "peak": tf_sust, "unit": "TFLOP/s", "frac": round(achieved / tf_sust, 4),
                     "peak_source": f"{src} bf16 sustained", "traffic": None,
                     "gemm_ms_per_step": round(gemm_ms / args.steps, 3),
                     "gemm_share_of_step": round(gemm_ms / ms, 4) if ms > 0 else None},
        "gpu_launches": int(launches), "clocks": clk,
        "one_off": {"load_s": round(load_s, 2), "capture_and_directions_ms": round(capture_ms, 2)},
        "kl_last": kls[-1] if kls else None,
    }
    if not args.no_cpu_baseline:
        po, pd = trials[-1]
        cpu_s, cpu_kl, cores = c1_cpu_trial(spec, w, dirs, good, po, pd, 1)
        line["cpu_baseline"] = {"value": round(tokens / cpu_s, 2), "unit": "tokens/s", "cores": cores,
                                "kind": "port", "s_per_trial": round(cpu_s, 3),
                                "sample": f"one whole C1 trial (edit GEMVs, forward of {P} x {S} tokens with "
                                          f"the deltas, KL over {spec['vocab']} logits) on the oracle",
                                "kl": cpu_kl, "kl_device_same_trial": kls[-1]}
    print(json.dumps(line), flush=True)
    model.close()


C4 = dict(n_layers=48, hidden=2048, heads=32, kv_heads=4, head_dim=128, inter=768, vocab=151936, eps=1e-6,
          rope_theta=1e6, qk_norm=1, n_experts=128, top_k=8, moe_inter=768, norm_topk=1)


def build_c4_model(dev, spec, seed, max_seq, ep_rank=0, ep_world=1):
    """Seeded N(0, 0.02) weights: attention, router, embedding and LM head in
    bf16, routed experts quantised to MXFP4 (natural layout) on the GPU."""
    import torch

    import ditch_b200
    from ditch_b200 import Tensor

    g = torch.Generator(device="cuda").manual_seed(seed)
    H, V, L, E, mi = spec["hidden"], spec["vocab"], spec["n_layers"], spec["n_experts"], spec["moe_inter"]
    hd = spec["head_dim"]
    qd, kvd = spec["heads"] * hd, spec["kv_heads"] * hd
    keep, tensors = [], []

    def bf16(shape):
        return (torch.randn(shape, generator=g, device="cuda", dtype=torch.float32) * 0.02).to(torch.bfloat16)

    def add_bf16(name, rows, cols):
        w = bf16((rows, cols))
        keep.append(w)
        tensors.append(Tensor(name, "bf16", rows, cols, w))

    def add_experts(name, rows, cols):
        packed, scales = [], []
        for e0 in range(0, E, 32):  # bounded temporaries
            w = bf16((32 * rows, cols))
            p_, s_ = mxfp4_packed(w)
            packed.append(p_)
            scales.append(s_)
            del w
        p_, s_ = torch.cat(packed), torch.cat(scales)
        keep.extend([p_, s_])
        tensors.append(Tensor(name, "mxfp4", rows, cols, p_, slabs=E, scales=s_))

    ones = torch.ones(max(H, hd), dtype=torch.bfloat16, device="cuda")
    keep.append(ones)
    add_bf16("embed", V, H)
    add_bf16("lm_head", V, H)
    tensors.append(Tensor("final_norm", "bf16", H, 1, ones[:H]))
    for i in range(L):
        tensors += [Tensor(f"L{i}.input_norm", "bf16", H, 1, ones[:H]),
                    Tensor(f"L{i}.post_norm", "bf16", H, 1, ones[:H]),
                    Tensor(f"L{i}.q_norm", "bf16", hd, 1, ones[:hd]), Tensor(f"L{i}.k_norm", "bf16", hd, 1, ones[:hd])]
        add_bf16(f"L{i}.q", qd, H)
        add_bf16(f"L{i}.k", kvd, H)
        add_bf16(f"L{i}.v", kvd, H)
        add_bf16(f"L{i}.o", H, qd)
        add_bf16(f"L{i}.router", E, H)
        add_experts(f"L{i}.e_gate", mi, H)
        add_experts(f"L{i}.e_up", mi, H)
        add_experts(f"L{i}.e_down", H, mi)
    torch.cuda.synchronize()
    model = ditch_b200.Model(dev, spec, tensors, max_seq=max_seq, ep_rank=ep_rank, ep_world=ep_world)
    del keep, tensors
    torch.cuda.empty_cache()
    return model


def c4_flops(spec, tokens):
    """Algorithmic FLOPs of one forward (counted per unit of work: linear layers of
    the attention, the router, top-k experts' SwiGLU, attention scores/values
    over causal prompts, the LM head on the last rows)."""
    H, L, E, k, mi = spec["hidden"], spec["n_layers"], spec["n_experts"], spec["top_k"], spec["moe_inter"]
    qd, kvd = spec["heads"] * spec["head_dim"], spec["kv_heads"] * spec["head_dim"]
    per_tok = 2 * (H * (qd + 2 * kvd) + qd * H + E * H + k * 3 * mi * H)
    return L * per_tok * tokens


def run_c4(args, dev, world=1, rank=0, dist=None):
    """C4 on `world` GPUs: expert-parallel (each rank owns 128 / world experts,
    rows exchanged over NVLink peer memory) and data-parallel over prompts
    (each rank routes its own 256 prompts; the library sums the residuals and
    the KL over the ranks through a second peer group)."""
    import torch

    import ditch_b200
    from bench import Clocks, all_reduce, measured_peaks, trial_params

    spec = dict(C4, n_layers=args.layers or C4["n_layers"], moe_layers=[True] * (args.layers or C4["n_layers"]))
    L, V, S = spec["n_layers"], spec["vocab"], args.seq
    P = args.prompts or 256
    t0 = time.time()
    model = build_c4_model(dev, spec, args.seed, max_seq=S, ep_rank=rank, ep_world=world)
    group = None
    if world > 1:
        def exchange(h):
            out = [None] * world
            dist.all_gather_object(out, h)
            return out

        group = ditch_b200.Group(dev, rank, world, model.group_bytes(P * S), exchange)
        model.set_group(group, P * S)
        dp_group = ditch_b200.Group(dev, rank, world, model.dp_group_bytes(P), exchange)
        model.set_dp_group(dp_group)
        dist.barrier()
    load_s = time.time() - t0
    rng = np.random.default_rng(args.seed + 1000 * (rank + 1))
    good = [rng.integers(0, V, S).astype(np.uint32) for _ in range(P)]
    bad = [rng.integers(0, V, S).astype(np.uint32) for _ in range(P)]
    kl_prompts = [rng.integers(0, V, S).astype(np.uint32) for _ in range(P)]
    dev.synchronize()
    dev.timer_start()
    gs, gc = model.residual_sums(good, window=1, batch_size=P)  # every rank's prompts (data-parallel group)
    bs, bc = model.residual_sums(bad, window=1, batch_size=P)
    model.directions(gs, gc, bs, bc, True)
    capture_ms = dev.timer_stop()
    model.kl_init(kl_prompts)
    tokens_flat = np.concatenate(kl_prompts).astype(np.uint32)
    offs = np.zeros(P + 1, np.uintp)
    offs[1:] = np.cumsum([len(p) for p in kl_prompts])
    trial_rng = np.random.default_rng(args.seed + 7)
    kls = []

    def step(e2e):
        po, pd, di = trial_params(trial_rng, L)
        model.apply_expert_edit(po, pd, di, n_experts=spec["top_k"], strength=1.0)
        # the mean KL over every rank's prompts
        kls.append(model.kl_score_prompts(tokens_flat, offs, P) if e2e else model.kl_score())

    def timed(e2e, steps):
        if dist:
            dist.barrier()
        torch.cuda.synchronize()
        dev.synchronize()
        dev.timer_start()
        for _ in range(steps):
            step(e2e)
        ms = dev.timer_stop()
        return float(all_reduce(dist, np.array([ms], np.float64), op="max")[0])

    for _ in range(args.warmup):
        step(False)
    dev.set_profiling(True)
    dev.reset_stats()
    clocks = Clocks(torch.cuda.current_device())
    ms = timed(False, args.steps)
    clk = clocks.stop()
    gemm_ms, gemm_launches, gemm_flops = dev.gemm_stats()
    launches = dev.launches()
    dev.set_profiling(False)
    for _ in range(max(1, args.warmup // 2)):
        step(True)
    ms_e2e = timed(True, args.steps)
    hbm, tf_burst, tf_sust, src = measured_peaks()
    tokens = P * S
    fl = c4_flops(spec, tokens)
    if world > 1:
        # expert parallel: the owners' grouped GEMMs run over the exchange's
        # receive capacity (their row counts stay on the device), so the
        # launch records overcount; each rank's GEMM work is its own tokens'
        # linear layers (balanced routing), counted analytically
        gemm_flops = fl * args.steps
    achieved = gemm_flops / (gemm_ms / 1000.0) / 1e12 if gemm_ms > 0 else 0.0
    line = {
        "metric": "trial-eval forward tokens/s", "value": round(tokens * world * args.steps / (ms / 1000.0), 1),
        "unit": "tokens/s", "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": round(ms / args.steps, 3), "s_per_trial": round(ms / args.steps / 1000.0, 5),
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
        "dtype": "mxfp4 experts + bf16 attention, bf16 MMA, f32 accumulate", "data": "synthetic",
        "config": {"workload": "C4: Qwen3-MoE-shaped, 128 MXFP4 experts top-8, trial = expert-selective rank-1 edit "
                               "(o_proj + top-8 expert down per layer) + edited forward + first-token KL",
                   "layers": L, "prompts_per_gpu": P, "seq_len": S, "vocab": V,
                   "parallelism": (f"ep{world} (experts {spec['n_experts'] // world} per GPU, rows exchanged over "
                                   f"NVLink peer memory) x dp{world} (prompts; residual sums and KL summed by the "
                                   f"library's peer-group reduction)" if world > 1 else "dp1"),
                   "l2": "inputs larger than L2 (15.4 GB of MXFP4 experts per forward)"},
        "e2e": {"value": round(tokens * world * args.steps / (ms_e2e / 1000.0), 1), "unit": "tokens/s",
                "h2d_bytes_per_step": int(tokens * 4 + (P + 1) * 8), "d2h_bytes_per_step": 8,
                "ms_per_step": round(ms_e2e / args.steps, 3)},
        "roofline": {"bound": "tensor",
                     "kernel": ("gemm_kernel: tcgen05 grouped GEMM, MXFP4 decoded per tile" if args.stage_min_tokens == 0
                                else "gemm_kernel: tcgen05 grouped GEMM over each expert stack's bf16 copy (MXFP4 "
                                     "decoded once at first use and kept, memory permitting)"),
                     "achieved": round(achieved, 1), "peak": tf_sust, "unit": "TFLOP/s",
                     "frac": round(achieved / tf_sust, 4), "peak_source": f"{src} bf16 sustained", "traffic": None,
                     "gemm_ms_per_step": round(gemm_ms / args.steps, 3),
                     "gemm_share_of_step": round(gemm_ms / ms, 4) if ms > 0 else None,
                     "forward_tflop": round(fl / 1e12, 2),
                     "forward_tflops_per_s": round(fl * world * args.steps / (ms / 1000.0) / 1e12, 1)},
        "gpu_launches": int(launches), "clocks": clk,
        "one_off": {"load_s": round(load_s, 2), "capture_and_directions_ms": round(capture_ms, 2)},
        "kl_last": kls[-1] if kls else None,
    }
    if rank == 0:
        print(json.dumps(line), flush=True)
    model.set_dp_group(None)
    model.close()
    if group is not None:
        dist.barrier()
        group.close()
        dp_group.close()


C5 = dict(n_layers=80, hidden=8192, heads=64, kv_heads=8, head_dim=128, inter=28672, vocab=128256, eps=1e-5,
          rope_theta=5e5)


def build_c5_shards(dev, spec, seed, rank, world, max_seq):
    """The Llama-3-70B-shaped bf16 model as this rank's tensor-parallel shards:
    q / k / v / gate / up rows and o / down columns of the rank, each drawn
    N(0, 0.02) from a seed of (layer, tensor, rank), so the ranks together hold
    one consistent random model. Embedding, LM head and norms are replicated
    (same seed on every rank)."""
    import torch

    import ditch_b200
    from ditch_b200 import Tensor

    H, I, V, L = spec["hidden"], spec["inter"], spec["vocab"], spec["n_layers"]
    qd, kvd = spec["heads"] * spec["head_dim"], spec["kv_heads"] * spec["head_dim"]
    qs, ks, isz = qd // world, kvd // world, I // world
    keep, tensors = [], []

    def gen(tag, shape):
        g = torch.Generator(device="cuda").manual_seed(seed * 1000003 + tag)
        w = torch.empty(shape, dtype=torch.bfloat16, device="cuda")
        w.normal_(0.0, 0.02, generator=g)
        keep.append(w)
        return w

    ones = torch.ones(H, dtype=torch.bfloat16, device="cuda")
    keep.append(ones)
    tensors += [Tensor("embed", "bf16", V, H, gen(1, (V, H))), Tensor("lm_head", "bf16", V, H, gen(2, (V, H))),
                Tensor("final_norm", "bf16", H, 1, ones)]
    for i in range(L):
        base = 16 + (i * 8 + 0) * 64 + rank * 8
        tensors += [Tensor(f"L{i}.input_norm", "bf16", H, 1, ones), Tensor(f"L{i}.post_norm", "bf16", H, 1, ones),
                    Tensor(f"L{i}.q", "bf16", qs, H, gen(base + 0, (qs, H))),
                    Tensor(f"L{i}.k", "bf16", ks, H, gen(base + 1, (ks, H))),
                    Tensor(f"L{i}.v", "bf16", ks, H, gen(base + 2, (ks, H))),
                    Tensor(f"L{i}.o", "bf16", H, qs, gen(base + 3, (H, qs))),
                    Tensor(f"L{i}.gate", "bf16", isz, H, gen(base + 4, (isz, H))),
                    Tensor(f"L{i}.up", "bf16", isz, H, gen(base + 5, (isz, H))),
                    Tensor(f"L{i}.down", "bf16", H, isz, gen(base + 6, (H, isz)))]
    torch.cuda.synchronize()
    model = ditch_b200.Model(dev, spec, tensors, max_seq=max_seq, tp_rank=rank, tp_world=world)
    del keep, tensors
    torch.cuda.empty_cache()
    return model


def run_c5_tp(args, dev, world, rank, dist):
    """The C5 trial tensor-parallel over `world` GPUs (strong scaling: every
    rank works on the same 64 x 32 tokens with its shard of the weights): the
    none-mode edit of all o_proj / down_proj shards (A = v^T W per shard, no
    exchange), the edited forward with the o / down partial sums all-reduced
    over NVLink peer memory, and the first-token KL."""
    import torch

    import ditch_b200
    from bench import Clocks, all_reduce, measured_peaks, trial_params

    L = args.layers or C5["n_layers"]
    spec = dict(C5, n_layers=L)
    P, S = args.prompts or 64, 32
    H = spec["hidden"]
    t0 = time.time()
    model = build_c5_shards(dev, spec, args.seed, rank, world, max_seq=S)

    def exchange(h):
        out = [None] * world
        dist.all_gather_object(out, h)
        return out

    group = ditch_b200.Group(dev, rank, world, model.group_bytes(P * S), exchange)
    model.set_group(group, P * S)
    dist.barrier()
    load_s = time.time() - t0
    rng = np.random.default_rng(args.seed + 5)
    kl_prompts = [rng.integers(0, spec["vocab"], S).astype(np.uint32) for _ in range(P)]  # same on every rank
    dirs = rng.standard_normal((L + 1, H)).astype(np.float32)
    dirs /= np.linalg.norm(dirs, axis=1, keepdims=True)  # r_l = normalise(N(0, 1))
    model.set_directions(dirs)
    model.kl_init(kl_prompts)
    tokens_flat = np.concatenate(kl_prompts).astype(np.uint32)
    offs = np.zeros(P + 1, np.uintp)
    offs[1:] = np.cumsum([len(p) for p in kl_prompts])
    trial_rng = np.random.default_rng(args.seed + 7)
    kls = []

    def step(e2e):
        po, pd, di = trial_params(trial_rng, L)
        model.apply_edit(po, pd, None)
        kls.append(model.kl_score_prompts(tokens_flat, offs, P) if e2e else model.kl_score())

    def timed(e2e, steps):
        dist.barrier()
        torch.cuda.synchronize()
        dev.synchronize()
        dev.timer_start()
        for _ in range(steps):
            step(e2e)
        ms = dev.timer_stop()
        return float(all_reduce(dist, np.array([ms], np.float64), op="max")[0])

    for _ in range(args.warmup):
        step(False)
    dev.set_profiling(True)
    dev.reset_stats()
    clocks = Clocks(torch.cuda.current_device())
    ms = timed(False, args.steps)
    clk = clocks.stop()
    gemm_ms, gemm_launches, gemm_flops = dev.gemm_stats()
    launches = dev.launches()
    dev.set_profiling(False)
    for _ in range(max(1, args.warmup // 2)):
        step(True)
    ms_e2e = timed(True, args.steps)
    hbm, tf_burst, tf_sust, src = measured_peaks()
    tokens = P * S
    achieved = gemm_flops / (gemm_ms / 1000.0) / 1e12 if gemm_ms > 0 else 0.0
    line = {
        "metric": "trial-eval forward tokens/s", "value": round(tokens * args.steps / (ms / 1000.0), 1),
        "unit": "tokens/s", "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": round(ms / args.steps, 3), "s_per_trial": round(ms / args.steps / 1000.0, 5),
        "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "bf16 weights, f32 accumulate",
        "data": "synthetic",
        "config": {"workload": "C5: Llama-3-70B-shaped bf16, trial = none-mode rank-1 edit of every o_proj/down_proj "
                               "shard + edited forward + first-token KL",
                   "layers": L, "prompts": P, "seq_len": S, "vocab": spec["vocab"],
                   "parallelism": f"tp{world} (heads and MLP columns; o/down partials all-reduced over NVLink peer "
                                  f"memory)",
                   "l2": f"weights {141.1 / world:.1f} GB per GPU, read once per forward"},
        "e2e": {"value": round(tokens * args.steps / (ms_e2e / 1000.0), 1), "unit": "tokens/s",
                "h2d_bytes_per_step": int(tokens * 4 + (P + 1) * 8), "d2h_bytes_per_step": 8,
                "ms_per_step": round(ms_e2e / args.steps, 3)},
        "roofline": {"bound": "tensor", "kernel": "gemm_kernel: tcgen05 bf16 MMA (this rank's shards)",
                     "achieved": round(achieved, 1), "peak": tf_sust, "unit": "TFLOP/s",
                     "frac": round(achieved / tf_sust, 4), "peak_source": f"{src} bf16 sustained", "traffic": None,
                     "gemm_ms_per_step": round(gemm_ms / args.steps, 3),
                     "gemm_share_of_step": round(gemm_ms / ms, 4) if ms > 0 else None},
        "gpu_launches": int(launches), "clocks": clk, "one_off": {"load_s": round(load_s, 2)},
        "kl_last": kls[-1] if kls else None,
    }
    if rank == 0:
        print(json.dumps(line), flush=True)
    model.close()
    dist.barrier()
    group.close()


def run_gen(args, dev):
    """Greedy generation on the C2 model (see the module docstring)."""
    from bench import C2, Clocks, build_c2_model, measured_peaks

    spec = dict(C2, n_layers=args.layers or C2["n_layers"])
    P, S, N = args.prompts or 128, args.seq, args.max_new
    t0 = time.time()
    model = build_c2_model(dev, spec, args.seed, max_seq=S + N)
    load_s = time.time() - t0
    rng = np.random.default_rng(args.seed + 5)
    ps = [rng.integers(0, spec["vocab"], S).astype(np.uint32) for _ in range(P)]
    for _ in range(args.warmup):
        out = model.generate(ps, N)
    dev.set_profiling(True)
    dev.reset_stats()
    clocks = Clocks(dev.ordinal)
    dev.synchronize()
    dev.timer_start()
    n_gen = 0
    for _ in range(args.steps):
        out = model.generate(ps, N)
        n_gen += sum(len(o) for o in out)
    ms = dev.timer_stop()
    clk = clocks.stop()
    gemm_ms, gemm_launches, gemm_flops = dev.gemm_stats()
    launches = dev.launches()
    dev.set_profiling(False)
    hbm, tf_burst, tf_sust, src = measured_peaks()
    # weight bytes streamed per decode step: the FP8 linear weights (1 B per
    # element plus 4 B per 128 x 128 block) and the bf16 LM head
    H, I, V, L = spec["hidden"], spec["inter"], spec["vocab"], spec["n_layers"]
    qd, kvd = spec["heads"] * spec["head_dim"], spec["kv_heads"] * spec["head_dim"]
    per_layer = (qd + 2 * kvd) * H + H * qd + 2 * I * H + H * I
    w_bytes = L * per_layer * (1 + 4 / (128 * 128)) + V * H * 2
    steps_per_call = N - 1
    line = {
        "metric": "greedy generation tokens/s", "value": round(n_gen / (ms / 1000.0), 1), "unit": "tokens/s",
        "n_gpus": 1, "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms / args.steps, 3),
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
        "dtype": "fp8-e4m3 weights, bf16 MMA, f32 accumulate, f32 KV cache", "data": "synthetic",
        "config": {"workload": "gen", "model": "llama-3-8b-shape fp8", "prompts": P, "seq_len": S, "max_new": N,
                   "layers": L, "l2": "weights and KV cache larger than L2"},
        "tokens_per_call": n_gen // max(args.steps, 1),
        "roofline": {"bound": "hbm", "kernel": "decode step: every weight read once per step",
                     "weight_gb_per_decode_step": round(w_bytes / 1e9, 3),
                     "achieved_weight_gbs": round(w_bytes * steps_per_call * args.steps / (ms / 1000.0) / 1e9, 1),
                     "peak": hbm, "unit": "GB/s", "peak_source": f"{src} HBM",
                     "gemm_ms_per_step": round(gemm_ms / args.steps, 3),
                     "gemm_share_of_step": round(gemm_ms / ms, 4) if ms > 0 else None},
        "gpu_launches": int(launches), "clocks": clk, "one_off": {"load_s": round(load_s, 2)},
        "first_tokens": out[0][:8],
    }
    line["roofline"]["frac"] = round(line["roofline"]["achieved_weight_gbs"] / hbm, 4)
    print(json.dumps(line), flush=True)
    model.close()


def run(args):
    import torch

    import ditch_b200
    from bench import dist_setup

    world, rank, local, dist = dist_setup(args.gpus)
    if world > 1 and args.config not in ("c4", "c5"):
        # only C4 shards (expert parallel); the others run on rank 0
        if rank != 0:
            dist.barrier()
            dist.destroy_process_group()
            return 0
    torch.cuda.set_device(local)
    dev = ditch_b200.Device(local)
    if args.stage_min_tokens is not None:
        dev.set_decode_staging(args.stage_min_tokens)
    dev.set_deterministic(args.deterministic)
    dev.set_cta_pairs(args.cta_pairs)
    dev.set_attention_tc(args.attention_tc)
    if args.config == "c4" or (args.config == "c5" and world > 1):
        if args.config == "c4":
            run_c4(args, dev, world, rank, dist)
        else:
            run_c5_tp(args, dev, world, rank, dist)
        dev.close()
        if dist:
            dist.barrier()
            dist.destroy_process_group()
        return 0
    if args.config == "gemm":
        run_gemm(args, dev)
    elif args.config == "c1":
        run_c1(args, dev)
    elif args.config == "c3":
        run_c3(args, dev)
    elif args.config == "c5":
        run_c5(args, dev)
    elif args.config == "gen":
        run_gen(args, dev)
    elif args.config == "hbm":
        run_hbm(args, dev)
    else:
        raise SystemExit(f"config {args.config} is not implemented")
    dev.close()
    if dist:
        dist.barrier()
        dist.destroy_process_group()
    return 0
