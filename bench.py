"""Trial-evaluation benchmark of ditch's hot path on B200.

Workload (per GPU, weak scaling): a Llama-3-8B-shaped decoder (32 layers,
hidden 4096, 32/8 heads, SwiGLU 14336, vocab 128256, RoPE theta 5e5) with
random N(0, 0.02) weights quantised to FP8 E4M3 with 128x128 f32 block scales
(embedding, LM head and norms bf16), 128 prompts x 64 uniform random token
ids. Synthetic data: there is no network for checkpoints; the reference's
config is itself synthetic.

One-off per study (reported, not timed as a step): residual capture over a
good and a bad batch (128 prompts each), an all-reduce of the f64 residual sums
across ranks, and the refusal directions.

One step = one trial: decode a seeded parameter vector (src/search.zig:108-139),
the none-mode rank-1 edit of every o_proj and down_proj (A = v^T W on the FP8
weights, src/abliterate.zig:264-280), the edited forward of the 128 KL prompts
with the deltas in the GEMM epilogues, and the first-token KL against the
unedited model (src/scorers.zig:378-402), all-reduced across ranks.

value = forward tokens per trial x ranks x steps / max-over-ranks device time.
"""
import argparse
import json
import math
import os
import statistics
import subprocess
import sys
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

C2 = dict(n_layers=32, hidden=4096, heads=32, kv_heads=8, head_dim=128, inter=14336, vocab=128256, eps=1e-5,
          rope_theta=5e5)


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=10)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="ditch_b200", choices=["ditch_b200", "reference"])
    ap.add_argument("--prompts", type=int, default=None, help="prompts per GPU (default: the config's)")
    ap.add_argument("--seq", type=int, default=64)
    ap.add_argument("--layers", type=int, default=None, help="decoder layers (default: the config's)")
    ap.add_argument("--cpu-sample-s", type=float, default=15.0, help="CPU baseline sample budget (seconds)")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--seed", type=int, default=1234)
    ap.add_argument("--config", default="c2", choices=["c2", "c1", "c3", "c4", "c5", "gemm", "gen", "hbm"],
                    help="c2 (default): the FP8 dense trial loop; c1: the Qwen2-0.5B fp32 trial loop with the "
                         "whole-trial CPU baseline; c3: dequant + GEMM sweep; c4: the Qwen3-MoE MXFP4 "
                         "trial loop (expert-selective edit); c5: Llama-3-70B-shaped in-place edit sweep; gemm: one "
                         "GEMM; hbm: the standalone decoders and the bf16 edit, one at a time")
    ap.add_argument("--max-new", type=int, default=100, help="gen: tokens generated per prompt")
    ap.add_argument("--row-normalization", default="none", choices=["none", "pre", "full"],
                    help="c1 / c2: the edit's row normalisation (full: rank-3 delta from the randomised SVD)")
    ap.add_argument("--cta-pairs", type=int, default=2,
                    help="dense bf16 GEMMs of 512+ tokens on CTA pairs (tcgen05 cta_group::2): 0 never, 1 products "
                         "with one accumulator, 2 SwiGLU products too (the library's default)")
    ap.add_argument("--attention-tc", type=int, default=2,
                    help="prefill attention of prompts up to 128 tokens on tcgen05: 0 never (mma.sync), 1 one CTA per "
                         "SM, 2 two CTAs per SM for prompts up to 64 tokens (the library's default)")
    ap.add_argument("--deterministic", type=int, default=0,
                    help="1: K splits summed in a fixed order (stream-K) instead of atomically")
    ap.add_argument("--fmt", default="fp8", help="gemm mode: bf16 | fp8 | mxfp4 | int4")
    ap.add_argument("--rows", type=int, default=4096)
    ap.add_argument("--cols", type=int, default=4096)
    ap.add_argument("--m", type=int, default=8192)
    ap.add_argument("--stage-min-tokens", type=int, default=None,
                    help="GEMMs over quantised weights with at least this many tokens decode the weight once to "
                         "bf16 first (0 = decode inside the GEMM always; default: the library's 1024)")
    args = ap.parse_args()
    if args.config == "c2":
        args.layers = args.layers or C2["n_layers"]
        args.prompts = args.prompts or 128
    return args


def dist_setup(gpus):
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    pg = None
    if world > 1:
        import datetime

        import torch
        import torch.distributed as dist

        torch.cuda.set_device(local)
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300), device_id=torch.device("cuda", local))
        pg = dist
    return world, rank, local, pg


def trial_params(rng, n_layers):
    """A seeded TPE-like parameter vector decoded as src/search.zig:108-139."""
    out = []
    for _ in range(2):  # attn.o_proj, mlp.down_proj
        max_w = float(rng.uniform(0.8, 1.5))
        max_pos = float(rng.uniform(0.6 * (n_layers - 1), n_layers - 1))
        min_frac = float(rng.uniform(0.0, 1.0))
        min_dist = float(rng.uniform(1.0, max(1.0, 0.6 * (n_layers - 1))))
        out.append((max_w, max_pos, min_frac * max_w, min_dist))
    scope_global = rng.random() < 0.5
    di = float(rng.uniform(0.4, 0.9) * (n_layers - 1)) if scope_global else None
    return out[0], out[1], di


# ---- synthetic model on the device (torch is the device-memory plumbing here) ----
def fp8_block_quant(w, block=128):
    """FP8 E4M3 with f32 block scales amax/448 (tools/make_fixture.py:109-127), on the GPU."""
    import torch

    rows, cols = w.shape
    rb, cb = -(-rows // block), -(-cols // block)
    wp = torch.nn.functional.pad(w.float(), (0, cb * block - cols, 0, rb * block - rows))
    blocks = wp.view(rb, block, cb, block)
    amax = blocks.abs().amax(dim=(1, 3)).clamp_min(1e-12)
    scale = (amax / 448.0).float()
    q = (blocks / scale[:, None, :, None]).to(torch.float8_e4m3fn)
    codes = q.view(rb * block, cb * block)[:rows, :cols].contiguous().view(torch.uint8)
    return codes, scale.contiguous()


def build_c2_model(dev, spec, seed, max_seq):
    import torch

    import ditch_b200
    from ditch_b200 import Tensor

    g = torch.Generator(device="cuda").manual_seed(seed)
    H, I, V, L = spec["hidden"], spec["inter"], spec["vocab"], spec["n_layers"]
    qd, kvd = spec["heads"] * spec["head_dim"], spec["kv_heads"] * spec["head_dim"]
    keep, tensors = [], []

    def bf16(shape):
        return (torch.randn(shape, generator=g, device="cuda", dtype=torch.float32) * 0.02).to(torch.bfloat16)

    def add_fp8(name, rows, cols):
        w = bf16((rows, cols))
        codes, scale = fp8_block_quant(w)
        del w
        keep.extend([codes, scale])
        tensors.append(Tensor(name, "fp8", rows, cols, codes, scales=scale, block_rows=128, block_cols=128))

    ones = torch.ones(H, dtype=torch.bfloat16, device="cuda")
    keep.append(ones)
    emb = bf16((V, H))
    lm = bf16((V, H))
    keep.extend([emb, lm])
    tensors += [Tensor("embed", "bf16", V, H, emb), Tensor("lm_head", "bf16", V, H, lm),
                Tensor("final_norm", "bf16", H, 1, ones)]
    model = None
    for i in range(L):
        tensors += [Tensor(f"L{i}.input_norm", "bf16", H, 1, ones), Tensor(f"L{i}.post_norm", "bf16", H, 1, ones)]
        add_fp8(f"L{i}.q", qd, H)
        add_fp8(f"L{i}.k", kvd, H)
        add_fp8(f"L{i}.v", kvd, H)
        add_fp8(f"L{i}.o", H, qd)
        add_fp8(f"L{i}.gate", I, H)
        add_fp8(f"L{i}.up", I, H)
        add_fp8(f"L{i}.down", H, I)
    torch.cuda.synchronize()
    model = ditch_b200.Model(dev, spec, tensors, max_seq=max_seq)
    del keep, tensors
    torch.cuda.empty_cache()
    return model


# ---- clocks ----
class Clocks:
    def __init__(self, index):
        self.p = None
        self.keep = bool(os.environ.get("DITCH_BENCH_CLOCKS_DIR"))
        import tempfile

        # the samples go to a private temporary file; DITCH_BENCH_CLOCKS_DIR
        # keeps them in a named folder instead
        keep = os.environ.get("DITCH_BENCH_CLOCKS_DIR")
        try:
            if keep:
                os.makedirs(keep, exist_ok=True)
                self.path = os.path.join(keep, f"clocks_bench_{index}_{os.getpid()}.csv")
            else:
                fd, self.path = tempfile.mkstemp(prefix=f"clocks_bench_{index}_", suffix=".csv")
                os.close(fd)
            self.f = open(self.path, "w")
            self.p = subprocess.Popen(
                ["nvidia-smi", "-i", str(index), "--query-gpu=index,clocks.sm,clocks.max.sm,power.draw,"
                 "clocks_event_reasons.active,clocks_event_reasons.hw_slowdown,"
                 "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,"
                 "clocks_event_reasons.sw_power_cap", "--format=csv,noheader,nounits", "-lms", "200"],
                stdout=self.f, stderr=subprocess.DEVNULL)
        except Exception:
            self.p = None

    def stop(self):
        if not self.p:
            return None
        self.p.terminate()
        try:
            self.p.wait(timeout=5)
        except Exception:
            self.p.kill()
        self.f.close()
        sm, mx, reasons = [], 0.0, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for line in open(self.path):
            parts = [x.strip() for x in line.split(",")]
            if len(parts) < 9:
                continue
            try:
                sm.append(float(parts[1]))
                mx = max(mx, float(parts[2]))
            except ValueError:
                continue
            for n, v in zip(names, parts[5:9]):
                if v.lower() == "active":
                    reasons.add(n)
        if not self.keep:
            try:
                os.unlink(self.path)
            except OSError:
                pass
        if not sm:
            return None
        load = [s for s in sm if s > 0.5 * max(sm)] or sm
        return {"sm_mhz": statistics.median(load), "sm_max_mhz": mx, "reasons": sorted(reasons), "samples": len(sm)}


def measured_peaks():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        d = json.load(open(p))
        return d["hbm_gbs"], d["bf16_tflops"], d["bf16_tflops_sustained"], "measured"
    return 6650.0, 1590.0, 1400.0, "fallback"


# ---- CPU baseline: the oracle (a C restatement of ditch's CPU engine) ----
def host_threads():
    """Host threads this process may run on (torchrun sets OMP_NUM_THREADS=1
    for its workers; the CPU baseline uses every core it is allowed)."""
    try:
        return len(os.sched_getaffinity(0))
    except AttributeError:
        return os.cpu_count() or 1


def cpu_baseline(args, reps=None, warmup=0):
    """Times ditch's CPU engine restated in C (oracle/, VL=16 FMA, all host
    threads) on a bounded sample: one decoder layer of the C2 shape over 8
    prompts, the LM head rows, the per-layer edit GEMVs and the KL rows,
    extrapolated to the whole trial (32 layers, `--prompts` prompts). The
    linear weights and the LM head are bf16, multiplied through ditch's
    half-precision path (rows converted to f32 per task, then the f32 tiles:
    src/tensor.zig:827-883), which is how ditch holds an FP8 checkpoint in
    mapped mode (decoded to bf16 once at load, src/dequant.zig:477-514; the
    decode is not timed). Values are random (timing does not depend on them)."""
    import oracle
    from oracle.model import OracleModel, flatten_batch

    L = oracle.lib()
    L.or_set_threads(host_threads())
    cores = L.or_get_threads()
    spec = dict(C2, n_layers=1)
    H, I, V = spec["hidden"], spec["inter"], spec["vocab"]
    qd, kvd = spec["heads"] * spec["head_dim"], spec["kv_heads"] * spec["head_dim"]
    rng = np.random.default_rng(args.seed)

    def w(r, c):
        return oracle.f32_to_bf16_bits(rng.standard_normal((r, c), dtype=np.float32) * np.float32(0.02))

    big = w(V, H)
    ones = np.ones(H, np.float32)
    weights = {"embed": oracle.bf16_bits_to_f32(big), "lm_head": big, "final_norm": ones, "L0.input_norm": ones,
               "L0.post_norm": ones, "L0.q": w(qd, H), "L0.k": w(kvd, H), "L0.v": w(kvd, H), "L0.o": w(H, qd),
               "L0.gate": w(I, H), "L0.up": w(I, H), "L0.down": w(H, I)}
    m = OracleModel(spec, weights, weights_bf16=True)
    p_cpu = 8
    sample = [rng.integers(0, V, args.seq).astype(np.uint32) for _ in range(p_cpu)]
    toks, rb, rp, cap, first, take, last = flatten_batch(sample)
    for _ in range(warmup):
        m.forward(toks, rb, rp, (), ())
    t0 = time.perf_counter()
    n = 0
    while True:  # `reps` timed samples, or as many as fit about half the sample budget
        m.forward(toks, rb, rp, (), ())
        n += 1
        if (reps is not None and n >= reps) or (reps is None and time.perf_counter() - t0 > args.cpu_sample_s * 0.5):
            break
    reps = n
    t_layer = (time.perf_counter() - t0) / reps
    hl = rng.standard_normal((p_cpu, H), dtype=np.float32)
    t0 = time.perf_counter()
    logits = oracle.matmul_t_bf16(hl, big)
    t_lm = time.perf_counter() - t0
    base = oracle.log_softmax(logits)
    t0 = time.perf_counter()
    oracle.kl_first_token(base, logits)
    t_kl = time.perf_counter() - t0
    v = rng.standard_normal(H).astype(np.float32)
    wo, wd = oracle.bf16_bits_to_f32(weights["L0.o"]), oracle.bf16_bits_to_f32(weights["L0.down"])
    t0 = time.perf_counter()  # the GEMV-T of the edit over the rows as f32 (the conversion is not timed)
    oracle.compute_delta_none(wo, v, 1.0)
    oracle.compute_delta_none(wd, v, 1.0)
    t_edit = time.perf_counter() - t0
    scale = args.prompts / p_cpu
    nl = args.layers
    s_trial = nl * t_layer * scale + (t_lm + t_kl) * scale + nl * t_edit
    tokens = args.prompts * args.seq
    return {
        "value": tokens / s_trial, "unit": "tokens/s", "cores": cores, "kind": "port",
        "s_per_trial": s_trial, "sample_layer_s": t_layer,
        "sample": (f"oracle (C restatement of ditch's CPU engine, bf16 weights through its half-precision path as "
                   f"in mapped mode), {cores} threads: 1 C2 decoder layer over {p_cpu} prompts x {args.seq} tokens "
                   f"({reps} reps, {t_layer:.3f} s), LM head + KL on {p_cpu} rows, o/down edit GEMVs of one layer; "
                   f"extrapolated to {nl} layers x {args.prompts} prompts"),
    }


def reference_arm(args):
    # one step = one timed sample (a C2 decoder layer over 8 prompts, the LM
    # head and KL rows, the edit GEMVs), after `warmup` untimed ones
    cb = cpu_baseline(args, reps=max(1, args.steps), warmup=args.warmup)
    tokens = args.prompts * args.seq
    v = cb["value"]
    line = {
        "impl": "reference", "metric": "trial-eval forward tokens/s", "value": round(v, 3), "unit": "tokens/s",
        "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
        # a step is one timed sample (the C2 decoder layer over 8 prompts);
        # value and s_per_trial extrapolate it to the whole trial
        "ms_per_step": round(cb["sample_layer_s"] * 1000.0, 3),
        "s_per_trial_extrapolated": round(cb["s_per_trial"], 3),
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "bf16 weights, f32 arithmetic", "data": "synthetic",
        "config": config_block(args),
        "cpu_baseline": cb,
        "e2e": {"value": round(v, 3), "unit": "tokens/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
        "note": "ditch is Zig and no zig toolchain exists on this image; the reference arm times the C restatement "
                "of its CPU engine (oracle/), checked against ditch's own fixtures",
    }
    return line


def config_block(args):
    return {"workload": "C2: Llama-3-8B-shaped, FP8 E4M3 128x128 block-scaled weights, trial = %s-mode edit of "
                        "o_proj/down_proj + edited forward + first-token KL" % args.row_normalization,
            "row_normalization": args.row_normalization,
            "gemm": {0: "one CTA per 128-row tile (tcgen05 cta_group::1)",
                     1: "CTA pairs (tcgen05 cta_group::2, 256 x 256 tiles) for qkv, o_proj and down_proj; SwiGLU "
                        "gate / up on one CTA per tile",
                     2: "CTA pairs for every dense GEMM of 512+ tokens"}[args.cta_pairs],
            "attention": {0: "mma.sync (bf16 hi/lo products)",
                          1: "tcgen05, one CTA per SM (bf16 hi/lo products, TMEM accumulators)",
                          2: "tcgen05, two CTAs per SM (bf16 hi/lo products, TMEM accumulators)"}[args.attention_tc],
            "layers": args.layers, "prompts_per_gpu": args.prompts, "seq_len": args.seq, "vocab": C2["vocab"],
            "parallelism": f"dp{args.gpus} (prompt batches; residual sums and KL summed over the ranks by the "
                           "library's peer-group reduction over NVLink)",
            "l2": "inputs larger than L2 (7 GB of FP8 weights read per trial)",
            "fp8_decode": ("staged: each GEMM with >= %d tokens runs the bf16 GEMM over its FP8 weight decoded once "
                           "to bf16 (decoded on first use, the copy kept across trials: the weights never change, "
                           "edits are separate deltas)"
                           % (1024 if args.stage_min_tokens is None else args.stage_min_tokens)
                           if args.stage_min_tokens != 0 else "inside the GEMM (tile by tile)")}


def all_reduce(dist, arr, op="sum"):
    """All-reduce of a numpy array across ranks (NCCL over the GPUs)."""
    if dist is None:
        return arr
    import torch

    t = torch.from_numpy(np.ascontiguousarray(arr)).cuda()
    dist.all_reduce(t, op=dist.ReduceOp.SUM if op == "sum" else dist.ReduceOp.MAX)
    return t.cpu().numpy()


def traffic_from_profiles():
    """DRAM bytes (read + write) per GEMM launch of the C2 trial, from the
    committed ncu summary of one decoder layer's GEMMs (every launch of the
    layer captured: qkv, o_proj, gate/up, down_proj, each at its own shape);
    the LM head's single launch per step is left out of the average."""
    import re

    rel = os.path.join("profiles", "gemm_traffic_c2.md")
    p = os.path.join(ROOT, rel)
    if not os.path.exists(p):
        return None, None
    m = re.search(r"traffic_bytes_per_layer_launch:\s*([0-9.eE+-]+)", open(p).read())
    return (float(m.group(1)), rel) if m else (None, None)


def main():
    args = parse()
    if args.config != "c2":
        import bench_configs

        return bench_configs.run(args)
    world, rank, local, dist = dist_setup(args.gpus)
    if args.impl == "reference":
        if rank == 0:
            print(json.dumps(reference_arm(args)), flush=True)
        if dist:
            dist.barrier()
            dist.destroy_process_group()
        return 0

    import torch

    import ditch_b200

    torch.cuda.set_device(local)
    dev = ditch_b200.Device(local)
    if args.stage_min_tokens is not None:
        dev.set_decode_staging(args.stage_min_tokens)
    dev.set_deterministic(args.deterministic)
    dev.set_cta_pairs(args.cta_pairs)
    dev.set_attention_tc(args.attention_tc)
    spec = dict(C2, n_layers=args.layers)
    L, V, P, S = spec["n_layers"], spec["vocab"], args.prompts, args.seq
    t0 = time.time()
    model = build_c2_model(dev, spec, args.seed, max_seq=S)  # identical weights on every rank
    load_s = time.time() - t0

    rng = np.random.default_rng(args.seed + 1000 * (rank + 1))
    good = [rng.integers(0, V, S).astype(np.uint32) for _ in range(P)]
    bad = [rng.integers(0, V, S).astype(np.uint32) for _ in range(P)]
    kl_prompts = [rng.integers(0, V, S).astype(np.uint32) for _ in range(P)]

    # data parallel: the library sums the residuals and the KL over the ranks
    # on the device (a peer group over NVLink); torch.distributed only carries
    # the group's IPC handles and the timing barrier
    group = None
    if dist:
        def exchange(h):
            out = [None] * world
            dist.all_gather_object(out, h)
            return out

        group = ditch_b200.Group(dev, rank, world, model.dp_group_bytes(P), exchange)
        model.set_dp_group(group)
        group.barrier()
        dist.barrier()

    # one-off per study: capture (residual sums over every rank's prompts), directions
    dev.synchronize()
    dev.timer_start()
    gs, gc = model.residual_sums(good, window=1, batch_size=P)
    bs, bc = model.residual_sums(bad, window=1, batch_size=P)
    model.directions(gs, gc, bs, bc, True)
    capture_ms = dev.timer_stop()
    model.kl_init(kl_prompts)
    if args.row_normalization != "none":
        model.set_row_normalization(args.row_normalization, lora_rank=3, seed=args.seed)

    tokens_flat = np.concatenate(kl_prompts).astype(np.uint32)
    offs = np.zeros(P + 1, np.uintp)
    offs[1:] = np.cumsum([len(p) for p in kl_prompts])
    trial_rng = np.random.default_rng(args.seed + 7)  # same trials on every rank
    kls = []

    def step(e2e):
        po, pd, di = trial_params(trial_rng, L)
        model.apply_edit(po, pd, di)
        # the mean KL over every rank's prompts (summed over the group on the device)
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
    clocks = Clocks(local)
    ms = timed(False, args.steps)
    clk = clocks.stop()
    gemm_ms, gemm_launches, gemm_flops = dev.gemm_stats()
    launches = dev.launches()
    dev.set_profiling(False)
    for _ in range(max(1, args.warmup // 2)):
        step(True)
    ms_e2e = timed(True, args.steps)

    tokens = P * S
    value = tokens * world * args.steps / (ms / 1000.0)
    value_e2e = tokens * world * args.steps / (ms_e2e / 1000.0)
    hbm, tf_burst, tf_sust, src = measured_peaks()
    achieved = gemm_flops / (gemm_ms / 1000.0) / 1e12 if gemm_ms > 0 else 0.0
    traffic, tsrc = traffic_from_profiles()
    staged = args.stage_min_tokens != 0 and P * S >= (args.stage_min_tokens or 1024)
    kernel_name = ("gemm_kernel: tcgen05 bf16 MMA over bf16 copies of the FP8 weights (decoded on first use and "
                   "kept; staged plan)" if staged else "gemm_kernel: tcgen05 bf16 MMA, FP8 decoded per tile inside the GEMM")
    line = {
        "metric": "trial-eval forward tokens/s", "value": round(value, 1), "unit": "tokens/s", "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms / args.steps, 3),
        "s_per_trial": round(ms / args.steps / 1000.0, 5), "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "fp8-e4m3 weights, bf16 MMA, f32 accumulate", "data": "synthetic",
        "config": config_block(args),
        "e2e": {"value": round(value_e2e, 1), "unit": "tokens/s", "h2d_bytes_per_step": int(tokens * 4 + (P + 1) * 8),
                "d2h_bytes_per_step": int(P * 8), "ms_per_step": round(ms_e2e / args.steps, 3)},
        "roofline": {"bound": "tensor", "kernel": kernel_name,
                     "achieved": round(achieved, 1), "peak": tf_sust, "unit": "TFLOP/s",
                     "frac": round(achieved / tf_sust, 4), "peak_source": f"{src} bf16 sustained",
                     "traffic": traffic, "traffic_source": tsrc,
                     "gemm_ms_per_step": round(gemm_ms / args.steps, 3),
                     "gemm_share_of_step": round(gemm_ms / ms, 4) if ms > 0 else None,
                     "gemm_tflop_per_step": round(gemm_flops / args.steps / 1e12, 3)},
        "gpu_launches": int(launches),
        "clocks": clk,
        "one_off": {"load_s": round(load_s, 2), "capture_and_directions_ms": round(capture_ms, 2)},
        "kl_last": kls[-1] if kls else None,
    }
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        cb = cpu_baseline(args)
        line["cpu_baseline"] = {k: (round(v, 3) if isinstance(v, float) else v) for k, v in cb.items()}
    if rank == 0:
        print(json.dumps(line), flush=True)
    model.set_dp_group(None)
    model.close()
    if group:
        group.barrier()
        group.close()
    dev.close()
    if dist:
        dist.barrier()
        dist.destroy_process_group()
    return 0


if __name__ == "__main__":
    sys.exit(main())
