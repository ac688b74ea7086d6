"""The data-parallel path of bench.py on CPU ranks (gloo, world size 2).

Prompt batches shard across ranks (src/engine.zig:383-435 treats prompts
independently). Each rank captures the residuals of its own prompts, the f64
sums and counts are all-reduced before the directions, and the per-prompt KL
sums are all-reduced per trial. The result must equal one process holding
every prompt: the same f64 sums up to summation order, hence the same
directions and the same KL. The oracle stands in for the device forward; the
all-reduce is bench.py's own helper."""
import os
import socket

import numpy as np
import pytest
import torch.multiprocessing as mp

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def _worker(rank, world, port, out_dir):
    import sys

    for p in (ROOT, os.path.join(ROOT, "tests")):
        if p not in sys.path:
            sys.path.insert(0, p)
    import datetime

    import torch
    import torch.distributed as dist

    import oracle
    from golden_loader import Golden
    from oracle.model import OracleModel, flatten_batch

    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=60))

    def all_reduce(arr):  # bench.py's reduction, on CPU tensors for gloo
        t = torch.from_numpy(np.ascontiguousarray(arr))
        dist.all_reduce(t)
        return t.numpy()

    g = Golden("qwen2")
    m = OracleModel(g.spec, g.f32_weights())
    rng = np.random.default_rng(5)
    good = [rng.integers(0, g.spec["vocab"], rng.integers(3, 9)).astype(np.uint32) for _ in range(6)]
    bad = [rng.integers(0, g.spec["vocab"], rng.integers(3, 9)).astype(np.uint32) for _ in range(6)]
    mine = slice(rank, None, world)
    sums = {}
    for name, ps in (("good", good[mine]), ("bad", bad[mine])):
        toks, rb, rp, cap, first, take, last = flatten_batch(ps, 1)
        res, _ = m.forward(toks, rb, rp, cap, ())
        sums[name] = (all_reduce(oracle.residual_sums(res, first, take)), all_reduce(np.array([len(ps)], np.float64)))
    dirs = oracle.compute_directions((sums["good"][0] / sums["good"][1][0]).astype(np.float32),
                                     (sums["bad"][0] / sums["bad"][1][0]).astype(np.float32), True)
    # per-trial KL on each rank's share of the KL prompts, all-reduced
    kp = good[mine]
    toks, rb, rp, cap, first, take, last = flatten_batch(kp, 1)
    _, base = m.forward(toks, rb, rp, (), last)
    w = g.f32_weights()
    for li in range(g.spec["n_layers"]):
        a, b = oracle.compute_delta_none(w[f"L{li}.o"], dirs[li + 1], 0.9)
        m.set_delta(li, "o", a, b)
    _, ed = m.forward(toks, rb, rp, (), last)
    kl_mean, _ = oracle.kl_first_token(oracle.log_softmax(base), ed)
    tot = all_reduce(np.array([kl_mean * len(kp), len(kp)], np.float64))
    if rank == 0:
        np.save(os.path.join(out_dir, "dirs.npy"), dirs)
        np.save(os.path.join(out_dir, "kl.npy"), np.array([tot[0] / tot[1]]))
    dist.barrier()
    dist.destroy_process_group()


def test_data_parallel_sums_directions_and_kl(tmp_path):
    import sys

    for p in (ROOT, os.path.join(ROOT, "tests")):
        if p not in sys.path:
            sys.path.insert(0, p)
    import oracle
    from golden_loader import Golden
    from oracle.model import OracleModel, flatten_batch

    mp.spawn(_worker, args=(2, _free_port(), str(tmp_path)), nprocs=2, join=True)
    dirs = np.load(tmp_path / "dirs.npy")
    kl = float(np.load(tmp_path / "kl.npy")[0])
    # one process, every prompt
    g = Golden("qwen2")
    m = OracleModel(g.spec, g.f32_weights())
    rng = np.random.default_rng(5)
    good = [rng.integers(0, g.spec["vocab"], rng.integers(3, 9)).astype(np.uint32) for _ in range(6)]
    bad = [rng.integers(0, g.spec["vocab"], rng.integers(3, 9)).astype(np.uint32) for _ in range(6)]
    means = []
    for ps in (good, bad):
        toks, rb, rp, cap, first, take, last = flatten_batch(ps, 1)
        res, _ = m.forward(toks, rb, rp, cap, ())
        means.append((oracle.residual_sums(res, first, take) / len(ps)).astype(np.float32))
    want = oracle.compute_directions(means[0], means[1], True)
    np.testing.assert_allclose(dirs, want, atol=1e-5)
    toks, rb, rp, cap, first, take, last = flatten_batch(good, 1)
    _, base = m.forward(toks, rb, rp, (), last)
    w = g.f32_weights()
    for li in range(g.spec["n_layers"]):
        a, b = oracle.compute_delta_none(w[f"L{li}.o"], want[li + 1], 0.9)
        m.set_delta(li, "o", a, b)
    _, ed = m.forward(toks, rb, rp, (), last)
    kl_want, _ = oracle.kl_first_token(oracle.log_softmax(base), ed)
    assert kl > 0
    assert abs(kl - kl_want) <= 1e-6 + 1e-4 * abs(kl_want)
