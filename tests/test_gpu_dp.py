"""Data parallelism over a peer group (ditch_cuda_model_set_dp_group).

Each rank evaluates its own share of the prompts; the residual sums
(src/engine.zig:314-438) and the KL (src/scorers.zig:378-402) come back
summed over the ranks on the device. On one GPU a one-rank group must give
the single-device results bit for bit (the reduction adds nothing and sums
the per-prompt KL values in the host's order). On 2, 4 or 8 GPUs (one
process each, skipped with fewer) every rank must hold the same bits, equal
within f32 rounding to one device evaluating every prompt (the ranks' GEMMs
see other token counts, so their K splits, and the last bits of the
residuals, can differ).
"""
import os
import socket

import numpy as np
import pytest

import ditch_b200
from synth import make_model, prompts

pytestmark = pytest.mark.gpu

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
LENGTHS = [40, 17, 64, 3, 70, 33, 9, 51, 64, 28, 12, 47, 5, 60, 22, 38]


def _all_prompts(vocab):
    return prompts(77, LENGTHS, vocab)


def _shard(ps, rank, world):
    return ps[rank::world]


@pytest.fixture
def deterministic(device):
    """K splits summed in a fixed order, so repeated forwards give the same bits."""
    device.set_deterministic(True)
    yield device
    device.set_deterministic(False)


def test_one_rank_group_matches_single_device(deterministic):
    device = deterministic
    spec, f32, tensors = make_model(310, n_layers=2, hidden=256, head_dim=64, heads=4, kv_heads=2)
    ps = _all_prompts(spec["vocab"])
    m = ditch_b200.Model(device, spec, tensors, max_seq=128)
    dirs = np.random.default_rng(3).standard_normal((spec["n_layers"] + 1, spec["hidden"])).astype(np.float32)
    dirs /= np.linalg.norm(dirs, axis=1, keepdims=True)
    m.set_directions(dirs)
    m.kl_init(ps)
    # one edit for every pass below (recomputing it would add the GEMV-T's
    # row splits in another order: the same deltas to the last bits only)
    m.apply_edit((1.2, 1.0, 0.5, 2.0), (0.9, 0.0, 0.3, 2.0))
    sums0, n0 = m.residual_sums(ps, window=2, batch_size=5)
    kl0 = m.kl_score()
    g = ditch_b200.Group(device, 0, 1, m.dp_group_bytes(len(ps)), lambda h: [h])
    m.set_dp_group(g)
    sums1, n1 = m.residual_sums(ps, window=2, batch_size=5)
    kl1 = m.kl_score()
    assert n1 == n0 == len(ps)
    assert np.array_equal(sums1, sums0)
    assert kl1 == kl0 and kl0 > 0
    # and twice more: the reductions alternate between the two halves of the region
    assert m.kl_score() == kl0
    assert np.array_equal(m.residual_sums(ps, window=2, batch_size=5)[0], sums0)
    np.testing.assert_array_equal(g.allreduce_f64([1.5, -2.0, 3.25]), [1.5, -2.0, 3.25])
    m.set_dp_group(None)
    m.close()
    g.close()


def test_dp_group_too_small_is_refused(device):
    spec, f32, tensors = make_model(311, n_layers=1, hidden=128, head_dim=32, heads=4, kv_heads=2, inter=256)
    m = ditch_b200.Model(device, spec, tensors, max_seq=64)
    g = ditch_b200.Group(device, 0, 1, 1024, lambda h: [h])  # room for a reduction, not for 200 KL values
    m.set_dp_group(g)
    ps = prompts(5, [8] * 200, spec["vocab"])
    m.kl_init(ps)
    with pytest.raises(ditch_b200.DitchCudaError, match="too small"):
        m.kl_score()
    m.set_dp_group(None)
    assert abs(m.kl_score()) < 1e-6  # the base model, scored without the group
    m.close()
    g.close()


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

    torch.cuda.set_device(rank)
    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=120))
    dev = ditch_b200.Device(rank)
    dev.set_deterministic(True)  # repeated forwards give the same bits
    spec, f32, tensors = make_model(312, n_layers=2, hidden=256, head_dim=64, heads=4, kv_heads=2, fmt="fp8",
                                    block=(64, 64))
    ps = _all_prompts(spec["vocab"])
    mine = _shard(ps, rank, world)
    m = ditch_b200.Model(dev, spec, tensors, max_seq=128)
    dirs = np.random.default_rng(3).standard_normal((spec["n_layers"] + 1, spec["hidden"])).astype(np.float32)
    dirs /= np.linalg.norm(dirs, axis=1, keepdims=True)
    m.set_directions(dirs)
    # one device, every prompt
    sums_one, n_one = m.residual_sums(ps, window=1)
    m.kl_init(ps)
    m.apply_edit((1.2, 1.0, 0.5, 2.0), (0.9, 0.0, 0.3, 2.0))
    kl_one = m.kl_score()
    m.reset_edits()

    def exchange(h):
        out = [None] * world
        dist.all_gather_object(out, h)
        return out

    g = ditch_b200.Group(dev, rank, world, m.dp_group_bytes(len(mine)), exchange)
    m.set_dp_group(g)
    dist.barrier()
    sums_dp, n_dp = m.residual_sums(mine, window=1)
    m.kl_init(mine)
    m.apply_edit((1.2, 1.0, 0.5, 2.0), (0.9, 0.0, 0.3, 2.0))
    kl_dp = m.kl_score()
    kl_dp2 = m.kl_score()
    red = g.allreduce_f64(np.arange(5, dtype=np.float64) + rank)
    g.barrier()
    np.savez(os.path.join(out_dir, f"r{rank}.npz"), sums_one=sums_one, n_one=n_one, kl_one=kl_one, sums_dp=sums_dp,
             n_dp=n_dp, kl_dp=kl_dp, kl_dp2=kl_dp2, red=red)
    m.set_dp_group(None)
    m.close()
    dist.barrier()
    g.close()
    dev.close()
    dist.destroy_process_group()


@pytest.mark.parametrize("world", [2, 4, 8])
def test_data_parallel_ranks_agree_with_one_gpu(tmp_path, world):
    import torch
    import torch.multiprocessing as mp

    if torch.cuda.device_count() < world:
        pytest.skip(f"needs {world} GPUs")
    os.environ.setdefault("NCCL_NVLS_ENABLE", "0")
    mp.spawn(_worker, args=(world, _free_port(), str(tmp_path)), nprocs=world, join=True)
    z = [np.load(tmp_path / f"r{r}.npz") for r in range(world)]
    for r in range(world):
        assert int(z[r]["n_dp"]) == len(LENGTHS)
        assert np.array_equal(z[r]["sums_dp"], z[0]["sums_dp"]), r  # the same bits on every rank
        assert float(z[r]["kl_dp"]) == float(z[0]["kl_dp"]) == float(z[r]["kl_dp2"]), r
        np.testing.assert_array_equal(z[r]["red"], np.arange(5) * world + world * (world - 1) / 2)
    one, dp = z[0]["sums_one"], z[0]["sums_dp"]
    assert np.abs(dp - one).max() <= 1e-5 * np.abs(one).max()
    kl1, kld = float(z[0]["kl_one"]), float(z[0]["kl_dp"])
    assert kl1 > 0 and abs(kld - kl1) <= 1e-5 * kl1, (kld, kl1)
