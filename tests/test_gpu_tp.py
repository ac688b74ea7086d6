"""Tensor parallelism over a peer group on 2, 4 and 8 GPUs (one process each).

Each rank loads the whole tensors and keeps its shard: 1 / world of the query
and kv heads (q / k / v rows, o columns) and of the MLP columns (gate / up
rows, down columns). The o_proj and down_proj partial sums are all-reduced over
NVLink peer memory after every layer. Both ranks run the same prompts and
must hold identical residual streams and logits (every element is one sum in
rank order); against the single-GPU model the products are split over K, so
the results agree to rounding: within the forward bound of
`test_gpu_model.py`, max |err| <= 2e-3 + 2e-2 max |ref|, and in practice far
closer. The none-mode edit of o_proj / down_proj is local to each shard
(src/abliterate.zig:264-280: A = v^T W splits by columns with W), so the
edited forward must agree the same way; so must the pre-normalised edit (row
norms summed over the shards) and the full one (src/abliterate.zig:324-350:
its randomised SVD over the column shards, the same sketch as one GPU).

Each world size needs that many GPUs; skipped otherwise."""
import os
import socket

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

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

    import ditch_b200
    from oracle.model import flatten_batch
    from synth import make_model, prompts

    torch.cuda.set_device(rank)
    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=120))
    dev = ditch_b200.Device(rank)
    # 8 query and 8 kv heads and 512 MLP columns: shards for every world size up to 8
    spec, f32, tensors = make_model(500, n_layers=3, hidden=256, head_dim=64, heads=8, kv_heads=8, inter=512,
                                    qkv_bias=True)
    ps = prompts(77, [40, 17, 64, 3, 70], spec["vocab"])  # the same prompts on every rank
    toks, rb, rp, cap, first, take, last = flatten_batch(ps, 2)
    max_tokens = 256

    def exchange(h):
        out = [None] * world
        dist.all_gather_object(out, h)
        return out

    one = ditch_b200.Model(dev, spec, tensors, max_seq=128)
    tp = ditch_b200.Model(dev, spec, tensors, max_seq=128, tp_rank=rank, tp_world=world)
    group = ditch_b200.Group(dev, rank, world, tp.group_bytes(max_tokens), exchange)
    tp.set_group(group, max_tokens)
    dist.barrier()
    res1, log1 = one.forward(toks, rb, rp, cap, last)
    res2, log2 = tp.forward(toks, rb, rp, cap, last)
    rng = np.random.default_rng(3)
    dirs = rng.standard_normal((spec["n_layers"] + 1, spec["hidden"])).astype(np.float32)
    dirs /= np.linalg.norm(dirs, axis=1, keepdims=True)
    for m in (one, tp):
        m.set_directions(dirs)
        m.apply_edit((1.2, 1.5, 0.5, 2.0), (1.1, 1.0, 0.4, 2.0), None)
    res3, log3 = one.forward(toks, rb, rp, cap, last)
    res4, log4 = tp.forward(toks, rb, rp, cap, last)
    # row_normalization = pre: the row norms of o_proj / down_proj summed over
    # the ranks' column shards (one all-reduce per matrix)
    for m in (one, tp):
        m.set_row_normalization("pre")
        m.apply_edit((1.2, 1.5, 0.5, 2.0), (1.1, 1.0, 0.4, 2.0), None)
    res5, log5 = one.forward(toks, rb, rp, cap, last)
    res6, log6 = tp.forward(toks, rb, rp, cap, last)
    # row_normalization = full (the product default): the randomised SVD of
    # each matrix's delta over the column shards, with the partial sums over
    # columns reduced over the group and the column vectors gathered whole
    for m in (one, tp):
        m.set_row_normalization("full", lora_rank=2, seed=5)
        m.apply_edit((1.2, 1.5, 0.5, 2.0), (1.1, 1.0, 0.4, 2.0), None)
    res7, log7 = one.forward(toks, rb, rp, cap, last)
    res8, log8 = tp.forward(toks, rb, rp, cap, last)
    for m in (one, tp):
        m.set_row_normalization("none")
    group.barrier()
    np.savez(os.path.join(out_dir, f"r{rank}.npz"), res1=res1, log1=log1, res2=res2, log2=log2, res3=res3, log3=log3,
             res4=res4, log4=log4, res5=res5, log5=log5, res6=res6, log6=log6, res7=res7, log7=log7, res8=res8,
             log8=log8)
    tp.close()
    one.close()
    dist.barrier()
    group.close()
    dev.close()
    dist.destroy_process_group()


@pytest.mark.parametrize("world", [2, 4, 8])
def test_tensor_parallel_forward_matches_one_gpu(tmp_path, world):
    import torch
    import torch.multiprocessing as mp

    if torch.cuda.device_count() < world:
        pytest.skip(f"needs {world} GPUs")
    os.environ.setdefault("NCCL_NVLS_ENABLE", "0")
    mp.spawn(_worker, args=(world, _free_port(), str(tmp_path)), nprocs=world, join=True)
    z = [np.load(tmp_path / f"r{r}.npz") for r in range(world)]
    z0 = z[0]
    for r in range(1, world):
        for key in ("res2", "log2", "res4", "log4", "res6", "log6", "res8", "log8"):
            assert np.array_equal(z0[key], z[r][key]), (r, key)  # replicated streams are identical
    for a, b in (("res1", "res2"), ("log1", "log2"), ("res3", "res4"), ("log3", "log4"), ("res5", "res6"),
                 ("log5", "log6"), ("res7", "res8"), ("log7", "log8")):
        ref, got = z0[a], z0[b]
        err = float(np.abs(got - ref).max())
        bound = 2e-3 + 2e-2 * float(np.abs(ref).max())
        assert err <= bound, (a, b, err, bound)
        print(f"{a} vs {b}: max |err| {err:.3e} (bound {bound:.3e})")
    assert not np.array_equal(z0["log1"], z0["log3"]), "the edit changed nothing"
    assert not np.array_equal(z0["log3"], z0["log5"]), "row normalisation changed nothing"
    assert not np.array_equal(z0["log5"], z0["log7"]), "full row normalisation changed nothing"


def _timeout_worker(rank, world, port, out_dir):
    import sys

    for p in (ROOT, os.path.join(ROOT, "tests")):
        if p not in sys.path:
            sys.path.insert(0, p)
    import datetime

    import torch
    import torch.distributed as dist

    import ditch_b200
    from synth import make_model

    torch.cuda.set_device(rank)
    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=120))
    dev = ditch_b200.Device(rank)
    spec, f32, tensors = make_model(510, n_layers=2, hidden=256, head_dim=64, heads=8, kv_heads=8, inter=512)

    def exchange(h):
        out = [None] * world
        dist.all_gather_object(out, h)
        return out

    tp = ditch_b200.Model(dev, spec, tensors, max_seq=64, tp_rank=rank, tp_world=world)
    group = ditch_b200.Group(dev, rank, world, tp.group_bytes(64), exchange)
    tp.set_group(group, 64)
    group.set_wait_budget(1.0)
    dist.barrier()
    codes = []
    if rank == 0:
        # rank 1 never joins: the row-norm collective runs out of its budget
        # (a flag nothing sets), twice: the failed call kept no norms
        for _ in range(2):
            try:
                tp.set_row_normalization("pre")
                codes.append(0)
            except ditch_b200.DitchCudaError as e:
                codes.append(e.code)
        # the context is still usable: a decode on the device after the failures
        q = np.arange(256, dtype=np.uint8).reshape(16, 16) & 0x77  # no NaN codes
        got = dev.dequant_fp8(q, np.full((1, 1), 0.5, np.float32), 16, 16)
        codes.append(int(np.asarray(got).any()))
    np.save(os.path.join(out_dir, f"t{rank}.npy"), np.asarray(codes, np.int64))
    dist.barrier()  # no kernel of either rank is in flight past this point
    tp.close()
    group.close()
    dev.close()
    dist.destroy_process_group()


def test_tensor_parallel_wait_runs_out_and_keeps_no_norms(tmp_path):
    """A rank that does not join a collective makes the peer's waits run out
    after the group's budget (1 s here): set_row_normalization returns
    DITCH_CUDA_DEVICE_FAILED, and a second call fails the same way instead of
    reusing row norms from the failed one. The device stays usable."""
    import torch
    import torch.multiprocessing as mp

    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    os.environ.setdefault("NCCL_NVLS_ENABLE", "0")
    mp.spawn(_timeout_worker, args=(2, _free_port(), str(tmp_path)), nprocs=2, join=True)
    codes = np.load(tmp_path / "t0.npy")
    assert list(codes) == [2, 2, 1], codes  # DEVICE_FAILED twice, then a decode that ran
