"""Expert parallelism over a peer group on 2, 4 and 8 GPUs (one process each).

Each rank keeps 1 / world of the routed experts (16 experts: 8, 4 or 2 per
rank), routes its own prompts and
exchanges (token, expert) rows with the other ranks over NVLink; the combine
runs in the same expert-index order as on one GPU, and every per-row product
is the same product, so the expert-parallel forward must equal the
single-GPU forward of the same prompts bit for bit. After the
expert-selective edit (moe.applyExpertSelective, src/moe.zig:1373-1477) the
gathered scores must pick the same experts as one GPU does and the edited
forwards must agree bit for bit too: each expert's A = v^T W_down comes from
the same fixed row chunks summed in the same order on either layout.

Each world size needs that many GPUs; skipped otherwise. The ranks exchange IPC handles over a
gloo process group on 127.0.0.1."""
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
    dev.set_deterministic(True)  # K splits summed in a fixed order: the two models must agree bit for bit
    spec, f32, tensors = make_model(300, n_layers=2, hidden=256, head_dim=64, heads=4, kv_heads=2, fmt="mxfp4",
                                    moe=dict(experts=16, top_k=4, inter=128))
    ps = prompts(40 + rank, [40, 17, 64, 3, 70][: 5 - rank % 4], spec["vocab"])  # a different batch per rank
    toks, rb, rp, cap, first, take, last = flatten_batch(ps, 2)
    max_tokens = 256

    def exchange(h):
        out = [None] * world
        dist.all_gather_object(out, h)
        return out

    one = ditch_b200.Model(dev, spec, tensors, max_seq=128)
    ep = ditch_b200.Model(dev, spec, tensors, max_seq=128, ep_rank=rank, ep_world=world)
    group = ditch_b200.Group(dev, rank, world, ep.group_bytes(max_tokens), exchange)
    ep.set_group(group, max_tokens)
    dist.barrier()

    res1, log1 = one.forward(toks, rb, rp, cap, last)
    res2, log2 = ep.forward(toks, rb, rp, cap, last)

    # the same directions and edit on both models (scores gathered across ranks)
    rng = np.random.default_rng(9)
    dirs = rng.standard_normal((spec["n_layers"] + 1, spec["hidden"])).astype(np.float32)
    dirs /= np.linalg.norm(dirs, axis=1, keepdims=True)
    for m in (one, ep):
        m.set_directions(dirs)
        m.apply_expert_edit((1.2, 1.0, 0.5, 2.0), (1.1, 0.5, 0.4, 2.0), None, n_experts=3, strength=1.0)
    res3, log3 = one.forward(toks, rb, rp, cap, last)
    res4, log4 = ep.forward(toks, rb, rp, cap, last)
    # row_normalization = full: every edited expert's rank-2 delta, its sketch
    # seeded by the matrix's index on one device whichever rank owns it
    for m in (one, ep):
        m.set_row_normalization("full", lora_rank=2, seed=5)
        m.apply_expert_edit((1.2, 1.0, 0.5, 2.0), (1.1, 0.5, 0.4, 2.0), None, n_experts=3, strength=1.0)
    res5, log5 = one.forward(toks, rb, rp, cap, last)
    res6, log6 = ep.forward(toks, rb, rp, cap, last)
    for m in (one, ep):
        m.set_row_normalization("none")
    order1 = one.rank_experts(1, dirs[2])
    order2 = ep.rank_experts(1, dirs[2])
    # greedy generation with the edited experts: the same tokens as one GPU.
    # Odd ranks stop early on an EOS (the second token of each of their
    # prompts), so their later steps run on the placeholder row while the
    # other ranks still decode.
    first = one.generate(ps, 6)
    eos = sorted({int(t[1]) for t in first if len(t) > 1}) if rank % 2 else []
    gen1 = one.generate(ps, 6, eos_ids=eos)
    gen2 = ep.generate(ps, 6, eos_ids=eos)
    flat = lambda g: np.concatenate([np.asarray(t, np.int64) for t in g] + [np.asarray([len(t) for t in g])])
    group.barrier()
    np.savez(os.path.join(out_dir, f"r{rank}.npz"), res1=res1, log1=log1, res2=res2, log2=log2, res3=res3, log3=log3,
             res4=res4, log4=log4, res5=res5, log5=log5, res6=res6, log6=log6, order1=np.asarray(order1[0]),
             order2=np.asarray(order2[0]), gen1=flat(gen1), gen2=flat(gen2),
             early=np.asarray([int(rank % 2 == 1 and any(len(t) < 6 for t in gen1))]))
    ep.close()
    one.close()
    dist.barrier()
    group.close()
    dev.close()
    dist.destroy_process_group()


@pytest.mark.parametrize("world", [2, 4, 8])
def test_expert_parallel_forward_equals_one_gpu(tmp_path, world):
    import torch
    import torch.multiprocessing as mp

    if torch.cuda.device_count() < world:
        pytest.skip(f"needs {world} GPUs")
    os.environ.setdefault("NCCL_NVLS_ENABLE", "0")
    mp.spawn(_worker, args=(world, _free_port(), str(tmp_path)), nprocs=world, join=True)
    for r in range(world):
        z = np.load(tmp_path / f"r{r}.npz")
        for a, b in (("res1", "res2"), ("log1", "log2"), ("res3", "res4"), ("log3", "log4"), ("res5", "res6"),
                     ("log5", "log6")):
            diff = float(np.abs(z[a] - z[b]).max()) if z[a].size else 0.0
            assert np.array_equal(z[a], z[b]), (r, a, b, diff)
        assert not np.array_equal(z["log1"], z["log3"]), "the edit changed nothing"
        assert not np.array_equal(z["log3"], z["log5"]), "full row normalisation changed nothing"
        assert np.array_equal(z["order1"], z["order2"])
        assert np.array_equal(z["gen1"], z["gen2"]), r
    assert any(int(np.load(tmp_path / f"r{r}.npz")["early"][0]) for r in range(1, world, 2)), "no rank stopped early"
