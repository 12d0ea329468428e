"""Multi-rank host logic on CPU: two gloo ranks split batch x heads, compute
their shards (with the CPU oracle standing in for the GPU kernel), and the
gathered result equals the single-process result; timing is max over ranks."""
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from monarch_attention_b200.shard import (gather_shards, max_over_ranks, shard_mask,
                                          shard_range, take_shard)


@pytest.mark.parametrize("E,H,world", [(4, 3, 2), (3, 5, 2), (2, 16, 8), (1, 7, 4)])
def test_shard_ranges_partition(E, H, world):
    ranges = [shard_range(E, H, world, r) for r in range(world)]
    assert ranges[0][0] == 0 and ranges[-1][1] == E * H
    for (a, b), (c, d) in zip(ranges, ranges[1:]):
        assert b == c
    sizes = [b - a for a, b in ranges]
    assert max(sizes) - min(sizes) <= (H if E % world == 0 else 1)


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def _worker(rank, world, port, result_path):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        from oracle.ma_oracle import monarch_attention_oracle
        g = torch.Generator().manual_seed(5)
        E, H, N, D, B, T = 3, 2, 40, 8, 8, 2
        q, k, v = (torch.randn(E, H, N, D, generator=g) for _ in range(3))
        mask = torch.ones(E, N, dtype=torch.bool)
        mask[1, 25:] = False
        a, b = shard_range(E, H, world, rank)
        qs, ks, vs = (take_shard(t, a, b) for t in (q, k, v))
        ms = shard_mask(mask, H, a, b)
        # per-head oracle call for each (e, h) of the shard (mask row per head)
        outs = []
        for i in range(b - a):
            o = monarch_attention_oracle(qs[:, i:i + 1].numpy(), ks[:, i:i + 1].numpy(),
                                         vs[:, i:i + 1].numpy(), ms[:, i].numpy(), T, B, False)
            outs.append(torch.from_numpy(o))
        shard_out = torch.cat(outs, dim=1)
        full = gather_shards(shard_out, E, H)
        t = max_over_ranks(float(rank + 1))
        if rank == 0:
            ref = monarch_attention_oracle(q.numpy(), k.numpy(), v.numpy(), mask.numpy(),
                                           T, B, False)
            err = float(np.abs(full.numpy() - ref).max())
            with open(result_path, "w") as f:
                f.write(f"{err} {t}")
    finally:
        dist.destroy_process_group()


def test_two_rank_gather_matches_single_process(tmp_path):
    world = 2
    path = str(tmp_path / "res.txt")
    mp.spawn(_worker, args=(world, _free_port(), path), nprocs=world, join=True)
    err, t = map(float, open(path).read().split())
    assert err < 1e-6
    assert t == float(world)


def _problem_worker(rank, world, port, result_path):
    """shard_problem + gather_shards exactly as bench.py uses them, with the
    oracle standing in for the kernel: each shard is run as its own (E', H')
    problem with its own mask rows."""
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        from oracle.ma_oracle import monarch_attention_oracle
        from monarch_attention_b200.shard import shard_problem
        g = torch.Generator().manual_seed(9)
        E, H, N, D, B, T = 2, 3, 40, 8, 8, 2
        q, k, v = (torch.randn(E, H, N, D, generator=g) for _ in range(3))
        mask = torch.ones(E, N, dtype=torch.bool)
        mask[1, 17:] = False
        scales = tuple(torch.rand(E, H, generator=g) for _ in range(3))
        qs, ks, vs, ms, ss, (a, b) = shard_problem(q, k, v, mask, scales, world, rank)
        assert qs.shape[0] * qs.shape[1] == b - a and qs.is_contiguous()
        # the scales follow the heads
        assert torch.equal(ss[0].reshape(-1), scales[0].reshape(-1)[a:b])
        o = monarch_attention_oracle(qs.numpy(), ks.numpy(), vs.numpy(), ms.numpy(), T, B, False)
        full = gather_shards(torch.from_numpy(o), E, H)
        if rank == 0:
            ref = monarch_attention_oracle(q.numpy(), k.numpy(), v.numpy(), mask.numpy(),
                                           T, B, False)
            with open(result_path, "w") as f:
                f.write(f"{float(np.abs(full.numpy() - ref).max())}")
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world", [2, 3])
def test_shard_problem_gather_matches_single_process(world, tmp_path):
    """world 2 splits whole batch rows; world 3 splits inside a batch row
    (the (n, 1) layout with per-head mask rows)."""
    path = str(tmp_path / "res.txt")
    mp.spawn(_problem_worker, args=(world, _free_port(), path), nprocs=world, join=True)
    assert float(open(path).read()) < 1e-6
