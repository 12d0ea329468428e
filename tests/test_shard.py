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
