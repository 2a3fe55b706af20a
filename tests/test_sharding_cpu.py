"""Multi-GPU partitioning (maskahead_b200.shard) of the bench workloads, checked on CPU
with gloo ranks.

* KV-head sharding (cfg4): every rank gets a disjoint, equal slice of the KV heads with
  their query heads, and the all-gather of the per-rank outputs reassembles the heads in
  the global order.
* Sequence sharding (cfg5): the ranks' contiguous ranges cover every sequence exactly once
  and every rank's total length is within one sequence of the ideal share.
"""

from __future__ import annotations

import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

import bench
from maskahead_b200.shard import HeadGather, head_shard, sequence_shard


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _gather_worker(rank: int, world: int, port: int, result):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        cfg = bench.CONFIGS["cfg4"]
        share = bench.rank_share(cfg, rank, world)
        hq = share["Hq"]
        # each query head's block filled with its global head index
        heads = torch.arange(rank * hq, (rank + 1) * hq, dtype=torch.float32)
        out = heads.view(1, hq, 1, 1).expand(1, hq, 4, 8).contiguous()
        gather = HeadGather(world)
        full = gather(out)
        again = torch.empty_like(full)
        gather(out * 2, out=again)                   # the receive buffer is reused
        result[rank] = (full[0, :, 0, 0].tolist(), again[0, :, 0, 0].tolist())
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world", [2, 4])
def test_head_shards_gather_in_global_order(world):
    cfg = bench.CONFIGS["cfg4"]
    shares = [bench.rank_share(cfg, r, world) for r in range(world)]
    assert sum(s["H"] for s in shares) == cfg["H"]
    assert [s["head0"] for s in shares] == [r * cfg["H"] // world for r in range(world)]
    assert all(s["Hq"] * cfg["H"] == s["H"] * cfg["Hq"] for s in shares), "query heads follow their KV heads"
    mgr = mp.Manager()
    result = mgr.dict()
    mp.spawn(_gather_worker, args=(world, _free_port(), result), nprocs=world, join=True)
    for r in range(world):
        assert result[r][0] == [float(h) for h in range(cfg["Hq"])]
        assert result[r][1] == [2.0 * h for h in range(cfg["Hq"])]
    hs = [head_shard(cfg["H"], cfg["Hq"], world, r) for r in range(world)]
    assert [h.hq0 for h in hs] == [r * cfg["Hq"] // world for r in range(world)]


@pytest.mark.parametrize("world", [1, 2, 4, 8])
def test_sequence_shards_cover_and_balance(world):
    cfg = bench.CONFIGS["cfg5"]
    lens = bench.sequence_lengths(cfg)
    assert len(lens) == 256 and min(lens) >= 4096 and max(lens) <= 16384
    parts = [bench.rank_share(cfg, r, world)["lens"] for r in range(world)]
    assert [x for p in parts for x in p] == lens, "contiguous ranges covering every sequence once"
    totals = [sum(p) for p in parts]
    ideal = sum(lens) / world
    assert all(abs(t - ideal) <= max(lens) for t in totals), "every share within one sequence of its ideal"
    shards = [sequence_shard(lens, world, r) for r in range(world)]
    assert [s.lo for s in shards[1:]] == [s.hi for s in shards[:-1]] and shards[-1].hi == len(lens)


def test_shard_arguments_are_checked():
    with pytest.raises(ValueError):
        head_shard(8, 32, 3, 0)
    with pytest.raises(ValueError):
        sequence_shard([5, 6], 2, 2)
