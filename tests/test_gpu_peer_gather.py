"""KV-head sharding's head-output exchange by this library's own kernel (ma_head_gather,
shard.PeerHeadGather) on two GPUs: one process per GPU, NCCL only for the handle exchange.

Every rank's rows land at their head offset in every rank's output, call after call (the
two receive slots alternate), equal to the NCCL all-gather (shard.HeadGather) bit for bit;
and a rank that skips a call makes the other rank's bounded wait give up, reported by
device_status() -- the failure made on the host (a missing call), no GPU fault. Skipped
with fewer than two GPUs.
"""

from __future__ import annotations

import os
import socket

import pytest
import torch

pytestmark = [pytest.mark.gpu,
              pytest.mark.skipif(not torch.cuda.is_available() or torch.cuda.device_count() < 2,
                                 reason="needs two GPUs")]


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank_main(rank: int, world: int, port: int, mode: str, result):
    import datetime

    import torch.distributed as dist

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    os.environ["NCCL_NVLS_ENABLE"] = "0"
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, device_id=dev,
                            timeout=datetime.timedelta(seconds=60))
    import maskahead_b200
    from maskahead_b200 import MaError
    from maskahead_b200._lib import MA_ERR_TIMEOUT
    from maskahead_b200.shard import HeadGather, PeerHeadGather

    ok = True
    try:
        peer, nccl = PeerHeadGather(world, rank), HeadGather(world)
        if mode == "exchange":
            for call in range(5):
                g = torch.Generator(device=dev).manual_seed(100 * call + rank)
                part = torch.randn(2, 8, 32, 128, generator=g, device=dev).to(torch.bfloat16)
                got = peer(part)
                want = nccl(part)
                torch.cuda.synchronize(dev)
                ok = ok and torch.equal(got, want)
                ok = ok and torch.equal(got[:, 8 * rank: 8 * (rank + 1)], part)
            maskahead_b200.device_status(dev)
        else:   # rank 1 skips the second call: rank 0's wait gives up
            part = torch.ones(1, 4, 32, 128, device=dev, dtype=torch.bfloat16) * (rank + 1)
            peer(part)
            torch.cuda.synchronize(dev)
            maskahead_b200.device_status(dev)
            if rank == 0:
                prev = maskahead_b200.set_peer_wait_ns(2_000_000)   # 2 ms
                peer(part)
                try:
                    maskahead_b200.device_status(dev)
                    ok = False
                except MaError as exc:
                    ok = exc.status == MA_ERR_TIMEOUT
                maskahead_b200.set_peer_wait_ns(prev)
            dist.barrier()
        peer.close()
    finally:
        dist.destroy_process_group()
    result[rank] = bool(ok)


def _run(mode: str):
    import torch.multiprocessing as mp

    ctx = mp.get_context("spawn")
    mgr = ctx.Manager()
    result = mgr.dict()
    port = _free_port()
    procs = [ctx.Process(target=_rank_main, args=(r, 2, port, mode, result)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=300)
    for p in procs:
        if p.is_alive():
            p.kill()
    assert all(p.exitcode == 0 for p in procs), [p.exitcode for p in procs]
    return dict(result)


def test_peer_gather_equals_the_nccl_all_gather():
    assert _run("exchange") == {0: True, 1: True}


def test_a_missing_peer_is_reported_by_device_status():
    assert _run("missing") == {0: True, 1: True}
