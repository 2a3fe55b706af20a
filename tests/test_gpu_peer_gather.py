"""KV-head sharding's head-output exchange by this library's own kernel (ma_head_gather,
shard.PeerHeadGather) on two GPUs: one process per GPU, NCCL only for the handle exchange.

Every rank's rows land at their head offset in every rank's output, call after call (the
two receive slots alternate), equal to the NCCL all-gather (shard.HeadGather) bit for bit;
the same when the exchange runs inside the attention launch (splitk_attention's
head_gather: the split merge stores the rows into every rank's region), for a step-0 call
with prefix statistics, the probe-merged step 0 (only the block's rows exchanged), a
sub-step and a plan of more CTAs than one wave (exchanged by the separate kernels after
it), with the separate exchange interleaved (shared counters); and a rank that skips a
call makes the other rank's bounded wait give up, reported by device_status() -- the
failure made on the host (a missing call), no GPU fault. Skipped with fewer than two GPUs.
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
        elif mode == "fused":
            from maskahead_b200.kernels import splitk_attention
            from maskahead_b200.layouts import Prefix

            cases = [  # B, KV heads of the rank, G, T, Tg, n, Tc, causal block, prefix statistics
                (1, 4, 4, 32, 32, 8192, 32, 0, True),     # step 0 of a cfg4 rank (shorter prefix)
                (1, 4, 4, 96, 32, 8192, 96, 32, True),    # the probe merged into step 0: the block's rows
                (1, 4, 4, 32, 32, 4096, 32, 0, False),    # a sub-step over a compact cache
                (40, 4, 4, 32, 32, 2048, 32, 0, False),   # 160 CTAs, more than one wave: the separate exchange
            ]
            for call, (B, Hk, G, T, Tg, n, Tc, causal, stats) in enumerate(cases * 2):
                g = torch.Generator(device=dev).manual_seed(100 * call + rank)
                q = torch.randn(B, Hk * G, T, 128, generator=g, device=dev).to(torch.bfloat16)
                k, v = (torch.randn(B, Hk, n, 128, generator=g, device=dev).to(torch.bfloat16) for _ in range(2))
                kc, vc = (torch.randn(B, Hk, Tc, 128, generator=g, device=dev).to(torch.bfloat16) for _ in range(2))
                pre = Prefix.dense(k, v)
                gout = torch.empty(B, Hk * G * world, Tg, 128, device=dev, dtype=torch.bfloat16)
                out, _ = splitk_attention(q, pre, kc, vc, causal_block=causal, q_pos0=Tc - T, want_prefix=stats,
                                          head_gather=(peer, gout))
                plain, _ = splitk_attention(q, pre, kc, vc, causal_block=causal, q_pos0=Tc - T, want_prefix=stats)
                want = nccl(out[:, :, :Tg].contiguous())
                torch.cuda.synchronize(dev)
                ok = ok and torch.equal(gout, want)
                ok = ok and torch.allclose(out.float(), plain.float(), rtol=2e-2, atol=2e-2)
                if call % 3 == 1:   # the separate exchange shares the counters
                    again = peer(out[:, :, :Tg])
                    torch.cuda.synchronize(dev)
                    ok = ok and torch.equal(again, want)
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


def test_attention_with_the_exchange_in_its_launch_equals_the_nccl_all_gather():
    assert _run("fused") == {0: True, 1: True}


def test_a_missing_peer_is_reported_by_device_status():
    assert _run("missing") == {0: True, 1: True}
