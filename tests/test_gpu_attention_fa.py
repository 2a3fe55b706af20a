"""GPU parity of the 128-key-tile attention kernel (TMA-fed dense bf16 prefix and current
block) and of the 64-key-tile kernel it replaces there, against the CPU oracle.

The pipelined kernel runs with one 128-row M tile per CTA and with a pair of M tiles per
CTA sharing the K/V tiles (R > 128), and the 64-key kernel on the same inputs
(``ma_set_attention_kernel`` 2, 3 and 1); each is compared with
``oracle.prefix_attention`` at the bf16 bar of the other attention tests (atol = rtol =
2e-2: bf16 output rounding plus the bf16 P operand of P.V); the prefix-only statistics
(max, sum, normalized output) are compared the same way. The sizes cover: an empty prefix,
prefixes shorter than one tile, one key past a tile boundary, several splits, a
current block longer than one tile, one and two 128-row M tiles, several row tiles
(R = G*T > 256), and query blocks whose length neither divides nor is a multiple of 128
(T = 96, 160: the row tile is loaded as four 32-row pieces). The splits of a row block
merge in one launch: in a thread-block cluster (each CTA pulling its share of the rows
from the others' shared memory, or -- when every split is at most one key tile, as in the
sub-steps -- each CTA pushing its rows into the shared memory of the CTA that merges
them), else through global memory in a cooperative launch, else in a separate pass.
"""

from __future__ import annotations

import numpy as np
import pytest
import torch

import oracle

pytestmark = pytest.mark.gpu

DEV = "cuda"
TOL = 2e-2


def _lib():
    from maskahead_b200._lib import load_library

    return load_library()


def _run(which, q, k, v, kc, vc, causal, q_pos0, c_pos0, want_prefix):
    from maskahead_b200.kernels import splitk_attention
    from maskahead_b200.layouts import Prefix

    prev = _lib().ma_set_attention_kernel(which)
    try:
        pre = Prefix.dense(k, v)
        out, st = splitk_attention(q, pre, kc, vc, causal_block=causal, q_pos0=q_pos0, c_pos0=c_pos0,
                                   want_prefix=want_prefix)
        torch.cuda.synchronize()
    finally:
        _lib().ma_set_attention_kernel(prev)
    return out, st


@pytest.mark.parametrize("B,Hq,H,T,n,Tc,causal", [
    (1, 4, 1, 32, 0, 32, 32),        # current block only
    (1, 4, 1, 32, 1, 32, 0),         # one prefix key
    (2, 6, 2, 64, 127, 64, 32),      # one partial tile
    (1, 7, 1, 32, 129, 32, 32),      # a tile boundary + 1, R = 224 (two M tiles)
    (1, 28, 4, 32, 1100, 32, 32),    # cfg2-like heads, several splits
    (1, 28, 4, 32, 1024, 32, 32),    # cfg2's sub-step: nine one-tile splits push their rows
    (3, 8, 2, 32, 300, 32, 32),      # one-tile splits, six clusters, R = 128
    (2, 8, 2, 32, 256, 32, 0),       # one-tile splits, R = 128 over three CTAs per cluster
    (1, 8, 2, 128, 5000, 160, 64),   # current block longer than a tile, R = 512 (two row tiles)
    (1, 4, 4, 256, 2048, 256, 128),  # T = 256: one query head per row tile
    (1, 16, 4, 96, 3000, 96, 32),    # T = 96 (a block + two probe blocks): 32-row query pieces
    (2, 4, 4, 96, 700, 96, 32),      # T = 96, one head per group: R = 96 < one row tile
    (1, 6, 2, 160, 1000, 160, 32),   # T = 160: pieces straddle row tiles, R = 480
    (8, 28, 4, 32, 8192, 32, 32),    # 192 CTAs: no single wave, the separate (half-warp) merge
])
def test_fa_kernel_matches_oracle_and_tc(B, Hq, H, T, n, Tc, causal):
    gen = torch.Generator().manual_seed(1000 * n + T + Hq)
    D = 128
    q = torch.randn(B, Hq, T, D, generator=gen).to(torch.bfloat16)
    k = torch.randn(B, H, n, D, generator=gen).to(torch.bfloat16)
    v = torch.randn(B, H, n, D, generator=gen).to(torch.bfloat16)
    kc = torch.randn(B, H, Tc, D, generator=gen).to(torch.bfloat16)
    vc = torch.randn(B, H, Tc, D, generator=gen).to(torch.bfloat16)
    q_pos0 = Tc - T                  # the queries are the last T positions of the block
    want, (mp, lp, op) = oracle.prefix_attention(q, k, v, kc, vc, causal_block=causal, q_pos0=q_pos0, c_pos0=0)
    dev = [x.to(DEV) for x in (q, k, v, kc, vc)]
    outs = {}
    for which in (2, 3, 1):
        out, st = _run(which, *dev, causal, q_pos0, 0, n > 0)
        np.testing.assert_allclose(out.float().cpu().numpy(), want.float().numpy(), rtol=TOL, atol=TOL,
                                   err_msg=f"kernel {which}")
        if n > 0:
            np.testing.assert_allclose(st[0].cpu().numpy(), mp.numpy(), rtol=1e-5, atol=1e-5)
            np.testing.assert_allclose(st[1].cpu().numpy(), lp.numpy(), rtol=TOL, atol=TOL)
            np.testing.assert_allclose(st[2].cpu().numpy(), op.numpy(), rtol=TOL, atol=TOL)
        outs[which] = out.float().cpu()
    # the kernels differ only in summation order and the lazy-rescale reference (a pair's
    # warp group takes every key tile of its rows, one M tile's two groups alternate tiles
    # and merge, and the pair's plan has twice the splits)
    np.testing.assert_allclose(outs[2].numpy(), outs[1].numpy(), rtol=TOL, atol=TOL)
    np.testing.assert_allclose(outs[3].numpy(), outs[2].numpy(), rtol=TOL, atol=TOL)


@pytest.mark.parametrize("which,Hq", [(2, 8), (3, 16)])
def test_fa_kernel_large_logits_rescale(which, Hq):
    """Logits growing along the keys force the lazy rescale of O on nearly every tile (one
    M tile per CTA, and a pair: R = 256)."""
    gen = torch.Generator().manual_seed(7)
    B, H, T, n, D = 1, 2, 32, 3000, 128
    q = torch.randn(B, Hq, T, D, generator=gen).to(torch.bfloat16)
    ramp = torch.linspace(0.0, 6.0, n)[None, None, :, None]
    k = (torch.randn(B, H, n, D, generator=gen) * 0.5 + ramp * q.float().mean(dim=(1, 2))[:, None, None, :].sign())
    k = k.to(torch.bfloat16)
    v = torch.randn(B, H, n, D, generator=gen).to(torch.bfloat16)
    kc = torch.randn(B, H, T, D, generator=gen).to(torch.bfloat16)
    vc = torch.randn(B, H, T, D, generator=gen).to(torch.bfloat16)
    want, _ = oracle.prefix_attention(q, k, v, kc, vc, causal_block=32)
    out, _ = _run(which, *[x.to(DEV) for x in (q, k, v, kc, vc)], 32, 0, 0, False)
    np.testing.assert_allclose(out.float().cpu().numpy(), want.float().numpy(), rtol=TOL, atol=TOL)


@pytest.mark.parametrize("n", [8192, 1024])
def test_fa_kernel_repeated_calls_are_identical(n):
    """The fused merge's counters reset between calls, and the pushed merge's barriers
    start afresh: the same inputs give the same bits."""
    gen = torch.Generator().manual_seed(3)
    B, Hq, H, T, D = 1, 28, 4, 32, 128
    dev = [torch.randn(*s, generator=gen).to(torch.bfloat16).to(DEV)
           for s in ((B, Hq, T, D), (B, H, n, D), (B, H, n, D), (B, H, T, D), (B, H, T, D))]
    first, _ = _run(0, *dev, 32, 0, 0, False)
    for _ in range(3):
        again, _ = _run(0, *dev, 32, 0, 0, False)
        assert torch.equal(first, again)


@pytest.mark.parametrize("which,B,Hq,H,n,ragged", [
    (0, 16, 28, 4, 1024, False),   # cfg5's sub-step shape: one split per row block, rows written directly
    (3, 16, 28, 4, 1024, False),   # the same with pairs of M tiles
    (2, 8, 28, 4, 8192, False),    # two 32-tile splits, the block folded into the second, merged in one launch
    (3, 8, 28, 4, 8192, True),     # pairs, ragged lengths (some sequences end in the first split)
    (0, 24, 28, 4, 6000, True),    # ragged, more CTAs than one wave: the separate merge
])
def test_fa_folded_block_matches_oracle(which, B, Hq, H, n, ragged):
    """Without prefix-only statistics (the sub-steps) the current block is the last prefix
    split's final key tile instead of a split of its own; a single split per row block then
    writes its rows as the output. Compared with the oracle per sequence, and with the same
    call asking for the statistics (block as its own split)."""
    from maskahead_b200.kernels import splitk_attention
    from maskahead_b200.layouts import Prefix

    gen = torch.Generator().manual_seed(11 * n + B + which)
    T = Tc = 32
    D = 128
    q = torch.randn(B, Hq, T, D, generator=gen).to(torch.bfloat16)
    k = torch.randn(B, H, n, D, generator=gen).to(torch.bfloat16)
    v = torch.randn(B, H, n, D, generator=gen).to(torch.bfloat16)
    kc = torch.randn(B, H, Tc, D, generator=gen).to(torch.bfloat16)
    vc = torch.randn(B, H, Tc, D, generator=gen).to(torch.bfloat16)
    lens = (torch.randint(1, n + 1, (B,), generator=gen) if ragged else torch.full((B,), n)).to(torch.int32)
    if ragged:
        lens[0] = 1            # one key
        lens[-1] = n           # every key
    dq, dk, dv, dkc, dvc = (x.to(DEV) for x in (q, k, v, kc, vc))
    pre = Prefix(kf=dk, vf=dv, nf=n, lens=lens.to(DEV) if ragged else None)
    prev = _lib().ma_set_attention_kernel(which)
    try:
        out, _ = splitk_attention(dq, pre, dkc, dvc)
        out_split, _ = splitk_attention(dq, pre, dkc, dvc, want_prefix=True)
        torch.cuda.synchronize()
    finally:
        _lib().ma_set_attention_kernel(prev)
    for bi in range(B):
        L = int(lens[bi])
        want, _ = oracle.prefix_attention(q[bi:bi + 1], k[bi:bi + 1, :, :L], v[bi:bi + 1, :, :L], kc[bi:bi + 1],
                                          vc[bi:bi + 1])
        np.testing.assert_allclose(out[bi:bi + 1].float().cpu().numpy(), want.float().numpy(), rtol=TOL, atol=TOL,
                                   err_msg=f"sequence {bi} (length {L})")
    np.testing.assert_allclose(out.float().cpu().numpy(), out_split.float().cpu().numpy(), rtol=TOL, atol=TOL)
