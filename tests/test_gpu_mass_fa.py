"""GPU parity of the TMA-pipelined prefix-mass / value-score kernel (dense bf16 caches)
against the CPU oracle and against the general (cp.async-staged) kernel.

Bars: mass a_j to fp32 rounding (rtol 2e-5 against the oracle's fp32 restatement, whose
statistics M_p, L_p come from the same device attention call); the value score
a_j ||v_j - c|| to rtol 5e-5. The two device kernels sum in different orders, so they
are compared at the same bars. Sizes cover several tiles per CTA, a ragged last tile,
selection-row counts that pad the MMA's N (1, 32, 224 rows) and a live-slot mask.
"""

from __future__ import annotations

import numpy as np
import pytest
import torch

import oracle

pytestmark = pytest.mark.gpu

DEV = "cuda"


def _lib():
    from maskahead_b200._lib import load_library

    return load_library()


def _scores(which, q, pre, st, rows):
    from maskahead_b200.kernels import prefix_scores

    prev = _lib().ma_set_attention_kernel(which)
    try:
        mass, score = prefix_scores(q, pre, st, rows, value=True)
        torch.cuda.synchronize()
    finally:
        _lib().ma_set_attention_kernel(prev)
    return mass.cpu(), score.cpu()


@pytest.mark.parametrize("B,Hq,H,T,n,rows,masked", [
    (1, 28, 4, 32, 8192, list(range(32)), False),     # cfg2 shape: R2 = 224
    (1, 8, 2, 32, 40000, list(range(0, 32, 4)), False),   # several tiles per CTA, R2 = 32
    (2, 4, 4, 16, 3001, [5], True),                  # one selection row, ragged tail, mask
])
def test_mass_fa_matches_oracle_and_general_kernel(B, Hq, H, T, n, rows, masked):
    from maskahead_b200.kernels import splitk_attention
    from maskahead_b200.layouts import Prefix

    gen = torch.Generator().manual_seed(n + Hq)
    D = 128
    q = torch.randn(B, Hq, T, D, generator=gen).to(torch.bfloat16)
    k = torch.randn(B, H, n, D, generator=gen).to(torch.bfloat16)
    v = torch.randn(B, H, n, D, generator=gen).to(torch.bfloat16)
    live = (torch.rand(B, H, n, generator=gen) > 0.2) if masked else None
    qd, kd, vd = q.to(DEV), k.to(DEV), v.to(DEV)
    pre = Prefix.dense(kd, vd, mask=None if live is None else live.to(DEV))
    _, st = splitk_attention(qd, pre, None, None, want_prefix=True)
    torch.cuda.synchronize()
    rows_t = torch.tensor(rows, dtype=torch.int32, device=DEV)
    mass0, score0 = _scores(0, qd, pre, st, rows_t)
    mass1, score1 = _scores(1, qd, pre, st, rows_t)
    want_mass = oracle.prefix_mass(q, k, st[0].cpu(), st[1].cpu(), rows, live_mask=live)
    np.testing.assert_allclose(mass0.numpy(), want_mass.numpy(), rtol=2e-5, atol=1e-9)
    np.testing.assert_allclose(mass1.numpy(), want_mass.numpy(), rtol=2e-5, atol=1e-9)
    want_score = oracle.value_score(want_mass, v)
    np.testing.assert_allclose(score0.numpy(), want_score.numpy(), rtol=5e-5, atol=1e-9)
    np.testing.assert_allclose(score0.numpy(), score1.numpy(), rtol=5e-5, atol=1e-9)


def test_mass_fa_repeated_calls_are_identical():
    """The centre counters and generations reset between calls: same inputs, same bits."""
    from maskahead_b200.kernels import prefix_scores, splitk_attention
    from maskahead_b200.layouts import Prefix

    gen = torch.Generator().manual_seed(11)
    q = torch.randn(1, 28, 32, 128, generator=gen).to(torch.bfloat16).to(DEV)
    k = torch.randn(1, 4, 20000, 128, generator=gen).to(torch.bfloat16).to(DEV)
    v = torch.randn(1, 4, 20000, 128, generator=gen).to(torch.bfloat16).to(DEV)
    pre = Prefix.dense(k, v)
    _, st = splitk_attention(q, pre, None, None, want_prefix=True)
    rows = torch.arange(32, dtype=torch.int32, device=DEV)
    m0, s0 = prefix_scores(q, pre, st, rows, value=True)
    for _ in range(3):
        m1, s1 = prefix_scores(q, pre, st, rows, value=True)
        assert torch.equal(m0, m1) and torch.equal(s0, s1)


@pytest.mark.parametrize("lanes,n", [(160, 1000), (24, 3000)])
def test_value_score_after_mass_calls_of_other_head_counts(lanes, n):
    """value_score over many lanes (one CTA per lane when lanes >= SMs, else several) right
    after a mass call of 4 heads and a value score of 3 lanes on the same workspace: the
    per-lane counters must not pick up the other calls' centres or partials (a stale
    counter makes a lane wait for a centre that never comes and score NaN)."""
    from maskahead_b200.hotpath import value_score
    from maskahead_b200.kernels import prefix_scores, splitk_attention
    from maskahead_b200.layouts import Prefix

    gen = torch.Generator().manual_seed(lanes + n)
    q = torch.randn(1, 28, 32, 128, generator=gen).to(torch.bfloat16).to(DEV)
    k = torch.randn(1, 4, 4096, 128, generator=gen).to(torch.bfloat16).to(DEV)
    vv = torch.randn(1, 4, 4096, 128, generator=gen).to(torch.bfloat16).to(DEV)
    pre = Prefix.dense(k, vv)
    _, st = splitk_attention(q, pre, None, None, want_prefix=True)
    prefix_scores(q, pre, st, torch.arange(32, dtype=torch.int32, device=DEV), value=True)
    value_score(torch.rand(3, n, generator=gen).to(DEV), torch.randn(3, n, 128, generator=gen).to(torch.bfloat16).to(DEV))
    a = torch.rand(lanes, n, generator=gen)
    v = torch.randn(lanes, n, 128, generator=gen).to(torch.bfloat16)
    for _ in range(2):
        got = value_score(a.to(DEV), v.to(DEV)).cpu()
        torch.cuda.synchronize()
        want = oracle.value_score(a, v)
        np.testing.assert_allclose(got.numpy(), want.numpy(), rtol=5e-5, atol=1e-9)


@pytest.mark.parametrize("B,n,cap", [
    (16, 16384, 0),   # a ragged serving batch (64 heads): CTAs of at most 16 tiles, score in a second launch
    (40, 9000, 8),    # more heads than SMs, 8-tile CTAs
])
def test_mass_fa_ragged_batch_split_matches_oracle(B, n, cap):
    """A ragged batch (ma_kv.lens) spreads each head over CTAs of a few tiles -- the longest
    sequences' heads no longer set the launch's time -- with the centre reduced by each
    head's last CTA and the score in a second launch of phase 2 alone. Same bars as above,
    per sequence against the oracle, and against one CTA per head (ma_set_mass_tiles(-1))."""
    from maskahead_b200.kernels import prefix_scores, splitk_attention
    from maskahead_b200.layouts import Prefix

    gen = torch.Generator().manual_seed(n + B)
    Hq, H, T, D = 28, 4, 32, 128
    q = torch.randn(B, Hq, T, D, generator=gen).to(torch.bfloat16)
    k = torch.randn(B, H, n, D, generator=gen).to(torch.bfloat16)
    v = torch.randn(B, H, n, D, generator=gen).to(torch.bfloat16)
    lens = torch.randint(1, n + 1, (B,), generator=gen).to(torch.int32)
    lens[0], lens[1] = 1, n
    qd = q.to(DEV)
    pre = Prefix(kf=k.to(DEV), vf=v.to(DEV), nf=n, lens=lens.to(DEV))
    _, st = splitk_attention(qd, pre, None, None, want_prefix=True)
    rows = list(range(T))
    rows_t = torch.tensor(rows, dtype=torch.int32, device=DEV)
    out = {}
    for setting in (cap, -1):
        prev = _lib().ma_set_mass_tiles(setting)
        try:
            mass, score = prefix_scores(qd, pre, st, rows_t, value=True)
            torch.cuda.synchronize()
        finally:
            _lib().ma_set_mass_tiles(prev)
        out[setting] = (mass.cpu(), score.cpu())
    mass, score = out[cap]
    for bi in range(B):
        L = int(lens[bi])
        mp, lp = st[0][bi:bi + 1].cpu(), st[1][bi:bi + 1].cpu()
        want_mass = oracle.prefix_mass(q[bi:bi + 1], k[bi:bi + 1, :, :L], mp, lp, rows)
        np.testing.assert_allclose(mass[bi:bi + 1, :, :L].numpy(), want_mass.numpy(), rtol=2e-5, atol=1e-9,
                                   err_msg=f"sequence {bi} (length {L})")
        want_score = oracle.value_score(want_mass, v[bi:bi + 1, :, :L])
        np.testing.assert_allclose(score[bi:bi + 1, :, :L].numpy(), want_score.numpy(), rtol=5e-5, atol=1e-9,
                                   err_msg=f"sequence {bi} (length {L})")
        assert not mass[bi, :, L:].any() and not score[bi, :, L:].any(), "slots past the length must be 0"
    np.testing.assert_allclose(mass.numpy(), out[-1][0].numpy(), rtol=2e-5, atol=1e-9)
    np.testing.assert_allclose(score.numpy(), out[-1][1].numpy(), rtol=5e-5, atol=1e-9)
