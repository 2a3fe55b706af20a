"""GPU parity of the sm_100a hot path against the CPU oracle and the reference fixtures.

Bars (stated per assertion):
  * index work (top-k read set, retained set, gather) -- bit-exact; the read set of a
    full step 0 may differ from the oracle only on slots whose oracle score is within
    1e-5 (relative) of the k-th score, where two fp32 summation orders can flip ranks;
  * prefix mass and value score -- fp32 rounding (rtol 2e-5 / 5e-5);
  * attention outputs -- fp32 queries 1e-4; bf16 queries: bf16 output rounding plus the
    bf16 P operand of the tensor-core P.V (atol = rtol = 2e-2).
"""

from __future__ import annotations

from pathlib import Path

import numpy as np
import pytest
import torch

import oracle
from gen_inputs import CASES, make_retain_case
from gpu_cases import band_equal, device_prefix, load_case

pytestmark = pytest.mark.gpu

GOLDEN = Path(__file__).resolve().parent / "golden"
DEV = "cuda"


def _golden(name):
    return dict(np.load(GOLDEN / f"{name}.npz"))


def _out_tol(dtype):
    return (1e-4, 1e-4) if dtype == torch.float32 else (2e-2, 2e-2)


@pytest.mark.parametrize("name", list(CASES))
def test_step0_matches_reference(name):
    from maskahead_b200.hotpath import fast_step0

    g = _golden(name)
    case, k, v, extra = load_case(name)
    spec = case["spec"]
    D = spec["D"]
    q, kc, vc, rows = case["query"], case["current_key"], case["current_value"], case["rows"]
    prefix = device_prefix(case, k, v, extra)
    topk = int(g["topk"])
    res = fast_step0(q.to(DEV), prefix, kc.to(DEV), vc.to(DEV), query_indices=rows, topk=topk,
                     value_aware=True, scaling=D ** -0.5)
    torch.cuda.synchronize()
    live = case.get("live_mask")
    mass = res.mass.cpu()
    if live is not None:
        mass = mass.masked_fill(~live, 0.0)
    np.testing.assert_allclose(mass.numpy(), g["importance"], rtol=2e-5, atol=1e-9)
    np.testing.assert_allclose(res.score.cpu().numpy(), g["value_score"], rtol=5e-5, atol=1e-9)
    band_equal(res.indices.cpu().numpy(), g["value_indices"], g["value_score"], topk)
    assert (np.diff(res.indices.cpu().numpy(), axis=-1) > 0).all(), "read set must be ascending"
    atol, rtol = _out_tol(q.dtype)
    np.testing.assert_allclose(res.out.float().cpu().numpy(), g["dense_out"], rtol=rtol, atol=atol)


@pytest.mark.parametrize("name", list(CASES))
def test_sparse_substep_matches_reference(name):
    from maskahead_b200.hotpath import compact_attention

    g = _golden(name)
    case, k, v, extra = load_case(name)
    q, kc, vc = case["query"], case["current_key"], case["current_value"]
    prefix = device_prefix(case, k, v, extra)
    idx = torch.from_numpy(g["value_indices"]).to(DEV)
    out = compact_attention(q.to(DEV), prefix, idx, kc.to(DEV), vc.to(DEV), scaling=case["spec"]["D"] ** -0.5)
    torch.cuda.synchronize()
    atol, rtol = _out_tol(q.dtype)
    np.testing.assert_allclose(out.float().cpu().numpy(), g["compact_out"], rtol=rtol, atol=atol)


@pytest.mark.parametrize("name", list(CASES))
def test_compact_cache_substep_matches_reference(name):
    """The session's path: the read set gathered once into a compact cache (dequantized),
    every sub-step attending [compact | block] as a contiguous cache."""
    from maskahead_b200.hotpath import compact_attention, gather_read_set

    g = _golden(name)
    case, k, v, extra = load_case(name)
    q, kc, vc = case["query"], case["current_key"], case["current_value"]
    prefix = device_prefix(case, k, v, extra)
    idx = torch.from_numpy(g["value_indices"]).to(DEV)
    compact = gather_read_set(prefix, idx, dtype=q.dtype)
    out = compact_attention(q.to(DEV), compact, None, kc.to(DEV), vc.to(DEV), scaling=case["spec"]["D"] ** -0.5)
    torch.cuda.synchronize()
    atol, rtol = _out_tol(q.dtype)
    np.testing.assert_allclose(out.float().cpu().numpy(), g["compact_out"], rtol=rtol, atol=atol)


@pytest.mark.parametrize("name", ["small_bf16", "small_k4v4_token", "small_k4v4_channel", "cfg1"])
def test_gather_is_bit_exact(name):
    from maskahead_b200.kernels import gather_packed_kv

    g = _golden(name)
    case, k, v, extra = load_case(name)
    prefix = device_prefix(case, k, v, extra, mask=False)
    idx = torch.from_numpy(g["value_indices"])
    ok_, ov = gather_packed_kv(prefix, idx.to(DEV), dtype=k.dtype)
    torch.cuda.synchronize()
    np.testing.assert_array_equal(ok_.cpu().float().numpy(), oracle.gather_per_kv_head(k, idx).float().numpy())
    np.testing.assert_array_equal(ov.cpu().float().numpy(), oracle.gather_per_kv_head(v, idx).float().numpy())


def test_selector_topk_api_matches_reference():
    from maskahead_b200.kernels import selector_topk

    for name in ("small_bf16", "small_bf16_live", "small_k4v4_channel"):
        g = _golden(name)
        case, k, v, extra = load_case(name)
        prefix = device_prefix(case, k, v, extra, mask=False)
        live = case.get("live_mask")
        res = selector_topk(case["query"].to(DEV), prefix, query_indices=case["rows"], topk=int(g["topk"]),
                            scaling=case["spec"]["D"] ** -0.5, return_importance=True,
                            live_mask=None if live is None else live.to(DEV))
        torch.cuda.synchronize()
        np.testing.assert_allclose(res.importance.cpu().numpy(), g["importance"], rtol=2e-5, atol=1e-9)
        band_equal(res.indices.cpu().numpy(), g["mass_indices"], g["importance"], int(g["topk"]))


def test_retention_matches_reference():
    from maskahead_b200.hotpath import lookahead_survivors, value_score

    g = _golden("retain")
    r = make_retain_case()
    a = (r["a1"] + r["a_probe"]).to(DEV)
    score = value_score(a, r["v_live"].to(DEV))
    torch.cuda.synchronize()
    np.testing.assert_allclose(score.cpu().numpy(), g["score"], rtol=2e-5, atol=1e-12)
    keep = lookahead_survivors(r["pos"].to(DEV), torch.from_numpy(g["score"]).to(DEV), r["C"],
                               recent_window=r["W"], sink_tokens=r["sinks"])
    torch.cuda.synchronize()
    np.testing.assert_array_equal(keep.cpu().numpy(), g["keep"])


@pytest.mark.parametrize("n,k", [(1, 1), (7, 3), (100, 100), (1000, 17), (5000, 1024), (20000, 3000),
                                 (40000, 4096), (65536, 4096), (70000, 4096), (131072, 8192), (140000, 512)])
def test_select_topk_bit_exact_with_ties(n, k):
    from maskahead_b200.kernels import select_topk_indices

    gen = torch.Generator().manual_seed(n + k)
    # few distinct values: many exact ties at the k-th score
    s = torch.randint(-20, 20, (2, 3, n), generator=gen).float() / 4.0
    s[0, 0, : n // 3] = float("-inf")
    live = torch.rand(2, 3, n, generator=gen) > 0.2
    live[..., :k] = True
    for mask in (None, live):
        want_i, want_v = oracle.topk_sorted(s, k, mask)
        got_i, got_v = select_topk_indices(s.to(DEV), k, None if mask is None else mask.to(DEV))
        torch.cuda.synchronize()
        np.testing.assert_array_equal(got_i.cpu().numpy(), want_i.numpy())
        np.testing.assert_array_equal(got_v.cpu().numpy(), want_v.numpy())


@pytest.mark.parametrize("live,C,W,sinks", [(600, 256, 64, 4), (5000, 2048, 64, 4), (300, 300, 64, 0),
                                            (1000, 50, 64, 4), (9000, 8192, 128, 4)])
def test_survivors_bit_exact(live, C, W, sinks):
    from maskahead_b200.hotpath import lookahead_survivors

    gen = torch.Generator().manual_seed(live + C)
    L, B, H = 2, 1, 3
    score = torch.randint(0, 50, (L, B, H, live), generator=gen).float()      # ties included
    pos = torch.empty(L, B, H, live, dtype=torch.int32)
    for i in range(L * B * H):
        p = torch.randperm(4 * live, generator=gen)[:live].sort().values
        pos.view(-1, live)[i] = p.to(torch.int32)
    pos[..., :2] = torch.tensor([0, 2], dtype=torch.int32)
    want = oracle.survivors_lookahead(pos, score, C, recent_window=W, sink_tokens=sinks)
    got = lookahead_survivors(pos.to(DEV), score.to(DEV), C, recent_window=W, sink_tokens=sinks)
    torch.cuda.synchronize()
    np.testing.assert_array_equal(got.cpu().numpy(), want.numpy())
    # positions not monotone along the live axis: output still ordered by position
    perm = torch.randperm(live, generator=gen)
    want = oracle.survivors_lookahead(pos[..., perm], score[..., perm], C, recent_window=W, sink_tokens=sinks)
    got = lookahead_survivors(pos[..., perm].contiguous().to(DEV), score[..., perm].contiguous().to(DEV), C,
                              recent_window=W, sink_tokens=sinks)
    torch.cuda.synchronize()
    np.testing.assert_array_equal(got.cpu().numpy(), want.numpy())


@pytest.mark.parametrize("live,C,W,sinks", [(65536, 8192, 128, 4), (20000, 4096, 64, 0), (4096, 4096, 64, 4),
                                            (70, 64, 64, 2), (5000, 1000, 0, 3)])
def test_survivors_large_and_physical_slots(live, C, W, sinks):
    """Rows of the cfg4 size (a cluster of CTAs per lane), a window filling the capacity, no
    window, and scores given per physical slot through phys (the paged cache): the same keep
    as the oracle on the scores gathered per live entry. Positions strictly increase along
    the live axis, and once with one repeated position (the general path)."""
    from maskahead_b200.hotpath import lookahead_survivors

    gen = torch.Generator().manual_seed(7 * live + C + W)
    L, B, H = 1, 2, 2
    n_phys = live + 100
    score_phys = torch.randint(0, 1000, (L, B, H, n_phys), generator=gen).float()   # ties included
    phys = torch.stack([torch.randperm(n_phys, generator=gen)[:live] for _ in range(L * B * H)])
    phys = phys.reshape(L, B, H, live).to(torch.int32)
    pos = torch.empty(L, B, H, live, dtype=torch.int32)
    for i in range(L * B * H):
        pos.view(-1, live)[i] = torch.randperm(2 * live, generator=gen)[:live].sort().values.to(torch.int32)
    score_live = torch.gather(score_phys, -1, phys.long())
    for p in (pos, torch.cat([pos[..., :1], pos[..., :-1]], dim=-1)):   # the second repeats position 0
        want = oracle.survivors_lookahead(p, score_live, C, recent_window=W, sink_tokens=sinks)
        got = lookahead_survivors(p.to(DEV), score_live.to(DEV), C, recent_window=W, sink_tokens=sinks)
        got_p = lookahead_survivors(p.to(DEV), score_phys.to(DEV), C, recent_window=W, sink_tokens=sinks,
                                    phys=phys.to(DEV))
        torch.cuda.synchronize()
        np.testing.assert_array_equal(got.cpu().numpy(), want.numpy())
        np.testing.assert_array_equal(got_p.cpu().numpy(), want.numpy())


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32])
@pytest.mark.parametrize("n", [0, 1, 31, 33, 257, 1100])
def test_prefix_attention_edges(dtype, n):
    """Ragged prefix lengths, empty prefix, prefix stats and the block-causal probe mask."""
    from maskahead_b200.kernels import splitk_attention

    gen = torch.Generator().manual_seed(n)
    B, Hq, H, T, D = 2, 6, 2, 64, 128
    q = torch.randn(B, Hq, T, D, generator=gen).to(dtype)
    k = torch.randn(B, H, n, D, generator=gen).to(dtype)
    v = torch.randn(B, H, n, D, generator=gen).to(dtype)
    kc = torch.randn(B, H, T, D, generator=gen).to(dtype)
    vc = torch.randn(B, H, T, D, generator=gen).to(dtype)
    live = torch.rand(B, H, n, generator=gen) > 0.3 if n > 1 else None
    from maskahead_b200.layouts import Prefix
    for causal in (0, 32):
        pre = Prefix.dense(k.to(DEV), v.to(DEV), mask=None if live is None else live.to(DEV))
        out, st = splitk_attention(q.to(DEV), pre, kc.to(DEV), vc.to(DEV), causal_block=causal,
                                   want_prefix=n > 0)
        torch.cuda.synchronize()
        want, (mp, lp, op) = oracle.prefix_attention(q, k, v, kc, vc, live_mask=live, causal_block=causal)
        atol, rtol = _out_tol(dtype)
        np.testing.assert_allclose(out.float().cpu().numpy(), want.float().numpy(), rtol=rtol, atol=atol)
        if n > 0:
            has = lp > 0
            np.testing.assert_allclose(st[0].cpu()[has].numpy(), mp[has].numpy(), rtol=1e-5, atol=1e-5)
            np.testing.assert_allclose(st[1].cpu()[has].numpy(), lp[has].numpy(), rtol=rtol, atol=rtol)
            np.testing.assert_allclose(st[2].cpu()[has].numpy(), op[has].numpy(), rtol=rtol, atol=atol)


def test_bad_arguments_raise_without_launching():
    from maskahead_b200 import MaError
    from maskahead_b200.kernels import select_topk_indices, splitk_attention
    from maskahead_b200.layouts import Prefix

    s = torch.zeros(1, 1, 8, device=DEV)
    with pytest.raises(ValueError):
        select_topk_indices(s, 9)
    q = torch.zeros(1, 4, 8, 96, device=DEV, dtype=torch.bfloat16)       # head_dim 96: unsupported
    k = torch.zeros(1, 2, 16, 96, device=DEV, dtype=torch.bfloat16)
    with pytest.raises(MaError):
        splitk_attention(q, Prefix.dense(k, k), k[:, :, :8], k[:, :, :8])
    torch.cuda.synchronize()
