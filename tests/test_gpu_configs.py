"""Parity of the composed block-step at the benchmarked configurations.

Each test runs what bench.py times for one layer -- step 0 through the public API
(``fast_step0(gather=True)``: attention, mass, value score, ascending read set, the read
set gathered into the compact cache) followed by three sparse sub-steps over that compact
cache (``compact_attention``) -- and compares every product with the CPU oracle on the
same seeded inputs:

  cfg2   one layer: prefix 8192, 28 q / 4 KV heads, bf16, read budget 1024; also against
         the reference's own outputs (tests/golden/cfg2_layer.npz, make_golden.py)
  cfg3   the same shape in k4v4 token mode (1% of the key channels x8 before quantizing);
         also against the reference's outputs (cfg3_layer.npz)
  cfg4   one layer: prefix 65536, 32 q / 8 KV heads, read budget 4096, the probe of two
         lookahead blocks (T = 96, block-causal), the lookahead value score and the
         survivors at capacity 8192
  cfg5   a slice of the serving batch: 16 sequences of U[4096, 16384] slots, k4v4 token
         mode in a shuffled pool of 64-slot pages (grids of several waves: the separate
         split merge)

plus the dense-layer bypass (session.py:456-467, 1378-1393): dense-prefix layers and a
budget covering the prefix attend densely.

Bars: mass rtol 2e-5, value score 5e-5 (fp32 summation order), read sets equal outside the
1e-5 tie band of the k-th score, the compact cache bit-exact, attention outputs 2e-2 (bf16
output, bf16 P operand, bf16 split partials), retained sets bit-exact on the same scores.
The packed cases are quantized on the CPU by the oracle (whose payloads the reference
fixtures pin), so no expected value comes from a device kernel.
"""

from __future__ import annotations

from pathlib import Path

import numpy as np
import pytest
import torch

import oracle
from gpu_cases import band_equal, device_prefix, load_case

pytestmark = pytest.mark.gpu

DEV = "cuda"
GOLDEN = Path(__file__).resolve().parent / "golden"
ATOL = RTOL = 2e-2


def _substep_inputs(seed, B, Hq, H, T, D, steps):
    g = torch.Generator().manual_seed(seed)
    return [(torch.randn(B, Hq, T, D, generator=g).to(torch.bfloat16),
             torch.randn(B, H, T, D, generator=g).to(torch.bfloat16),
             torch.randn(B, H, T, D, generator=g).to(torch.bfloat16)) for _ in range(steps)]


def _block_step(prefix, steps, rows, topk, scale):
    """step 0 + the sub-steps over the compact cache, as bench.py's Workload.block_step."""
    from maskahead_b200.hotpath import compact_attention, fast_step0

    q0, kc0, vc0 = (t.to(DEV) for t in steps[0])
    res = fast_step0(q0, prefix, kc0, vc0, query_indices=rows, topk=topk, value_aware=True, scaling=scale,
                     gather=True)
    subs = [compact_attention(q.to(DEV), res.compact, None, kc.to(DEV), vc.to(DEV), scaling=scale)
            for q, kc, vc in steps[1:]]
    torch.cuda.synchronize()
    return res, subs


def _check_against_oracle(res, subs, steps, k, v, rows, topk, scale, b=None):
    """Every product of one sequence's block-step (b: its batch row) against the oracle."""
    sl = slice(None) if b is None else slice(b, b + 1)
    n = k.shape[2]
    q0, kc0, vc0 = (t[sl] for t in steps[0])
    imp = oracle.selector_importance(q0, k, query_indices=rows, scale=scale)
    mass = res.mass[sl].cpu()
    np.testing.assert_allclose(mass[..., :n].numpy(), imp.numpy(), rtol=2e-5, atol=1e-9)
    assert (mass[..., n:] == 0).all(), "slots past the sequence carry no mass"
    vs = oracle.rescore_by_value(imp, v)
    np.testing.assert_allclose(res.score[sl].cpu()[..., :n].numpy(), vs.numpy(), rtol=5e-5, atol=1e-9)
    want_idx, _ = oracle.topk_sorted(vs, topk)
    idx = res.indices[sl].cpu()
    band_equal(idx.numpy(), want_idx.numpy(), vs.numpy(), topk)
    assert (np.diff(idx.numpy(), axis=-1) > 0).all(), "read set must be ascending"
    assert int(idx.max()) < n, "a read set never reaches past its sequence"
    want_out = oracle.dense_attention(q0, k, v, kc0, vc0, scale=scale)
    np.testing.assert_allclose(res.out[sl].float().cpu().numpy(), want_out.float().numpy(), rtol=RTOL, atol=ATOL)
    # the compact cache holds the read set's rows exactly
    ck = oracle.gather_per_kv_head(k, idx)
    cv = oracle.gather_per_kv_head(v, idx)
    assert torch.equal(res.compact.kf[sl].cpu(), ck.to(torch.bfloat16))
    assert torch.equal(res.compact.vf[sl].cpu(), cv.to(torch.bfloat16))
    for got, (q, kc, vc) in zip(subs, steps[1:]):
        q, kc, vc = q[sl], kc[sl], vc[sl]
        want = oracle.sdpa_compact(q.float(), torch.cat([ck, kc], 2).float(), torch.cat([cv, vc], 2).float())
        np.testing.assert_allclose(got[sl].float().cpu().numpy(), want.numpy(), rtol=RTOL, atol=ATOL)
    return imp, vs


@pytest.mark.parametrize("name", ["cfg2_layer", "cfg3_layer"])
def test_cfg2_cfg3_layer_block_step(name):
    """cfg2 / cfg3 one layer: the composed step against the reference's fixture and the
    oracle; the first sub-step repeats step 0's inputs, so it must equal the reference's
    sdpa_compact over the reference's read set."""
    g = dict(np.load(GOLDEN / f"{name}.npz"))
    case, k, v, extra = load_case(name)
    spec = case["spec"]
    D, T, topk = spec["D"], spec["T"], int(g["topk"])
    scale = D ** -0.5
    rows = case["rows"]
    first = (case["query"], case["current_key"], case["current_value"])
    steps = [first, first] + _substep_inputs(spec["seed"] + 1, 1, spec["Hq"], spec["H"], T, D, 2)
    res, subs = _block_step(device_prefix(case, k, v, extra), steps, rows, topk, scale)
    # the reference's own outputs
    np.testing.assert_allclose(res.mass.cpu().numpy(), g["importance"], rtol=2e-5, atol=1e-9)
    np.testing.assert_allclose(res.score.cpu().numpy(), g["value_score"], rtol=5e-5, atol=1e-9)
    rows_cmp, flips = band_equal(res.indices.cpu().numpy(), g["value_indices"], g["value_score"], topk)
    assert rows_cmp == spec["H"]
    np.testing.assert_allclose(res.out.float().cpu().numpy(), g["dense_out"], rtol=RTOL, atol=ATOL)
    if flips == 0:
        np.testing.assert_allclose(subs[0].float().cpu().numpy(), g["compact_out"], rtol=RTOL, atol=ATOL)
    _check_against_oracle(res, subs, steps, k, v, rows, topk, scale)


def _survivor_band(keep, want, score, pos, capacity, window, sinks):
    """Retained sets equal, except slots whose score lies within 1e-5 (relative) of the
    (capacity - window - sinks)-th score among the entries outside the window and sinks."""
    live = pos.shape[-1]
    for i in range(keep.shape[0]):
        a, b = set(keep[i].tolist()), set(want[i].tolist())
        if a == b:
            continue
        p = pos[i]
        recent = set(np.argsort(p, kind="stable")[live - window:].tolist())
        rest = [j for j in range(live) if j not in recent and p[j] >= sinks]
        n_sink = int((p < sinks).sum())
        r = capacity - window - n_sink
        kth = np.sort(score[i][rest])[::-1][r - 1]
        band = 1e-5 * max(abs(float(kth)), 1e-30)
        for j in a ^ b:
            assert abs(float(score[i][j]) - float(kth)) <= band, f"lane {i}: slot {j} differs outside the band"


def test_cfg4_layer_block_step_and_retention():
    """cfg4 one layer (one GPU holds all 8 KV heads): block-step, then the retention pass --
    the probe of two lookahead blocks, a = a_step0 + a_probe, the value score and the
    survivors at capacity 8192 (eviction.py:364-409; session.py:1985-2034)."""
    from maskahead_b200.hotpath import lookahead_survivors, probe_attention, value_score

    B, Hq, H, D, T, n, topk, C, W, sinks = 1, 32, 8, 128, 32, 65536, 4096, 8192, 64, 4
    scale = D ** -0.5
    gen = torch.Generator().manual_seed(404)
    k = torch.randn(B, H, n, D, generator=gen).to(torch.bfloat16)
    v = torch.randn(B, H, n, D, generator=gen).to(torch.bfloat16)
    steps = _substep_inputs(405, B, Hq, H, T, D, 4)
    rows = list(range(T))
    from maskahead_b200.layouts import Prefix

    prefix = Prefix.dense(k.to(DEV), v.to(DEV))
    res, subs = _block_step(prefix, steps, rows, topk, scale)
    imp, _ = _check_against_oracle(res, subs, steps, k, v, rows, topk, scale)

    # the probe forward: [block | 2 probe blocks] block-causal over [prefix | itself]
    tp = T * 3
    qp = torch.randn(B, Hq, tp, D, generator=gen).to(torch.bfloat16)
    kcp = torch.randn(B, H, tp, D, generator=gen).to(torch.bfloat16)
    vcp = torch.randn(B, H, tp, D, generator=gen).to(torch.bfloat16)
    prow = torch.arange(T, tp, dtype=torch.int32, device=DEV)
    pout, pmass = probe_attention(qp.to(DEV), prefix, kcp.to(DEV), vcp.to(DEV), block_size=T, scaling=scale,
                                  probe_rows=prow)
    torch.cuda.synchronize()
    want_pout, (mp, lp, _) = oracle.prefix_attention(qp, k, v, kcp, vcp, scale=scale, causal_block=T, q_pos0=0,
                                                     c_pos0=0)
    np.testing.assert_allclose(pout.float().cpu().numpy(), want_pout.float().numpy(), rtol=RTOL, atol=ATOL)
    want_pmass = oracle.prefix_mass(qp, k, mp, lp, list(range(T, tp)), scale=scale) * 2
    np.testing.assert_allclose(pmass.cpu().numpy(), want_pmass.numpy(), rtol=1e-4, atol=1e-9)

    a = res.mass + pmass
    score = value_score(a, prefix.vf)
    pos = torch.arange(n, dtype=torch.int32).expand(1, B, H, n).contiguous()
    keep = lookahead_survivors(pos.to(DEV), score.unsqueeze(0), C, recent_window=W, sink_tokens=sinks)
    torch.cuda.synchronize()
    want_score = oracle.lookahead_score(imp, want_pmass, v)
    np.testing.assert_allclose(score.cpu().numpy(), want_score.numpy(), rtol=2e-4, atol=1e-9)
    # the survivors kernel on the device's scores: bit-exact with the oracle's selection
    got = keep.cpu()
    same = oracle.survivors_lookahead(pos, score.unsqueeze(0).cpu(), C, recent_window=W, sink_tokens=sinks)
    assert torch.equal(got, same)
    # and against the oracle's own scores, outside the tie band
    want = oracle.survivors_lookahead(pos, want_score.unsqueeze(0), C, recent_window=W, sink_tokens=sinks)
    _survivor_band(got.reshape(-1, C).numpy(), want.reshape(-1, C).numpy(), want_score.reshape(-1, n).numpy(),
                   pos.reshape(-1, n).numpy(), C, W, sinks)


@pytest.mark.parametrize("probe_blocks,Hq,H", [(1, 28, 4), (2, 32, 8)], ids=["cfg2_probe1", "cfg4_probe2"])
def test_merged_probe_step0(probe_blocks, Hq, H):
    """lookahead_merge: step 0 over [block | probe blocks] in one launch, block-causal. The
    block's rows select as usual (their keys: the block only), the probe rows' prefix mass
    times the probe blocks, and the outputs of every row against the oracle's
    prefix_attention(causal_block=32) + prefix_mass; the probe mass equals the separate
    probe pass's (the same attention launch)."""
    from maskahead_b200.hotpath import fast_step0, probe_attention
    from maskahead_b200.layouts import Prefix

    B, D, T, n, topk = 1, 128, 32, 8192, 1024
    tp = T * (1 + probe_blocks)
    scale = D ** -0.5
    gen = torch.Generator().manual_seed(808 + probe_blocks)
    k = torch.randn(B, H, n, D, generator=gen).to(torch.bfloat16)
    v = torch.randn(B, H, n, D, generator=gen).to(torch.bfloat16)
    q = torch.randn(B, Hq, tp, D, generator=gen).to(torch.bfloat16)
    kc = torch.randn(B, H, tp, D, generator=gen).to(torch.bfloat16)
    vc = torch.randn(B, H, tp, D, generator=gen).to(torch.bfloat16)
    prefix = Prefix.dense(k.to(DEV), v.to(DEV))
    rows = list(range(T))
    res = fast_step0(q.to(DEV), prefix, kc.to(DEV), vc.to(DEV), query_indices=rows, topk=topk, scaling=scale,
                     probe_blocks=probe_blocks, block_size=T)
    _, sep = probe_attention(q.to(DEV), prefix, kc.to(DEV), vc.to(DEV), block_size=T, scaling=scale)
    torch.cuda.synchronize()
    want, (mp, lp, _) = oracle.prefix_attention(q, k, v, kc, vc, scale=scale, causal_block=T, q_pos0=0, c_pos0=0)
    np.testing.assert_allclose(res.out.float().cpu().numpy(), want.float().numpy(), rtol=RTOL, atol=ATOL)
    imp = oracle.prefix_mass(q, k, mp, lp, rows, scale=scale)
    np.testing.assert_allclose(res.mass.cpu().numpy(), imp.numpy(), rtol=2e-5, atol=1e-9)
    vs = oracle.rescore_by_value(imp, v)
    np.testing.assert_allclose(res.score.cpu().numpy(), vs.numpy(), rtol=5e-5, atol=1e-9)
    want_idx, _ = oracle.topk_sorted(vs, topk)
    band_equal(res.indices.cpu().numpy(), want_idx.numpy(), vs.numpy(), topk)
    pm = oracle.prefix_mass(q, k, mp, lp, list(range(T, tp)), scale=scale) * probe_blocks
    np.testing.assert_allclose(res.probe_mass.cpu().numpy(), pm.numpy(), rtol=1e-4, atol=1e-9)
    assert torch.equal(res.probe_mass, sep), "the merged probe mass is the separate pass's"


def _paged_k4v4_batch(lens, H, D, page, seed):
    """Sequences quantized on the CPU by the oracle (token-mode keys with their own divisor,
    1% of the key channels x8 as outliers), their payloads scattered into a shuffled pool of
    pages; the oracle's dequantized K/V per sequence."""
    from maskahead_b200.layouts import Prefix

    gen = torch.Generator().manual_seed(seed)
    need = [(n + page - 1) // page for n in lens]
    P = sum(need) + 3                                   # spare pages stay unused
    order = torch.randperm(P, generator=gen)
    table = torch.full((len(lens), max(need)), -1, dtype=torch.int32)
    pool = {"kq": torch.zeros(P, H, page, D // 32, 16, dtype=torch.uint8),
            "ks": torch.zeros(P, H, page, D // 32, dtype=torch.float16),
            "kz": torch.zeros(P, H, page, D // 32, dtype=torch.float16)}
    pool.update({"v" + key[1]: t.clone() for key, t in pool.items()})
    kchans, ref_k, ref_v = [], [], []
    nxt = 0
    for b, n in enumerate(lens):
        k = torch.randn(1, H, n, D, generator=gen)
        for h in range(H):
            k[0, h, :, torch.randperm(D, generator=gen)[: max(1, D // 100)]] *= 8.0
        k = k.to(torch.bfloat16)
        v = torch.randn(1, H, n, D, generator=gen).to(torch.bfloat16)
        kchan = oracle.key_channel_divisor(k)
        kq, ks, kz = oracle.quantize_keys_token(k, kchan)
        vq, vs, vz = oracle.quantize_values(v)
        kchans.append(kchan[0])
        ref_k.append(oracle.dequantize_keys_token(kq, ks, kz, kchan))
        ref_v.append(oracle.dequantize_values(vq, vs, vz))
        src = {"kq": kq, "ks": ks, "kz": kz, "vq": vq, "vs": vs, "vz": vz}
        for p in range(need[b]):
            slot = int(order[nxt])
            nxt += 1
            table[b, p] = slot
            lo, hi = p * page, min(n, (p + 1) * page)
            for key, t in src.items():
                pool[key][slot, :, : hi - lo] = t[0, :, lo:hi]
    d = {key: t.to(DEV) for key, t in pool.items()}
    prefix = Prefix(kq=d["kq"], ks=d["ks"], kz=d["kz"], vq=d["vq"], vs=d["vs"], vz=d["vz"], nq=max(lens), kb=4, vb=4,
                    kg=32, vg=32, kmode=1, kch=torch.stack(kchans).to(DEV), pages=table.to(DEV), page_size=page,
                    lens=torch.tensor(lens, dtype=torch.int32, device=DEV))
    return prefix, ref_k, ref_v


def test_cfg5_paged_slice_block_step():
    """cfg5 slice: 16 sequences of the cfg3 shape, lengths U[4096, 16384], k4v4 token mode
    in a shuffled pool of 64-slot pages; the step-0 grid spans several waves, so the splits
    merge in the separate combine launch."""
    B, Hq, H, D, T, topk, page = 16, 28, 4, 128, 32, 1024, 64
    scale = D ** -0.5
    gen = torch.Generator().manual_seed(505)
    lens = torch.randint(4096, 16385, (B,), generator=gen).tolist()
    lens[0], lens[1] = 16384, 4096                      # both ends of the range
    prefix, ref_k, ref_v = _paged_k4v4_batch(lens, H, D, page, 506)
    steps = _substep_inputs(507, B, Hq, H, T, D, 4)
    rows = list(range(T))
    res, subs = _block_step(prefix, steps, rows, topk, scale)
    for b in range(B):
        _check_against_oracle(res, subs, steps, ref_k[b], ref_v[b], rows, topk, scale, b=b)


def test_dense_layers_bypass_selection():
    """Dense-prefix layers and a budget covering the prefix (session.py:456-467): step 0
    attends without selecting (fast_step0(select=False)) and every sub-step attends the
    whole prefix (fast_attend, session.py:1378-1393); with mass rows fast_attend also gives
    their prefix mass."""
    from maskahead_b200.hotpath import dense_required, fast_attend, fast_step0
    from maskahead_b200.layouts import Prefix

    assert dense_required(0, dense_prefix_layers=2, old_cache_len=8192, topk=1024, query_indices=[0])
    assert dense_required(5, dense_prefix_layers=2, old_cache_len=900, topk=1024, query_indices=[0])
    assert not dense_required(5, dense_prefix_layers=2, old_cache_len=8192, topk=1024, query_indices=[0])
    assert not dense_required(5, dense_prefix_layers=2, old_cache_len=900, topk=1024, query_indices=[0],
                              eviction=True, live_cache_len=900)
    assert dense_required(5, dense_prefix_layers=2, old_cache_len=8192, topk=1024, query_indices=[])

    B, Hq, H, D, T, n = 1, 28, 4, 128, 32, 900
    scale = D ** -0.5
    gen = torch.Generator().manual_seed(606)
    k = torch.randn(B, H, n, D, generator=gen).to(torch.bfloat16)
    v = torch.randn(B, H, n, D, generator=gen).to(torch.bfloat16)
    steps = _substep_inputs(607, B, Hq, H, T, D, 2)
    prefix = Prefix.dense(k.to(DEV), v.to(DEV))
    q0, kc0, vc0 = (t.to(DEV) for t in steps[0])
    res = fast_step0(q0, prefix, kc0, vc0, query_indices=list(range(T)), topk=1024, scaling=scale, select=False)
    q1, kc1, vc1 = steps[1]
    out1, mass1 = fast_attend(q1.to(DEV), prefix, kc1.to(DEV), vc1.to(DEV), scaling=scale,
                              mass_rows=list(range(T)))
    torch.cuda.synchronize()
    assert res.indices is None and res.mass is None and res.compact is None
    want0 = oracle.dense_attention(*steps[0][:1], k, v, *steps[0][1:], scale=scale)
    np.testing.assert_allclose(res.out.float().cpu().numpy(), want0.float().numpy(), rtol=RTOL, atol=ATOL)
    want1 = oracle.dense_attention(q1, k, v, kc1, vc1, scale=scale)
    np.testing.assert_allclose(out1.float().cpu().numpy(), want1.float().numpy(), rtol=RTOL, atol=ATOL)
    imp = oracle.selector_importance(q1, k, query_indices=list(range(T)), scale=scale)
    np.testing.assert_allclose(mass1.cpu().numpy(), imp.numpy(), rtol=2e-5, atol=1e-9)
    # a covering budget that still selects (eviction on): every slot, ascending, and the
    # sub-step over that compact cache equals the dense attention
    sel = fast_step0(q0, prefix, kc0, vc0, query_indices=list(range(T)), topk=1024, scaling=scale, gather=True)
    torch.cuda.synchronize()
    assert torch.equal(sel.indices.cpu(), torch.arange(n).expand(B, H, n))
    out_c, _ = fast_attend(q1.to(DEV), sel.compact, kc1.to(DEV), vc1.to(DEV), scaling=scale)
    torch.cuda.synchronize()
    np.testing.assert_allclose(out_c.float().cpu().numpy(), want1.float().numpy(), rtol=RTOL, atol=ATOL)
