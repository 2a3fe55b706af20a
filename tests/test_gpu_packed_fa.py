"""The pipelined kernels reading token-mode k4v4 prefixes in place (unpack=False; the
default attention route unpacks first, which measured faster on B200).

The producer warps of attn_partial_fa and prefix_mass_fa dequantize the packed rows into
the same bf16 tiles an unpack followed by TMA loads would give them (fma(code, scale,
zero) in fp32, times the key divisor, one rounding to bf16), under the same split plan, so
every output -- attention rows, prefix statistics, mass, value score -- must equal the
unpacked path's bit for bit. Cases: contiguous prefixes (one and several row tiles, one
and several splits, a partial last tile), a ragged batch in a shuffled pool of 64-slot
pages with page-straddling tiles, the block-causal probe (T = 96), the value-score pass
with given a_j, and a prefix the kernels cannot read in place (a dense tail) which is
unpacked first. The packed payloads come from the oracle's quantizers on the CPU and the
oracle checks the step on the contiguous case.
"""

from __future__ import annotations

import numpy as np
import pytest
import torch

import oracle

pytestmark = pytest.mark.gpu

DEV = "cuda"


def _packed(B, H, n, D=128, seed=0, lens=None, page=None):
    """A token-mode prefix quantized by the oracle (per sequence divisor, 1% of the key
    channels x8), contiguous or in a shuffled page pool; with the oracle's bf16 K/V."""
    from maskahead_b200.layouts import Prefix

    g = torch.Generator().manual_seed(seed)
    lens = lens or [n] * B
    k = torch.randn(B, H, n, D, generator=g)
    for b in range(B):
        for h in range(H):
            k[b, h, :, torch.randperm(D, generator=g)[:2]] *= 8.0
    k = k.to(torch.bfloat16)
    v = torch.randn(B, H, n, D, generator=g).to(torch.bfloat16)
    kchan = torch.stack([oracle.key_channel_divisor(k[b : b + 1, :, : lens[b]])[0] for b in range(B)])
    kq, ks, kz = oracle.quantize_keys_token(k, kchan)
    vq, vs, vz = oracle.quantize_values(v)
    ref_k = oracle.dequantize_keys_token(kq, ks, kz, kchan)
    ref_v = oracle.dequantize_values(vq, vs, vz)
    arrays = dict(kq=kq, ks=ks, kz=kz, vq=vq, vs=vs, vz=vz)
    lens_t = torch.tensor(lens, dtype=torch.int32, device=DEV) if any(x != n for x in lens) else None
    if page is None:
        d = {key: t.to(DEV) for key, t in arrays.items()}
        pre = Prefix(**d, nq=n, kb=4, vb=4, kg=32, vg=32, kmode=1, kch=kchan.to(DEV), lens=lens_t)
        return pre, ref_k, ref_v
    need = [(x + page - 1) // page for x in lens]
    P = sum(need) + 2
    order = torch.randperm(P, generator=g)
    table = torch.full((B, max(need)), -1, dtype=torch.int32)
    pool = {key: torch.zeros((P, H, page) + tuple(t.shape[3:]), dtype=t.dtype) for key, t in arrays.items()}
    at = 0
    for b in range(B):
        for p in range(need[b]):
            slot = int(order[at])
            at += 1
            table[b, p] = slot
            lo, hi = p * page, min(lens[b], (p + 1) * page)
            for key, t in arrays.items():
                pool[key][slot, :, : hi - lo] = t[b, :, lo:hi]
    d = {key: t.to(DEV) for key, t in pool.items()}
    pre = Prefix(**d, nq=n, kb=4, vb=4, kg=32, vg=32, kmode=1, kch=kchan.to(DEV), pages=table.to(DEV), page_size=page,
                 lens=torch.tensor(lens, dtype=torch.int32, device=DEV))
    return pre, ref_k, ref_v


def _inputs(B, Hq, H, T, D=128, seed=1):
    g = torch.Generator().manual_seed(seed)
    q = torch.randn(B, Hq, T, D, generator=g).to(torch.bfloat16).to(DEV)
    kc = torch.randn(B, H, T, D, generator=g).to(torch.bfloat16).to(DEV)
    vc = torch.randn(B, H, T, D, generator=g).to(torch.bfloat16).to(DEV)
    return q, kc, vc


def _read_in_place(pre, B, H):
    from maskahead_b200._lib import lib
    from maskahead_b200.layouts import kv_descriptor

    desc = kv_descriptor(pre, batch=B, heads=H, head_dim=128)
    return lib().ma_kv_read_in_place(desc.kv, 128) == 1


def _same(a, b):
    assert torch.equal(a, b), f"max |diff| {(a.float() - b.float()).abs().max().item()}"


CASES = [
    dict(B=1, Hq=28, H=4, n=320, T=32),             # one split, a partial last tile
    dict(B=1, Hq=28, H=4, n=8192, T=32),            # cfg3's layer: 2 row tiles x 17 splits
    dict(B=1, Hq=32, H=8, n=20480, T=32),           # R = 128: one row tile, long splits
    dict(B=3, Hq=8, H=2, n=5000, T=32, lens=[5000, 3001, 777], page=64),   # ragged, paged
    dict(B=2, Hq=8, H=2, n=2000, T=96, causal=32),  # the probe shape, block-causal
]


@pytest.mark.parametrize("which", [2, 3], ids=["one_m_tile", "m_tile_pairs"])
@pytest.mark.parametrize("case", CASES, ids=[f"n{c['n']}_T{c['T']}{'_paged' if 'page' in c else ''}" for c in CASES])
def test_packed_attention_and_scores_equal_the_unpacked_path(case, which):
    """With one M tile per CTA and with pairs of M tiles (ma_set_attention_kernel 2, 3)."""
    from maskahead_b200._lib import lib

    prev = lib().ma_set_attention_kernel(which)
    try:
        _packed_equals_unpacked(case)
    finally:
        lib().ma_set_attention_kernel(prev)


def _packed_equals_unpacked(case):
    from maskahead_b200.hotpath import unpacked_prefix
    from maskahead_b200.kernels import prefix_scores, splitk_attention

    B, Hq, H, n, T = (case[x] for x in ("B", "Hq", "H", "n", "T"))
    cb = case.get("causal", 0)
    pre, _, _ = _packed(B, H, n, seed=n, lens=case.get("lens"), page=case.get("page"))
    assert _read_in_place(pre, B, H)
    q, kc, vc = _inputs(B, Hq, H, T, seed=n + 1)
    rows = list(range(T)) if cb == 0 else list(range(32, T))
    out_p, st_p = splitk_attention(q, pre, kc, vc, causal_block=cb, want_prefix=True)
    mass_p, score_p = prefix_scores(q, pre, st_p, rows, value=True)
    un = unpacked_prefix(pre, B, H, 128)
    un = type(un)(**{s: getattr(un, s) for s in type(un).__slots__})   # hold the scratch's views
    kf, vf = un.kf.clone(), un.vf.clone()
    un.kf, un.vf = kf, vf
    out_u, st_u = splitk_attention(q, un, kc, vc, causal_block=cb, want_prefix=True)
    mass_u, score_u = prefix_scores(q, un, st_u, rows, value=True)
    torch.cuda.synchronize()
    _same(out_p, out_u)
    for a, b in zip(st_p[:3], st_u[:3]):
        _same(a, b)
    _same(mass_p, mass_u)
    _same(score_p, score_u)


@pytest.mark.parametrize("unpack", [None, False], ids=["unpacked_first", "in_place"])
def test_packed_step0_matches_the_oracle(unpack):
    """fast_step0 over a packed prefix, unpacked first (the default) or read in place by
    the producer warps (unpack=False)."""
    from maskahead_b200.hotpath import fast_step0

    B, Hq, H, n, T, topk = 1, 28, 4, 4096, 32, 512
    pre, k, v = _packed(B, H, n, seed=99)
    q, kc, vc = _inputs(B, Hq, H, T, seed=100)
    res = fast_step0(q, pre, kc, vc, query_indices=list(range(T)), topk=topk, scaling=128 ** -0.5, gather=True,
                     unpack=unpack)
    torch.cuda.synchronize()
    qc, kcc, vcc = q.cpu(), kc.cpu(), vc.cpu()
    imp = oracle.selector_importance(qc, k, query_indices=list(range(T)), scale=128 ** -0.5)
    np.testing.assert_allclose(res.mass.cpu().numpy(), imp.numpy(), rtol=2e-5, atol=1e-9)
    vs = oracle.rescore_by_value(imp, v)
    np.testing.assert_allclose(res.score.cpu().numpy(), vs.numpy(), rtol=5e-5, atol=1e-9)
    want = oracle.dense_attention(qc, k, v, kcc, vcc, scale=128 ** -0.5)
    np.testing.assert_allclose(res.out.float().cpu().numpy(), want.float().numpy(), rtol=2e-2, atol=2e-2)
    idx = res.indices.cpu()
    assert torch.equal(res.compact.kf.cpu(), oracle.gather_per_kv_head(k, idx))
    assert torch.equal(res.compact.vf.cpu(), oracle.gather_per_kv_head(v, idx))


@pytest.mark.parametrize("n", [3000, 40000])
def test_packed_value_score_with_given_mass_equals_unpacked(n):
    """The retention pass's value score (given a_j: only V is read) in place and after an
    unpack: the same numbers (40000 slots: more tiles per CTA than its slots hold, so the
    score pass reads the packed rows directly)."""
    from maskahead_b200.hotpath import value_score_prefix

    pre, _, v = _packed(1, 4, n, seed=n + 5)
    g = torch.Generator().manual_seed(n)
    a = torch.rand(1, 4, n, generator=g).to(DEV)
    got = value_score_prefix(a, pre)
    want = value_score_prefix(a, pre, unpack=True)
    torch.cuda.synchronize()
    _same(got, want)
    np.testing.assert_allclose(got.cpu().numpy(), oracle.value_score(a.cpu(), v).numpy(), rtol=5e-5, atol=1e-9)


def test_prefix_with_a_dense_tail_is_unpacked_first():
    """A packed prefix with a bf16 tail is not read in place (ma_kv_read_in_place = 0):
    fast_step0 unpacks it and still matches the oracle."""
    from maskahead_b200.hotpath import fast_step0
    from maskahead_b200.layouts import Prefix

    B, Hq, H, nq, nf, T = 1, 8, 2, 512, 40, 32
    pre, k, v = _packed(B, H, nq, seed=7)
    g = torch.Generator().manual_seed(8)
    kt = torch.randn(B, H, nf, 128, generator=g).to(torch.bfloat16)
    vt = torch.randn(B, H, nf, 128, generator=g).to(torch.bfloat16)
    tail = Prefix(kq=pre.kq, ks=pre.ks, kz=pre.kz, vq=pre.vq, vs=pre.vs, vz=pre.vz, kf=kt.to(DEV), vf=vt.to(DEV),
                  nq=nq, nf=nf, kb=4, vb=4, kg=32, vg=32, kmode=1, kch=pre.kch)
    assert not _read_in_place(tail, B, H)
    q, kc, vc = _inputs(B, Hq, H, T, seed=9)
    res = fast_step0(q, tail, kc, vc, query_indices=list(range(T)), topk=64, scaling=128 ** -0.5)
    torch.cuda.synchronize()
    kk, vv = torch.cat([k, kt], 2), torch.cat([v, vt], 2)
    imp = oracle.selector_importance(q.cpu(), kk, query_indices=list(range(T)), scale=128 ** -0.5)
    np.testing.assert_allclose(res.mass.cpu().numpy(), imp.numpy(), rtol=2e-5, atol=1e-9)
    want = oracle.dense_attention(q.cpu(), kk, vv, kc.cpu(), vc.cpu(), scale=128 ** -0.5)
    np.testing.assert_allclose(res.out.float().cpu().numpy(), want.float().numpy(), rtol=2e-2, atol=2e-2)
