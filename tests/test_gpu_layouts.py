"""GPU parity of the device quantizer and of the paged, ragged cache layout.

* The quantize-on-append kernels must reproduce the reference's own k4v4 payloads,
  fp16 scales/zeros and token-mode divisor bit for bit (fixtures made by running the
  reference's quantizers, tests/golden/make_golden.py).
* A paged cache (pages of 64 slots, shuffled in a pool, a page table per sequence) with
  ragged lengths must give, per sequence, what the oracle gives on that sequence's
  contiguous prefix: attention outputs within the bf16 bar, mass and value score to
  fp32 rounding, read sets bit-exact up to fp32 ties; slots past a sequence's length
  are dead (mass 0, never selected).
"""

from __future__ import annotations

from pathlib import Path

import numpy as np
import pytest
import torch

import oracle
from gen_inputs import make_case
from gpu_cases import band_equal

pytestmark = pytest.mark.gpu

GOLDEN = Path(__file__).resolve().parent / "golden"
DEV = "cuda"


@pytest.mark.parametrize("name", ["small_k4v4_token", "small_k4v4_channel"])
def test_quantizer_matches_reference_payloads(name):
    from maskahead_b200.layouts import key_divisor, quantize_keys_channel, quantize_tokens

    g = dict(np.load(GOLDEN / f"{name}.npz"))
    case = make_case(name)
    kf, vf = case["key_fp"].to(DEV), case["value_fp"].to(DEV)
    vq, vs, vz = quantize_tokens(vf)
    if case["spec"]["packed"] == "token":
        kchan = key_divisor(kf)
        np.testing.assert_array_equal(kchan.cpu().numpy(), g["packed_kchan"])
        kq, ks, kz = quantize_tokens(kf, kchan)
    else:
        kq, ks, kz = quantize_keys_channel(kf)
    torch.cuda.synchronize()
    for got, key in ((kq, "kq"), (ks, "ks"), (kz, "kz"), (vq, "vq"), (vs, "vs"), (vz, "vz")):
        a = got.cpu()
        if a.dtype == torch.float16:
            a = a.view(torch.int16)
        np.testing.assert_array_equal(a.numpy(), g[f"packed_{key}"], err_msg=key)


def test_quantizer_float32_matches_oracle():
    """fp32 inputs quantize in fp32 (no intermediate rounding), as the oracle does."""
    from maskahead_b200.layouts import quantize_keys_channel, quantize_tokens

    gen = torch.Generator().manual_seed(5)
    x = torch.randn(2, 3, 64, 128, generator=gen) * 3.0
    x[0, 0, 5] = 0.25   # a constant group: scale clamps at 1e-8
    pq, ps, pz = quantize_tokens(x.to(DEV))
    wq, ws, wz = oracle.quantize_values(x)
    np.testing.assert_array_equal(pq.cpu().numpy(), wq.numpy())
    np.testing.assert_array_equal(ps.cpu().view(torch.int16).numpy(), ws.view(torch.int16).numpy())
    np.testing.assert_array_equal(pz.cpu().view(torch.int16).numpy(), wz.view(torch.int16).numpy())
    cq, cs, cz = quantize_keys_channel(x.to(DEV))
    wq, ws, wz = oracle.quantize_keys(x)
    np.testing.assert_array_equal(cq.cpu().numpy(), wq.numpy())
    np.testing.assert_array_equal(cs.cpu().view(torch.int16).numpy(), ws.view(torch.int16).numpy())


def _paged_batch(mode: str, lens=(448, 320, 200), H=2, Hq=8, D=128, T=32, page=64, seed=21):
    """Per-sequence contiguous inputs and the same data in a shuffled page pool."""
    from maskahead_b200.layouts import Prefix, key_divisor, quantize_tokens

    gen = torch.Generator().manual_seed(seed)
    B = len(lens)
    cap = max(lens)
    max_pages = (cap + page - 1) // page
    need = [(n + page - 1) // page for n in lens]
    P = sum(need) + 2                                   # two spare pages stay unused
    order = torch.randperm(P, generator=gen)
    table = torch.full((B, max_pages), -1, dtype=torch.int32)
    seq_k, seq_v = [], []
    pool_k = torch.zeros(P, H, page, D, dtype=torch.bfloat16)
    pool_v = torch.zeros_like(pool_k)
    owner = torch.zeros(P, dtype=torch.int64)
    nxt = 0
    for b, n in enumerate(lens):
        k = torch.randn(H, n, D, generator=gen).to(torch.bfloat16)
        v = torch.randn(H, n, D, generator=gen).to(torch.bfloat16)
        seq_k.append(k)
        seq_v.append(v)
        for p in range(need[b]):
            slot = int(order[nxt])
            nxt += 1
            table[b, p] = slot
            owner[slot] = b
            lo, hi = p * page, min(n, (p + 1) * page)
            pool_k[slot, :, : hi - lo] = k[:, lo:hi]
            pool_v[slot, :, : hi - lo] = v[:, lo:hi]
    q = torch.randn(B, Hq, T, D, generator=gen).to(torch.bfloat16)
    kc = torch.randn(B, H, T, D, generator=gen).to(torch.bfloat16)
    vc = torch.randn(B, H, T, D, generator=gen).to(torch.bfloat16)
    lens_t = torch.tensor(lens, dtype=torch.int32)
    if mode == "dense":
        prefix = Prefix(kf=pool_k.to(DEV), vf=pool_v.to(DEV), nf=cap, pages=table.to(DEV), page_size=page,
                        lens=lens_t.to(DEV))
        ref_k, ref_v = seq_k, seq_v
    else:
        # token-mode k4v4: the divisor of each sequence (over its live slots), pages
        # quantized in place with their owner's divisor
        kchan = torch.stack([key_divisor(k.unsqueeze(0).to(DEV))[0] for k in seq_k])      # [B, H, D]
        vq, vs, vz = quantize_tokens(pool_v.to(DEV))
        kq, ks, kz = quantize_tokens(pool_k.to(DEV), kchan[owner.to(DEV)])
        prefix = Prefix(kq=kq, ks=ks, kz=kz, vq=vq, vs=vs, vz=vz, nq=cap, kb=4, vb=4, kg=32, vg=32, kmode=1,
                        kch=kchan, pages=table.to(DEV), page_size=page, lens=lens_t.to(DEV))
        ref_k, ref_v = [], []
        for b, n in enumerate(lens):
            pk = oracle.pages_to_contiguous(kq.cpu(), table[b], n, page)
            psk = oracle.pages_to_contiguous(ks.cpu(), table[b], n, page)
            pzk = oracle.pages_to_contiguous(kz.cpu(), table[b], n, page)
            pv = oracle.pages_to_contiguous(vq.cpu(), table[b], n, page)
            psv = oracle.pages_to_contiguous(vs.cpu(), table[b], n, page)
            pzv = oracle.pages_to_contiguous(vz.cpu(), table[b], n, page)
            ref_k.append(oracle.dequantize_keys_token(pk.unsqueeze(0), psk.unsqueeze(0), pzk.unsqueeze(0),
                                                      kchan[b : b + 1].cpu())[0])
            ref_v.append(oracle.dequantize_values(pv.unsqueeze(0), psv.unsqueeze(0), pzv.unsqueeze(0))[0])
    return dict(prefix=prefix, q=q, kc=kc, vc=vc, ref_k=ref_k, ref_v=ref_v, lens=lens, D=D, T=T)


@pytest.mark.parametrize("mode", ["dense", "k4v4_token"])
def test_paged_ragged_step0_and_substep(mode):
    from maskahead_b200.hotpath import compact_attention, fast_step0

    c = _paged_batch(mode)
    D, T, topk = c["D"], c["T"], 96
    rows = list(range(T))
    scale = D ** -0.5
    res = fast_step0(c["q"].to(DEV), c["prefix"], c["kc"].to(DEV), c["vc"].to(DEV), query_indices=rows,
                     topk=topk, value_aware=True, scaling=scale)
    sub = compact_attention(c["q"].to(DEV), c["prefix"], res.indices, c["kc"].to(DEV), c["vc"].to(DEV),
                            scaling=scale)
    torch.cuda.synchronize()
    mass, score, idx = res.mass.cpu(), res.score.cpu(), res.indices.cpu()
    for b, n in enumerate(c["lens"]):
        q, kc, vc = c["q"][b : b + 1], c["kc"][b : b + 1], c["vc"][b : b + 1]
        k, v = c["ref_k"][b].unsqueeze(0), c["ref_v"][b].unsqueeze(0)
        want_out = oracle.dense_attention(q, k, v, kc, vc, scale=scale)
        np.testing.assert_allclose(res.out[b : b + 1].float().cpu().numpy(), want_out.float().numpy(),
                                   rtol=2e-2, atol=2e-2)
        imp = oracle.selector_importance(q, k, query_indices=rows, scale=scale)
        np.testing.assert_allclose(mass[b, :, :n].numpy(), imp[0].numpy(), rtol=2e-5, atol=1e-9)
        assert (mass[b, :, n:] == 0).all(), "slots past the sequence length must carry no mass"
        vs = oracle.rescore_by_value(imp, v)
        np.testing.assert_allclose(score[b, :, :n].numpy(), vs[0].numpy(), rtol=5e-5, atol=1e-9)
        want_idx, _ = oracle.topk_sorted(vs, topk)
        band_equal(idx[b : b + 1].numpy(), want_idx.numpy(), vs.numpy(), topk)
        assert (idx[b] < n).all(), "a read set never reaches past its sequence"
        sel = idx[b : b + 1].to(torch.int64)
        sk = torch.cat([oracle.gather_per_kv_head(k, sel), kc], dim=2)
        sv = torch.cat([oracle.gather_per_kv_head(v, sel), vc], dim=2)
        want_sub = oracle.sdpa_compact(q.float(), sk.float(), sv.float())
        np.testing.assert_allclose(sub[b : b + 1].float().cpu().numpy(), want_sub.numpy(), rtol=2e-2, atol=2e-2)


def test_bad_page_entries_read_as_dead():
    """A page-table entry outside the pool never addresses memory: the slot is dead."""
    from maskahead_b200.hotpath import fast_step0

    c = _paged_batch("dense", lens=(128, 128), seed=3)
    pre = c["prefix"]
    table = pre.pages.clone()
    table[1, 1] = 10_000                                # sequence 1, slots 64..127
    pre.pages = table
    res = fast_step0(c["q"].to(DEV), pre, c["kc"].to(DEV), c["vc"].to(DEV), query_indices=list(range(32)),
                     topk=32, value_aware=True, scaling=128 ** -0.5)
    torch.cuda.synchronize()
    assert (res.mass[1, :, 64:128].cpu() == 0).all()
    assert (res.indices[1].cpu() < 64).all()
    assert torch.isfinite(res.out.float()).all()


def test_unpack_prefix_writes_the_live_slots_only():
    """ma_unpack_prefix (the step-0 unpack of a ragged batch): the slots below each
    sequence's length equal ma_gather_kv's whole-prefix dequantization, bit for bit, and the
    slots past it keep what the buffer held (a sentinel here); without lens every slot is
    written. The unpacked prefix then gives the same step 0 as the packed one."""
    from maskahead_b200._lib import i64, lib as get_lib
    from maskahead_b200.hotpath import unpacked_prefix
    from maskahead_b200.kernels.splitk import dequantize_prefix
    from maskahead_b200.layouts import kv_descriptor

    c = _paged_batch("k4v4_token", lens=(448, 320, 200))
    pre, lens = c["prefix"], c["lens"]
    B, H, D = len(lens), 2, c["D"]          # _paged_batch's default H
    n = max(lens)
    want_k, want_v = dequantize_prefix(pre, B, H, D)
    ko = torch.full((B, H, n, D), 7.0, dtype=torch.bfloat16, device=DEV)
    vo = torch.full_like(ko, -3.0)
    lib = get_lib()
    desc = kv_descriptor(pre, batch=B, heads=H, head_dim=D)
    rc = lib.ma_unpack_prefix(desc.kv, B, H, D, ko.data_ptr(), vo.data_ptr(), i64(*ko.stride()[:3]),
                              i64(*vo.stride()[:3]), torch.cuda.current_stream().cuda_stream)
    assert rc == 0
    torch.cuda.synchronize()
    for b, L in enumerate(lens):
        assert torch.equal(ko[b, :, :L].cpu(), want_k[b, :, :L].cpu())
        assert torch.equal(vo[b, :, :L].cpu(), want_v[b, :, :L].cpu())
        assert bool((ko[b, :, L:] == 7.0).all()) and bool((vo[b, :, L:] == -3.0).all())
    un = unpacked_prefix(pre, B, H, D)
    for b, L in enumerate(lens):
        assert torch.equal(un.kf[b, :, :L].cpu(), want_k[b, :, :L].cpu())
        assert torch.equal(un.vf[b, :, :L].cpu(), want_v[b, :, :L].cpu())


@pytest.mark.parametrize("live_only", [True, False], ids=["unpack_prefix", "dequantize_prefix"])
def test_long_batch_unpack_equals_the_per_sequence_unpack(live_only):
    """Above 2^20 slot-heads a token-mode batch is unpacked by the staged kernel (bulk-copied
    raw rows, all warps converting); each sequence unpacked alone takes the per-slot kernel.
    Both are the same dequantization: equal bit for bit below lens[b] (and zeros past it
    when every slot is written), on a ragged batch in a shuffled pool of 64-slot pages."""
    from maskahead_b200._lib import i64, lib as get_lib
    from maskahead_b200.kernels.splitk import dequantize_prefix
    from maskahead_b200.layouts import Prefix, key_divisor, kv_descriptor, quantize_tokens

    g = torch.Generator(device=DEV).manual_seed(5)
    B, H, D, page, n = 24, 4, 128, 64, 16384
    lens = torch.randint(4096, n + 1, (B,), generator=torch.Generator().manual_seed(6)).tolist()
    need = [(x + page - 1) // page for x in lens]
    P = sum(need) + 3
    order = torch.randperm(P, generator=torch.Generator().manual_seed(7))
    table = torch.full((B, n // page), -1, dtype=torch.int32)
    owner = torch.zeros(P, dtype=torch.int64)
    at = 0
    for b, m in enumerate(need):
        table[b, :m] = order[at:at + m].to(torch.int32)
        owner[order[at:at + m]] = b
        at += m
    kpool = torch.randn(P, H, page, D, generator=g, device=DEV).to(torch.bfloat16)
    vpool = torch.randn(P, H, page, D, generator=g, device=DEV).to(torch.bfloat16)
    kchan = torch.rand(B, H, D, generator=g, device=DEV) + 0.5
    kq, ks, kz = quantize_tokens(kpool, kchan[owner.to(DEV)])
    vq, vs, vz = quantize_tokens(vpool)
    arrays = dict(kq=kq, ks=ks, kz=kz, vq=vq, vs=vs, vz=vz, nq=n, kb=4, vb=4, kg=32, vg=32, kmode=1, page_size=page)
    lens_t = torch.tensor(lens, dtype=torch.int32, device=DEV)
    pre = Prefix(**arrays, kch=kchan, pages=table.to(DEV), lens=lens_t)
    lib = get_lib()

    def unpack(p, batch):
        if not live_only:
            return dequantize_prefix(p, batch, H, D)
        ko = torch.full((batch, H, n, D), 7.0, dtype=torch.bfloat16, device=DEV)
        vo = torch.full_like(ko, -3.0)
        desc = kv_descriptor(p, batch=batch, heads=H, head_dim=D)
        assert lib.ma_unpack_prefix(desc.kv, batch, H, D, ko.data_ptr(), vo.data_ptr(), i64(*ko.stride()[:3]),
                                    i64(*vo.stride()[:3]), torch.cuda.current_stream().cuda_stream) == 0
        return ko, vo

    got_k, got_v = unpack(pre, B)
    torch.cuda.synchronize()
    for b in range(0, B, 5):
        one = Prefix(**arrays, kch=kchan[b:b + 1], pages=table[b:b + 1].to(DEV), lens=lens_t[b:b + 1])
        want_k, want_v = unpack(one, 1)
        torch.cuda.synchronize()
        L = lens[b]
        assert torch.equal(got_k[b, :, :L], want_k[0, :, :L])
        assert torch.equal(got_v[b, :, :L], want_v[0, :, :L])
        if live_only:
            assert bool((got_k[b, :, L:] == 7.0).all()) and bool((got_v[b, :, L:] == -3.0).all())
        else:
            assert not bool(got_k[b, :, L:].any()) and not bool(got_v[b, :, L:].any())
