"""GPU parity of the cache compaction after an eviction (ma_compact_tokens).

* On the reference's own caches (fixtures recorded by running PackedKVCache.compact_tokens
  on a token-mode k4v4 cache and PackedKVCache.compact on a bf16 cache,
  tests/golden/make_golden.py) the device compaction must give the reference's arrays
  bit for bit, every layer in one call (the layer axis merged into the batch axis).
* On larger random caches it must equal the oracle's compaction bit for bit for any keep
  order, out-of-range keep entries (zero rows), strided sources and a destination with
  more slots than kept (slots past C untouched).
"""

from __future__ import annotations

from pathlib import Path

import numpy as np
import pytest
import torch

import oracle
from test_oracle_golden import load_compact

pytestmark = pytest.mark.gpu

DEV = "cuda"
GOLDEN = Path(__file__).resolve().parent / "golden"


def _merge_layers(t: torch.Tensor) -> torch.Tensor:
    """[L, B, H, ...] -> [L*B, H, ...] (the C ABI's batch axis covers every layer)."""
    return t.reshape(t.shape[0] * t.shape[1], *t.shape[2:])


def _bytes(t: torch.Tensor) -> torch.Tensor:
    return t.contiguous().view(torch.uint8)


def test_token_mode_matches_reference_compact_tokens():
    from maskahead_b200.layouts import Prefix, compact_tokens

    f = load_compact("compact_token")
    dev = {k: _merge_layers(v).to(DEV) for k, v in f.items()}
    n = dev["before_k_q"].shape[2]
    src = Prefix(kq=dev["before_k_q"], ks=dev["before_k_scale"], kz=dev["before_k_zero"],
                 vq=dev["before_v_q"], vs=dev["before_v_scale"], vz=dev["before_v_zero"], nq=n, kb=4, vb=4,
                 kmode=1, kch=dev["k_chan"])
    out = compact_tokens(src, dev["keep"])
    torch.cuda.synchronize()
    for ours, name in ((out.kq, "k_q"), (out.ks, "k_scale"), (out.kz, "k_zero"), (out.vq, "v_q"),
                       (out.vs, "v_scale"), (out.vz, "v_zero")):
        want = _merge_layers(f[f"after_{name}"])
        assert torch.equal(_bytes(ours.cpu()), _bytes(want)), name
    assert out.nq == f["keep"].shape[-1]


def test_bf16_matches_reference_compact():
    from maskahead_b200.layouts import Prefix, compact_tokens

    f = load_compact("compact_bf16")
    kf, vf = _merge_layers(f["before_k_fp"]).to(DEV), _merge_layers(f["before_v_fp"]).to(DEV)
    out = compact_tokens(Prefix.dense(kf, vf), _merge_layers(f["keep"]).to(DEV))
    torch.cuda.synchronize()
    assert torch.equal(_bytes(out.kf.cpu()), _bytes(_merge_layers(f["after_k_fp"])))
    assert torch.equal(_bytes(out.vf.cpu()), _bytes(_merge_layers(f["after_v_fp"])))


def _random_keep(B, H, n, C, gen, *, sorted_=True, bad=0):
    keep = torch.stack([torch.randperm(n, generator=gen)[:C] for _ in range(B * H)]).view(B, H, C)
    if sorted_:
        keep = keep.sort(-1).values
    if bad:
        flat = keep.view(-1)
        pos = torch.randperm(flat.numel(), generator=gen)[:bad]
        flat[pos[: bad // 2]] = -1
        flat[pos[bad // 2:]] = n + 7
    return keep


@pytest.mark.parametrize("sorted_,bad", [(True, 0), (False, 64)])
def test_token_mode_random_matches_oracle(sorted_, bad):
    from maskahead_b200.layouts import Prefix, compact_tokens, pack_prefix

    gen = torch.Generator().manual_seed(31)
    B, H, n, D, C, cap = 2, 4, 20000, 128, 4096, 5000
    k = torch.randn(B, H, n, D, generator=gen).to(torch.bfloat16).to(DEV)
    v = torch.randn(B, H, n, D, generator=gen).to(torch.bfloat16).to(DEV)
    src = pack_prefix(k, v, key_mode="token")
    keep = _random_keep(B, H, n, C, gen, sorted_=sorted_, bad=bad)
    # destination with more slots than kept: slots >= C keep their sentinel
    dst = Prefix(kq=torch.full((B, H, cap, D // 32, 16), 0xA5, dtype=torch.uint8, device=DEV),
                 ks=torch.full((B, H, cap, D // 32), 3.0, dtype=torch.float16, device=DEV),
                 kz=torch.full((B, H, cap, D // 32), 3.0, dtype=torch.float16, device=DEV),
                 vq=torch.full((B, H, cap, D // 32, 16), 0xA5, dtype=torch.uint8, device=DEV),
                 vs=torch.full((B, H, cap, D // 32), 3.0, dtype=torch.float16, device=DEV),
                 vz=torch.full((B, H, cap, D // 32), 3.0, dtype=torch.float16, device=DEV),
                 nq=cap, kb=4, vb=4, kmode=1, kch=src.kch)
    before = {name: getattr(dst, name).cpu() for name in ("kq", "ks", "kz", "vq", "vs", "vz")}
    out = compact_tokens(src, keep.to(DEV), out=dst)
    torch.cuda.synchronize()
    assert out is dst and out.nq == C
    for name in ("kq", "ks", "kz", "vq", "vs", "vz"):
        want = oracle.compact_slots(getattr(src, name).cpu(), keep)
        got = getattr(out, name).cpu()
        assert torch.equal(_bytes(got[:, :, :C]), _bytes(want)), name
        assert torch.equal(_bytes(got[:, :, C:]), _bytes(before[name][:, :, C:])), f"{name}: slots past C written"


@pytest.mark.parametrize("dtype,D", [(torch.bfloat16, 128), (torch.float32, 64)])
def test_dense_strided_source_matches_oracle(dtype, D):
    from maskahead_b200.layouts import Prefix, compact_tokens

    gen = torch.Generator().manual_seed(32)
    B, H, n, cap, C = 3, 2, 3000, 3500, 1000
    kbuf = torch.randn(B, H, cap, D, generator=gen).to(dtype).to(DEV)
    vbuf = torch.randn(B, H, cap, D, generator=gen).to(dtype).to(DEV)
    src = Prefix.dense(kbuf[:, :, :n], vbuf[:, :, :n])          # strided: capacity > live
    keep = _random_keep(B, H, n, C, gen, sorted_=False, bad=10)
    out = compact_tokens(src, keep.to(DEV))
    torch.cuda.synchronize()
    assert torch.equal(out.kf.cpu(), oracle.compact_slots(kbuf[:, :, :n].cpu(), keep))
    assert torch.equal(out.vf.cpu(), oracle.compact_slots(vbuf[:, :, :n].cpu(), keep))


def test_rejected_requests():
    from maskahead_b200._lib import MaError
    from maskahead_b200.layouts import Prefix, compact_tokens, pack_prefix

    k = torch.randn(1, 2, 256, 128, device=DEV).to(torch.bfloat16)
    v = torch.randn(1, 2, 256, 128, device=DEV).to(torch.bfloat16)
    keep = torch.arange(64, device=DEV).expand(1, 2, 64).contiguous()
    with pytest.raises(NotImplementedError):
        compact_tokens(pack_prefix(k, v, key_mode="channel"), keep)
    with pytest.raises(ValueError):
        compact_tokens(Prefix.dense(k[:, :, :32], v[:, :, :32]), keep)
    src = Prefix.dense(k, v)
    with pytest.raises(MaError):
        compact_tokens(src, keep, out=src)                       # in place is refused
    empty = compact_tokens(src, keep[:, :, :0])
    assert empty.nf == 0


REBUILD_ARRAYS = ("k_q", "k_scale", "k_zero", "v_q", "v_scale", "v_zero", "k_residual", "v_residual")


def _rebuilt_regions(out, g_total, st):
    gk = out.kg
    return {"k_q": out.kq[:, :, :g_total], "k_scale": out.ks[:, :, :g_total], "k_zero": out.kz[:, :, :g_total],
            "v_q": out.vq[:, :, :g_total * gk], "v_scale": out.vs[:, :, :g_total * gk],
            "v_zero": out.vz[:, :, :g_total * gk], "k_residual": out.kf[:, :, :st], "v_residual": out.vf[:, :, :st]}


def _channel_prefix(a: dict):
    from maskahead_b200.layouts import Prefix

    return Prefix(kq=a["k_q"], ks=a["k_scale"], kz=a["k_zero"], vq=a["v_q"], vs=a["v_scale"], vz=a["v_zero"],
                  kf=a["k_residual"], vf=a["v_residual"], nq=a["v_q"].shape[2], nf=a["k_residual"].shape[2],
                  kb=4, vb=4, kmode=0)


def test_rebuild_matches_reference():
    """The device rebuild of a channel-mode cache gives the reference's rebuild
    (cache.py:236-335) bit for bit: kept groups moved, sparse survivors re-encoded,
    undecided slots staged in bf16, and the remap."""
    from maskahead_b200.layouts import rebuild

    f = load_compact("rebuild_channel")
    before = {name: _merge_layers(f[f"before_{name}"]).to(DEV) for name in REBUILD_ARRAYS}
    idx = [_merge_layers(f[k]).to(DEV) for k in ("groups_before", "encode", "groups_after", "stage")]
    out, remap = rebuild(_channel_prefix(before), *idx)
    torch.cuda.synchronize()
    g_total = f["after_k_q"].shape[3]
    st = f["after_k_residual"].shape[3]
    assert out.nq == g_total * 32 and out.nf == st
    for name, t in _rebuilt_regions(out, g_total, st).items():
        assert torch.equal(_bytes(t.cpu()), _bytes(_merge_layers(f[f"after_{name}"]))), name
    assert torch.equal(remap.cpu(), _merge_layers(f["remap"]))


def test_rebuild_random_matches_oracle():
    """A larger channel-mode cache (8 lanes, 64 key groups + a 40-slot bf16 residual) with
    per-lane index lists of different lengths: device rebuild == oracle, bit for bit."""
    from maskahead_b200.layouts import pack_prefix, rebuild

    gen = torch.Generator().manual_seed(41)
    B, H, ng, rl, D, gk = 2, 4, 64, 40, 128, 32
    k = torch.randn(B, H, ng * gk, D, generator=gen).to(torch.bfloat16).to(DEV)
    v = torch.randn(B, H, ng * gk, D, generator=gen).to(torch.bfloat16).to(DEV)
    p = pack_prefix(k, v, key_mode="channel")
    arrays = {"k_q": p.kq, "k_scale": p.ks, "k_zero": p.kz, "v_q": p.vq, "v_scale": p.vs, "v_zero": p.vz,
              "k_residual": torch.randn(B, H, rl, D, generator=gen).to(torch.bfloat16).to(DEV),
              "v_residual": torch.randn(B, H, rl, D, generator=gen).to(torch.bfloat16).to(DEV)}
    lists = {"gb": [], "enc": [], "ga": [], "st": []}
    for _ in range(B * H):
        perm = torch.randperm(ng - 2, generator=gen)
        kept = perm[: int(torch.randint(10, 30, (1,), generator=gen))].sort().values
        sparse = perm[30:40]
        slots = (sparse.view(-1, 1) * gk + torch.arange(gk)).view(-1)
        slots = slots[torch.rand(slots.numel(), generator=gen) < 0.3].sort().values
        lists["gb"].append(kept)
        lists["enc"].append(slots)
        lists["ga"].append(torch.tensor([ng - 2, ng - 1]))
        lists["st"].append(torch.randperm(rl, generator=gen)[: int(torch.randint(5, 30, (1,), generator=gen))]
                           .sort().values + ng * gk)

    def padded(rows):
        w = max(r.numel() for r in rows)
        out = torch.full((len(rows), w), -1, dtype=torch.int64)
        for i, r in enumerate(rows):
            out[i, : r.numel()] = r
        return out.view(B, H, w)

    idx = [padded(lists[key]) for key in ("gb", "enc", "ga", "st")]
    out, remap = rebuild(_channel_prefix(arrays), *[t.to(DEV) for t in idx])
    torch.cuda.synchronize()
    want, want_remap = oracle.rebuild_channel({k2: t.cpu() for k2, t in arrays.items()}, *idx)
    g_total = want["k_q"].shape[2]
    st = want["k_residual"].shape[2]
    for name, t in _rebuilt_regions(out, g_total, st).items():
        assert torch.equal(_bytes(t.cpu()), _bytes(want[name])), name
    assert torch.equal(remap.cpu(), want_remap)


@pytest.mark.parametrize("layout", ["bf16", "k4v4_token"])
def test_attention_after_compaction_equals_masked_attention(layout):
    """Round trip at the cfg2 layer size (n = 8192, 4 KV heads, 28 query heads, C = 2048):
    attention over the compacted cache equals attention over the original cache with
    every slot but the kept ones masked dead (attention does not depend on the order of
    the keys), within the bf16 output bar of the attention tests (atol = rtol = 2e-2)."""
    from maskahead_b200.kernels.splitk import splitk_attention
    from maskahead_b200.layouts import Prefix, as_prefix, compact_tokens, pack_prefix

    gen = torch.Generator().manual_seed(43)
    B, H, G, T, n, C, D = 1, 4, 7, 32, 8192, 2048, 128
    k = torch.randn(B, H, n, D, generator=gen).to(torch.bfloat16).to(DEV)
    v = torch.randn(B, H, n, D, generator=gen).to(torch.bfloat16).to(DEV)
    q = torch.randn(B, H * G, T, D, generator=gen).to(torch.bfloat16).to(DEV)
    kc = torch.randn(B, H, T, D, generator=gen).to(torch.bfloat16).to(DEV)
    vc = torch.randn(B, H, T, D, generator=gen).to(torch.bfloat16).to(DEV)
    src = Prefix.dense(k, v) if layout == "bf16" else pack_prefix(k, v, key_mode="token")
    keep = _random_keep(B, H, n, C, gen).to(DEV)
    compacted = compact_tokens(src, keep)
    mask = torch.zeros(B, H, n, dtype=torch.uint8, device=DEV)
    mask.scatter_(-1, keep, 1)
    got, _ = splitk_attention(q, compacted, kc, vc)
    want, _ = splitk_attention(q, as_prefix(src, mask=mask), kc, vc)
    torch.cuda.synchronize()
    torch.testing.assert_close(got.float(), want.float(), atol=2e-2, rtol=2e-2)


def test_evict_plan_matches_reference():
    """ma_evict_plan on the reference's own _evict_to case (evict_channel.npz): the same
    kept groups, encoded and staged slots, bit for bit, and the remap ma_rebuild_remap
    builds from them equals the reference rebuild's."""
    from maskahead_b200._lib import i64, lib as get_lib
    from maskahead_b200.layouts import evict_plan

    g = dict(np.load(GOLDEN / "evict_channel.npz"))
    gb, enc, ga, stg = evict_plan(torch.from_numpy(g["phys"]).to(DEV), torch.from_numpy(g["pos"]).to(DEV),
                                  quantized_length=int(g["quantized_length"]), recent_window=int(g["recent_window"]),
                                  repack_below=float(g["repack_below"]), compaction=str(g["compaction"]))
    for got, key in ((gb, "groups_before"), (enc, "encode"), (ga, "groups_after"), (stg, "stage")):
        np.testing.assert_array_equal(got.cpu().numpy(), g[key], err_msg=key)
    L, B, H, old_len = g["remap"].shape
    remap = torch.empty((L * B, H, old_len), dtype=torch.int64, device=DEV)
    parts = [t.reshape(L * B, H, -1).contiguous() for t in (gb, enc, ga, stg)]
    rc = get_lib().ma_rebuild_remap(L * B, H, old_len, 32, parts[0].data_ptr(), parts[0].shape[-1], parts[1].data_ptr(),
                                    parts[1].shape[-1], parts[2].data_ptr(), parts[2].shape[-1], parts[3].data_ptr(),
                                    parts[3].shape[-1], remap.data_ptr(), torch.cuda.current_stream().cuda_stream)
    assert rc == 0
    torch.cuda.synchronize()
    np.testing.assert_array_equal(remap.cpu().numpy().reshape(g["remap"].shape), g["remap"])


@pytest.mark.parametrize("mode", ["lazy", "full", "tail_groups", "tail_stage", "no_window"])
def test_evict_plan_matches_oracle(mode):
    """Larger lanes (2 x 2 x 4, 3000 live of 9000 slots, 280 key groups) against the
    oracle's restatement: lazy and full compaction, a tail of unadmitted groups placed
    after or staged, no recent window."""
    from maskahead_b200.layouts import evict_plan

    gen = torch.Generator().manual_seed(77)
    L, B, H, n, live, ql = 2, 2, 4, 9000, 3000, 8960
    lanes = L * B * H
    phys = torch.empty(lanes, live, dtype=torch.int32)
    for i in range(lanes):
        base = torch.arange(n)
        for _ in range(200):
            a, b = torch.randint(0, n, (2,), generator=gen).tolist()
            base[a], base[b] = base[b].clone(), base[a].clone()
        whole = torch.randperm(ql // 32, generator=gen)[:12]
        forced = torch.cat([(base // 32 == int(x)).nonzero().flatten() for x in whole])
        fset = set(forced.tolist())
        rest = torch.tensor([j for j in torch.randperm(n, generator=gen).tolist() if j not in fset][: live - forced.numel()])
        sel = torch.cat([forced, rest]).sort().values
        phys[i] = base[sel].to(torch.int32)
    pos = (torch.arange(live) * 5 + 11).expand(lanes, live).contiguous().to(torch.int64)
    phys, pos = phys.view(L, B, H, live), pos.view(L, B, H, live)
    kw = dict(quantized_length=ql, recent_window=0 if mode == "no_window" else 64,
              compaction="full" if mode == "full" else "lazy")
    if mode.startswith("tail"):
        kw.update(tail=64, tail_stage=mode == "tail_stage", cache_length=n)
    got = evict_plan(phys.to(DEV), pos.to(DEV), **kw)
    want = oracle.evict_plan(phys, pos, **kw)
    for a, b, name in zip(got, want, ("groups_before", "encode", "groups_after", "stage")):
        np.testing.assert_array_equal(a.cpu().numpy(), b.numpy(), err_msg=name)


def test_evict_plan_rejects_positions_out_of_order():
    from maskahead_b200.layouts import evict_plan

    phys = torch.arange(200, dtype=torch.int32).view(1, 1, 1, 200)
    pos = torch.arange(200, dtype=torch.int64).flip(-1).view(1, 1, 1, 200)
    with pytest.raises(ValueError):
        evict_plan(phys.to(DEV), pos.to(DEV), quantized_length=192)
