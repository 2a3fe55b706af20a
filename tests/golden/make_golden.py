"""Generate the golden fixtures in this folder from the REFERENCE implementation.

Run where the reference package's source tree is available, naming its ``src``
directory (the folder that holds the ``maskahead`` package):

    MASKAHEAD_REF_SRC=<reference checkout>/src python tests/golden/make_golden.py

For each case of gen_inputs.CASES it builds the reference's LayerCacheView on the
seeded inputs and records what the reference's own CPU (torch) path returns:

* selector_topk(backend="torch", return_importance=True)     kernels/ops.py:333-521
* BitSieveSession._rescore_by_value (value_center="attn")     runtime/session.py:870-954
* dense_attention_reference over [live prefix | block]       reference.py:279-296
* sdpa_compact over [value-aware read set | block]           reference.py:403-426
* value_score (BITSIEVE_VSCORE_FP32=1) + EvictionState.survivors (lookahead)
                                                              session.py:27-40, eviction.py:325-409
* quantize_values / quantize_keys payloads                    reference.py:58-90, 182-213
* PackedKVCache.compact_tokens (token-mode k4v4) and .compact (bf16) after an
  eviction decision                                           cache.py:659-678, 342-365
* PackedKVCache.rebuild (KIVI channel-mode keys: kept groups copied, sparse groups
  re-encoded, undecided slots staged in bf16)                 cache.py:236-335
* BitSieveSession._evict_to planning a rebuild after an eviction (the group decision and
  the index lists it hands to rebuild)                         runtime/session.py:270-361

Outputs go to <case>.npz next to this script, with the SHA-256 of the inputs.
"""

from __future__ import annotations

import os
import sys
import types
from pathlib import Path

import numpy as np
import torch

HERE = Path(__file__).resolve().parent
sys.path.insert(0, str(HERE))
_REF_SRC = os.environ.get("MASKAHEAD_REF_SRC")
if not _REF_SRC or not (Path(_REF_SRC) / "maskahead").is_dir():
    raise SystemExit("set MASKAHEAD_REF_SRC to the reference's src directory (the folder holding maskahead/)")
sys.path.insert(0, _REF_SRC)
os.environ["BITSIEVE_VSCORE_FP32"] = "1"

from gen_inputs import CASES, LARGE, digest, make_case, make_retain_case  # noqa: E402

from maskahead.cache import LayerCacheView, PackedKVCache  # noqa: E402
from maskahead.config import QuantizationConfig  # noqa: E402
from maskahead.eviction import EvictionConfig, EvictionState  # noqa: E402
from maskahead.kernels.ops import selector_topk  # noqa: E402
from maskahead.reference import (  # noqa: E402
    dense_attention_reference, dequantize_keys, dequantize_values, gather_per_kv_head,
    quantize_keys, quantize_values, sdpa_compact, selector_importance_reference,
    PackedKeys, PackedValues,
)
from maskahead.runtime.session import BitSieveSession, value_score  # noqa: E402


def _view(case) -> tuple[LayerCacheView, torch.Tensor, torch.Tensor, dict]:
    """Reference cache view of the case, plus the prefix K/V as the reference reads them."""
    spec = case["spec"]
    n, D = spec["n"], spec["D"]
    extra = {}
    packed = spec.get("packed")
    if not packed:
        k, v = case["key"], case["value"]
        view = LayerCacheView(k_bits=16, v_bits=16, length=n, quantized_length=0, residual_length=0,
                              key_token_group=32, value_channel_group=32, k_q=None, k_scale=None,
                              k_zero=None, v_q=None, v_scale=None, v_zero=None, k_fp=k, v_fp=v,
                              k_residual=None, v_residual=None, head_dim=D)
        return view, k, v, extra
    kf, vf = case["key_fp"], case["value_fp"]
    pv = quantize_values(vf, bits=4, channel_group=32)
    extra.update(vq=pv.payload, vs=pv.scale, vz=pv.zero)
    v = dequantize_values(pv, dtype=torch.bfloat16)
    if packed == "channel":
        pk = quantize_keys(kf, bits=4, token_group=32)
        extra.update(kq=pk.payload, ks=pk.scale, kz=pk.zero)
        k = dequantize_keys(pk, dtype=torch.bfloat16)
        view = LayerCacheView(k_bits=4, v_bits=4, length=n, quantized_length=n, residual_length=0,
                              key_token_group=32, value_channel_group=32, k_q=pk.payload, k_scale=pk.scale,
                              k_zero=pk.zero, v_q=pv.payload, v_scale=pv.scale, v_zero=pv.zero, k_fp=None,
                              v_fp=None, k_residual=None, v_residual=None, head_dim=D)
        return view, k, v, extra
    # token mode: c_i = sqrt(max_t |K|) (cache.py:488-490), keys / c quantized like values
    # (cache.py:491-497); dequant = fp32(code*s+z) * c, one cast (splitk.py:389-395)
    kchan = kf.abs().amax(dim=2).float().clamp_min(1e-4).sqrt()
    kn = (kf.float() / kchan.unsqueeze(2)).to(torch.bfloat16)
    pk = quantize_values(kn, bits=4, channel_group=32)
    extra.update(kq=pk.payload, ks=pk.scale, kz=pk.zero, kchan=kchan)
    k = (dequantize_values(pk, dtype=torch.float32) * kchan.unsqueeze(2)).to(torch.bfloat16)
    return None, k, v, extra


def _rescore(importance, k, v, live_mask, topk):
    """Run the reference's BitSieveSession._rescore_by_value on a minimal stand-in."""
    sel = types.SimpleNamespace(value_center="attn", value_joint=False, value_per_query=False,
                                value_set="none", value_caote=False, sort_indices=True)
    stub = types.SimpleNamespace(
        cache=types.SimpleNamespace(dequantize_layer=lambda layer: (k, v)),
        config=types.SimpleNamespace(collect_diagnostics=False, selector=sel),
    )
    from maskahead.kernels.ops import SelectorResult
    res = BitSieveSession._rescore_by_value(stub, 0, SelectorResult(indices=None, values=None,
                                                                     importance=importance),
                                            topk, live_mask)
    return res.indices, stub._last_value_score


def build_case(name: str) -> dict:
    case = make_case(name)
    spec = case["spec"]
    view, k, v, extra = _view(case)
    q, kc, vc, rows = case["query"], case["current_key"], case["current_value"], case["rows"]
    live = case.get("live_mask")
    D = spec["D"]
    n_live = spec["n"] if live is None else int(live[0, 0].sum())
    topk = min(spec["k"], n_live)
    if view is not None:
        res = selector_topk(q, view, query_indices=rows, topk=topk, backend="torch", live_mask=live,
                            return_importance=True, scaling=D ** -0.5)
        importance, mass_idx = res.importance, res.indices
    else:
        importance = selector_importance_reference(q, k, query_indices=rows, scale=D ** -0.5,
                                                   live_mask=live)
        rank_on = importance if live is None else importance.masked_fill(~live, float("-inf"))
        mass_idx = torch.topk(rank_on, k=topk, dim=-1, sorted=False).indices.sort(dim=-1).values
    vidx, vscore = _rescore(importance, k, v, live, topk)
    # dense step-0 attention over the live prefix and the block (session.py:1472-1504, 1506+)
    if live is None:
        k_used, v_used = k, v
    else:
        pos = live.nonzero()[:, -1].reshape(live.shape[0], live.shape[1], -1)
        k_used, v_used = gather_per_kv_head(k, pos), gather_per_kv_head(v, pos)
    dense_out = dense_attention_reference(q, k_used, v_used, kc, vc, scale=D ** -0.5)
    # sparse sub-step over [read set | block] (session.py:1286-1336)
    sk = torch.cat([gather_per_kv_head(k, vidx), kc.to(k.dtype)], dim=2)
    sv = torch.cat([gather_per_kv_head(v, vidx), vc.to(v.dtype)], dim=2)
    compact_out = sdpa_compact(q.to(k.dtype), sk, sv).to(q.dtype)
    inputs = {key: val for key, val in case.items() if isinstance(val, torch.Tensor)}
    inputs.update({key: val for key, val in extra.items()})
    out = dict(
        digest=np.array(digest(inputs)),
        importance=importance.float().numpy(),
        mass_indices=mass_idx.numpy(),
        value_score=vscore.float().numpy(),
        value_indices=vidx.numpy(),
        dense_out=dense_out.float().numpy(),
        compact_out=compact_out.float().numpy(),
        topk=np.array(topk),
    )
    for key in ("kq", "ks", "kz", "vq", "vs", "vz", "kchan"):
        if key in extra and name not in LARGE:
            t = extra[key]
            out["packed_" + key] = t.view(torch.int16).numpy() if t.dtype in (torch.float16, torch.bfloat16) else t.numpy()
    return out


def build_retain() -> dict:
    r = make_retain_case()
    a = r["a1"] + r["a_probe"]                                   # session.py:2017-2021
    score = value_score(a, r["v_live"])                          # session.py:2025 (fp32 centre)
    L, B, H, live = r["pos"].shape
    st = EvictionState(num_layers=L, batch_size=B, num_kv_heads=H, capacity=live, device="cpu")
    st.append(list(range(live)))
    st.pos[..., :live] = r["pos"]
    cfg = EvictionConfig(policy="lookahead", recent_window=r["W"], capacity_floor=r["C"],
                         sink_tokens=r["sinks"], lookahead_blocks=1)
    keep = st.survivors(cfg, r["C"], None, score)
    inputs = {key: val for key, val in r.items() if isinstance(val, torch.Tensor)}
    return dict(digest=np.array(digest(inputs)), score=score.numpy(), keep=keep.numpy())


_COMPACT_ARRAYS = ("k_q", "k_scale", "k_zero", "v_q", "v_scale", "v_zero", "k_fp", "v_fp")


def build_compact(mode: str, seed: int, L: int, B: int, H: int, n: int, C: int) -> dict:
    """A reference cache filled by its own append path (begin_append / stage_layer /
    commit_append quantize the staged bf16 rows), then compacted to the slots `keep`
    (an ascending random subset per lane, as eviction keeps them): the cache's arrays
    before (slots < n) and after (slots < C)."""
    g = torch.Generator().manual_seed(seed)
    D = 128
    quant = QuantizationConfig(key_mode="token") if mode == "token" else QuantizationConfig(k_bits=16, v_bits=16)
    cache = PackedKVCache(num_layers=L, batch_size=B, num_kv_heads=H, head_dim=D, max_tokens=4096,
                          quant=quant, device="cpu", backend="torch")
    cache.begin_append(n)
    for layer in range(L):
        k = torch.randn(B, H, n, D, generator=g).to(torch.bfloat16)
        v = torch.randn(B, H, n, D, generator=g).to(torch.bfloat16)
        cache.stage_layer(layer, k, v)
    cache.commit_append()
    out = {}
    for name in _COMPACT_ARRAYS:
        t = getattr(cache, name, None)
        if t is not None:
            out[f"before_{name}"] = t[:, :, :, :n].clone()
    if mode == "token":
        out["k_chan"] = cache.k_chan.clone()
    keep = torch.stack([torch.randperm(n, generator=g)[:C].sort().values for _ in range(L * B * H)])
    keep = keep.view(L, B, H, C)
    if mode == "token":
        cache.compact_tokens(keep)                                 # cache.py:659-678
    else:
        cache.compact(keep)                                        # cache.py:342-365
    for name in _COMPACT_ARRAYS:
        t = getattr(cache, name, None)
        if t is not None:
            out[f"after_{name}"] = t[:, :, :, :C].clone()
    out["keep"] = keep
    res = {}
    for key, val in out.items():
        res[key] = val.view(torch.int16).numpy() if val.dtype in (torch.bfloat16, torch.float16) else val.numpy()
    res["dtypes"] = np.array([f"{key}:{str(val.dtype)}" for key, val in out.items()])
    return res


def _padded(rows: list, width: int) -> torch.Tensor:
    out = torch.full((len(rows), width), -1, dtype=torch.int64)
    for i, r in enumerate(rows):
        out[i, : len(r)] = torch.as_tensor(r, dtype=torch.int64)
    return out


def build_rebuild(seed: int = 23, L: int = 2, B: int = 1, H: int = 2, n: int = 333) -> dict:
    """A channel-mode k4v4 reference cache (its own append path: 288 quantized slots in
    9 key groups, 45 in the bf16 residual), rebuilt by PackedKVCache.rebuild from
    per-lane index lists of different lengths padded with -1, as the session's _evict_to
    makes them (session.py:303-361): kept groups ascending, encoded and staged slots
    ascending by position. Records the arrays before, the index lists, the arrays after
    (the regions rebuild defines) and the remap."""
    g = torch.Generator().manual_seed(seed)
    D, gk = 128, 32
    quant = QuantizationConfig(key_mode="channel")
    cache = PackedKVCache(num_layers=L, batch_size=B, num_kv_heads=H, head_dim=D, max_tokens=4096,
                          quant=quant, device="cpu", backend="torch")
    cache.begin_append(n)
    for layer in range(L):
        k = torch.randn(B, H, n, D, generator=g).to(torch.bfloat16)
        v = torch.randn(B, H, n, D, generator=g).to(torch.bfloat16)
        cache.stage_layer(layer, k, v)
    cache.commit_append()
    ql, rl, ng = cache.quantized_length, cache.residual_length, cache.quantized_length // gk
    out = {}
    for name in ("k_q", "k_scale", "k_zero"):
        out[f"before_{name}"] = getattr(cache, name)[:, :, :, :ng].clone()
    for name in ("v_q", "v_scale", "v_zero"):
        out[f"before_{name}"] = getattr(cache, name)[:, :, :, :ql].clone()
    for name in ("k_residual", "v_residual"):
        out[f"before_{name}"] = getattr(cache, name)[:, :, :, :rl].clone()
    gb, enc, ga, stg = [], [], [], []
    for _ in range(L * B * H):
        perm = torch.randperm(ng - 1, generator=g)             # the last group goes "after"
        kept = sorted(perm[: int(torch.randint(3, 6, (1,), generator=g))].tolist())
        sparse = sorted(perm[6:8].tolist())
        slots = sorted(s for grp in sparse for s in range(grp * gk, grp * gk + gk)
                       if torch.rand(1, generator=g).item() < 0.4)
        gb.append(kept)
        enc.append(slots)
        ga.append([ng - 1])
        stg.append(sorted(torch.randperm(rl, generator=g)[: int(torch.randint(3, 8, (1,), generator=g))]
                          .add(ql).tolist()))
    groups_before = _padded(gb, max(map(len, gb))).view(L, B, H, -1)
    encode = _padded(enc, max(map(len, enc))).view(L, B, H, -1)
    groups_after = _padded(ga, 1).view(L, B, H, -1)
    stage = _padded(stg, max(map(len, stg))).view(L, B, H, -1)
    remap = cache.rebuild(groups_before, encode, groups_after, stage)    # cache.py:236-335
    g1, m, g3, st = (t.shape[-1] for t in (groups_before, encode, groups_after, stage))
    total = g1 + -(-m // gk) + g3
    for name in ("k_q", "k_scale", "k_zero"):
        out[f"after_{name}"] = getattr(cache, name)[:, :, :, :total].clone()
    for name in ("v_q", "v_scale", "v_zero"):
        out[f"after_{name}"] = getattr(cache, name)[:, :, :, :total * gk].clone()
    for name in ("k_residual", "v_residual"):
        out[f"after_{name}"] = getattr(cache, name)[:, :, :, :st].clone()
    out.update(groups_before=groups_before, encode=encode, groups_after=groups_after, stage=stage,
               remap=remap)
    res = {}
    for key, val in out.items():
        res[key] = val.view(torch.int16).numpy() if val.dtype in (torch.bfloat16, torch.float16) else val.numpy()
    res["dtypes"] = np.array([f"{key}:{str(val.dtype)}" for key, val in out.items()])
    return res


def build_evict(seed: int = 31, L: int = 2, B: int = 1, H: int = 2, n: int = 333, C: int = 190,
                W: int = 40) -> dict:
    """A channel-mode reference cache (288 quantized slots in 9 key groups, 45 staged), an
    EvictionState whose live entries have increasing positions and physical slots that are
    a near-identity permutation, then BitSieveSession._evict_to with per-lane survivor sets
    (three whole key groups plus random entries, ascending) on a stub session. Records the
    live entries' slots and positions after the eviction's compaction, the index lists
    _evict_to hands to cache.rebuild, its remap and the live entries' new slots."""
    g = torch.Generator().manual_seed(seed)
    D, gk = 128, 32
    quant = QuantizationConfig(key_mode="channel")
    cache = PackedKVCache(num_layers=L, batch_size=B, num_kv_heads=H, head_dim=D, max_tokens=4096,
                          quant=quant, device="cpu", backend="torch")
    cache.begin_append(n)
    for layer in range(L):
        cache.stage_layer(layer, torch.randn(B, H, n, D, generator=g).to(torch.bfloat16),
                          torch.randn(B, H, n, D, generator=g).to(torch.bfloat16))
    cache.commit_append()
    phys0 = torch.arange(n)
    for _ in range(12):                                     # a few slots moved by earlier rebuilds
        i, j = torch.randint(0, n, (2,), generator=g).tolist()
        phys0[i], phys0[j] = phys0[j].clone(), phys0[i].clone()
    positions = torch.arange(n) * 3 + 7
    st = EvictionState(num_layers=L, batch_size=B, num_kv_heads=H, capacity=n, device="cpu")
    st.append(positions, phys=phys0)
    keep = torch.empty(L, B, H, C, dtype=torch.int64)
    for lane in range(L * B * H):
        whole = torch.randperm(8, generator=g)[:3]
        forced = torch.cat([(phys0 // gk == int(x)).nonzero().flatten() for x in whole])
        rest = torch.tensor([i for i in torch.randperm(n, generator=g).tolist() if i not in set(forced.tolist())])
        keep.view(-1, C)[lane] = torch.cat([forced, rest[: C - forced.numel()]]).sort().values
    captured = {}
    orig = cache.rebuild

    def rebuild(gb, enc, ga, stg):
        captured.update(groups_before=gb.clone(), encode=enc.clone(), groups_after=ga.clone(), stage=stg.clone())
        remap = orig(gb, enc, ga, stg)
        captured["remap"] = remap.clone()
        return remap

    cache.rebuild = rebuild
    compact = st.compact

    def compact_and_record(k):
        compact(k)
        captured.update(phys=st.phys[..., : st.live].clone(), pos=st.pos[..., : st.live].clone())

    st.compact = compact_and_record
    cfg = EvictionConfig(policy="lookahead", recent_window=W, capacity_floor=C)
    stub = types.SimpleNamespace(_eviction=st, config=types.SimpleNamespace(eviction=cfg), _attn_log=None,
                                 _phys_compact=True, cache=cache, _next_position=cache.get_seq_length(),
                                 trace=types.SimpleNamespace(add_counter=lambda *a, **k: None))
    BitSieveSession._evict_to(stub, keep)
    out = {key: val.numpy() for key, val in captured.items()}
    out.update(keep=keep.numpy(), new_phys=st.phys[..., : st.live].numpy(), quantized_length=np.array(288),
               recent_window=np.array(W), repack_below=np.array(cfg.repack_below), compaction=np.array(cfg.compaction))
    return out


def main() -> None:
    only = set(sys.argv[1:])
    if "evict_channel" in only:
        np.savez_compressed(HERE / "evict_channel.npz", **build_evict())
        print("wrote evict_channel")
        return
    for name in CASES:
        if only and name not in only:
            continue
        np.savez_compressed(HERE / f"{name}.npz", **build_case(name))
        print("wrote", name)
    if only:
        return
    np.savez_compressed(HERE / "retain.npz", **build_retain())
    print("wrote retain")
    np.savez_compressed(HERE / "compact_token.npz", **build_compact("token", 21, 2, 1, 2, 300, 96))
    np.savez_compressed(HERE / "compact_bf16.npz", **build_compact("bf16", 22, 1, 1, 2, 160, 48))
    print("wrote compact_token, compact_bf16")
    np.savez_compressed(HERE / "rebuild_channel.npz", **build_rebuild())
    print("wrote rebuild_channel")
    np.savez_compressed(HERE / "evict_channel.npz", **build_evict())
    print("wrote evict_channel")


if __name__ == "__main__":
    main()
