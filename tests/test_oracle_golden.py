"""Pin the CPU oracle against outputs recorded from the reference implementation.

The fixtures (tests/golden/*.npz) were produced by tests/golden/make_golden.py, which
runs the reference's own torch CPU path on the seeded inputs of gen_inputs.py.
"""

from __future__ import annotations

from pathlib import Path

import numpy as np
import pytest
import torch

import oracle
from gen_inputs import CASES, digest, make_case, make_retain_case

GOLDEN = Path(__file__).resolve().parent / "golden"


def _load(name):
    return dict(np.load(GOLDEN / f"{name}.npz"))


def oracle_case(name):
    """Inputs of a case plus the prefix K/V as the hot path reads them (dequantized)."""
    case = make_case(name)
    spec = case["spec"]
    packed = spec.get("packed")
    extra = {}
    if not packed:
        return case, case["key"], case["value"], extra
    kf, vf = case["key_fp"], case["value_fp"]
    vq, vs, vz = oracle.quantize_values(vf)
    extra.update(vq=vq, vs=vs, vz=vz)
    v = oracle.dequantize_values(vq, vs, vz)
    if packed == "channel":
        kq, ks, kz = oracle.quantize_keys(kf)
        extra.update(kq=kq, ks=ks, kz=kz)
        k = oracle.dequantize_keys(kq, ks, kz)
    else:
        kchan = oracle.key_channel_divisor(kf)
        kq, ks, kz = oracle.quantize_keys_token(kf, kchan)
        extra.update(kq=kq, ks=ks, kz=kz, kchan=kchan)
        k = oracle.dequantize_keys_token(kq, ks, kz, kchan)
    return case, k, v, extra


@pytest.mark.parametrize("name", list(CASES))
def test_oracle_matches_reference(name):
    g = _load(name)
    case, k, v, extra = oracle_case(name)
    inputs = {key: val for key, val in case.items() if isinstance(val, torch.Tensor)}
    inputs.update(extra)
    # same inputs, bit for bit (packed payloads included)
    assert digest(inputs) == str(g["digest"])
    for key in ("kq", "ks", "kz", "vq", "vs", "vz", "kchan"):
        if key in extra and "packed_" + key in g:
            t = extra[key]
            t = t.view(torch.int16) if t.dtype in (torch.float16, torch.bfloat16) else t
            np.testing.assert_array_equal(t.numpy(), g["packed_" + key])

    spec = case["spec"]
    D = spec["D"]
    q, kc, vc, rows = case["query"], case["current_key"], case["current_value"], case["rows"]
    live = case.get("live_mask")
    topk = int(g["topk"])

    imp = oracle.selector_importance(q, k, query_indices=rows, scale=D ** -0.5, live_mask=live)
    np.testing.assert_allclose(imp.numpy(), g["importance"], rtol=1e-6, atol=1e-12)

    idx, _ = oracle.topk_sorted(imp, topk, live)
    np.testing.assert_array_equal(idx.numpy(), g["mass_indices"])

    vs = oracle.rescore_by_value(imp, v, live)
    np.testing.assert_allclose(vs.numpy(), g["value_score"], rtol=1e-5, atol=1e-10)
    vidx, _ = oracle.topk_sorted(vs, topk, live)
    np.testing.assert_array_equal(vidx.numpy(), g["value_indices"])

    # the step-0 output, through the prefix-statistics restatement used by the kernels
    out, (mp, lp, op) = oracle.prefix_attention(q, k, v, kc, vc, scale=D ** -0.5, live_mask=live)
    tol = 1e-5 if q.dtype == torch.float32 else 1.6e-2
    np.testing.assert_allclose(out.float().numpy(), g["dense_out"], rtol=tol, atol=tol)
    # prefix mass from the statistics equals the selector importance (splitk.py:582-614)
    a = oracle.prefix_mass(q, k, mp, lp, rows, scale=D ** -0.5, live_mask=live)
    np.testing.assert_allclose(a.numpy(), g["importance"], rtol=2e-5, atol=1e-10)

    sk = torch.cat([oracle.gather_per_kv_head(k, vidx), kc.to(k.dtype)], dim=2)
    sv = torch.cat([oracle.gather_per_kv_head(v, vidx), vc.to(v.dtype)], dim=2)
    cout = oracle.sdpa_compact(q.to(k.dtype), sk, sv).to(q.dtype)
    np.testing.assert_allclose(cout.float().numpy(), g["compact_out"], rtol=1e-6, atol=1e-6)


def test_retention_matches_reference():
    g = _load("retain")
    r = make_retain_case()
    inputs = {key: val for key, val in r.items() if isinstance(val, torch.Tensor)}
    assert digest(inputs) == str(g["digest"])
    score = oracle.lookahead_score(r["a1"], r["a_probe"], r["v_live"])
    np.testing.assert_allclose(score.numpy(), g["score"], rtol=1e-6, atol=1e-12)
    keep = oracle.survivors_lookahead(r["pos"], torch.from_numpy(g["score"]), r["C"],
                                      recent_window=r["W"], sink_tokens=r["sinks"])
    np.testing.assert_array_equal(keep.numpy(), g["keep"])


def test_topk_tie_rule_lowest_index_first():
    s = torch.tensor([[1.0, 3.0, 3.0, 2.0, 3.0, 3.0]])
    idx, val = oracle.topk_sorted(s, 3)
    assert idx.tolist() == [[1, 2, 4]]
    assert val.tolist() == [[3.0, 3.0, 3.0]]
    live = torch.tensor([[True, False, True, True, True, True]])
    idx, _ = oracle.topk_sorted(s, 3, live)
    assert idx.tolist() == [[2, 4, 5]]


def test_order_keys_monotone():
    x = np.array([-np.inf, -3.5, -1e-30, -0.0, 0.0, 1e-30, 2.0, np.inf], dtype=np.float32)
    k = oracle.order_keys(x)
    assert np.all(np.diff(k.astype(np.int64)) >= 0)
    assert k[3] < k[4]          # -0.0 orders below +0.0


def test_pack_roundtrip():
    g = torch.Generator().manual_seed(3)
    codes = torch.randint(0, 16, (5, 7, 32), generator=g, dtype=torch.uint8)
    p = oracle.pack_last_dim(codes, 4)
    assert p.shape == (5, 7, 16)
    assert int(p[0, 0, 0]) == int(codes[0, 0, 0]) | (int(codes[0, 0, 1]) << 4)
    np.testing.assert_array_equal(oracle.unpack_last_dim(p, 4, 32).numpy(), codes.numpy())


def test_pages_to_contiguous():
    g = torch.Generator().manual_seed(4)
    H, ps, D = 2, 4, 8
    seq = torch.randn(H, 10, D, generator=g)
    table = torch.tensor([5, 1, 3], dtype=torch.int32)
    pool = torch.zeros(6, H, ps, D)
    for lp, pp in enumerate(table.tolist()):
        chunk = seq[:, lp * ps:(lp + 1) * ps]
        pool[pp, :, :chunk.shape[1]] = chunk
    np.testing.assert_array_equal(oracle.pages_to_contiguous(pool, table, 10, ps).numpy(), seq.numpy())


def load_compact(name):
    """A compaction fixture: arrays before/after as torch tensors of their recorded dtype."""
    z = _load(name)
    dt = dict(s.split(":") for s in z.pop("dtypes").tolist())
    out = {}
    for key, arr in z.items():
        t = torch.from_numpy(arr)
        if dt[key] in ("torch.bfloat16", "torch.float16"):
            t = t.view(getattr(torch, dt[key].split(".")[1]))
        out[key] = t
    return out


@pytest.mark.parametrize("name", ["compact_token", "compact_bf16"])
def test_compaction_matches_reference(name):
    """compact_slots (the oracle's compaction) reproduces the reference cache's
    compact_tokens / compact bit-exactly on every stored array."""
    f = load_compact(name)
    keep = f["keep"]
    names = [k[len("before_"):] for k in f if k.startswith("before_")]
    assert names
    for arr in names:
        got = oracle.compact_slots(f[f"before_{arr}"], keep, slot_dim=3)
        want = f[f"after_{arr}"]
        assert got.dtype == want.dtype
        assert torch.equal(got.view(torch.uint8) if got.dtype != torch.uint8 else got,
                           want.view(torch.uint8) if want.dtype != torch.uint8 else want), arr


def test_compaction_out_of_range_rows_are_zero():
    t = torch.arange(2 * 3 * 5 * 4, dtype=torch.int16).view(2, 3, 5, 4)
    keep = torch.tensor([4, -1, 0, 5]).expand(2, 3, 4)
    got = oracle.compact_slots(t, keep)
    assert torch.equal(got[:, :, 0], t[:, :, 4]) and torch.equal(got[:, :, 2], t[:, :, 0])
    assert int(got[:, :, 1].abs().sum()) == 0 and int(got[:, :, 3].abs().sum()) == 0


REBUILD_ARRAYS = ("k_q", "k_scale", "k_zero", "v_q", "v_scale", "v_zero", "k_residual", "v_residual")


def test_rebuild_matches_reference():
    """rebuild_channel (the oracle's group-preserving rebuild) reproduces the reference
    cache's rebuild bit-exactly: kept groups, re-encoded groups, the bf16 residual and
    the remap (every layer at once, the layer axis merged into the batch axis)."""
    f = load_compact("rebuild_channel")

    def merge(t):
        return t.reshape(t.shape[0] * t.shape[1], *t.shape[2:])

    before = {name: merge(f[f"before_{name}"]) for name in REBUILD_ARRAYS}
    idx = [merge(f[k]) for k in ("groups_before", "encode", "groups_after", "stage")]
    got, remap = oracle.rebuild_channel(before, *idx)
    for name in REBUILD_ARRAYS:
        want = merge(f[f"after_{name}"])
        assert got[name].shape == want.shape, name
        assert torch.equal(got[name].contiguous().view(torch.uint8), want.contiguous().view(torch.uint8)), name
    assert torch.equal(remap, merge(f["remap"]))


def test_oracle_evict_plan_matches_reference():
    """The eviction planning of BitSieveSession._evict_to (session.py:303-356), recorded
    from the reference on a channel-mode cache: the kept groups, the re-encoded and staged
    slots in position order, and the live entries' slots after the reference's rebuild."""
    g = _load("evict_channel")
    gb, enc, ga, stg = oracle.evict_plan(torch.from_numpy(g["phys"]), torch.from_numpy(g["pos"]),
                                         quantized_length=int(g["quantized_length"]),
                                         recent_window=int(g["recent_window"]),
                                         repack_below=float(g["repack_below"]), compaction=str(g["compaction"]))
    for got, key in ((gb, "groups_before"), (enc, "encode"), (ga, "groups_after"), (stg, "stage")):
        np.testing.assert_array_equal(got.numpy(), g[key], err_msg=key)
    new_phys = torch.from_numpy(g["remap"]).gather(-1, torch.from_numpy(g["phys"]).long())
    np.testing.assert_array_equal(new_phys.numpy(), g["new_phys"])
