"""Split-K attention over [prefix | current block] and the prefix scores, on sm_100a.

Drop-in counterparts of src/maskahead/kernels/splitk.py in the reference:

    out, stats = splitk_attention(q, prefix, kc, vc, want_prefix=True)
    mass, score = prefix_scores(q, prefix, stats, q_rows, value=True)

Same signatures and return shapes. The reference's tuning keywords (block sizes,
dequantization thresholds) are accepted and ignored: there is one kernel family. O_p is
returned in fp32. The value score's centre is c = sum_j a_j v_j / sum_j a_j in fp32
over the live slots (session.py:27-40 with the fp32 centre), which equals the mean of
O_p over the selection rows that the reference uses (splitk.py:600-601).
"""

from __future__ import annotations

import torch

from .. import _lib
from ..layouts import Prefix, as_prefix, kv_descriptor
from ._common import block_struct, rows_struct

__all__ = ["Prefix", "splitk_attention", "prefix_scores", "dequantize_prefix"]


def splitk_attention(query, prefix, current_key, current_value, *, scaling=None,
                     causal_block: int = 0, q_pos0: int = 0, c_pos0: int = 0, want_prefix: bool = False,
                     stats_out=None, head_gather=None, **_tuning):
    """softmax over [prefix | current] for every query row (splitk.py:493-579).

    Returns (out [B,Hq,T,D] in the query dtype, stats) with stats = (M_p, L_p, O_p,
    prefix) when want_prefix: prefix-only max and sum [B,Hkv,R] and normalized output
    [B,Hkv,R,D] fp32 per row r = g*T + t. causal_block > 0: query q_pos0+t sees current
    key c_pos0+j only if (c_pos0+j)//causal_block <= (q_pos0+t)//causal_block.
    stats_out = (M_p, L_p) or (M_p, L_p, O_p): contiguous fp32 buffers of those shapes to
    write the statistics into (e.g. one layer's slice of layer-stacked buffers); O_p is
    then computed only if given. Implies want_prefix.
    head_gather = (gather, gathered): KV-head sharding (maskahead_b200.shard.PeerHeadGather
    of the process group, every rank making the same calls): this rank's output rows
    t < gathered.shape[2] are exchanged with every rank's in the same launch (the split
    merge stores them into every rank's receive region) and gathered holds all of them,
    [B, world * Hq, Tg, D] bf16, when the call returns on the stream.
    """
    lib = _lib.lib()
    prefix = as_prefix(prefix)
    b, hq, t, d = query.shape
    if current_key is not None:
        hkv = current_key.shape[1]
    else:
        hkv = (prefix.kf if prefix.kf is not None else prefix.vq).shape[1]
    g = hq // hkv
    r = g * t
    dev = query.device
    rows, qkeep = rows_struct(query)
    cur, ckeep = block_struct(current_key, current_value, query.dtype)
    if prefix.n:
        desc = kv_descriptor(prefix, batch=b, heads=hkv, head_dim=d)
        kv = desc.kv
    else:
        desc, kv = None, _lib.MaKV()
        kv.layout, kv.dtype = _lib.MA_KV_DENSE, rows.dtype
    out = torch.empty_like(query)
    if stats_out is not None:
        mp, lp = stats_out[0], stats_out[1]
        op = stats_out[2] if len(stats_out) > 2 else None
        for x, shape in ((mp, (b, hkv, r)), (lp, (b, hkv, r)), (op, (b, hkv, r, d))):
            if x is not None and (tuple(x.shape) != shape or x.dtype != torch.float32 or not x.is_contiguous()
                                  or x.device != dev):
                raise ValueError(f"stats_out: need contiguous float32 {shape} tensors on {dev}")
        want_prefix = True
    elif want_prefix:
        mp = torch.empty((b, hkv, r), device=dev, dtype=torch.float32)
        lp = torch.empty_like(mp)
        op = torch.empty((b, hkv, r, d), device=dev, dtype=torch.float32)
    else:
        mp = lp = op = None
    nbytes = lib.ma_prefix_attention_workspace(b, hkv, r, prefix.n, d, cur.Tc)
    ws = _lib.workspace(dev, "attention", nbytes)
    scale = float(scaling if scaling is not None else d ** -0.5)
    if head_gather is not None:
        gather, gout = head_gather
        tg = gout.shape[2]
        if (gout.dtype != torch.bfloat16 or gout.device != dev or tuple(gout.shape) != (b, hq * gather.world, tg, d)
                or gout.stride(-1) != 1 or not 0 < tg <= t):
            raise ValueError(f"head_gather: need a bfloat16 [{b}, {hq * gather.world}, Tg <= {t}, {d}] tensor on {dev}")
        bases, gws = gather.region(dev, b, hq * gather.world, tg)
        _lib.check("ma_prefix_attention_gather", lib.ma_prefix_attention_gather(
            rows, kv, hkv, cur, scale, int(causal_block), int(q_pos0), int(c_pos0),
            out.data_ptr(), _lib.i64(*out.stride()[:3]), _lib.ptr(mp), _lib.ptr(lp), _lib.ptr(op),
            ws.data_ptr(), ws.numel(), gather.world, gather.rank, bases, tg, gout.data_ptr(),
            _lib.i64(*gout.stride()[:3]), gws.data_ptr(), gws.numel(), _lib.stream_handle(dev)))
    else:
        _lib.check("ma_prefix_attention", lib.ma_prefix_attention(
            rows, kv, hkv, cur, scale, int(causal_block), int(q_pos0), int(c_pos0),
            out.data_ptr(), _lib.i64(*out.stride()[:3]), _lib.ptr(mp), _lib.ptr(lp), _lib.ptr(op),
            ws.data_ptr(), ws.numel(), _lib.stream_handle(dev)))
    del qkeep, ckeep, desc
    return out, ((mp, lp, op, prefix) if want_prefix else None)


def prefix_scores(query, prefix, stats, q_rows, *, value: bool, scaling=None, **_tuning):
    """Per prefix slot: mass a_j (mean prefix-softmax over the selection rows) and, with
    value=True, a_j * ||v_j - c|| with c = sum_j a_j v_j / sum_j a_j (splitk.py:582-614).

    q_rows: positions t within the block (int tensor or list); every query head of the
    KV head contributes. Returns (mass, score) as [B, Hkv, n] fp32 (score None when
    value=False). Dead slots score 0.
    """
    lib = _lib.lib()
    b, hq, t, d = query.shape
    mp, lp, _op, used = stats
    prefix = used if used is not None else as_prefix(prefix)
    hkv = mp.shape[1]
    n = prefix.n
    dev = query.device
    mass = torch.empty((b, hkv, n), device=dev, dtype=torch.float32)
    if n == 0:
        return mass, (torch.empty_like(mass) if value else None)
    if isinstance(q_rows, torch.Tensor) and q_rows.is_cuda and q_rows.dtype == torch.int32:
        rows_t = q_rows.contiguous()
    else:
        rows_t = torch.as_tensor(q_rows, dtype=torch.int32).to(dev).contiguous()
    rows, qkeep = rows_struct(query)
    desc = kv_descriptor(prefix, batch=b, heads=hkv, head_dim=d)
    scale = float(scaling if scaling is not None else d ** -0.5)
    score = torch.empty_like(mass) if value else None
    ws = _lib.workspace(dev, "value_score", lib.ma_value_score_workspace(b, hkv, n, d))
    _lib.check("ma_prefix_scores", lib.ma_prefix_scores(
        rows, desc.kv, hkv, rows_t.data_ptr(), int(rows_t.numel()), mp.data_ptr(), lp.data_ptr(), scale,
        mass.data_ptr(), _lib.i64(mass.stride(0), mass.stride(1)), _lib.ptr(score),
        _lib.i64(*(score.stride()[:2] if value else (0, 0))), ws.data_ptr(), ws.numel(),
        _lib.stream_handle(dev)))
    del qkeep, rows_t
    return mass, score


def dequantize_prefix(prefix, b: int, hkv: int, d: int, dtype=torch.bfloat16, block_n: int = 64, *, out=None):
    """The whole prefix as contiguous [B, Hkv, n, D] tensors (splitk.py:465-480): every slot
    dequantized (packed part) or copied (dense tail) in one launch; slots past lens[b] or on
    a bad page are zeros. out = (key, value) buffers of that shape (optional). block_n (the
    reference's Triton tile) is accepted and ignored."""
    lib = _lib.lib()
    prefix = as_prefix(prefix)
    n = prefix.n
    dev = (prefix.kq if prefix.nq else prefix.kf).device
    if out is not None:
        ko, vo = out
    else:
        ko = torch.empty((b, hkv, n, d), device=dev, dtype=dtype)
        vo = torch.empty_like(ko)
    if n == 0:
        return ko, vo
    unmasked = Prefix(**{s: getattr(prefix, s) for s in Prefix.__slots__})
    unmasked.mask = None
    desc = kv_descriptor(unmasked, batch=b, heads=hkv, head_dim=d)
    _lib.check("ma_gather_kv", lib.ma_gather_kv(
        desc.kv, b, hkv, d, None, n, None, ko.data_ptr(), vo.data_ptr(), _lib.i64(*ko.stride()[:3]),
        _lib.i64(*vo.stride()[:3]), _lib.dtype_code(ko.dtype), _lib.stream_handle(dev)))
    return ko, vo