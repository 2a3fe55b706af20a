"""Session-level hot path: step 0, sparse sub-steps and lookahead retention.

These functions are what the reference session's fast path does per layer
(src/maskahead/runtime/session.py), written against the sm_100a operators:

  dense_required      _dense_required (456-467): whether a layer skips selection and
                      attends densely (dense-prefix layers, a budget covering the prefix).
  fast_attend         _fast_attend (1378-1393): the dense layers' sub-steps, attention over
                      [live prefix | block], optionally with the prefix mass of some rows.
  fast_step0          _fast_step0 (1403-1454): dense attention over [live prefix |
                      block], the block's prefix mass, the value-aware score, the
                      ascending top-k read set and (gather=True) the read set's K/V rows
                      gathered once into a compact dense cache (1438-1447, gather_dequant
                      1174-1190).
  step0_attention     fast_step0's attention half (the prefix statistics optionally into
                      the caller's layer-stacked buffers).
  select_step0        fast_step0's selection half on the step-0 statistics, for one layer
                      or for every layer of the step at once, stacked along the batch
                      axis (the session's finish_step0, 1264-1285: nothing reads a layer's
                      read set before its first sub-step, so the selection of all layers
                      can follow the step-0 forward as one pass).
  gather_read_set     that gather on its own.
  compact_attention   _compact_attention / sdpa_compact (1286-1336; reference.py:403-426):
                      attention over [read set | block], from the compact cache (as the
                      reference does) or by index straight from the cache.
  probe_attention     the lookahead probe (2317-2332): block-causal attention of the probe
                      forward plus the prefix mass of the probe rows.
  value_score         value_score (27-40) with the fp32 centre, over dense values;
  value_score_prefix  the same over any cache layout (packed values dequantized in place).
  lookahead_survivors EvictionState.survivors for the lookahead policy (eviction.py:364-409).
"""

from __future__ import annotations

from dataclasses import dataclass

import torch

from . import _lib
from .kernels._common import block_struct, rows_struct
from .kernels.ops import gather_packed_kv, select_topk_indices
from .kernels.splitk import prefix_scores, splitk_attention
from .layouts import Prefix, as_prefix, kv_descriptor

__all__ = ["Step0Result", "dense_required", "fast_attend", "fast_step0", "step0_attention", "select_step0",
           "unpacked_prefix", "gather_read_set", "compact_attention", "probe_attention", "value_score",
           "value_score_prefix", "lookahead_survivors"]


@dataclass(slots=True)
class Step0Result:
    out: torch.Tensor | None             # [B, Hq, T, D] attention output (None from select_step0)
    indices: torch.Tensor | None         # [B, Hkv, k] ascending read set (None: dense layer)
    mass: torch.Tensor | None            # [B, Hkv, n] prefix mass of the selection rows
    score: torch.Tensor | None           # [B, Hkv, n] value-aware score (value_aware only)
    compact: Prefix | None = None        # the read set's rows, gathered (gather=True only)
    probe_mass: torch.Tensor | None = None   # [B, Hkv, n] merged probe's prefix mass (probe_blocks > 0)


def dense_required(layer_idx: int, *, dense_prefix_layers: int, old_cache_len: int, topk: int,
                   query_indices, eviction: bool = False, live_cache_len: int | None = None,
                   semantic: str = "A") -> bool:
    """Whether layer `layer_idx` attends densely instead of through a read set
    (session.py:456-467): the dense semantic, the first `dense_prefix_layers` layers, an
    empty cache or no selection rows, and -- without eviction -- a budget `topk` (the
    selector's effective top-k for this cache length) that covers the whole prefix. With
    eviction the cache is the live set and a covering budget still selects."""
    if semantic == "dense" or layer_idx < dense_prefix_layers:
        return True
    if eviction:
        return (live_cache_len or 0) == 0 or not query_indices
    return old_cache_len == 0 or int(topk) >= old_cache_len or not query_indices


def fast_attend(query: torch.Tensor, prefix, current_key: torch.Tensor, current_value: torch.Tensor, *,
                scaling: float | None = None, causal: int = 0, q_pos0: int = 0, mass_rows=None):
    """Attention over [live prefix | current block] and, with mass_rows, the prefix mass of
    those rows (session.py:1378-1393): what a dense layer's sub-steps run. Returns
    (out, mass or None)."""
    prefix = as_prefix(prefix)
    out, stats = splitk_attention(query, prefix, current_key, current_value, scaling=scaling, causal_block=causal,
                                  q_pos0=q_pos0, c_pos0=q_pos0, want_prefix=mass_rows is not None)
    if mass_rows is None or prefix.n == 0:
        return out, None
    mass, _ = prefix_scores(query, prefix, stats, mass_rows, value=False, scaling=scaling)
    return out, mass


def _needs_unpack(prefix: Prefix, batch: int, heads: int, head_dim: int, unpack) -> bool:
    """Whether an attention pass (step 0, the probe) unpacks a packed prefix to bf16 first.

    unpack=None (automatic) and True: yes. On B200 the unpack kernel followed by the
    TMA-fed bf16 kernels is the faster route for attention: the unpack does the
    dequantization once on every SM, and its output of a layer stays in L2 for the
    attention, scoring and gather passes, while dequantizing producer warps inside the
    attention kernel compete with its softmax warps for issue slots and are repeated by
    every row tile of a head (measured: a cfg3 layer's step-0 attention 29 us unpacked
    against 36 us in place, 16 paged cfg5 sequences 0.16 + unpack against 0.76 ms).
    unpack=False reads the prefix in place: the pipelined kernels' producer warps for a
    token-mode layout they accept (ma_kv_read_in_place), the general kernels otherwise;
    that route moves only the packed bytes (160 per slot and head)."""
    return prefix.nq > 0 and unpack is not False


def fast_step0(query: torch.Tensor, prefix, current_key: torch.Tensor, current_value: torch.Tensor, *,
               query_indices, topk: int, value_aware: bool = True, scaling: float | None = None,
               select: bool = True, want_mass: bool = False, gather: bool = False,
               compact_out: tuple[torch.Tensor, torch.Tensor] | None = None, unpack: bool | None = None,
               probe_blocks: int = 0, block_size: int = 32, probe_rows: torch.Tensor | None = None) -> Step0Result:
    """Step 0 of one layer: attention output, mass, score and the read set (session.py:1403-1454).

    The read set is the top min(topk, live) slots by score (value_aware) or mass, dead
    slots never chosen, as ascending slot indices. gather=True also gathers the read set's
    K/V rows (dequantized to the query dtype) into a compact dense cache for the
    sub-steps, optionally into the caller's buffers compact_out = (key, value), each
    [B, Hkv, >= k, D] (the session's state.key / state.value).

    A packed (k4v4) prefix is dequantized once into a contiguous bf16 copy (a per-device
    scratch) that the attention, scoring and gather passes then read, as the reference's
    pass 1 unpacks it (splitk.py:465-480; session.py:1438-1441 gathers from that read); the
    copy keeps the prefix's mask and lengths. unpack=False reads the packed prefix in place
    instead (_needs_unpack has the trade-off); either way the values read are the same
    bf16 numbers.

    probe_blocks > 0 merges the lookahead probe into this pass (lookahead_merge,
    eviction.py:125-128; session.py:1949-1960): query and the current keys/values hold
    [block | probe_blocks blocks of block_size], one attention launch covers every row,
    block-causal by block_size as the probe forward attends (session.py:2326: the block's
    rows see only its own keys, probe block i the blocks <= i), the block's selection rows
    (query_indices, positions < block_size) score and select as usual, and probe_mass is the
    prefix mass of the probe rows (positions block_size.., or the device int32 probe_rows)
    times probe_blocks (session.py:2331). That replaces the separate probe_attention pass
    over the prefix.

    fast_step0 = step0_attention, then select_step0 on its statistics.
    """
    need_stats = select or want_mass or probe_blocks > 0
    out, stats = step0_attention(query, prefix, current_key, current_value, scaling=scaling, want_stats=need_stats,
                                 unpack=unpack, probe_blocks=probe_blocks, block_size=block_size)
    if stats is None:
        return Step0Result(out, None, None, None)
    res = select_step0(query, prefix, stats, query_indices=query_indices, topk=topk, value_aware=value_aware,
                       scaling=scaling, select=select, want_mass=want_mass, gather=gather,
                       compact_out=compact_out, probe_blocks=probe_blocks, block_size=block_size,
                       probe_rows=probe_rows)
    res.out = out
    return res


def step0_attention(query: torch.Tensor, prefix, current_key: torch.Tensor, current_value: torch.Tensor, *,
                    scaling: float | None = None, want_stats: bool = True,
                    stats_out: tuple[torch.Tensor, torch.Tensor] | None = None, unpack: bool | None = None,
                    unpack_out: tuple[torch.Tensor, torch.Tensor] | None = None,
                    probe_blocks: int = 0, block_size: int = 32, head_gather=None):
    """fast_step0's attention half: the output over [live prefix | block] (block-causal by
    block_size when probe_blocks > 0 merges the probe) and, with want_stats, the prefix
    statistics stats = (M_p, L_p, O_p, prefix read) that select_step0 takes (None for an
    empty prefix or without want_stats). A packed prefix is unpacked first as fast_step0
    says (the stats then name the unpacked copy, which the next call's unpack overwrites).

    stats_out = (M_p, L_p): contiguous fp32 [B, Hkv, G*T] buffers -- one layer's slice of
    layer-stacked buffers -- that receive the statistics instead (O_p is not computed):
    the session's step-0 forward, whose selection select_step0 runs for every layer at once
    over the stacked statistics and the layer-stacked cache. unpack_out = (key, value): the
    buffers a packed prefix is unpacked into (unpacked_prefix's out), so that the
    selection can read every layer's unpacked copy. head_gather = (gather, gathered): the
    KV-head-sharded exchange of the output rows t < gathered.shape[2] in the same launch
    (splitk_attention).
    """
    prefix = as_prefix(prefix)
    if query.dtype == torch.bfloat16 and _needs_unpack(prefix, query.shape[0], current_key.shape[1], query.shape[3],
                                                         unpack):
        prefix = unpacked_prefix(prefix, query.shape[0], current_key.shape[1], query.shape[3], out=unpack_out)
    causal = block_size if probe_blocks > 0 else 0
    if prefix.n == 0:
        out, _ = splitk_attention(query, prefix, current_key, current_value, scaling=scaling, causal_block=causal,
                                  head_gather=head_gather)
        return out, None
    out, stats = splitk_attention(query, prefix, current_key, current_value, scaling=scaling, causal_block=causal,
                                  want_prefix=want_stats, stats_out=stats_out, head_gather=head_gather)
    return out, stats


def select_step0(query: torch.Tensor, prefix, stats, *, query_indices, topk: int, value_aware: bool = True,
                 scaling: float | None = None, select: bool = True, want_mass: bool = False,
                 gather: bool = False, compact_out: tuple[torch.Tensor, torch.Tensor] | None = None,
                 probe_blocks: int = 0, block_size: int = 32,
                 probe_rows: torch.Tensor | None = None) -> Step0Result:
    """The selection half of fast_step0 (session.py:1424-1454): from the step-0 prefix
    statistics stats = (M_p, L_p, ...) of splitk_attention, the mass, score, read set,
    compact cache and merged probe's mass, as fast_step0 returns them (out None).

    Several layers at once: stack them along the batch axis -- query [L*B, Hq, T, D] (the
    step-0 queries), prefix over [L*B, Hkv, n, D] (a layer-stacked cache), stats of
    [L*B, Hkv, G*T] (each layer's attention writing its slice through stats_out) and
    compact_out [L*B, Hkv, >= k, D] -- and one launch per kernel serves every layer: the
    mass of 4 KV heads at a time is a few CTAs per launch, of 28 layers' at once a wave.
    Every slot's mass is the same number either way (its sum over the rows does not depend
    on the launch), and so are the read sets up to ties of the value-aware score, whose
    head centre is summed in a launch-dependent order.
    """
    prefix = as_prefix(prefix)
    if len(stats) < 4 or stats[3] is None:
        stats = (stats[0], stats[1], None, prefix)
    probe_mass = None
    if probe_blocks > 0:
        rows = probe_rows if probe_rows is not None else list(range(block_size, query.shape[2]))
        probe_mass, _ = prefix_scores(query, prefix, stats, rows, value=False, scaling=scaling)
        probe_mass = probe_mass * probe_blocks
        if not (select or want_mass):
            return Step0Result(None, None, None, None, probe_mass=probe_mass)
    value = select and value_aware
    mass, score = prefix_scores(query, prefix, stats, query_indices, value=value, scaling=scaling)
    idx = None
    if select:
        live = prefix.n if prefix.mask is None else None
        k = int(topk) if live is None else min(int(topk), live)
        rank = score if value else mass
        idx, _ = select_topk_indices(rank, k, prefix.mask, want_values=False, lens=prefix.lens)
    compact = None
    if select and gather:
        compact = gather_read_set(stats[3], idx, dtype=query.dtype, out=compact_out)
    return Step0Result(None, idx, mass, score, compact, probe_mass)


def unpacked_prefix(prefix, batch: int, heads: int, head_dim: int, *,
                    out: tuple[torch.Tensor, torch.Tensor] | None = None) -> Prefix:
    """The prefix dequantized into contiguous bf16 [B, Hkv, n, D] K/V held in a per-device
    scratch (reused by the next call), or in out = (key, value) -- e.g. one layer's slice
    of layer-stacked buffers that a later select_step0 reads -- with the prefix's mask and
    lengths."""
    from .kernels.splitk import dequantize_prefix

    prefix = as_prefix(prefix)
    n = prefix.n
    dev = (prefix.kq if prefix.nq else prefix.kf).device
    nbytes = batch * heads * n * head_dim * 2
    if out is not None:
        kb, vb = out
        for x in (kb, vb):
            if (tuple(x.shape) != (batch, heads, n, head_dim) or x.dtype != torch.bfloat16 or not x.is_contiguous()
                    or x.device != dev):
                raise ValueError(f"out: need contiguous bfloat16 {(batch, heads, n, head_dim)} tensors on {dev}")
    else:
        kb = _lib.workspace(dev, "unpack_k", nbytes)[:nbytes].view(torch.bfloat16).view(batch, heads, n, head_dim)
        vb = _lib.workspace(dev, "unpack_v", nbytes)[:nbytes].view(torch.bfloat16).view(batch, heads, n, head_dim)
    rc = _lib.MA_ERR_UNSUPPORTED
    if n > 0 and prefix.lens is not None:
        # a ragged batch: only the slots below each sequence's length are written (every
        # consumer of the returned Prefix honours its lens)
        unmasked = Prefix(**{s: getattr(prefix, s) for s in Prefix.__slots__})
        unmasked.mask = None
        desc = kv_descriptor(unmasked, batch=batch, heads=heads, head_dim=head_dim)
        rc = _lib.lib().ma_unpack_prefix(desc.kv, batch, heads, head_dim, kb.data_ptr(), vb.data_ptr(),
                                         _lib.i64(*kb.stride()[:3]), _lib.i64(*vb.stride()[:3]),
                                         _lib.stream_handle(dev))
        if rc != _lib.MA_ERR_UNSUPPORTED:
            _lib.check("ma_unpack_prefix", rc)
    if rc == _lib.MA_ERR_UNSUPPORTED:
        dequantize_prefix(prefix, batch, heads, head_dim, out=(kb, vb))
    return Prefix(kf=kb, vf=vb, nf=n, mask=prefix.mask, lens=prefix.lens)


def gather_read_set(prefix, indices: torch.Tensor, *, dtype: torch.dtype = torch.bfloat16,
                    out: tuple[torch.Tensor, torch.Tensor] | None = None) -> Prefix:
    """The read set's K/V rows per KV head, dequantized into contiguous [B, Hkv, k, D]
    tensors -- the session's compact cache (session.py:1174-1190, 1438-1447) -- as a dense
    Prefix for compact_attention. out = (key, value) buffers of at least k rows."""
    k = indices.shape[2]
    ok = ov = None
    if out is not None:
        ok, ov = out[0][:, :, :k, :], out[1][:, :, :k, :]
    ck, cv = gather_packed_kv(prefix, indices, dtype=dtype, out_key=ok, out_value=ov)
    return Prefix.dense(ck, cv)


def compact_attention(query: torch.Tensor, prefix, indices: torch.Tensor | None, current_key: torch.Tensor,
                      current_value: torch.Tensor, *, scaling: float | None = None, head_gather=None) -> torch.Tensor:
    """Attention of every query row over [prefix[indices] | current block] (sdpa_compact
    over the gathered read set, session.py:1286-1336). indices=None: prefix is the
    compact cache itself (gather_read_set / fast_step0(gather=True)), attended as a
    contiguous dense cache; else the selected slots are read straight from the (packed or
    dense) cache by index. head_gather = (gather, gathered): with indices=None, the
    KV-head-sharded exchange of the output in the same launch (splitk_attention)."""
    if indices is None:
        out, _ = splitk_attention(query, prefix, current_key, current_value, scaling=scaling, head_gather=head_gather)
        return out
    if head_gather is not None:
        raise ValueError("head_gather: only for the compact cache (indices=None)")
    lib = _lib.lib()
    prefix = as_prefix(prefix)
    b, hq, t, d = query.shape
    hkv = current_key.shape[1]
    desc = kv_descriptor(Prefix(**{s: getattr(prefix, s) for s in Prefix.__slots__ if s != "mask"}),
                         batch=b, heads=hkv, head_dim=d)
    rows, qkeep = rows_struct(query)
    cur, ckeep = block_struct(current_key, current_value, query.dtype)
    idx = indices if indices.dtype == torch.int64 and indices.stride(-1) == 1 else indices.to(torch.int64).contiguous()
    k = idx.shape[2]
    out = torch.empty_like(query)
    nbytes = lib.ma_sparse_attention_workspace(b, hkv, (hq // hkv) * t, k, d, cur.Tc)
    ws = _lib.workspace(query.device, "attention", nbytes)
    scale = float(scaling if scaling is not None else d ** -0.5)
    _lib.check("ma_sparse_attention", lib.ma_sparse_attention(
        rows, desc.kv, hkv, idx.data_ptr(), k, _lib.i64(idx.stride(0), idx.stride(1)), cur, scale,
        out.data_ptr(), _lib.i64(*out.stride()[:3]), ws.data_ptr(), ws.numel(),
        _lib.stream_handle(query.device)))
    del qkeep, ckeep
    return out


def probe_attention(query: torch.Tensor, prefix, current_key: torch.Tensor, current_value: torch.Tensor, *,
                    block_size: int = 32, scaling: float | None = None, probe_rows: torch.Tensor | None = None,
                    unpack: bool | None = None):
    """Lookahead probe of one layer (session.py:2317-2332): block-causal attention of the
    probe forward [block k+1 | probe blocks] over [live prefix | itself], and the prefix
    mass of the probe rows (positions block_size..T) times the number of probe blocks.
    probe_rows: those positions as a device int32 tensor (optional; avoids a host copy,
    e.g. under CUDA-graph capture). unpack: as for fast_step0 (a packed prefix is unpacked
    once to bf16 first unless unpack=False)."""
    t = query.shape[2]
    prefix = as_prefix(prefix)
    if query.dtype == torch.bfloat16 and _needs_unpack(prefix, query.shape[0], current_key.shape[1], query.shape[3],
                                                         unpack):
        prefix = unpacked_prefix(prefix, query.shape[0], current_key.shape[1], query.shape[3])
    out, stats = splitk_attention(query, prefix, current_key, current_value, scaling=scaling,
                                  causal_block=block_size, q_pos0=0, c_pos0=0, want_prefix=True)
    rows = probe_rows if probe_rows is not None else list(range(block_size, t))
    if len(rows) == 0:
        return out, None
    mass, _ = prefix_scores(query, prefix, stats, rows, value=False, scaling=scaling)
    return out, mass * max(1, (t - block_size) // block_size)


def value_score(a: torch.Tensor, v: torch.Tensor, live_mask: torch.Tensor | None = None) -> torch.Tensor:
    """a_i * ||v_i - c||, c = sum_j a_j v_j / max(sum_j a_j, 1e-12), fp32 (session.py:27-40).

    a [..., n], v [..., n, D] (float32 or bfloat16). Dead slots (live_mask False) are left
    out of the centre and score 0.
    """
    lib = _lib.lib()
    lead = a.shape[:-1]
    n, d = v.shape[-2], v.shape[-1]
    a3 = a.reshape(-1, 1, n).to(torch.float32).contiguous()
    v4 = v.reshape(-1, 1, n, d)
    if v4.stride(-1) != 1:
        v4 = v4.contiguous()
    mask = None if live_mask is None else live_mask.reshape(-1, 1, n)
    desc = kv_descriptor(Prefix.dense(v4, v4, mask=mask))
    bb = a3.shape[0]
    score = torch.empty_like(a3)
    nbytes = lib.ma_value_score_workspace(bb, 1, n, d)
    ws = _lib.workspace(a.device, "value_score", nbytes)
    _lib.check("ma_value_score", lib.ma_value_score(
        desc.kv, bb, 1, d, a3.data_ptr(), _lib.i64(a3.stride(0), a3.stride(1)), score.data_ptr(),
        _lib.i64(score.stride(0), score.stride(1)), ws.data_ptr(), ws.numel(), _lib.stream_handle(a.device)))
    return score.reshape(*lead, n)


def value_score_prefix(a: torch.Tensor, prefix, *, unpack: bool | None = None) -> torch.Tensor:
    """value_score over a cache layout (dense, packed k4v4 or paged): a [B, Hkv, n] fp32,
    the values read (dequantized) from the prefix; dead slots score 0 (session.py:27-40,
    with the live values _live_values dequantizes, runtime/session.py:263-268). The
    reference's _live_values returns the values in the compute dtype (bf16): unpack=None
    (automatic) reads a packed prefix in place through the pipelined kernel's producer
    warps when it can (the same bf16 values), unpack=True dequantizes it into the bf16
    scratch of unpacked_prefix first; unpack=False reads the packed values in place with
    whichever kernel serves the layout."""
    lib = _lib.lib()
    prefix = as_prefix(prefix)
    b, h, n = a.shape
    desc = kv_descriptor(prefix, batch=b, heads=h)
    # only V is read here: in place the producer warps' dequantization replaces the unpack's
    # (cfg3 layer: 78 against 118 us)
    in_place = prefix.nq > 0 and unpack is None and lib.ma_kv_read_in_place(desc.kv, desc.head_dim) == 1
    if unpack is not False and not in_place and prefix.nq > 0 and (prefix.vf is None or
                                                                  prefix.vf.dtype == torch.bfloat16):
        prefix = unpacked_prefix(prefix, b, h, desc.head_dim)
        desc = kv_descriptor(prefix, batch=b, heads=h)
    a3 = a.to(torch.float32)
    if a3.stride(-1) != 1:
        a3 = a3.contiguous()
    score = torch.empty((b, h, n), device=a.device, dtype=torch.float32)
    nbytes = lib.ma_value_score_workspace(b, h, n, desc.head_dim)
    ws = _lib.workspace(a.device, "value_score", nbytes)
    _lib.check("ma_value_score", lib.ma_value_score(
        desc.kv, b, h, desc.head_dim, a3.data_ptr(), _lib.i64(a3.stride(0), a3.stride(1)), score.data_ptr(),
        _lib.i64(score.stride(0), score.stride(1)), ws.data_ptr(), ws.numel(), _lib.stream_handle(a.device)))
    return score


def lookahead_survivors(pos: torch.Tensor, score: torch.Tensor, capacity: int, *, recent_window: int,
                        sink_tokens: int = 0, phys: torch.Tensor | None = None) -> torch.Tensor:
    """Live-axis indices to keep [L, B, H, capacity] int64, ordered by position.

    pos [L,B,H,live] int; score [L,B,H,live] fp32 (or per physical slot [L,B,H,n_phys]
    with phys [L,B,H,live] the slot of each live entry). Keeps the
    W = min(recent_window, capacity) newest, the sinks (pos < sink_tokens) and the best
    remaining entries by score (eviction.py:364-409).
    """
    lib = _lib.lib()
    live = pos.shape[-1]
    lanes = pos.numel() // live if live else 0
    if capacity > live:
        raise ValueError(f"capacity {capacity} exceeds the live set {live}")
    p = pos.to(torch.int32).contiguous()
    s = score.to(torch.float32).contiguous()
    ph = None if phys is None else phys.to(torch.int32).contiguous()
    keep = torch.empty((*pos.shape[:-1], capacity), device=pos.device, dtype=torch.int64)
    _lib.check("ma_retain", lib.ma_retain(
        s.data_ptr(), _lib.ptr(ph), int(s.shape[-1]) if ph is not None else 0, p.data_ptr(), lanes, live,
        int(capacity), int(recent_window), int(sink_tokens), keep.data_ptr(), _lib.stream_handle(pos.device)))
    return keep
