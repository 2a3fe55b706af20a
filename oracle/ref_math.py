"""CPU restatement of the MaskAhead hot-path math (test infrastructure, see package doc).

Conventions (same as the reference):
  query          [B, Hq, T, D]     block queries; Hq = G * Hkv (GQA)
  key / value    [B, Hkv, n, D]    the prefix (dequantized to the compute dtype)
  rows           r = g * T + t     the G query heads of one KV head, then positions
All floating-point arithmetic is torch fp32 on the CPU, as in the reference's torch path.
"""

from __future__ import annotations

import math

import numpy as np
import torch

__all__ = [
    "pack_last_dim", "unpack_last_dim",
    "quantize_values", "dequantize_values", "quantize_keys", "dequantize_keys",
    "key_channel_divisor", "quantize_keys_token", "dequantize_keys_token",
    "query_indices", "selected_queries", "selector_importance",
    "value_score", "rescore_by_value", "order_keys", "topk_sorted", "topk_reference_torch",
    "dense_attention", "prefix_attention", "prefix_mass", "sdpa_compact", "gather_per_kv_head",
    "survivors_lookahead", "lookahead_score", "effective_topk",
    "pages_to_contiguous", "compact_slots", "rebuild_channel", "evict_plan",
]


# ----------------------------------------------------------------------------- packing
def pack_last_dim(q: torch.Tensor, bits: int = 4) -> torch.Tensor:
    """Codes [..., m] -> bytes [..., m*bits/8]; element i of a byte sits at bits i*bits.

    Follows reference.py:35-45 (element 2i in the low nibble for 4-bit codes).
    """
    vpb = 8 // bits
    x = q.to(torch.int16).reshape(*q.shape[:-1], q.shape[-1] // vpb, vpb)
    shifts = torch.arange(vpb, dtype=torch.int16) * bits
    return torch.sum(x << shifts, dim=-1).to(torch.uint8)


def unpack_last_dim(payload: torch.Tensor, bits: int, size: int) -> torch.Tensor:
    """Inverse of pack_last_dim (reference.py:48-55)."""
    vpb = 8 // bits
    shifts = torch.arange(vpb, dtype=torch.int16) * bits
    x = payload.to(torch.int16).unsqueeze(-1)
    q = (x >> shifts) & ((1 << bits) - 1)
    return q.reshape(*payload.shape[:-1], size).to(torch.uint8)


# ------------------------------------------------------------------------ quantization
def quantize_values(value: torch.Tensor, bits: int = 4, channel_group: int = 32,
                    param_dtype: torch.dtype = torch.float16):
    """Per-token asymmetric quantization over channel groups (reference.py:182-213).

    scale = max((max - min) / (2^bits - 1), 1e-8), zero = min, code = round((x-min)/scale)
    (torch.round: half to even). Returns payload [B,H,T,D/cg,cg*bits/8] u8, scale and
    zero [B,H,T,D/cg] in param_dtype.
    """
    b, h, t, d = value.shape
    x = value.reshape(b, h, t, d // channel_group, channel_group)
    mn = x.amin(dim=-1, keepdim=True)
    mx = x.amax(dim=-1, keepdim=True)
    scale = ((mx - mn) / float((1 << bits) - 1)).clamp_min(1e-8)
    q = torch.round((x - mn) / scale).clamp_(0, (1 << bits) - 1).to(torch.uint8)
    return (pack_last_dim(q, bits).contiguous(), scale.squeeze(-1).to(param_dtype).contiguous(),
            mn.squeeze(-1).to(param_dtype).contiguous())


def dequantize_values(payload: torch.Tensor, scale: torch.Tensor, zero: torch.Tensor, *,
                      bits: int = 4, channel_group: int = 32,
                      dtype: torch.dtype = torch.bfloat16) -> torch.Tensor:
    """x = code * f32(scale) + f32(zero), cast to dtype (reference.py:259-268)."""
    q = unpack_last_dim(payload, bits, channel_group)
    x = q.to(torch.float32) * scale.float().unsqueeze(-1) + zero.float().unsqueeze(-1)
    b, h, t, ng, cg = x.shape
    return x.reshape(b, h, t, ng * cg).to(dtype)


def quantize_keys(key: torch.Tensor, bits: int = 4, token_group: int = 32,
                  param_dtype: torch.dtype = torch.float16):
    """KIVI per-channel key quantization over token groups (reference.py:58-90).

    Returns payload [B,H,ng,D,tg*bits/8] u8 and scale/zero [B,H,ng,D].
    """
    b, h, t, d = key.shape
    ng = t // token_group
    x = key.reshape(b, h, ng, token_group, d).permute(0, 1, 2, 4, 3)
    mn = x.amin(dim=-1, keepdim=True)
    mx = x.amax(dim=-1, keepdim=True)
    scale = ((mx - mn) / float((1 << bits) - 1)).clamp_min(1e-8)
    q = torch.round((x - mn) / scale).clamp_(0, (1 << bits) - 1).to(torch.uint8)
    return (pack_last_dim(q, bits).contiguous(), scale.squeeze(-1).to(param_dtype).contiguous(),
            mn.squeeze(-1).to(param_dtype).contiguous())


def dequantize_keys(payload, scale, zero, *, bits: int = 4, token_group: int = 32,
                    dtype: torch.dtype = torch.bfloat16) -> torch.Tensor:
    """Inverse of quantize_keys (reference.py:168-179). Returns [B,H,ng*tg,D]."""
    q = unpack_last_dim(payload, bits, token_group)
    x = q.to(torch.float32) * scale.float().unsqueeze(-1) + zero.float().unsqueeze(-1)
    b, h, ng, d, tg = x.shape
    return x.permute(0, 1, 2, 4, 3).reshape(b, h, ng * tg, d).to(dtype)


def key_channel_divisor(key: torch.Tensor) -> torch.Tensor:
    """Token-mode key divisor c_i = sqrt(max_t |K_t,i|), clamped at 1e-4 before the root.

    Follows cache.py:488-490 (computed once from the first append). [B,H,D] fp32.
    """
    return key.abs().amax(dim=2).float().clamp_min(1e-4).sqrt()


def quantize_keys_token(key: torch.Tensor, kchan: torch.Tensor, bits: int = 4,
                        channel_group: int = 32, compute_dtype: torch.dtype = torch.bfloat16):
    """Token-mode keys: (K / c) in the compute dtype, then quantized like values.

    Follows cache.py:491-497.
    """
    kn = (key.float() / kchan.unsqueeze(2)).to(compute_dtype)
    return quantize_values(kn, bits=bits, channel_group=channel_group)


def dequantize_keys_token(payload, scale, zero, kchan, *, bits: int = 4, channel_group: int = 32,
                          dtype: torch.dtype = torch.bfloat16) -> torch.Tensor:
    """Token-mode key dequantization: f32(code*scale + zero) * c, one rounding to dtype.

    The reference has no CPU path for these keys (cache.py:692-715 assumes the channel
    layout); this follows its GPU unpack, splitk.py:389-395 (fp32 dequant times the
    per-channel divisor, then a single cast).
    """
    x = dequantize_values(payload, scale, zero, bits=bits, channel_group=channel_group,
                          dtype=torch.float32)
    return (x * kchan.float().unsqueeze(2)).to(dtype)


# ------------------------------------------------------------------------ selection rows
def query_indices(masked_positions, block_size: int, mode: str = "all") -> list[int]:
    """Selection rows within the block (config.py:185-203; fast path: "all" or "middle")."""
    positions = sorted(set(int(x) for x in masked_positions if 0 <= int(x) < block_size))
    if not positions:
        return []
    if mode == "all":
        return positions
    if mode == "middle":
        center = (block_size - 1) / 2.0
        return [min(positions, key=lambda x: (abs(x - center), x))]
    raise ValueError(f"selector mode {mode!r} is not on the hot path")


def selected_queries(query: torch.Tensor, qidx: list[int], hkv: int) -> torch.Tensor:
    """[B,Hq,T,D] -> [B,Hkv,G*m,D], head-major within the KV group (ops.py:320-330)."""
    b, hq, _, d = query.shape
    q = query[:, :, qidx, :].reshape(b, hkv, hq // hkv, len(qidx), d)
    return q.reshape(b, hkv, -1, d).contiguous()


def effective_topk(old_cache_len: int, topk: int = 512, topk_percent: float | None = None,
                   topk_floor: int | None = None) -> int:
    """Read budget (config.py:172-183)."""
    if old_cache_len <= 0:
        return 0
    if topk_percent is not None:
        return min(old_cache_len, max(topk_floor or 1, int(math.ceil(old_cache_len * topk_percent / 100.0))))
    return min(old_cache_len, topk)


# ------------------------------------------------------------------------------ scoring
def selector_importance(query: torch.Tensor, old_key: torch.Tensor, *, query_indices: list[int],
                        scale: float | None = None,
                        live_mask: torch.Tensor | None = None) -> torch.Tensor:
    """Mean prefix-softmax mass per prefix entry (reference.py:318-366, domain "prefix").

    logits = (q . k) * scale in fp32; dead entries -> -inf BEFORE the softmax
    (reference.py:345-348); importance_j = mean over (g, m) of softmax_j. [B,Hkv,n] fp32.
    """
    b, hq, _, d = query.shape
    hkv = old_key.shape[1]
    g = hq // hkv
    q = query[:, :, query_indices, :].reshape(b, hkv, g, len(query_indices), d)
    logits = torch.einsum("bhgmd,bhnd->bhgmn", q.float(), old_key.float())
    logits = logits * (scale if scale is not None else d ** -0.5)
    if live_mask is not None:
        logits = logits.masked_fill(~live_mask[:, :, None, None, :], float("-inf"))
    return torch.softmax(logits, dim=-1).mean(dim=(2, 3))


def value_score(a: torch.Tensor, v: torch.Tensor) -> torch.Tensor:
    """a_i * ||v_i - c||, c = sum_j a_j v_j / sum_j a_j, all fp32.

    The fp32-centre variant of session.py:27-40 (BITSIEVE_VSCORE_FP32=1 branch, 34-37).
    """
    v = v.float()
    c = (a.unsqueeze(-1) * v).sum(-2, keepdim=True) / a.sum(-1, keepdim=True).clamp_min(1e-12).unsqueeze(-1)
    return a * (v - c).norm(dim=-1)


def rescore_by_value(importance: torch.Tensor, value: torch.Tensor,
                     live_mask: torch.Tensor | None = None) -> torch.Tensor:
    """Value-aware read-set score with value_center="attn" (session.py:870-899, 935).

    w = importance (0 on dead entries), v fp32 (0 on dead entries), centre = sum w v /
    clamp(sum w, 1e-12), score = w * ||v - centre||. Dead entries rank -inf afterwards
    (session.py:940-941); that masking is left to the top-k.
    """
    n = importance.shape[-1]
    v = value[:, :, :n, :].to(torch.float32)
    w = importance.to(torch.float32)
    if live_mask is not None:
        live = live_mask[..., :n]
        w = w.masked_fill(~live, 0.0)
        v = v.masked_fill(~live.unsqueeze(-1), 0.0)
    center = (w.unsqueeze(-1) * v).sum(dim=2, keepdim=True) / w.sum(dim=-1, keepdim=True).clamp_min(1e-12).unsqueeze(-1)
    return w * (v - center).norm(dim=-1)


# ------------------------------------------------------------------------------ top-k
def order_keys(x: np.ndarray) -> np.ndarray:
    """fp32 -> uint32 keys whose unsigned order is the float order (-inf < ... < +inf)."""
    u = np.ascontiguousarray(x, dtype=np.float32).view(np.uint32)
    neg = (u >> 31).astype(bool)
    return np.where(neg, ~u, u | np.uint32(0x80000000)).astype(np.uint32)


def topk_sorted(score: torch.Tensor, k: int, live_mask: torch.Tensor | None = None):
    """Top-k per row, returned as indices sorted ascending (+ their scores).

    The reference ranks with torch.topk then sorts the indices (ops.py:377-380, 509-516;
    session.py:944-946). Its order among exactly equal scores is an artefact of the
    CPU partial sort, so this restatement fixes the rule: larger score first, and
    among equal scores the lower index first. Dead entries rank below every live entry,
    -inf included (the reference masks them to -inf, ops.py:374-380, so that they are
    never chosen while a live entry is left). Returns (indices int64 [..., k], values
    fp32 [..., k]) with the values of the live entries.
    """
    s = score.detach().to(torch.float32).contiguous()
    flat = s.reshape(-1, s.shape[-1]).numpy()
    dead = None if live_mask is None else (~live_mask).reshape(-1, s.shape[-1]).numpy()
    out_i = np.empty((flat.shape[0], k), dtype=np.int64)
    out_v = np.empty((flat.shape[0], k), dtype=np.float32)
    for row in range(flat.shape[0]):
        keys = order_keys(flat[row])
        if dead is not None:
            keys = np.where(dead[row], np.uint32(0), keys)
        # stable sort on (-key, index): lexsort uses the last key as primary
        order = np.lexsort((np.arange(keys.size), -keys.astype(np.int64)))[:k]
        order = np.sort(order)
        out_i[row] = order
        out_v[row] = flat[row][order]
    shape = (*s.shape[:-1], k)
    return torch.from_numpy(out_i).reshape(shape), torch.from_numpy(out_v).reshape(shape)


def topk_reference_torch(score: torch.Tensor, k: int, live_mask: torch.Tensor | None = None):
    """The reference's own calls: torch.topk(sorted=False) then sort (ops.py:377-380, 514-516)."""
    rank_on = score if live_mask is None else score.masked_fill(~live_mask, float("-inf"))
    values, indices = torch.topk(rank_on, k=k, dim=-1, sorted=False)
    indices, order = torch.sort(indices, dim=-1)
    return indices, torch.gather(values, -1, order)


# ---------------------------------------------------------------------------- attention
def _repeat_kv(x: torch.Tensor, hq: int) -> torch.Tensor:
    """reference.py:271-276."""
    if x.shape[1] == hq:
        return x
    return x.repeat_interleave(hq // x.shape[1], dim=1)


def dense_attention(query, old_key, old_value, current_key, current_value, *,
                    scale: float | None = None) -> torch.Tensor:
    """softmax(q [k_old|k_cur]^T * scale) [v_old|v_cur] in fp32, cast to query dtype.

    reference.py:279-296.
    """
    key = _repeat_kv(torch.cat([old_key, current_key], dim=2), query.shape[1])
    value = _repeat_kv(torch.cat([old_value, current_value], dim=2), query.shape[1])
    if scale is None:
        scale = query.shape[-1] ** -0.5
    scores = torch.matmul(query.float(), key.float().transpose(-1, -2)) * scale
    prob = torch.softmax(scores, dim=-1)
    return torch.matmul(prob, value.float()).to(query.dtype)


def prefix_attention(query, key, value, current_key, current_value, *, scale=None,
                     live_mask=None, causal_block: int = 0, q_pos0: int = 0, c_pos0: int = 0):
    """Attention over [prefix | current] plus the prefix-only softmax statistics.

    Semantics of splitk_attention (splitk.py:493-579, kernels 115-318): dead prefix
    slots (live_mask False) are never attended; with causal_block > 0 a query at
    q_pos0+t sees current key c_pos0+j only if (c_pos0+j)//cb <= (q_pos0+t)//cb.
    Returns out [B,Hq,T,D] (query dtype) and (M_p, L_p [B,Hkv,R], O_p [B,Hkv,R,D] fp32)
    over rows r = g*T + t: prefix-only max, sum of exp(s - M_p) and normalized output.
    Rows with no live prefix entry get M_p = -inf, L_p = 0, O_p = 0.
    """
    b, hq, t, d = query.shape
    hkv = key.shape[1]
    g = hq // hkv
    sc = scale if scale is not None else d ** -0.5
    q = query.float().reshape(b, hkv, g * t, d)
    s_p = torch.einsum("bhrd,bhnd->bhrn", q, key.float()) * sc
    if live_mask is not None:
        s_p = s_p.masked_fill(~live_mask[:, :, None, :], float("-inf"))
    s_c = torch.einsum("bhrd,bhnd->bhrn", q, current_key.float()) * sc
    if causal_block > 0:
        tq = (q_pos0 + torch.arange(t)) // causal_block
        tc = (c_pos0 + torch.arange(current_key.shape[2])) // causal_block
        vis = (tc[None, :] <= tq[:, None]).repeat(g, 1)           # [R, nc]
        s_c = s_c.masked_fill(~vis[None, None], float("-inf"))
    m_p = s_p.amax(dim=-1) if s_p.shape[-1] else torch.full(s_p.shape[:-1], float("-inf"))
    m_safe = torch.where(torch.isinf(m_p), torch.zeros_like(m_p), m_p)
    e_p = torch.exp(s_p - m_safe.unsqueeze(-1))
    l_p = e_p.sum(dim=-1)
    o_p = torch.einsum("bhrn,bhnd->bhrd", e_p, value.float()) / torch.where(l_p > 0, l_p, torch.ones_like(l_p)).unsqueeze(-1)
    full = torch.softmax(torch.cat([s_p, s_c], dim=-1), dim=-1)
    out = torch.einsum("bhrn,bhnd->bhrd", full, torch.cat([value.float(), current_value.float()], dim=2))
    out = out.reshape(b, hkv, g, t, d).reshape(b, hq, t, d).to(query.dtype)
    return out, (m_p, l_p, o_p)


def prefix_mass(query, key, m_p, l_p, q_rows, *, scale=None, live_mask=None) -> torch.Tensor:
    """a_j = mean over selection rows (every query head g, positions t in q_rows) of
    exp(s_rj - M_p,r) / L_p,r, with s over the prefix; dead slots get 0.

    Follows splitk.py:320-359 (pass 2 of the split-K path) and session.py:2326-2331.
    """
    b, hq, t, d = query.shape
    hkv = key.shape[1]
    g = hq // hkv
    sc = scale if scale is not None else d ** -0.5
    rows = (torch.arange(g).unsqueeze(1) * t + torch.as_tensor(list(q_rows)).unsqueeze(0)).reshape(-1)
    q = query.float().reshape(b, hkv, g * t, d)[:, :, rows]
    s = torch.einsum("bhrd,bhnd->bhrn", q, key.float()) * sc
    mp = m_p[:, :, rows]
    lp = l_p[:, :, rows]
    p = torch.exp(s - mp.unsqueeze(-1)) / torch.where(lp > 0, lp, torch.ones_like(lp)).unsqueeze(-1)
    a = p.mean(dim=2)
    if live_mask is not None:
        a = a.masked_fill(~live_mask, 0.0)
    return a


def sdpa_compact(query, key, value) -> torch.Tensor:
    """SDPA over a compact [selected | current] buffer with GQA (reference.py:403-426)."""
    return torch.nn.functional.scaled_dot_product_attention(
        query, _repeat_kv(key, query.shape[1]), _repeat_kv(value, query.shape[1]),
        attn_mask=None, dropout_p=0.0, is_causal=False)


def gather_per_kv_head(x: torch.Tensor, indices: torch.Tensor) -> torch.Tensor:
    """x [B,H,n,D], indices [B,H,k] -> [B,H,k,D] (reference.py:396-400)."""
    gi = indices.unsqueeze(-1).expand(*indices.shape, x.shape[-1])
    return torch.gather(x, 2, gi)


# ----------------------------------------------------------------------------- retention
def lookahead_score(a1: torch.Tensor, a_probe: torch.Tensor | None, v_live: torch.Tensor) -> torch.Tensor:
    """score = value_score(a1 + a_probe, v) on the live axis (session.py:2011-2025)."""
    a = a1 if a_probe is None else a1 + a_probe
    return value_score(a, v_live)


def survivors_lookahead(pos: torch.Tensor, score: torch.Tensor, capacity: int, *,
                        recent_window: int, sink_tokens: int = 0) -> torch.Tensor:
    """Live-axis indices to keep, [L,B,H,capacity] int64, sorted by position.

    Follows EvictionState.survivors for the lookahead policy (eviction.py:364-409):
    the W = min(recent_window, C) newest by position are kept; sinks (pos < sink_tokens)
    rank +inf; the window ranks -inf in the contest for the other C - W slots; the
    union is ordered by position. Ranking ties use the rule of topk_sorted.
    """
    live = pos.shape[-1]
    w = min(recent_window, capacity)
    lanes = pos.reshape(-1, live).numpy().astype(np.int64)
    sc = score.reshape(-1, live).to(torch.float32).numpy()
    keep = np.empty((lanes.shape[0], capacity), dtype=np.int64)
    for i in range(lanes.shape[0]):
        p = lanes[i]
        recent = np.argsort(-p, kind="stable")[:w] if w else np.empty(0, dtype=np.int64)
        rest = capacity - w
        chosen = recent
        if rest > 0:
            rank = sc[i].copy()
            if sink_tokens:
                rank[p < sink_tokens] = np.inf
            rank[recent] = -np.inf
            keys = order_keys(rank)
            extra = np.lexsort((np.arange(live), -keys.astype(np.int64)))[:rest]
            chosen = np.concatenate([recent, extra])
        keep[i] = chosen[np.argsort(p[chosen], kind="stable")]
    return torch.from_numpy(keep).reshape(*pos.shape[:-1], capacity)


# -------------------------------------------------------------------------- paged layout
def pages_to_contiguous(pool: torch.Tensor, page_table: torch.Tensor, length: int,
                        page_size: int) -> torch.Tensor:
    """Gather one sequence's pages into a contiguous [H, length, ...] tensor.

    pool [P, H, page_size, ...]; page_table [max_pages] int32 (logical page -> pool
    page). The reference has no paged layout; this is the restatement the paged
    kernels are checked against (contiguous equivalent, then the oracle per sequence).
    """
    npages = (length + page_size - 1) // page_size
    pages = pool[page_table[:npages].long()]                       # [np, H, ps, ...]
    x = pages.transpose(0, 1).reshape(pool.shape[1], npages * page_size, *pool.shape[3:])
    return x[:, :length]


# ------------------------------------------------------------------ compaction (eviction)
def compact_slots(t: torch.Tensor, keep: torch.Tensor, slot_dim: int = 2) -> torch.Tensor:
    """Slots keep[..., j] of t, in keep's order, for every trailing element of a slot.

    Restates PackedKVCache.compact_tokens (cache.py:659-678: ``t.gather(3, idx)`` over
    [L, B, H, slot, ...] for each stored array) and the gather of PackedKVCache.compact
    (cache.py:342-365: bf16 survivors re-staged unchanged). keep has t's leading
    dimensions up to the slot axis; an index outside [0, n) gives a zero row (the
    device kernel's convention, where the reference's gather raises)."""
    n = t.shape[slot_dim]
    k = keep.to(torch.int64)
    bad = (k < 0) | (k >= n)
    safe = k.clamp(0, max(n - 1, 0))
    idx = safe.reshape(*safe.shape, *([1] * (t.dim() - slot_dim - 1))).expand(*safe.shape, *t.shape[slot_dim + 1:])
    out = t.gather(slot_dim, idx)
    if bool(bad.any()):
        out = out.masked_fill(bad.reshape(*bad.shape, *([1] * (t.dim() - slot_dim - 1))), 0)
    return out


def rebuild_channel(arrays: dict, groups_before: torch.Tensor, encode: torch.Tensor,
                    groups_after: torch.Tensor, stage: torch.Tensor, token_group: int = 32) -> tuple[dict, torch.Tensor]:
    """The group-preserving rebuild of a KIVI channel-mode k4v4 cache (cache.py:236-335).

    arrays: k_q [B,H,ng,D,16], k_scale/k_zero [B,H,ng,D], v_q [B,H,ql,D/32,16],
    v_scale/v_zero [B,H,ql,D/32], k_residual/v_residual [B,H,rl,D] (bf16). Index tensors
    [B,H,*] padded with -1; a padded entry copies group / slot 0 (clamp at 0) or is zero,
    as in the reference. Returns the new arrays over the regions the rebuild defines
    (groups [0, g1+g2+g3), value slots [0, ql'), residual [0, st)) and remap [B,H,old_len].
    """
    gk = token_group
    kq, ks, kz = arrays["k_q"], arrays["k_scale"], arrays["k_zero"]
    vq, vs, vz = arrays["v_q"], arrays["v_scale"], arrays["v_zero"]
    kr, vr = arrays["k_residual"], arrays["v_residual"]
    B, H = kq.shape[:2]
    ql_old, rl = vq.shape[2], kr.shape[2]
    old_len = ql_old + rl
    g1, m, g3, st = (t.shape[-1] for t in (groups_before, encode, groups_after, stage))
    g2 = -(-m // gk)
    ql = (g1 + g2 + g3) * gk
    keys = torch.cat([dequantize_keys(kq, ks, kz, token_group=gk, dtype=kr.dtype), kr], 2)
    vals = torch.cat([dequantize_values(vq, vs, vz, dtype=vr.dtype), vr], 2)
    remap = torch.full((B, H, old_len + 1), -1, dtype=torch.int64)
    ar = torch.arange(gk)
    parts = {name: [] for name in ("k_q", "k_scale", "k_zero", "v_q", "v_scale", "v_zero")}

    def copy_groups(gid, at):
        n = gid.shape[-1]
        safe = gid.clamp_min(0)
        tok = (safe.unsqueeze(-1) * gk + ar).reshape(B, H, n * gk)
        for name, src, idx in (("k_q", kq, safe), ("k_scale", ks, safe), ("k_zero", kz, safe),
                               ("v_q", vq, tok), ("v_scale", vs, tok), ("v_zero", vz, tok)):
            parts[name].append(compact_slots(src, idx))
        new_slot = ((torch.arange(n) + at).view(1, 1, n, 1) * gk + ar).expand(B, H, n, gk)
        valid = (gid >= 0).unsqueeze(-1).expand(-1, -1, -1, gk)
        idx = torch.where(valid, tok.view(B, H, n, gk), old_len)
        remap.scatter_(-1, idx.reshape(B, H, -1), new_slot.reshape(B, H, -1))

    copy_groups(groups_before, 0)
    safe = encode.clamp_min(0)
    dead = (encode < 0).unsqueeze(-1)
    pad = g2 * gk - m
    src_k = torch.nn.functional.pad(compact_slots(keys, safe).masked_fill(dead, 0), (0, 0, 0, pad))
    src_v = torch.nn.functional.pad(compact_slots(vals, safe).masked_fill(dead, 0), (0, 0, 0, pad))
    for name, t in zip(("k_q", "k_scale", "k_zero"), quantize_keys(src_k, token_group=gk)):
        parts[name].append(t)
    for name, t in zip(("v_q", "v_scale", "v_zero"), quantize_values(src_v)):
        parts[name].append(t)
    remap.scatter_(-1, torch.where(encode >= 0, encode, old_len),
                   torch.arange(m).view(1, 1, m).expand(B, H, m) + g1 * gk)
    copy_groups(groups_after, g1 + g2)
    safe = stage.clamp_min(0)
    dead = (stage < 0).unsqueeze(-1)
    out = {name: torch.cat(ts, 2) for name, ts in parts.items()}
    out["k_residual"] = compact_slots(keys, safe).masked_fill(dead, 0)
    out["v_residual"] = compact_slots(vals, safe).masked_fill(dead, 0)
    remap.scatter_(-1, torch.where(stage >= 0, stage, old_len), torch.arange(st).view(1, 1, st).expand(B, H, st) + ql)
    return out, remap[..., :old_len]


# ----------------------------------------------------------------- eviction planning
def evict_plan(phys: torch.Tensor, pos: torch.Tensor, *, quantized_length: int, token_group: int = 32,
               repack_below: float = 1.0, compaction: str = "lazy", recent_window: int = 64,
               tail: int = 0, tail_stage: bool = False, cache_length: int | None = None):
    """The index lists of a group-preserving rebuild after an eviction decision.

    Restates the planning part of BitSieveSession._evict_to for a channel-mode packed cache
    (session.py:303-356): phys / pos [L,B,H,live] are the live entries' physical slots and
    positions (after EvictionState.compact). A key group with at least
    max(1, ceil(repack_below * gk)) live entries is kept whole ("lazy"; none with
    "full"), except the unadmitted tail's groups; staged entries (slot >= ql) among the
    recent_window newest positions stay staged; every other live entry is re-encoded.
    Returns (groups_before, encode, groups_after, stage) as [L,B,H,*] int64 padded with -1
    to the largest count over lanes -- the arguments of PackedKVCache.rebuild. Encoded and
    staged slots are ordered by position (then slot); the tail's slots are staged after
    the others (cache.stage) or its groups placed after everything (tail_groups).
    """
    gk, ql = token_group, quantized_length
    phys = phys.to(torch.int64)
    posl = pos.to(torch.int64)
    L, B, H, live = phys.shape
    in_q = phys < ql
    ng = max(1, ql // gk)
    grp = torch.where(in_q, phys // gk, torch.full_like(phys, ng))
    counts = torch.zeros((L, B, H, ng + 1), dtype=torch.int64)
    counts.scatter_add_(-1, grp, torch.ones_like(grp))
    counts = counts[..., :ng]
    if compaction == "lazy":
        need = max(1, int(math.ceil(repack_below * gk)))
        keep_g = counts >= need
    else:
        keep_g = torch.zeros_like(counts, dtype=torch.bool)
    tail_groups = 0
    if tail and not tail_stage:
        tail_groups = tail // gk
        keep_g[..., ng - tail_groups:] = False
    in_kept = in_q & keep_g.gather(-1, grp.clamp_max(ng - 1)) & (grp < ng)
    w = min(recent_window, live)
    if w:
        thr = posl.topk(w, dim=-1).values.amin(-1, keepdim=True)
    else:
        thr = torch.full((L, B, H, 1), 1 << 60, dtype=torch.int64)
    undecided = ~in_q & (posl >= thr)
    encode = ~in_kept & ~undecided
    big = 1 << 62

    def packed(sel, key):
        n = int(sel.sum(-1).max().item()) if sel.numel() else 0
        k2 = torch.where(sel, key, big).sort(dim=-1).values[..., :n]
        return torch.where(k2 >= big, -1, k2)

    def slots_by_pos(sel):
        k2 = packed(sel, posl * (1 << 24) + phys)
        return torch.where(k2 < 0, -1, k2 % (1 << 24))

    groups_before = packed(keep_g, torch.arange(ng).expand(L, B, H, ng))
    enc = slots_by_pos(encode)
    stage = slots_by_pos(undecided)
    empty = torch.empty((L, B, H, 0), dtype=torch.int64)
    groups_after = empty
    if tail and tail_stage:
        tail_slots = torch.arange(cache_length - tail, cache_length).view(1, 1, 1, -1).expand(L, B, H, tail)
        stage = torch.cat([stage, tail_slots], -1)
    elif tail:
        groups_after = torch.arange(ng - tail_groups, ng).expand(L, B, H, -1)
    return groups_before, enc, groups_after, stage
