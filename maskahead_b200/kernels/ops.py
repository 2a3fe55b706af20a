"""Operator API of the select + attend path, sm_100a kernels only.

Drop-in counterparts of src/maskahead/kernels/ops.py in the reference, with the same
signatures: ``selector_topk`` (333-521, 790-832), ``gather_packed_kv`` (570-662,
835-855), ``dense_packed_attention`` (130-264, 766-787) and the cache's quantizers
``quantize_key_groups_into`` (665-712) and ``quantize_values_into`` (715-763); plus
``sdpa_compact`` (src/maskahead/reference.py:403-426), the attention over a session's
compact buffer. ``backend``,
``kernel_variant``, ``scratch`` and ``logits_dtype`` are accepted for compatibility and
ignored: there is a single backend, logits never leave registers, and its scratch lives
in per-device workspaces. There is no CPU path: without the built library or a CUDA
device these raise ``KernelUnavailableError`` (the reference's error type, ops.py:19).
Unlike the reference overlay, ``selector_topk`` honours ``live_mask`` on its fast path.
"""

from __future__ import annotations

from dataclasses import dataclass

import torch

from .. import _lib
from .._lib import KernelUnavailableError
from ..layouts import LayerCacheView, Prefix, as_prefix, kv_descriptor
from .splitk import prefix_scores, splitk_attention

__all__ = ["KernelUnavailableError", "SelectorResult", "SelectorScratch", "selector_topk",
           "gather_packed_kv", "dense_packed_attention", "select_topk_indices", "LayerCacheView",
           "quantize_key_groups_into", "quantize_values_into", "sdpa_compact"]


@dataclass(slots=True)
class SelectorResult:
    indices: torch.Tensor
    values: torch.Tensor
    importance: torch.Tensor | None = None


class SelectorScratch:
    """Accepted for signature compatibility (ops.py:274-317); scratch is managed per device."""


def _view_heads(view) -> int:
    for name in ("k_fp", "k_q", "k_residual", "kf", "kq"):
        t = getattr(view, name, None)
        if t is not None:
            return int(t.shape[1])
    raise ValueError("cannot infer the number of KV heads from the view")


def select_topk_indices(score: torch.Tensor, k: int, live_mask: torch.Tensor | None = None,
                        want_values: bool = True, lens: torch.Tensor | None = None):
    """Top-k per (b, h) row of score [B,H,n] among live slots, as ascending indices.

    Live: live_mask (optional [B,H,n]) and slot < lens[b] (optional int32 [B], ragged
    sequences). Ties at the k-th score go to the lower slot; dead slots rank below every
    live one. Returns (indices int64 [B,H,k], values fp32 [B,H,k] | None).
    """
    lib = _lib.lib()
    if score.ndim != 3 or score.dtype != torch.float32:
        raise ValueError("score must be a float32 [B, H, n] tensor")
    b, h, n = score.shape
    if not 0 <= k <= n:
        raise ValueError(f"k={k} outside [0, {n}]")
    s = score if score.stride(-1) == 1 else score.contiguous()
    dev = s.device
    idx = torch.empty((b, h, k), device=dev, dtype=torch.int64)
    vals = torch.empty((b, h, k), device=dev, dtype=torch.float32) if want_values else None
    m = None
    if live_mask is not None:
        m = live_mask.to(torch.uint8).contiguous()
        if tuple(m.shape) != (b, h, n):
            raise ValueError("live_mask must match score")
    ln = None
    if lens is not None:
        ln = lens.to(device=dev, dtype=torch.int32).contiguous()
        if tuple(ln.shape) != (b,):
            raise ValueError("lens must be [B]")
    if k:
        _lib.check("ma_select_topk", lib.ma_select_topk(
            s.data_ptr(), b, h, n, _lib.i64(s.stride(0), s.stride(1)), _lib.ptr(m), _lib.ptr(ln), k, idx.data_ptr(),
            _lib.ptr(vals), _lib.i64(idx.stride(0), idx.stride(1)), _lib.stream_handle(dev)))
    return idx, vals


def selector_topk(query: torch.Tensor, view, *, query_indices: list[int], topk: int,
                  current_key: torch.Tensor | None = None, domain: str = "prefix",
                  score_kind: str = "softmax", sort_indices: bool = True, scaling: float | None = None,
                  backend: str = "auto", live_mask: torch.Tensor | None = None,
                  return_importance: bool = False, scratch=None, kernel_variant: str = "blocked",
                  logits_dtype: torch.dtype = torch.float16) -> SelectorResult:
    """Top-k prefix entries per KV head by mean prefix-softmax mass of the query rows.

    importance_j = mean over query heads g and rows query_indices of
    softmax_j(q . k * scale) over the live prefix (reference.py:318-366); indices are the
    top min(topk, n) by importance (dead slots never chosen), ascending.
    """
    if domain != "prefix" or score_kind != "softmax":
        raise ValueError("the sm_100a selector implements domain='prefix', score_kind='softmax' "
                         "(the fast-path selector, session.py:62-63)")
    if not query_indices:
        raise ValueError("query_indices cannot be empty")
    prefix = as_prefix(view, mask=live_mask)
    if prefix.n <= 0:
        raise ValueError("selector requires a non-empty prefix")
    hkv = _view_heads(view)
    b, hq, t, d = query.shape
    if hq % hkv:
        raise ValueError("Hq must be divisible by Hkv")
    k = min(int(topk), prefix.n)
    _, stats = splitk_attention(query, prefix, None, None, scaling=scaling, want_prefix=True)
    importance, _ = prefix_scores(query, prefix, stats, query_indices, value=False, scaling=scaling)
    idx, vals = select_topk_indices(importance, k, live_mask)
    return SelectorResult(indices=idx, values=vals, importance=importance if return_importance else None)


def gather_packed_kv(view, indices: torch.Tensor, *, dtype: torch.dtype = torch.bfloat16,
                     backend: str = "auto", out_key: torch.Tensor | None = None,
                     out_value: torch.Tensor | None = None) -> tuple[torch.Tensor, torch.Tensor]:
    """Dequantized rows of the selected slots per KV head: [B,Hkv,k,D] each (ops.py:570-662)."""
    lib = _lib.lib()
    if indices.ndim != 3:
        raise ValueError("indices must have shape [B,Hkv,K]")
    prefix = as_prefix(view)
    desc = kv_descriptor(prefix)
    b, hkv, k = indices.shape
    d = desc.head_dim
    if out_key is None:
        out_key = torch.empty((b, hkv, k, d), device=indices.device, dtype=dtype)
    if out_value is None:
        out_value = torch.empty_like(out_key)
    if tuple(out_key.shape) != (b, hkv, k, d) or tuple(out_value.shape) != (b, hkv, k, d):
        raise ValueError("output buffer has the wrong shape")
    idx = indices.to(torch.int64)
    if idx.stride(-1) != 1:
        idx = idx.contiguous()
    _lib.check("ma_gather_kv", lib.ma_gather_kv(
        desc.kv, b, hkv, d, idx.data_ptr(), k, _lib.i64(idx.stride(0), idx.stride(1)),
        out_key.data_ptr(), out_value.data_ptr(), _lib.i64(*out_key.stride()[:3]),
        _lib.i64(*out_value.stride()[:3]), _lib.dtype_code(out_key.dtype), _lib.stream_handle(indices.device)))
    return out_key, out_value


def dense_packed_attention(query: torch.Tensor, view, current_key: torch.Tensor,
                           current_value: torch.Tensor, *, scaling: float | None = None,
                           backend: str = "auto", kernel_variant: str = "blocked") -> torch.Tensor:
    """softmax over [prefix | current] per query row, GQA (ops.py:130-264)."""
    if query.ndim != 4 or current_key.ndim != 4 or current_value.ndim != 4:
        raise ValueError("Q/K/V must be rank-4 [B,H,T,D]")
    if current_key.shape != current_value.shape:
        raise ValueError("current K and V shapes differ")
    if query.shape[1] % current_key.shape[1]:
        raise ValueError("Hq must be divisible by Hkv")
    length = getattr(view, "length", None)
    prefix = as_prefix(view) if length is None or length > 0 else Prefix()
    out, _ = splitk_attention(query, prefix, current_key, current_value, scaling=scaling)
    return out


def sdpa_compact(query: torch.Tensor, key: torch.Tensor, value: torch.Tensor) -> torch.Tensor:
    """softmax(q k^T / sqrt(D)) v over every key, no mask, GQA by head groups (reference.py:
    403-426): the sub-step attention over a session's compact buffer [selected | block]."""
    if query.ndim != 4 or key.ndim != 4 or key.shape != value.shape:
        raise ValueError("Q/K/V must be rank-4 [B,H,T,D] with matching K and V")
    if query.shape[1] % key.shape[1]:
        raise ValueError("Hq must be divisible by Hkv")
    out, _ = splitk_attention(query, Prefix.dense(key, value), None, None)
    return out


def _quant_outputs(payload: torch.Tensor, scale: torch.Tensor, zero: torch.Tensor, inner: tuple[int, ...]):
    if scale.dtype != torch.float16 or zero.dtype != torch.float16 or payload.dtype != torch.uint8:
        raise KernelUnavailableError("the sm_100a quantizers write uint8 payloads with float16 scale/zero "
                                     "(quant.param_dtype = float16)")
    if scale.stride() != zero.stride():
        raise ValueError("scale and zero must share one layout")
    if scale.stride(-1) != 1 or payload.stride(-1) != 1 or payload.stride(-2) != payload.shape[-1]:
        raise ValueError("the innermost output dimensions must be contiguous")
    if tuple(payload.shape[3:]) != inner:
        raise ValueError(f"payload inner shape {tuple(payload.shape[3:])}, expected {inner}")


def _quant_source(source: torch.Tensor, bits: int, group: int, what: str) -> torch.Tensor:
    if bits != 4 or group != 32:
        raise KernelUnavailableError(f"the sm_100a quantizers implement 4-bit {what} over groups of 32 "
                                     f"(got bits={bits}, group={group})")
    if source.ndim != 4 or not source.is_cuda or source.dtype not in (torch.bfloat16, torch.float32):
        raise ValueError("source must be a bfloat16 or float32 CUDA tensor [B, H, t, D]")
    return source if source.stride(-1) == 1 else source.contiguous()


def quantize_key_groups_into(source: torch.Tensor, out_payload: torch.Tensor, out_scale: torch.Tensor,
                             out_zero: torch.Tensor, *, bits: int, token_group: int, backend: str = "auto") -> None:
    """KIVI keys: per channel over groups of token_group tokens, computed in the source's
    dtype (reference.py:58-90), into payload [B,H,t/g,D,g*bits/8] u8 and scale/zero
    [B,H,t/g,D] fp16 -- views into the cache (cache.py:499-517)."""
    lib = _lib.lib()
    x = _quant_source(source, bits, token_group, "keys")
    b, h, t, d = x.shape
    if t % token_group or tuple(out_payload.shape[:3]) != (b, h, t // token_group):
        raise ValueError("invalid key quantization output geometry")
    _quant_outputs(out_payload, out_scale, out_zero, (d, token_group * bits // 8))
    if tuple(out_scale.shape) != (b, h, t // token_group, d):
        raise ValueError("invalid key scale geometry")
    if t == 0:
        return
    _lib.check("ma_quantize_keys_channel", lib.ma_quantize_keys_channel(
        x.data_ptr(), _lib.dtype_code(x.dtype), b, h, t, d, _lib.i64(*x.stride()[:3]), token_group,
        out_payload.data_ptr(), _lib.i64(*out_payload.stride()[:3]), out_scale.data_ptr(), out_zero.data_ptr(),
        _lib.i64(*out_scale.stride()[:3]), _lib.stream_handle(x.device)))


def quantize_values_into(source: torch.Tensor, out_payload: torch.Tensor, out_scale: torch.Tensor,
                         out_zero: torch.Tensor, *, bits: int, channel_group: int, backend: str = "auto") -> None:
    """Per token over groups of channel_group channels, computed in the source's dtype
    (reference.py:182-213), into payload [B,H,t,D/g,g*bits/8] u8 and scale/zero
    [B,H,t,D/g] fp16 -- values, and token-mode keys already divided by the channel
    divisor (cache.py:482-540)."""
    lib = _lib.lib()
    x = _quant_source(source, bits, channel_group, "tokens")
    b, h, t, d = x.shape
    if d % channel_group or tuple(out_payload.shape[:3]) != (b, h, t):
        raise ValueError("invalid value quantization output geometry")
    _quant_outputs(out_payload, out_scale, out_zero, (d // channel_group, channel_group * bits // 8))
    if tuple(out_scale.shape) != (b, h, t, d // channel_group):
        raise ValueError("invalid value scale geometry")
    if t == 0:
        return
    _lib.check("ma_quantize_tokens", lib.ma_quantize_tokens(
        x.data_ptr(), _lib.dtype_code(x.dtype), b, h, t, d, _lib.i64(*x.stride()[:3]), None, None, channel_group,
        out_payload.data_ptr(), _lib.i64(*out_payload.stride()[:3]), out_scale.data_ptr(), out_zero.data_ptr(),
        _lib.i64(*out_scale.stride()[:3]), _lib.stream_handle(x.device)))
