"""Cache views and their translation to the C ABI's ``ma_kv`` descriptor.

``LayerCacheView`` has the fields of the reference's view (src/maskahead/cache.py:37-61)
and ``Prefix`` the fields of its split-K prefix (src/maskahead/kernels/splitk.py:
408-462), so objects built by the reference cache can be passed in unchanged (any
object with these attributes works). Layouts (cache.py:142-189):

  bf16/fp32     k_fp, v_fp            [B, H, cap, D]
  packed V      v_q [B,H,cap,D/32,16] u8, v_scale / v_zero [B,H,cap,D/32] fp16
  token keys    k_q, k_scale, k_zero as V, plus k_chan [B,H,D] fp32
  channel keys  k_q [B,H,ng,D,16] u8, k_scale / k_zero [B,H,ng,D] fp16  (KIVI)
  tail          k_residual, v_residual [B, H, rcap, D] bf16

Paged storage (no counterpart in the reference; the serving batch uses it): the packed
part (or a dense cache) is a pool of pages whose first axis is the page instead of the
sequence -- e.g. v_q [P, H, page_size, D/32, 16] -- and ``pages`` [B, max_pages] int32
maps each sequence's logical page to a pool page; ``lens`` [B] int32 gives each
sequence's live length (ragged batches).
"""

from __future__ import annotations

import math
from dataclasses import dataclass

import torch

from . import _lib
from ._lib import MaKV, i64


@dataclass(slots=True)
class LayerCacheView:
    k_bits: int
    v_bits: int
    length: int
    quantized_length: int
    residual_length: int
    key_token_group: int
    value_channel_group: int
    k_q: torch.Tensor | None
    k_scale: torch.Tensor | None
    k_zero: torch.Tensor | None
    v_q: torch.Tensor | None
    v_scale: torch.Tensor | None
    v_zero: torch.Tensor | None
    k_fp: torch.Tensor | None
    v_fp: torch.Tensor | None
    k_residual: torch.Tensor | None
    v_residual: torch.Tensor | None
    head_dim: int | None = None
    key_mode: str = "channel"
    k_chan: torch.Tensor | None = None


class Prefix:
    """The prefix a kernel reads: packed (+ bf16 tail) or plain dense. [B, Hkv, n, D]."""

    __slots__ = ("kq", "ks", "kz", "vq", "vs", "vz", "kf", "vf", "nq", "nf", "kb", "vb", "kg", "vg", "mask",
                 "kmode", "kch", "pages", "page_size", "lens")

    def __init__(self, *, kq=None, ks=None, kz=None, vq=None, vs=None, vz=None, kf=None, vf=None,
                 nq=0, nf=0, kb=16, vb=16, kg=32, vg=32, mask=None, kmode=0, kch=None, pages=None,
                 page_size=0, lens=None):
        self.mask = mask          # optional uint8/bool [B, Hkv, n]: 0 = dead slot, never attended
        self.kmode, self.kch = kmode, kch    # kmode 1: per-token keys with divisor kch [B, Hkv, D]
        self.pages, self.page_size = pages, int(page_size)   # optional page table [B, max_pages] int32
        self.lens = lens          # optional live length per sequence [B] int32
        self.kq, self.ks, self.kz, self.vq, self.vs, self.vz = kq, ks, kz, vq, vs, vz
        self.kf, self.vf, self.nq, self.nf = kf, vf, int(nq), int(nf)
        self.kb, self.vb, self.kg, self.vg = kb, vb, kg, vg

    @property
    def n(self) -> int:
        return self.nq + self.nf

    @classmethod
    def from_view(cls, view) -> "Prefix":
        """splitk.py:427-436."""
        if view.k_bits == 16 and view.v_bits == 16:
            return cls(kf=view.k_fp, vf=view.v_fp, nf=view.length)
        if view.k_bits == 16 or view.v_bits == 16:
            raise NotImplementedError("mixed 16-bit / packed K,V")
        return cls(kq=view.k_q, ks=view.k_scale, kz=view.k_zero, vq=view.v_q, vs=view.v_scale, vz=view.v_zero,
                   kf=view.k_residual, vf=view.v_residual, nq=view.quantized_length, nf=view.residual_length,
                   kb=view.k_bits, vb=view.v_bits, kg=view.key_token_group, vg=view.value_channel_group,
                   kmode=1 if getattr(view, "key_mode", "channel") == "token" else 0,
                   kch=getattr(view, "k_chan", None))

    @classmethod
    def dense(cls, key: torch.Tensor, value: torch.Tensor, mask=None) -> "Prefix":
        return cls(kf=key, vf=value, nf=key.shape[2], mask=mask)


def as_prefix(view_or_prefix, mask=None) -> Prefix:
    if isinstance(view_or_prefix, Prefix):
        p = view_or_prefix
    elif hasattr(view_or_prefix, "k_bits"):
        p = Prefix.from_view(view_or_prefix)
    elif hasattr(view_or_prefix, "nq") and hasattr(view_or_prefix, "kf"):
        # another Prefix class with these fields (the reference's has no pages / lens)
        p = Prefix(**{s: getattr(view_or_prefix, s) for s in Prefix.__slots__ if hasattr(view_or_prefix, s)})
    else:
        raise TypeError(f"expected a LayerCacheView or Prefix, got {type(view_or_prefix).__name__}")
    if mask is not None:
        p = Prefix(**{s: getattr(p, s) for s in Prefix.__slots__})
        p.mask = mask
    return p


class KVDesc:
    """A filled ``ma_kv`` plus the tensors it points into (kept alive with it)."""

    def __init__(self, kv: MaKV, keep: list, device: torch.device, batch: int, heads: int, head_dim: int,
                 n: int):
        self.kv, self.keep, self.device = kv, keep, device
        self.batch, self.heads, self.head_dim, self.n = batch, heads, head_dim, n


def _inner_contig(t: torch.Tensor, dims: int, name: str) -> None:
    """The last `dims` dimensions must be densely packed (row-major)."""
    expect = 1
    for d in range(t.ndim - 1, t.ndim - 1 - dims, -1):
        if t.shape[d] > 1 and t.stride(d) != expect:
            raise ValueError(f"{name}: the innermost {dims} dimension(s) must be contiguous")
        expect *= t.shape[d]


def _strides3(t: torch.Tensor) -> tuple[int, int, int]:
    return t.stride(0), t.stride(1), t.stride(2)


def kv_descriptor(prefix: Prefix, *, batch: int | None = None, heads: int | None = None,
                  head_dim: int | None = None) -> KVDesc:
    """Translate a Prefix into the C descriptor; validates layouts (ValueError)."""
    kv = MaKV()
    keep: list = []
    dense_src = prefix.kf if prefix.kf is not None else prefix.kq
    if dense_src is None:
        raise ValueError("empty prefix: neither dense nor packed tensors given")
    device = dense_src.device
    kv.nq, kv.nf = int(prefix.nq), int(prefix.nf)
    kv.kgroup, kv.vgroup = int(prefix.kg), int(prefix.vg)
    paged = prefix.pages is not None
    if prefix.nq:
        if prefix.kb != 4 or prefix.vb != 4:
            raise NotImplementedError("packed caches: the kernels read 4-bit keys and values")
        kv.layout = _lib.MA_KV_PACKED_TOKEN if prefix.kmode == 1 else _lib.MA_KV_PACKED_CHANNEL
        B, H = prefix.vq.shape[0], prefix.vq.shape[1]
        pool = prefix.vq.shape[0]
        D = prefix.vq.shape[3] * prefix.vq.shape[4] * 2
        for name in ("kq", "vq"):
            t = getattr(prefix, name)
            if t.dtype != torch.uint8 or t.ndim != 5:
                raise ValueError(f"{name} must be a rank-5 uint8 tensor")
            _inner_contig(t, 2, name)
        for name in ("ks", "kz", "vs", "vz"):
            t = getattr(prefix, name)
            if t.dtype != torch.float16 or t.ndim != 4:
                raise ValueError(f"{name} must be a rank-4 float16 tensor (param_dtype float16)")
            _inner_contig(t, 1, name)
        if prefix.ks.stride() != prefix.kz.stride() or prefix.vs.stride() != prefix.vz.stride():
            raise ValueError("scale and zero tensors must share strides")
        kv.kq, kv.vq = prefix.kq.data_ptr(), prefix.vq.data_ptr()
        kv.ks, kv.kz = prefix.ks.data_ptr(), prefix.kz.data_ptr()
        kv.vs, kv.vz = prefix.vs.data_ptr(), prefix.vz.data_ptr()
        kv.skq, kv.sks = i64(*_strides3(prefix.kq)), i64(*_strides3(prefix.ks))
        kv.svq, kv.svs = i64(*_strides3(prefix.vq)), i64(*_strides3(prefix.vs))
        keep += [prefix.kq, prefix.ks, prefix.kz, prefix.vq, prefix.vs, prefix.vz]
        if prefix.kmode == 1:
            if prefix.kch is None:
                raise ValueError("token-mode keys need k_chan")
            kch = prefix.kch
            if kch.dtype != torch.float32 or kch.stride(-1) != 1:
                raise ValueError("k_chan must be float32 with a contiguous channel axis")
            kv.kchan, kv.skc = kch.data_ptr(), i64(kch.stride(0), kch.stride(1))
            keep.append(kch)
        kv.dtype = _lib.MA_BF16
        if prefix.nf:
            kv.dtype = _lib.dtype_code(prefix.kf.dtype)
    else:
        kv.layout = _lib.MA_KV_DENSE
        B, H, D = prefix.kf.shape[0], prefix.kf.shape[1], prefix.kf.shape[3]
        pool = prefix.kf.shape[0]
        kv.dtype = _lib.dtype_code(prefix.kf.dtype)
    if paged:
        pt = prefix.pages
        if pt.dtype != torch.int32 or pt.ndim != 2 or pt.stride(1) != 1:
            raise ValueError("pages must be an int32 [B, max_pages] tensor with a contiguous page axis")
        if prefix.page_size <= 0:
            raise ValueError("paged prefixes need page_size")
        B = pt.shape[0]
        kv.pages, kv.spg, kv.page_size, kv.num_pages = pt.data_ptr(), pt.stride(0), prefix.page_size, pool
        keep.append(pt)
    if prefix.lens is not None:
        ln = prefix.lens
        if ln.dtype != torch.int32 or tuple(ln.shape) != (B,) or ln.stride(0) != 1:
            raise ValueError("lens must be a contiguous int32 [B] tensor")
        kv.lens = ln.data_ptr()
        keep.append(ln)
    if prefix.nf:
        for name in ("kf", "vf"):
            t = getattr(prefix, name)
            if t.ndim != 4 or t.stride(-1) != 1:
                raise ValueError(f"{name} must be rank 4 with a contiguous head_dim")
            if t.dtype != prefix.kf.dtype:
                raise ValueError("dense K and V must share a dtype")
        kv.kf, kv.vf = prefix.kf.data_ptr(), prefix.vf.data_ptr()
        kv.skf, kv.svf = i64(*_strides3(prefix.kf)), i64(*_strides3(prefix.vf))
        keep += [prefix.kf, prefix.vf]
    if prefix.mask is not None:
        m = prefix.mask
        if m.dtype == torch.bool:
            m = m.to(torch.uint8)
        m = m.contiguous()
        if tuple(m.shape) != (B, H, prefix.n):
            raise ValueError(f"mask must be [B, Hkv, n] = {(B, H, prefix.n)}, got {tuple(m.shape)}")
        kv.mask = m.data_ptr()
        keep.append(m)
    if batch is not None and batch != B or heads is not None and heads != H:
        raise ValueError("prefix batch/heads do not match the query")
    if head_dim is not None and head_dim != D:
        raise ValueError("prefix head_dim does not match the query")
    return KVDesc(kv, keep, device, B, H, D, prefix.n)


# ------------------------------------------------------------------- quantize-on-append
def _check_rows(x: torch.Tensor, name: str) -> None:
    if x.ndim != 4 or x.stride(-1) != 1:
        raise ValueError(f"{name} must be rank 4 [B, H, n, D] with a contiguous head_dim")
    if x.dtype not in (torch.bfloat16, torch.float32):
        raise ValueError(f"{name} must be bfloat16 or float32")


def key_divisor(key: torch.Tensor) -> torch.Tensor:
    """Token-mode key divisor sqrt(max(max_t |K|, 1e-4)) per (b, h, channel), fp32
    [B, H, D] (cache.py:488-490)."""
    _check_rows(key, "key")
    lib = _lib.lib()
    b, h, n, d = key.shape
    out = torch.empty((b, h, d), device=key.device, dtype=torch.float32)
    _lib.check("ma_key_divisor", lib.ma_key_divisor(
        key.data_ptr(), _lib.dtype_code(key.dtype), b, h, n, d, i64(*_strides3(key)), out.data_ptr(),
        i64(out.stride(0), out.stride(1)), _lib.stream_handle(key.device)))
    return out


def quantize_tokens(x: torch.Tensor, kchan: torch.Tensor | None = None, group: int = 32):
    """Per-token 4-bit quantization over groups of 32 channels, computed in x's dtype as
    the reference does (reference.py:182-213; token-mode keys x / kchan first, cache.py:
    491-497). Returns payload [B,H,n,D/32,16] u8, scale and zero [B,H,n,D/32] fp16."""
    _check_rows(x, "x")
    lib = _lib.lib()
    b, h, n, d = x.shape
    pay = torch.empty((b, h, n, d // group, group // 2), device=x.device, dtype=torch.uint8)
    sc = torch.empty((b, h, n, d // group), device=x.device, dtype=torch.float16)
    zr = torch.empty_like(sc)
    kc = None
    if kchan is not None:
        kc = kchan.to(torch.float32)
        if kc.stride(-1) != 1:
            kc = kc.contiguous()
    _lib.check("ma_quantize_tokens", lib.ma_quantize_tokens(
        x.data_ptr(), _lib.dtype_code(x.dtype), b, h, n, d, i64(*_strides3(x)), _lib.ptr(kc),
        i64(kc.stride(0), kc.stride(1)) if kc is not None else None, group, pay.data_ptr(), i64(*_strides3(pay)),
        sc.data_ptr(), zr.data_ptr(), i64(*_strides3(sc)), _lib.stream_handle(x.device)))
    return pay, sc, zr


def quantize_keys_channel(key: torch.Tensor, group: int = 32):
    """KIVI per-channel 4-bit key quantization over groups of 32 tokens (reference.py:
    58-90). Returns payload [B,H,n/32,D,16] u8, scale and zero [B,H,n/32,D] fp16."""
    _check_rows(key, "key")
    lib = _lib.lib()
    b, h, n, d = key.shape
    ng = n // group
    pay = torch.empty((b, h, ng, d, group // 2), device=key.device, dtype=torch.uint8)
    sc = torch.empty((b, h, ng, d), device=key.device, dtype=torch.float16)
    zr = torch.empty_like(sc)
    _lib.check("ma_quantize_keys_channel", lib.ma_quantize_keys_channel(
        key.data_ptr(), _lib.dtype_code(key.dtype), b, h, n, d, i64(*_strides3(key)), group, pay.data_ptr(),
        i64(*_strides3(pay)), sc.data_ptr(), zr.data_ptr(), i64(*_strides3(sc)), _lib.stream_handle(key.device)))
    return pay, sc, zr


def pack_prefix(key: torch.Tensor, value: torch.Tensor, *, key_mode: str = "token", group: int = 32,
                kchan: torch.Tensor | None = None) -> Prefix:
    """A fully packed k4v4 prefix from dense K/V [B, H, n, D] on the device: values per
    token, keys per token (with the divisor, computed from K unless given) or per
    channel (KIVI)."""
    vq, vs, vz = quantize_tokens(value, group=group)
    n = key.shape[2]
    if key_mode == "token":
        kch = key_divisor(key) if kchan is None else kchan
        kq, ks, kz = quantize_tokens(key, kch, group=group)
        return Prefix(kq=kq, ks=ks, kz=kz, vq=vq, vs=vs, vz=vz, nq=n, kb=4, vb=4, kg=group, vg=group, kmode=1,
                      kch=kch)
    if key_mode == "channel":
        kq, ks, kz = quantize_keys_channel(key, group=group)
        return Prefix(kq=kq, ks=ks, kz=kz, vq=vq, vs=vs, vz=vz, nq=n, kb=4, vb=4, kg=group, vg=group, kmode=0)
    raise ValueError(f"key_mode must be 'token' or 'channel', got {key_mode!r}")


# ------------------------------------------------------------ compaction after eviction
def compact_tokens(prefix, keep: torch.Tensor, out: Prefix | None = None) -> Prefix:
    """Move the kept slots of a cache to the front: slot j of the result holds slot
    keep[b, h, j] of ``prefix``, every array moved bit-exactly (cache.py:659-678
    compact_tokens for token-mode packed caches; cache.py:342-365 compact for dense
    bf16/fp32 caches). keep [B, H, C] int64 physical slots. Out of place: the result goes
    to ``out`` (a Prefix of the same layout with at least C slots, whose arrays do not
    overlap the source's) or to new tensors of C slots. Channel-mode keys, paged storage
    and a packed cache with a dense tail raise (the reference requires a fully quantized
    cache, cache.py:662-663). The result carries no mask: every slot below C is live."""
    src = as_prefix(prefix)
    if keep.ndim != 3:
        raise ValueError("keep must have shape [B, H, C]")
    if src.pages is not None:
        raise NotImplementedError("compaction of paged storage")
    if src.nq and src.kmode != 1:
        raise NotImplementedError("channel-mode keys are rebuilt by key groups (cache.py:236-335)")
    if src.nq and src.nf:
        raise RuntimeError("compact_tokens needs a fully quantized cache")
    b, h, c = keep.shape
    if c > src.n:
        raise ValueError("compact cannot grow the cache")
    if out is None:
        def like(t):
            return torch.empty((b, h, c, *t.shape[3:]), device=t.device, dtype=t.dtype)
        if src.nq:
            out = Prefix(kq=like(src.kq), ks=like(src.ks), kz=like(src.kz), vq=like(src.vq), vs=like(src.vs),
                         vz=like(src.vz), nq=c, kb=src.kb, vb=src.vb, kg=src.kg, vg=src.vg, kmode=1, kch=src.kch)
        else:
            out = Prefix(kf=like(src.kf), vf=like(src.vf), nf=c)
    sdesc = kv_descriptor(Prefix(**{s: getattr(src, s) for s in Prefix.__slots__ if s not in ("mask", "lens")}))
    ddesc = kv_descriptor(out)
    if (sdesc.batch, sdesc.heads) != (b, h) or (ddesc.batch, ddesc.heads) != (b, h):
        raise ValueError("keep, source and destination disagree on [B, H]")
    idx = keep.to(torch.int64)
    if idx.stride(-1) != 1:
        idx = idx.contiguous()
    lib = _lib.lib()
    _lib.check("ma_compact_tokens", lib.ma_compact_tokens(
        sdesc.kv, ddesc.kv, b, h, sdesc.head_dim, idx.data_ptr(), c, i64(idx.stride(0), idx.stride(1)),
        _lib.stream_handle(keep.device)))
    if out.nq:
        out.nq = c
    else:
        out.nf = c
    return out


def _gather_rows_into(desc: KVDesc, slots: torch.Tensor, out_k: torch.Tensor, out_v: torch.Tensor) -> None:
    """out_k/out_v [B, H, k, D] bf16 <- the dequantized slots[b, h, :] of the cache (ma_gather_kv)."""
    b, h, k = slots.shape
    if k == 0:
        return
    _lib.check("ma_gather_kv", _lib.lib().ma_gather_kv(
        desc.kv, b, h, desc.head_dim, slots.data_ptr(), k, i64(slots.stride(0), slots.stride(1)),
        out_k.data_ptr(), out_v.data_ptr(), i64(*out_k.stride()[:3]), i64(*out_v.stride()[:3]),
        _lib.dtype_code(out_k.dtype), _lib.stream_handle(slots.device)))


def rebuild(prefix, groups_before: torch.Tensor, encode: torch.Tensor, groups_after: torch.Tensor,
            stage: torch.Tensor) -> tuple[Prefix, torch.Tensor]:
    """The group-preserving rebuild of a KIVI channel-mode k4v4 cache after an eviction
    (PackedKVCache.rebuild, cache.py:236-335), on the device.

    New physical layout [groups_before | encoded | groups_after] + a bf16 residual. The
    index tensors are [B, H, *] int64 padded with -1 (a padded entry is dead: it holds a
    copy of group / slot 0 or zeros, as in the reference, and the caller masks it):
    groups_before / groups_after are old key groups whose codes and scales of keys and
    values move bit-exactly (one compaction launch each); encode are old slots
    dequantized to bf16 and quantized into fresh groups (dead rows and the padding of
    the last group are zeros); stage are old slots kept in bf16 (the new residual).
    Returns the new cache (nq = its quantized slots, nf = the residual) and remap
    [B, H, old_length]: the new slot of every old slot, -1 if dropped. Every layer at once
    when the layer axis is merged into the batch axis."""
    src = as_prefix(prefix)
    if not src.nq or src.kmode != 0:
        raise NotImplementedError("rebuild is for packed caches with channel-mode (KIVI) keys")
    if src.pages is not None:
        raise NotImplementedError("rebuild of paged storage")
    gk = int(src.kg)
    B, H = src.vq.shape[0], src.vq.shape[1]
    D = src.vq.shape[3] * src.vq.shape[4] * 2
    dev = src.vq.device
    old_len, ql_old = src.n, src.nq
    idx = [t.to(device=dev, dtype=torch.int64) for t in (groups_before, encode, groups_after, stage)]
    for t in idx:
        if t.ndim != 3 or tuple(t.shape[:2]) != (B, H):
            raise ValueError("index tensors must be [B, H, *]")
    gb, enc, ga, stg = (t.contiguous() for t in idx)
    g1, m, g3, st = (t.shape[-1] for t in idx)
    g2 = -(-m // gk)
    ql = (g1 + g2 + g3) * gk
    cap = ql + st + 1024
    ng_cap = -(-cap // gk)
    kq = torch.empty((B, H, ng_cap, D, gk // 2), device=dev, dtype=torch.uint8)
    ks = torch.empty((B, H, ng_cap, D), device=dev, dtype=torch.float16)
    kz = torch.empty_like(ks)
    vq = torch.empty((B, H, cap, D // src.vg, src.vg // 2), device=dev, dtype=torch.uint8)
    vs = torch.empty((B, H, cap, D // src.vg), device=dev, dtype=torch.float16)
    vz = torch.empty_like(vs)
    rcap = max(st + 256, 64)
    tail_dtype = src.kf.dtype if src.nf else torch.bfloat16
    kr = torch.empty((B, H, rcap, D), device=dev, dtype=tail_dtype)
    vr = torch.empty_like(kr)
    remap = torch.empty((B, H, old_len), device=dev, dtype=torch.int64)
    sdesc = kv_descriptor(Prefix(**{s: getattr(src, s) for s in Prefix.__slots__ if s not in ("mask", "lens")}))
    lib = _lib.lib()

    def copy_groups(gid: torch.Tensor, at: int) -> None:
        n = gid.shape[-1]
        if n == 0:
            return
        safe = gid.clamp_min(0).contiguous()
        dst = Prefix(kq=kq[:, :, at:at + n], ks=ks[:, :, at:at + n], kz=kz[:, :, at:at + n],
                     vq=vq[:, :, at * gk:(at + n) * gk], vs=vs[:, :, at * gk:(at + n) * gk],
                     vz=vz[:, :, at * gk:(at + n) * gk], nq=n * gk, kb=4, vb=4, kg=gk, vg=src.vg, kmode=0)
        ddesc = kv_descriptor(dst)
        _lib.check("ma_compact_tokens", lib.ma_compact_tokens(
            sdesc.kv, ddesc.kv, B, H, D, safe.data_ptr(), n, i64(safe.stride(0), safe.stride(1)),
            _lib.stream_handle(dev)))

    copy_groups(gb, 0)
    copy_groups(ga, g1 + g2)
    if m:
        rows_k = torch.zeros((B, H, g2 * gk, D), device=dev, dtype=torch.bfloat16)
        rows_v = torch.zeros_like(rows_k)
        _gather_rows_into(sdesc, enc, rows_k[:, :, :m], rows_v[:, :, :m])     # -1 gathers a zero row
        pk, sk_ = kq[:, :, g1:g1 + g2], ks[:, :, g1:g1 + g2]
        _lib.check("ma_quantize_keys_channel", lib.ma_quantize_keys_channel(
            rows_k.data_ptr(), _lib.MA_BF16, B, H, g2 * gk, D, i64(*_strides3(rows_k)), gk, pk.data_ptr(),
            i64(*_strides3(pk)), sk_.data_ptr(), kz[:, :, g1:g1 + g2].data_ptr(), i64(*_strides3(sk_)),
            _lib.stream_handle(dev)))
        pv, sv_ = vq[:, :, g1 * gk:(g1 + g2) * gk], vs[:, :, g1 * gk:(g1 + g2) * gk]
        _lib.check("ma_quantize_tokens", lib.ma_quantize_tokens(
            rows_v.data_ptr(), _lib.MA_BF16, B, H, g2 * gk, D, i64(*_strides3(rows_v)), None, None, src.vg,
            pv.data_ptr(), i64(*_strides3(pv)), sv_.data_ptr(), vz[:, :, g1 * gk:(g1 + g2) * gk].data_ptr(),
            i64(*_strides3(sv_)), _lib.stream_handle(dev)))
    if st:
        _gather_rows_into(sdesc, stg, kr[:, :, :st], vr[:, :, :st])
    _lib.check("ma_rebuild_remap", lib.ma_rebuild_remap(
        B, H, old_len, gk, gb.data_ptr() if g1 else None, g1, enc.data_ptr() if m else None, m,
        ga.data_ptr() if g3 else None, g3, stg.data_ptr() if st else None, st, remap.data_ptr(),
        _lib.stream_handle(dev)))
    out = Prefix(kq=kq, ks=ks, kz=kz, vq=vq, vs=vs, vz=vz, kf=kr, vf=vr, nq=ql, nf=st, kb=4, vb=4, kg=gk,
                 vg=src.vg, kmode=0)
    return out, remap


def evict_plan(phys: torch.Tensor, pos: torch.Tensor, *, quantized_length: int, key_group: int = 32,
               repack_below: float = 1.0, compaction: str = "lazy", recent_window: int = 64, tail: int = 0,
               tail_stage: bool = False, cache_length: int | None = None):
    """The index lists of the rebuild after an eviction (_evict_to, session.py:303-356), on
    the device: phys [L,B,H,live] int32 (the live entries' slots) and pos [L,B,H,live]
    (their positions, increasing along the live axis as the eviction state keeps them).

    A key group with at least max(1, ceil(repack_below * key_group)) live entries is kept
    whole (compaction "lazy"; none with "full"), the unadmitted tail's groups excepted;
    staged entries among the recent_window newest positions stay staged; the others are
    re-encoded. Returns (groups_before, encode, groups_after, stage) as [L,B,H,*] int64
    padded with -1 to the largest count over lanes: the arguments of rebuild (and of the
    reference's PackedKVCache.rebuild). The lists are built by one kernel; their widths
    take one host read of three counts, as the reference's padding does
    (session.py:323-325)."""
    lib = _lib.lib()
    if phys.ndim != 4 or pos.shape != phys.shape:
        raise ValueError("phys and pos must be [L, B, H, live]")
    if compaction not in ("lazy", "full"):
        raise ValueError(f"compaction must be 'lazy' or 'full', got {compaction!r}")
    L, B, H, live = phys.shape
    lanes = L * B * H
    dev = phys.device
    gk, ql = int(key_group), int(quantized_length)
    ng = max(1, ql // gk)
    need = max(1, math.ceil(repack_below * gk)) if compaction == "lazy" else 0
    tail_groups = tail // gk if tail and not tail_stage else 0
    ph = phys.reshape(lanes, live).to(torch.int32).contiguous()
    ps = pos.reshape(lanes, live).to(torch.int64).contiguous()
    gb = torch.empty((lanes, ng), device=dev, dtype=torch.int64)
    enc = torch.empty((lanes, live), device=dev, dtype=torch.int64)
    stg = torch.empty((lanes, live), device=dev, dtype=torch.int64)
    counts = torch.empty((lanes, 3), device=dev, dtype=torch.int32)
    maxes = torch.empty(4, device=dev, dtype=torch.int32)
    _lib.check("ma_evict_plan", lib.ma_evict_plan(
        ph.data_ptr(), ps.data_ptr(), lanes, live, _lib.i64(live, live), ql, gk, need, tail_groups,
        int(recent_window), gb.data_ptr(), enc.data_ptr(), stg.data_ptr(), counts.data_ptr(), maxes.data_ptr(),
        _lib.stream_handle(dev)))
    g1, m, st, bad = maxes.tolist()
    if bad:
        raise ValueError(f"{bad} lane(s) hold live entries out of position order")
    groups_before = gb[:, :g1].reshape(L, B, H, g1)
    encode = enc[:, :m].reshape(L, B, H, m)
    stage = stg[:, :st].reshape(L, B, H, st)
    groups_after = torch.empty((L, B, H, 0), device=dev, dtype=torch.int64)
    if tail and tail_stage:
        tail_slots = torch.arange(cache_length - tail, cache_length, device=dev).view(1, 1, 1, -1)
        stage = torch.cat([stage, tail_slots.expand(L, B, H, tail)], -1)
    elif tail:
        groups_after = torch.arange(ng - tail_groups, ng, device=dev).expand(L, B, H, -1).contiguous()
    return groups_before, encode, groups_after, stage
