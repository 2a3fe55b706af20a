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
"""

from __future__ import annotations

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
                 "kmode", "kch")

    def __init__(self, *, kq=None, ks=None, kz=None, vq=None, vs=None, vz=None, kf=None, vf=None,
                 nq=0, nf=0, kb=16, vb=16, kg=32, vg=32, mask=None, kmode=0, kch=None):
        self.mask = mask          # optional uint8/bool [B, Hkv, n]: 0 = dead slot, never attended
        self.kmode, self.kch = kmode, kch    # kmode 1: per-token keys with divisor kch [B, Hkv, D]
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
        p = Prefix(**{s: getattr(view_or_prefix, s) for s in Prefix.__slots__})
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
    if prefix.nq:
        if prefix.kb != 4 or prefix.vb != 4:
            raise NotImplementedError("packed caches: the kernels read 4-bit keys and values")
        kv.layout = _lib.MA_KV_PACKED_TOKEN if prefix.kmode == 1 else _lib.MA_KV_PACKED_CHANNEL
        B, H = prefix.vq.shape[0], prefix.vq.shape[1]
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
        kv.dtype = _lib.dtype_code(prefix.kf.dtype)
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
