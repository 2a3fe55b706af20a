"""Helpers turning torch tensors into the C ABI's query/current-block descriptors."""

from __future__ import annotations

import torch

from .. import _lib


def _fix_inner(t: torch.Tensor) -> torch.Tensor:
    """Innermost dimension contiguous and row starts 16-byte aligned, copying if not."""
    es = t.element_size()
    ok = t.stride(-1) == 1 and t.data_ptr() % 16 == 0 and all((s * es) % 16 == 0 for s in t.stride()[:-1])
    return t if ok else t.contiguous()


def rows_struct(query: torch.Tensor):
    if query.ndim != 4:
        raise ValueError("query must have shape [B, Hq, T, D]")
    if not query.is_cuda:
        raise _lib.KernelUnavailableError("maskahead_b200 kernels need CUDA tensors")
    q = _fix_inner(query)
    r = _lib.MaRows()
    r.q = q.data_ptr()
    r.dtype = _lib.dtype_code(q.dtype)
    r.B, r.Hq, r.T, r.D = q.shape
    r.sq = _lib.i64(*q.stride()[:3])
    return r, q


def block_struct(key: torch.Tensor | None, value: torch.Tensor | None, dtype: torch.dtype):
    blk = _lib.MaBlock()
    if key is None or key.shape[2] == 0:
        blk.Tc = 0
        return blk, None
    if key.shape != value.shape:
        raise ValueError("current K and V shapes differ")
    k = _fix_inner(key.to(dtype))
    v = _fix_inner(value.to(dtype))
    blk.k, blk.v, blk.Tc = k.data_ptr(), v.data_ptr(), k.shape[2]
    blk.sk, blk.sv = _lib.i64(*k.stride()[:3]), _lib.i64(*v.stride()[:3])
    return blk, (k, v)
