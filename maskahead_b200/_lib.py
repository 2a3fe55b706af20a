"""ctypes binding of ``libmaskahead_b200.so`` (the C ABI of include/maskahead_b200.h).

The library is built in-tree by ``maskahead_b200.build``. There is no fallback: if the
library is missing or CUDA is unavailable, every operator raises
``KernelUnavailableError``.
"""

from __future__ import annotations

import ctypes
from pathlib import Path

import torch

LIB_PATH = Path(__file__).resolve().parent / "_lib" / "libmaskahead_b200.so"

MA_OK = 0
MA_ERR_UNSUPPORTED = -2
MA_ERR_CUDA = -4
MA_ERR_TIMEOUT = -5
MA_F32, MA_BF16, MA_F16 = 0, 1, 2
MA_KV_DENSE, MA_KV_PACKED_TOKEN, MA_KV_PACKED_CHANNEL = 0, 1, 2


class KernelUnavailableError(RuntimeError):
    """The sm_100a library or a CUDA device is not available (ops.py:19-21 in the reference)."""


class MaError(RuntimeError):
    """A C-ABI entry point returned a negative status."""

    def __init__(self, fn: str, status: int, detail: str):
        super().__init__(f"{fn} failed with status {status} ({detail})")
        self.status = status


c_i64_3 = ctypes.c_int64 * 3
c_i64_2 = ctypes.c_int64 * 2


class MaKV(ctypes.Structure):
    _fields_ = [
        ("layout", ctypes.c_int32), ("dtype", ctypes.c_int32), ("nq", ctypes.c_int32),
        ("nf", ctypes.c_int32), ("kgroup", ctypes.c_int32), ("vgroup", ctypes.c_int32),
        ("kf", ctypes.c_void_p), ("vf", ctypes.c_void_p), ("skf", c_i64_3), ("svf", c_i64_3),
        ("kq", ctypes.c_void_p), ("ks", ctypes.c_void_p), ("kz", ctypes.c_void_p),
        ("skq", c_i64_3), ("sks", c_i64_3),
        ("vq", ctypes.c_void_p), ("vs", ctypes.c_void_p), ("vz", ctypes.c_void_p),
        ("svq", c_i64_3), ("svs", c_i64_3),
        ("kchan", ctypes.c_void_p), ("skc", c_i64_2),
        ("mask", ctypes.c_void_p),
        ("pages", ctypes.c_void_p), ("spg", ctypes.c_int64), ("page_size", ctypes.c_int32),
        ("num_pages", ctypes.c_int32), ("lens", ctypes.c_void_p),
    ]


class MaRows(ctypes.Structure):
    _fields_ = [
        ("q", ctypes.c_void_p), ("dtype", ctypes.c_int32), ("B", ctypes.c_int32),
        ("Hq", ctypes.c_int32), ("T", ctypes.c_int32), ("D", ctypes.c_int32), ("sq", c_i64_3),
    ]


class MaBlock(ctypes.Structure):
    _fields_ = [
        ("k", ctypes.c_void_p), ("v", ctypes.c_void_p), ("Tc", ctypes.c_int32),
        ("sk", c_i64_3), ("sv", c_i64_3),
    ]


_P = ctypes.POINTER
_vp, _i32, _f32, _sz = ctypes.c_void_p, ctypes.c_int, ctypes.c_float, ctypes.c_size_t

_SIGNATURES = {
    "ma_version": (_i32, []),
    "ma_status_string": (ctypes.c_char_p, [_i32]),
    "ma_set_attention_kernel": (_i32, [_i32]),
    "ma_set_mass_tiles": (_i32, [_i32]),
    "ma_kv_read_in_place": (_i32, [_P(MaKV), _i32]),
    "ma_last_cuda_error": (ctypes.c_char_p, []),
    "ma_workspace_status": (_i32, [_vp, _sz, _vp]),
    "ma_set_peer_wait_ns": (ctypes.c_int64, [ctypes.c_int64]),
    "ma_value_score_noalloc_status": (_i32, [_vp]),
    "ma_prefix_attention_workspace": (_sz, [_i32] * 6),
    "ma_prefix_attention": (_i32, [_P(MaRows), _P(MaKV), _i32, _P(MaBlock), _f32, _i32, _i32, _i32,
                                   _vp, _P(ctypes.c_int64), _vp, _vp, _vp, _vp, _sz, _vp]),
    "ma_prefix_scores": (_i32, [_P(MaRows), _P(MaKV), _i32, _vp, _i32, _vp, _vp, _f32, _vp,
                                _P(ctypes.c_int64), _vp, _P(ctypes.c_int64), _vp, _sz, _vp]),
    "ma_value_score_workspace": (_sz, [_i32] * 4),
    "ma_value_score": (_i32, [_P(MaKV), _i32, _i32, _i32, _vp, _P(ctypes.c_int64), _vp,
                              _P(ctypes.c_int64), _vp, _sz, _vp]),
    "ma_value_score_noalloc": (_i32, [_P(MaKV), _i32, _i32, _i32, _vp, _P(ctypes.c_int64), _vp,
                                      _P(ctypes.c_int64), _vp]),
    "ma_select_topk": (_i32, [_vp, _i32, _i32, _i32, _P(ctypes.c_int64), _vp, _vp, _i32, _vp, _vp,
                              _P(ctypes.c_int64), _vp]),
    "ma_retain": (_i32, [_vp, _vp, _i32, _vp, _i32, _i32, _i32, _i32, _i32, _vp, _vp]),
    "ma_sparse_attention_workspace": (_sz, [_i32] * 6),
    "ma_sparse_attention": (_i32, [_P(MaRows), _P(MaKV), _i32, _vp, _i32, _P(ctypes.c_int64),
                                   _P(MaBlock), _f32, _vp, _P(ctypes.c_int64), _vp, _sz, _vp]),
    "ma_gather_kv": (_i32, [_P(MaKV), _i32, _i32, _i32, _vp, _i32, _P(ctypes.c_int64), _vp, _vp,
                            _P(ctypes.c_int64), _P(ctypes.c_int64), _i32, _vp]),
    "ma_unpack_prefix": (_i32, [_P(MaKV), _i32, _i32, _i32, _vp, _vp, _P(ctypes.c_int64), _P(ctypes.c_int64), _vp]),
    "ma_quantize_tokens": (_i32, [_vp, _i32, _i32, _i32, _i32, _i32, _P(ctypes.c_int64), _vp,
                                  _P(ctypes.c_int64), _i32, _vp, _P(ctypes.c_int64), _vp, _vp,
                                  _P(ctypes.c_int64), _vp]),
    "ma_quantize_keys_channel": (_i32, [_vp, _i32, _i32, _i32, _i32, _i32, _P(ctypes.c_int64), _i32, _vp,
                                        _P(ctypes.c_int64), _vp, _vp, _P(ctypes.c_int64), _vp]),
    "ma_key_divisor": (_i32, [_vp, _i32, _i32, _i32, _i32, _i32, _P(ctypes.c_int64), _vp,
                              _P(ctypes.c_int64), _vp]),
    "ma_compact_tokens": (_i32, [_P(MaKV), _P(MaKV), _i32, _i32, _i32, _vp, _i32, _P(ctypes.c_int64), _vp]),
    "ma_rebuild_remap": (_i32, [_i32, _i32, _i32, _i32, _vp, _i32, _vp, _i32, _vp, _i32, _vp, _i32, _vp, _vp]),
    "ma_evict_plan": (_i32, [_vp, _vp, _i32, _i32, _P(ctypes.c_int64), _i32, _i32, _i32, _i32, _i32, _vp, _vp, _vp,
                             _vp, _vp, _vp]),
    "ma_head_gather_region_bytes": (_sz, [_i32, _i32, _i32]),
    "ma_head_gather_workspace": (_sz, []),
    "ma_peer_alloc": (_i32, [_sz, _P(_vp)]),
    "ma_peer_free": (_i32, [_vp]),
    "ma_ipc_handle_bytes": (_sz, []),
    "ma_ipc_get_handle": (_i32, [_vp, _vp]),
    "ma_ipc_open_handle": (_i32, [_vp, _P(_vp)]),
    "ma_ipc_close_handle": (_i32, [_vp]),
    "ma_head_gather": (_i32, [_vp, _P(ctypes.c_int64), _i32, _i32, _i32, _i32, _i32, _i32, _P(_vp), _vp,
                              _P(ctypes.c_int64), _vp, _sz, _vp]),
    "ma_prefix_attention_gather": (_i32, [_P(MaRows), _P(MaKV), _i32, _P(MaBlock), _f32, _i32, _i32, _i32,
                                          _vp, _P(ctypes.c_int64), _vp, _vp, _vp, _vp, _sz, _i32, _i32, _P(_vp),
                                          _i32, _vp, _P(ctypes.c_int64), _vp, _sz, _vp]),
}

EXPORTED = tuple(_SIGNATURES)

_lib: ctypes.CDLL | None = None


def load_library() -> ctypes.CDLL:
    """Load (once) and return the C-ABI library; raises KernelUnavailableError."""
    global _lib
    if _lib is not None:
        return _lib
    if not LIB_PATH.exists():
        raise KernelUnavailableError(
            f"{LIB_PATH} is missing: build it with `python -m maskahead_b200.build`")
    lib = ctypes.CDLL(str(LIB_PATH))
    for name, (res, args) in _SIGNATURES.items():
        fn = getattr(lib, name)
        fn.restype = res
        fn.argtypes = args
    _lib = lib
    return lib


def lib() -> ctypes.CDLL:
    """The library, for a compute call: also requires a CUDA device."""
    if not torch.cuda.is_available():
        raise KernelUnavailableError("maskahead_b200 kernels need a CUDA device (sm_100a)")
    return load_library()


def check(fn: str, status: int) -> None:
    if status != MA_OK:
        lib_ = load_library()
        detail = lib_.ma_status_string(status).decode()
        if status == MA_ERR_CUDA:
            detail += ": " + lib_.ma_last_cuda_error().decode()
        raise MaError(fn, status, detail)


def dtype_code(dt: torch.dtype) -> int:
    if dt == torch.float32:
        return MA_F32
    if dt == torch.bfloat16:
        return MA_BF16
    raise ValueError(f"unsupported dtype {dt}: the kernels take float32 or bfloat16")


def ptr(t: torch.Tensor | None) -> int | None:
    return None if t is None else t.data_ptr()


def i64(*vals) -> ctypes.Array:
    return (ctypes.c_int64 * len(vals))(*[int(v) for v in vals])


def stream_handle(device: torch.device) -> int:
    return torch.cuda.current_stream(device).cuda_stream


# ------------------------------------------------------------------------ workspaces
_WORKSPACES: dict[tuple, torch.Tensor] = {}
# purposes whose buffers are C-ABI workspaces (an error word at their first 256-byte
# boundary); the others are plain data scratch (e.g. the unpacked prefix)
STATUS_WORKSPACES = frozenset({"attention", "value_score"})
# further C-ABI workspaces with an error word, owned by objects (device index, buffer)
STATUS_EXTRA: list[tuple[int, torch.Tensor]] = []


def device_status(device: torch.device | int | None = None) -> None:
    """Raise MaError(MA_ERR_TIMEOUT) if a bounded device-side wait of a kernel that used one
    of this module's workspaces on `device` gave up since the last check (its rows were
    written as NaN). Waits for the work queued on the device's current stream and clears
    the recorded errors."""
    dev = torch.device("cuda", torch.cuda.current_device() if device is None else
                       (device if isinstance(device, int) else device.index or 0))
    lib_ = lib()
    stream = stream_handle(dev)
    failed = []
    for (kind, index, purpose), buf in list(_WORKSPACES.items()):
        if kind != "cuda" or index != dev.index or purpose not in STATUS_WORKSPACES:
            continue
        rc = lib_.ma_workspace_status(buf.data_ptr(), buf.numel(), stream)
        if rc == MA_ERR_TIMEOUT:
            failed.append(purpose)
        elif rc != MA_OK:
            check("ma_workspace_status", rc)
    for index, buf in list(STATUS_EXTRA):
        if index != dev.index:
            continue
        rc = lib_.ma_workspace_status(buf.data_ptr(), buf.numel(), stream)
        if rc == MA_ERR_TIMEOUT:
            failed.append("head_gather")
        elif rc != MA_OK:
            check("ma_workspace_status", rc)
    if failed:
        detail = load_library().ma_status_string(MA_ERR_TIMEOUT).decode()
        raise MaError("device_status", MA_ERR_TIMEOUT, f"{detail} in the work of: {', '.join(sorted(failed))}")


def set_peer_wait_ns(ns: int) -> int:
    """Bound (ns) on a kernel CTA's wait for the other CTAs of its launch; <= 0 restores the
    default. Returns the previous bound (ma_set_peer_wait_ns)."""
    return int(load_library().ma_set_peer_wait_ns(int(ns)))


# Buffers a larger one replaced. They stay allocated for the life of the process: a CUDA
# graph captured before the growth still addresses them (its kernels keep their counters
# and error word there), and freed memory would be handed to other tensors while such a
# graph can still replay.
_RETIRED: list[torch.Tensor] = []


def workspace(device: torch.device, purpose: str, nbytes: int) -> torch.Tensor:
    """Grow-only, zero-initialized scratch per (device, purpose).

    Like the reference's module-level scratch pools (ops.py:274-317) it is shared by
    every call on the device, so calls that can overlap (several streams or threads)
    must bring their own workspace. A buffer that grows is replaced, never freed (graphs
    captured before keep using it); run the largest calls once before capturing a graph
    so that its kernels and later eager calls share one buffer.
    """
    key = (device.type, device.index, purpose)
    buf = _WORKSPACES.get(key)
    if buf is None or buf.numel() < nbytes:
        size = max(nbytes, 1 << 20)
        if buf is not None:
            _RETIRED.append(buf)
        buf = torch.zeros(size + 256, dtype=torch.uint8, device=device)
        _WORKSPACES[key] = buf
    return buf
