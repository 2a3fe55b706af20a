"""The workspace-free value score (ma_value_score_noalloc) against ma_value_score.

ma_value_score_noalloc exists for callers that cannot allocate device memory (a host
binding handed only its input and output buffers, or a framework that owns every device
allocation): it keeps its scratch in a static device array inside the library. This
test calls it through the C ABI twice in a row, on different inputs, and checks each
result against ma_value_score run with a caller workspace on the same inputs. The file
is named to be collected last.
"""

from __future__ import annotations

import ctypes

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu


def _inputs(seed, B, H, n, D):
    g = torch.Generator(device="cuda").manual_seed(seed)
    a = torch.softmax(torch.randn(B, H, n, generator=g, device="cuda") * 2.0, dim=-1)
    v = torch.randn(B, H, n, D, generator=g, device="cuda").to(torch.bfloat16)
    return a.contiguous(), v.contiguous()


def _kv(v):
    from maskahead_b200._lib import MA_BF16, MA_KV_DENSE, MaKV, i64

    kv = MaKV()
    kv.layout, kv.dtype, kv.nq, kv.nf = MA_KV_DENSE, MA_BF16, 0, v.shape[2]
    kv.kf = kv.vf = v.data_ptr()
    kv.skf = i64(*v.stride()[:3])
    kv.svf = i64(*v.stride()[:3])
    return kv


def _with_workspace(lib, kv, a, v, stream):
    from maskahead_b200._lib import i64

    B, H, n, D = v.shape
    ws = torch.zeros(lib.ma_value_score_workspace(B, H, n, D), dtype=torch.uint8, device="cuda")
    out = torch.empty_like(a)
    rc = lib.ma_value_score(kv, B, H, D, a.data_ptr(), i64(a.stride(0), a.stride(1)), out.data_ptr(),
                            i64(out.stride(0), out.stride(1)), ws.data_ptr(), ws.numel(), stream)
    assert rc == 0
    return out


def _no_alloc(lib, kv, a, v, stream):
    from maskahead_b200._lib import i64

    B, H, n, D = v.shape
    out = torch.full_like(a, float("nan"))
    rc = lib.ma_value_score_noalloc(kv, B, H, D, a.data_ptr(), i64(a.stride(0), a.stride(1)), out.data_ptr(),
                                    i64(out.stride(0), out.stride(1)), stream)
    assert rc == 0, f"ma_value_score_noalloc returned {rc}"
    return out


def test_value_score_noalloc_matches_workspace_version_twice():
    from maskahead_b200._lib import lib as get_lib

    lib = get_lib()
    stream = torch.cuda.current_stream().cuda_stream
    for seed, shape in ((5, (1, 4, 8192, 128)), (6, (2, 3, 1000, 64))):
        a, v = _inputs(seed, *shape)
        kv = _kv(v)
        want = _with_workspace(lib, kv, a, v, stream)
        got = _no_alloc(lib, kv, a, v, stream)
        torch.cuda.synchronize()
        np.testing.assert_allclose(got.cpu().numpy(), want.cpu().numpy(), rtol=2e-5, atol=1e-12)


def test_value_score_noalloc_rejects_sizes_beyond_its_scratch():
    from maskahead_b200._lib import i64, lib as get_lib

    lib = get_lib()
    a, v = _inputs(7, 1, 1, 64, 128)
    kv = _kv(v)
    kv.nf = 1 << 24           # 16M slots: scratch beyond 8 MiB, rejected before any launch
    out = torch.empty_like(a)
    rc = lib.ma_value_score_noalloc(kv, 1, 64, 128, a.data_ptr(), i64(a.stride(0), a.stride(1)),
                                    out.data_ptr(), i64(out.stride(0), out.stride(1)),
                                    ctypes.c_void_p(torch.cuda.current_stream().cuda_stream))
    assert rc == -2
    torch.cuda.synchronize()


def test_value_score_noalloc_status_reports_a_timeout():
    """A bounded wait of the no-alloc call that gives up (the centre wait, bounded here at
    1 ns) shows in ma_value_score_noalloc_status; the next call, with the bound restored,
    runs clean and matches ma_value_score again."""
    import maskahead_b200
    from maskahead_b200._lib import lib as get_lib

    lib = get_lib()
    stream = torch.cuda.current_stream().cuda_stream
    a, v = _inputs(8, 1, 4, 8192, 128)
    kv = _kv(v)
    want = _with_workspace(lib, kv, a, v, stream)
    assert lib.ma_value_score_noalloc_status(stream) == 0
    prev = maskahead_b200.set_peer_wait_ns(1)
    try:
        got = _no_alloc(lib, kv, a, v, stream)
        assert lib.ma_value_score_noalloc_status(stream) == -5
        assert bool(torch.isnan(got).any())
    finally:
        maskahead_b200.set_peer_wait_ns(prev)
    got = _no_alloc(lib, kv, a, v, stream)
    assert lib.ma_value_score_noalloc_status(stream) == 0
    np.testing.assert_allclose(got.cpu().numpy(), want.cpu().numpy(), rtol=2e-5, atol=1e-12)
