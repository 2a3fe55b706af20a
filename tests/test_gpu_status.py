"""Device-side timeouts reach the caller.

Every cross-CTA wait in the kernels is bounded (ma_set_peer_wait_ns). A CTA whose wait
gives up writes its rows as NaN and records the timeout in the workspace's error word;
ma_workspace_status (maskahead_b200.device_status) returns it as MA_ERR_TIMEOUT. These
tests shorten the bound to 1 ns, so the CTAs that arrive first at the split merge (step 0
at the cfg2 shape: 16 prefix splits + the block, merged in one cooperative launch) and at
the value-score centre give up at once -- nothing faults, traps or hangs -- then restore
it and check that the next calls run clean and give the same results as before.
"""

from __future__ import annotations

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu

DEV = "cuda"


def _cfg2_layer(seed=11):
    g = torch.Generator().manual_seed(seed)
    q = torch.randn(1, 28, 32, 128, generator=g).to(torch.bfloat16).to(DEV)
    k = torch.randn(1, 4, 8192, 128, generator=g).to(torch.bfloat16).to(DEV)
    v = torch.randn(1, 4, 8192, 128, generator=g).to(torch.bfloat16).to(DEV)
    kc = torch.randn(1, 4, 32, 128, generator=g).to(torch.bfloat16).to(DEV)
    vc = torch.randn(1, 4, 32, 128, generator=g).to(torch.bfloat16).to(DEV)
    return q, k, v, kc, vc


def _step0(q, k, v, kc, vc):
    from maskahead_b200.hotpath import fast_step0
    from maskahead_b200.layouts import Prefix

    res = fast_step0(q, Prefix.dense(k, v), kc, vc, query_indices=list(range(32)), topk=1024, scaling=128 ** -0.5)
    return res.out.float().cpu(), res.score.cpu()


def test_peer_wait_timeout_is_reported_and_recovers():
    import maskahead_b200
    from maskahead_b200 import MaError

    inputs = _cfg2_layer()
    maskahead_b200.device_status()               # nothing pending from earlier tests
    want_out, want_score = _step0(*inputs)
    maskahead_b200.device_status()
    prev = maskahead_b200.set_peer_wait_ns(1)
    try:
        out, score = _step0(*inputs)
        with pytest.raises(MaError) as err:
            maskahead_b200.device_status()
        assert err.value.status == -5
        assert bool(torch.isnan(out).any()) or bool(torch.isnan(score).any()), "timed-out rows are NaN"
    finally:
        maskahead_b200.set_peer_wait_ns(prev)
    out, score = _step0(*inputs)
    maskahead_b200.device_status()               # clean again: the counters stayed consistent
    np.testing.assert_array_equal(out.numpy(), want_out.numpy())
    np.testing.assert_array_equal(score.numpy(), want_score.numpy())


def test_workspace_status_of_a_clean_workspace():
    from maskahead_b200._lib import lib as get_lib

    lib = get_lib()
    ws = torch.zeros(1 << 16, dtype=torch.uint8, device=DEV)
    stream = torch.cuda.current_stream().cuda_stream
    assert lib.ma_workspace_status(ws.data_ptr(), ws.numel(), stream) == 0
    ws[:4] = torch.tensor([1, 0, 0, 0], dtype=torch.uint8)   # an error word set by a kernel
    assert lib.ma_workspace_status(ws.data_ptr(), ws.numel(), stream) == -5
    assert lib.ma_workspace_status(ws.data_ptr(), ws.numel(), stream) == 0   # cleared by the query
    assert lib.ma_workspace_status(ws.data_ptr(), 8, stream) == -1
