"""GPU parity of the retention pass's pieces over dense and packed (k4v4) prefixes: the
lookahead probe (block-causal attention of [block | probe blocks] over [prefix | itself]
plus the probe rows' prefix mass, session.py:2317-2332) and the value score over a cache
layout (a_j ||v_j - c||, session.py:27-40 with the live values in the compute dtype).

A packed prefix is quantized on the CPU by the oracle (token-mode keys with their
divisor), its payloads are what the device reads, and the oracle runs on its own bf16
dequantization of the same payloads -- no expected value comes from a device kernel. Bars: the attention
output at the bf16 bar of the other attention tests (2e-2), the probe mass to 1e-4 (the
oracle's own prefix statistics against the device's, which sum in another order), the
value score to 5e-5.
"""

from __future__ import annotations

import numpy as np
import pytest
import torch

import oracle

pytestmark = pytest.mark.gpu

DEV = "cuda"


def _inputs(seed, B=1, Hq=8, H=2, T=96, n=3000, D=128):
    gen = torch.Generator().manual_seed(seed)
    q = torch.randn(B, Hq, T, D, generator=gen).to(torch.bfloat16)
    k = torch.randn(B, H, n, D, generator=gen).to(torch.bfloat16)
    v = torch.randn(B, H, n, D, generator=gen).to(torch.bfloat16)
    kc = torch.randn(B, H, T, D, generator=gen).to(torch.bfloat16)
    vc = torch.randn(B, H, T, D, generator=gen).to(torch.bfloat16)
    return q, k, v, kc, vc


def _prefix(kind, k, v):
    from maskahead_b200.layouts import Prefix

    if kind == "dense":
        return Prefix.dense(k.to(DEV), v.to(DEV)), k, v
    kchan = oracle.key_channel_divisor(k)
    kq, ks, kz = oracle.quantize_keys_token(k, kchan)
    vq, vs, vz = oracle.quantize_values(v)
    pre = Prefix(kq=kq.to(DEV), ks=ks.to(DEV), kz=kz.to(DEV), vq=vq.to(DEV), vs=vs.to(DEV), vz=vz.to(DEV),
                 nq=k.shape[2], kb=4, vb=4, kg=32, vg=32, kmode=1, kch=kchan.to(DEV))
    return pre, oracle.dequantize_keys_token(kq, ks, kz, kchan), oracle.dequantize_values(vq, vs, vz)


@pytest.mark.parametrize("kind", ["dense", "packed"])
@pytest.mark.parametrize("T,probe_blocks", [(64, 1), (96, 2)])
def test_probe_attention_matches_oracle(kind, T, probe_blocks):
    from maskahead_b200.hotpath import probe_attention

    q, k, v, kc, vc = _inputs(T + (7 if kind == "packed" else 0), T=T)
    pre, kr, vr = _prefix(kind, k, v)
    rows = torch.arange(32, T, dtype=torch.int32, device=DEV)
    out, mass = probe_attention(q.to(DEV), pre, kc.to(DEV), vc.to(DEV), block_size=32, probe_rows=rows)
    torch.cuda.synchronize()
    want, (mp, lp, _) = oracle.prefix_attention(q, kr, vr, kc, vc, causal_block=32, q_pos0=0, c_pos0=0)
    np.testing.assert_allclose(out.float().cpu().numpy(), want.float().numpy(), rtol=2e-2, atol=2e-2)
    want_mass = oracle.prefix_mass(q, kr, mp, lp, list(range(32, T))) * probe_blocks
    np.testing.assert_allclose(mass.cpu().numpy(), want_mass.numpy(), rtol=1e-4, atol=1e-9)


@pytest.mark.parametrize("n", [3000, 9000])
def test_value_score_prefix_packed_matches_oracle(n):
    """The default (the packed values read in place by the producer warps of the value
    pass) and unpack=True score the bf16-dequantized values (the reference's compute
    dtype); unpack=False reads the packed values in place as well."""
    from maskahead_b200.hotpath import value_score_prefix

    _, k, v, _, _ = _inputs(n, H=4, n=n)
    pre, _, vr = _prefix("packed", k, v)
    gen = torch.Generator().manual_seed(n + 1)
    a = torch.rand(1, 4, n, generator=gen)
    got = value_score_prefix(a.to(DEV), pre).cpu()
    got_inplace = value_score_prefix(a.to(DEV), pre, unpack=False).cpu()
    torch.cuda.synchronize()
    want = oracle.value_score(a, vr)
    np.testing.assert_allclose(got.numpy(), want.numpy(), rtol=5e-5, atol=1e-9)
    np.testing.assert_allclose(got_inplace.numpy(), want.numpy(), rtol=2e-2, atol=1e-6)
