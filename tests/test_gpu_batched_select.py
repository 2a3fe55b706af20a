"""Step 0's selection run once for every layer (select_step0 over layer-stacked inputs)
against the per-layer fast_step0 it replaces.

The session's step-0 forward runs each layer's attention (step0_attention, the prefix
statistics written into that layer's slice of stacked buffers); the selection of all
layers then runs as one pass over the layer-stacked queries, cache and statistics (one
launch per kernel). Per layer the products must be those of fast_step0 on the same
inputs: the attention output and the mass bit for bit (a slot's mass does not depend on
how the launch splits the slots), the value-aware score within the fp32 reordering of
the head centre's sum (rtol 1e-5), the read sets equal up to that score's ties (band
1e-5 of the k-th score, the bar of the other selection tests) and the compact cache
bit-exact where the read sets agree; on a retention block the merged probe's mass bit
for bit as well. Cases: bf16 and k4v4 token-mode caches (the packed one stacked as one
allocation of all layers, read by the selection in place, or through the step's unpacked
copies that each layer's attention leaves in its slice of stacked buffers), four layers
of cfg2's heads.
"""

from __future__ import annotations

import numpy as np
import pytest
import torch

from gpu_cases import band_equal

pytestmark = pytest.mark.gpu

DEV = "cuda"
L, B, HQ, H, T, D, N, K = 4, 1, 28, 4, 32, 128, 2048, 256


def _caches(kind, g):
    from maskahead_b200.layouts import Prefix, pack_prefix

    def rnd(*shape):
        return torch.randn(*shape, generator=g, device=DEV).to(torch.bfloat16)

    if kind == "bf16":
        k, v = rnd(L, B, H, N, D), rnd(L, B, H, N, D)
        return [Prefix.dense(k[i], v[i]) for i in range(L)], Prefix.dense(k.flatten(0, 1), v.flatten(0, 1))
    packs = [pack_prefix(rnd(B, H, N, D), rnd(B, H, N, D), key_mode="token") for _ in range(L)]
    fields = ("kq", "ks", "kz", "vq", "vs", "vz", "kch")
    stacked = {f: torch.cat([getattr(p, f) for p in packs]) for f in fields}
    meta = {s: getattr(packs[0], s) for s in Prefix.__slots__
            if s not in fields and s not in ("kf", "vf", "mask", "pages", "lens")}
    per = [Prefix(**{f: stacked[f][i * B:(i + 1) * B] for f in fields}, **meta) for i in range(L)]
    return per, Prefix(**stacked, **meta)


@pytest.mark.parametrize("kind", ["bf16", "k4v4_token", "k4v4_token_unpacked"])
@pytest.mark.parametrize("probe_blocks", [0, 2])
def test_all_layers_selected_at_once_equal_the_per_layer_step0(kind, probe_blocks):
    from maskahead_b200.hotpath import fast_step0, select_step0, step0_attention

    g = torch.Generator(device=DEV).manual_seed(11 + probe_blocks)
    per, stacked = _caches("bf16" if kind == "bf16" else "k4v4_token", g)
    Tq = T * (1 + probe_blocks)
    q = torch.randn(L, B, HQ, Tq, D, generator=g, device=DEV).to(torch.bfloat16)
    kc = torch.randn(L, B, H, Tq, D, generator=g, device=DEV).to(torch.bfloat16)
    vc = torch.randn(L, B, H, Tq, D, generator=g, device=DEV).to(torch.bfloat16)
    rows = torch.arange(T, device=DEV, dtype=torch.int32)
    probe_rows = torch.arange(T, Tq, device=DEV, dtype=torch.int32)
    scale = D ** -0.5
    kw = dict(probe_blocks=probe_blocks, block_size=T)

    want = []
    for i in range(L):
        ck = torch.empty(B, H, K, D, device=DEV, dtype=torch.bfloat16)
        cv = torch.empty_like(ck)
        res = fast_step0(q[i], per[i], kc[i], vc[i], query_indices=rows, topk=K, scaling=scale, gather=True,
                         compact_out=(ck, cv), probe_rows=probe_rows, **kw)
        want.append((res.out.clone(), res.indices.clone(), res.mass.clone(), res.score.clone(), ck, cv,
                     None if res.probe_mass is None else res.probe_mass.clone()))

    G = HQ // H
    mp = torch.empty(L, B, H, G * Tq, device=DEV, dtype=torch.float32)
    lp = torch.empty_like(mp)
    outs = []
    uk = uv = None
    if kind == "k4v4_token_unpacked":
        from maskahead_b200.layouts import Prefix

        uk = torch.empty(L, B, H, N, D, device=DEV, dtype=torch.bfloat16)
        uv = torch.empty_like(uk)
    for i in range(L):
        out, _ = step0_attention(q[i], per[i], kc[i], vc[i], scaling=scale, stats_out=(mp[i], lp[i]),
                                 unpack_out=None if uk is None else (uk[i], uv[i]), **kw)
        outs.append(out)
    if uk is not None:
        stacked = Prefix.dense(uk.flatten(0, 1), uv.flatten(0, 1))
    CK = torch.empty(L, B, H, K, D, device=DEV, dtype=torch.bfloat16)
    CV = torch.empty_like(CK)
    got = select_step0(q.flatten(0, 1), stacked, (mp.flatten(0, 1), lp.flatten(0, 1)), query_indices=rows, topk=K,
                       scaling=scale, gather=True, compact_out=(CK.flatten(0, 1), CV.flatten(0, 1)),
                       probe_rows=probe_rows, **kw)
    torch.cuda.synchronize()
    assert got.out is None and got.indices.shape == (L * B, H, K)
    idx = got.indices.view(L, B, H, K)
    mass = got.mass.view(L, B, H, N)
    score = got.score.view(L, B, H, N)
    for i in range(L):
        w_out, w_idx, w_mass, w_score, w_ck, w_cv, w_probe = want[i]
        assert torch.equal(outs[i], w_out), f"layer {i}: attention output"
        assert torch.equal(mass[i], w_mass), f"layer {i}: mass"
        torch.testing.assert_close(score[i], w_score, rtol=1e-5, atol=1e-12)
        band_equal(idx[i].cpu().numpy(), w_idx.cpu().numpy(), w_score.cpu().numpy(), K, rel=1e-5)
        same = (idx[i] == w_idx).all(dim=-1)                 # [B, H]: rows whose read sets agree
        assert torch.equal(CK[i][same], w_ck[same]) and torch.equal(CV[i][same], w_cv[same])
        if probe_blocks:
            assert torch.equal(got.probe_mass.view(L, B, H, N)[i], w_probe), f"layer {i}: probe mass"
    np.testing.assert_equal(np.isfinite(score.cpu().numpy()).all(), True)
