"""The reference's own BitSieveSession with the sm_100a operators bound in (dropin.install).

One block loop runs twice on one set of seeded inputs, through the reference package's
public session API (begin_block / prepare_forward / attend / finish_step0 /
stage_if_committing / end_block, runtime/session.py:374-427, 1264-1285, 2254-2528, driven
as runtime/generator.py:339-494 drives it):

* first unpatched on the CPU: the reference's torch path (runtime/session.py:2310-2418:
  selector_topk + the value-aware rescoring + gather at step 0, dense_packed_attention on
  the dense layers, sdpa over the compact buffer at the sub-steps);
* then on the GPU with maskahead_b200.dropin installed, which the session serves through
  its fast path (runtime/session.py:1403-1459: splitk_attention + prefix_scores + top-k +
  gather_packed_kv at step 0, sdpa_compact at the sub-steps, splitk_attention on the
  dense layers), the prefill and the commit forwards appending through the cache's
  quantizers (cache.py:482-540) -- every operator one of ours.

Per block, step and layer the outputs agree within the bf16 tolerance (2e-2), and every
sparse layer's read set equals the CPU session's up to ties of the value-aware score
(the oracle's score over the CPU cache's own dequantized K/V, relative band 1e-4).
Configurations: the shipped bf16 cache and KIVI k4v4 (token-mode keys run on the fast
path only, session.py:189-190, so the CPU session cannot serve them). Skipped when the
reference package is not importable (tests/reference_pkg.py).
"""

from __future__ import annotations

import numpy as np
import pytest
import torch

import oracle
from gpu_cases import band_equal
from reference_pkg import reference_package

REF = reference_package()
pytestmark = [pytest.mark.gpu,
              pytest.mark.skipif(REF is None, reason="reference package not installed (baseline/_ref)")]

L, HQ, H, D, BLOCK, SMALL = 3, 8, 2, 128, 32, 8
N0, BLOCKS = 1000, 2
STEPS = BLOCK // SMALL               # step 0 + 3 sub-steps, SMALL positions revealed each


def _config(quant: dict, selector: dict):
    from maskahead.config import ExperimentConfig

    raw = dict(name="dropin", semantic="A", backend="auto", async_selector=False, max_cache_tokens=4096,
               quant=dict(key_token_group=32, value_channel_group=32, param_dtype="float16", **quant),
               selector={**dict(mode="all", topk=96, domain="prefix", score="softmax", dense_prefix_layers=1,
                                sort_indices=True), **selector},
               generation=dict(block_size=BLOCK, small_block_size=SMALL, max_new_tokens=BLOCK * BLOCKS),
               eviction=dict(policy="none"))
    return ExperimentConfig.from_dict(raw)


CASES = {
    "bf16_value_aware": (dict(k_bits=16, v_bits=16, residual_tokens=0),
                         dict(value_aware=True, value_center="attn")),
    "kivi4_value_aware": (dict(k_bits=4, v_bits=4, residual_tokens=32, key_mode="channel"),
                          dict(value_aware=True, value_center="attn")),
    "bf16_mass_middle": (dict(k_bits=16, v_bits=16, residual_tokens=0),
                         dict(value_aware=False, mode="middle")),
}


def _inputs(seed: int):
    g = torch.Generator().manual_seed(seed)

    def rnd(*shape, s=1.0):
        return (torch.randn(*shape, generator=g) * s).to(torch.bfloat16)

    prefill = [(rnd(1, H, N0, D), rnd(1, H, N0, D)) for _ in range(L)]
    blocks = []
    for _ in range(BLOCKS):
        steps = [[(rnd(1, HQ, BLOCK, D, s=2.0), rnd(1, H, BLOCK, D), rnd(1, H, BLOCK, D)) for _ in range(L)]
                 for _ in range(STEPS + 1)]          # the last one is the commit forward
        blocks.append(steps)
    return prefill, blocks


def _drive(cfg, prefill, blocks, device, record_kv: bool):
    from maskahead.cache import PackedKVCache
    from maskahead.runtime.session import BitSieveSession

    cache = PackedKVCache(num_layers=L, batch_size=1, num_kv_heads=H, head_dim=D, max_tokens=cfg.max_cache_tokens,
                          quant=cfg.quant, device=device, compute_dtype=torch.bfloat16, backend=cfg.backend)
    cache.begin_append(N0)
    for layer, (k, v) in enumerate(prefill):
        cache.stage_layer(layer, k.to(device), v.to(device))
    cache.commit_append()
    session = BitSieveSession(cache, cfg, num_q_heads=HQ, num_kv_heads=H, head_dim=D, compute_dtype=torch.bfloat16)
    outs, reads, kv, qidx = {}, {}, {}, {}
    for b, steps in enumerate(blocks):
        masked = list(range(BLOCK))
        session.begin_block(masked)
        qidx[b] = list(session.query_indices)
        if record_kv:
            kv[b] = [tuple(t.float().cpu() for t in cache.dequantize_layer(layer)) for layer in range(L)]
        for s in range(STEPS):
            session.prepare_forward(s, masked_positions=masked)
            for layer, (q, k, v) in enumerate(steps[s]):
                outs[(b, s, layer)] = session.attend(layer, q.to(device), k.to(device), v.to(device)).float().cpu()
            if s == 0:
                session.finish_step0()
                for layer in range(L):
                    st = session._states.get(layer)
                    if st is not None and st.indices is not None:
                        reads[(b, layer)] = st.indices.cpu().numpy()
            masked = masked[SMALL:]
        cache.begin_append(BLOCK)
        session.prepare_forward(STEPS, masked_positions=[], commit_current=True)
        for layer, (q, k, v) in enumerate(steps[STEPS]):
            outs[(b, "commit", layer)] = session.attend(layer, q.to(device), k.to(device),
                                                        v.to(device)).float().cpu()
            session.stage_if_committing(layer, k.to(device), v.to(device))
        cache.commit_append()
        session.end_block()
    return outs, reads, kv, qidx, session.fast


@pytest.mark.parametrize("name", list(CASES))
def test_reference_session_with_the_shim_matches_its_cpu_session(name):
    from maskahead_b200 import device_status, dropin

    quant, selector = CASES[name]
    prefill, blocks = _inputs(seed=len(name))
    want, want_reads, kv, qidx, fast_cpu = _drive(_config(quant, selector), prefill, blocks, "cpu", True)
    assert not fast_cpu
    inst = dropin.install()
    try:
        got, got_reads, _, _, fast_gpu = _drive(_config(quant, selector), prefill, blocks, "cuda", False)
        torch.cuda.synchronize()
        device_status()
    finally:
        inst.uninstall()
    assert fast_gpu, "the session did not take its fast path"
    assert got.keys() == want.keys()
    for key in want:
        torch.testing.assert_close(got[key], want[key], rtol=2e-2, atol=2e-2, msg=lambda m, key=key: f"{key}: {m}")
    assert got_reads.keys() == want_reads.keys() and want_reads
    for (b, layer), idx in want_reads.items():
        key_l, val_l = kv[b][layer]
        q0 = blocks[b][0][layer][0].float()
        imp = oracle.selector_importance(q0, key_l, query_indices=qidx[b], scale=D ** -0.5)
        score = oracle.rescore_by_value(imp, val_l) if selector.get("value_aware") else imp
        band_equal(np.sort(got_reads[(b, layer)], -1), np.sort(idx, -1), score.numpy(), idx.shape[-1], rel=1e-4)
