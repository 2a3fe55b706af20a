#!/usr/bin/env python
"""Benchmark of the MaskAhead select + attend block-step on B200.

Workloads (--config picks one, the default is the headline cfg2):

  cfg2  28 layers, batch 1, 28 query / 4 KV heads, head_dim 128, bf16 K/V, prefix 8192,
        a 32-token mask block denoised in 4 sub-steps, read budget 1024, retain budget
        2048, one lookahead block.  --gpus N: one sequence per rank (weak scaling).
  cfg3  cfg2 with the prefix in k4v4 token mode (4-bit K/V, fp16 scale/zero per token
        per 32-channel group, 1% of the key channels x8 as outliers before quantization).
  cfg4  32 layers, 32 query / 8 KV heads, bf16, prefix 65536, read budget 4096, retain
        8192, two lookahead blocks; --gpus N shards the KV heads (strong scaling) and
        all-gathers the head outputs of every layer step over NVLink (NCCL).
  cfg5  serving batch: 256 sequences of the cfg3 shape, prefix lengths U[4096, 16384],
        k4v4 token mode in a shuffled pool of 64-slot pages; --gpus N shards the
        sequences (strong scaling, no collective). Retention is not part of this step:
        the retention kernel takes one live length for all lanes.

One step = one block-step over all layers:
  step 0     score (prefix mass of the 32 mask queries x G query heads), value-aware
             score, top-k read set, dense attention over [prefix | block];
  3 sparse sub-steps: attention over [read set | block];
  retention (every 4th block, interval_blocks = 4): probe attention of the lookahead
             block(s), probe mass, lookahead value score, survivors.
Synthetic seeded inputs, N(0,1); every cache exceeds L2 (126 MB), so each step reads it
from HBM. `value` = tokens/s (32 tokens per block-step per sequence) over all ranks.

  python bench.py [--config cfg2] [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
"""

from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import threading
import time
from pathlib import Path

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

_BASE = dict(L=28, B=1, Hq=28, H=4, D=128, T=32, n=8192, k=1024, C=2048, substeps=4, probe_blocks=1,
             interval=4, W=64, sinks=4, seed=1234, kv="bf16", shard="seqs", scaling="weak", retention=True)
CONFIGS = {
    "cfg2": dict(_BASE, name="cfg2",
                 workload="cfg2: 28 layers, 28q/4kv heads, d128, bf16 K/V, prefix 8192, block 32 x 4 sub-steps, "
                          "k_r 1024, C 2048, 1 lookahead block, retention every 4 blocks"),
    "cfg3": dict(_BASE, name="cfg3", kv="k4v4_token",
                 workload="cfg3: cfg2 shape with k4v4 token-mode K/V (4-bit, fp16 scale/zero per token per "
                          "32-channel group, 1% key channels x8 outliers), retention every 4 blocks"),
    "cfg4": dict(_BASE, name="cfg4", L=32, Hq=32, H=8, n=65536, k=4096, C=8192, probe_blocks=2, shard="heads",
                 scaling="strong",
                 workload="cfg4: 32 layers, 32q/8kv heads, d128, bf16 K/V, prefix 65536, k_r 4096, C 8192, "
                          "2 lookahead blocks; KV heads sharded across ranks, NCCL all-gather of head outputs"),
    "cfg5": dict(_BASE, name="cfg5", B=256, n=16384, n_min=4096, kv="k4v4_token_paged", page=64,
                 scaling="strong", retention=False,
                 workload="cfg5: 256 sequences of the cfg3 shape, prefix U[4096,16384], k4v4 token mode in "
                          "64-slot pages (shuffled pool), sequences sharded across ranks; step 0 + 3 sub-steps"),
}
METRIC = "µs per block-step select+attend; achieved HBM GB/s vs peak; tokens/s at 1/2/4/8 GPU"
# DRAM bytes (read + write) per launch of the step-0 attention kernel, from the ncu captures
# summarized in profiles/attn_partial_fa_cfg2.md and profiles/attn_partial_fa_cfg4_step0.md
ATTN_TRAFFIC_BYTES = {"cfg2": 17_142_528, "cfg4": 273_547_264}


def parse_args():
    ap = argparse.ArgumentParser(description="MaskAhead select+attend block-step benchmark (B200)")
    ap.add_argument("--config", choices=sorted(CONFIGS), default="cfg2")
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=4)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--cpu-sample-layers", type=int, default=2)
    ap.add_argument("--layers", type=int, default=0,
                    help="override the config's layer count (profiling captures on a small device footprint; "
                         "the JSON line records it and is not the config's headline number)")
    ap.add_argument("--eager", action="store_true",
                    help="time eager block-steps instead of CUDA-graph replays (for launch lists: under ncu "
                         "the replay of a cooperative kernel node fails to launch)")
    return ap.parse_args()


# --------------------------------------------------------------------------- helpers
def peaks():
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return float(d["hbm_gbs"]), float(d["bf16_tflops"]), "measured"
    return 6650.0, 1590.0, "fallback"


class ClockSampler:
    """nvidia-smi clocks and throttle reasons sampled every 200 ms while running."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int):
        self.gpu = gpu_index
        self.samples: list[list[str]] = []
        self._stop = threading.Event()
        self._thr = threading.Thread(target=self._run, daemon=True)

    def _run(self):
        while not self._stop.is_set():
            try:
                out = subprocess.run(["nvidia-smi", "-i", str(self.gpu), f"--query-gpu={self.FIELDS}",
                                      "--format=csv,noheader,nounits"], capture_output=True, text=True,
                                     timeout=5).stdout.strip()
                if out:
                    self.samples.append([x.strip() for x in out.split(",")])
            except Exception:
                pass
            self._stop.wait(0.2)

    def __enter__(self):
        self._thr.start()
        return self

    def __exit__(self, *exc):
        self._stop.set()
        self._thr.join(timeout=10)

    def summary(self):
        if not self.samples:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"]}
        sm = [float(s[1]) for s in self.samples if s[1].replace(".", "").isdigit()]
        mx = [float(s[2]) for s in self.samples if s[2].replace(".", "").isdigit()]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for s in self.samples for i in range(4)
                          if len(s) > 5 + i and s[5 + i].lower().startswith("active")})
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": max(mx) if mx else None,
                "reasons": reasons, "samples": len(self.samples)}


def sequence_lengths(cfg: dict) -> list[int]:
    """Prefix length of every sequence of the job (seeded; the same on every rank)."""
    import torch

    if "n_min" not in cfg:
        return [cfg["n"]] * cfg["B"]
    g = torch.Generator().manual_seed(cfg["seed"] + 77)
    return torch.randint(cfg["n_min"], cfg["n"] + 1, (cfg["B"],), generator=g).tolist()


def rank_share(cfg: dict, rank: int, world: int) -> dict:
    """What one rank runs: its sequences (lengths) and KV heads."""
    lens = sequence_lengths(cfg)
    if cfg["shard"] == "heads":
        if cfg["H"] % world:
            raise SystemExit(f"{cfg['name']}: {cfg['H']} KV heads do not split over {world} ranks")
        h = cfg["H"] // world
        return dict(lens=lens, H=h, Hq=cfg["Hq"] // world, head0=rank * h)
    if cfg["scaling"] == "weak":
        return dict(lens=lens, H=cfg["H"], Hq=cfg["Hq"], head0=0)
    # strong scaling over sequences: contiguous ranges, each cut at the prefix sum nearest
    # to its ideal share of the total length (every share within one sequence of ideal)
    total = sum(lens)
    prefix = [0]
    for n in lens:
        prefix.append(prefix[-1] + n)
    bounds = [0]
    for r in range(1, world):
        goal = total * r / world
        i = min(range(bounds[-1], len(lens) + 1), key=lambda j: abs(prefix[j] - goal))
        bounds.append(i)
    bounds.append(len(lens))
    return dict(lens=lens[bounds[rank]:bounds[rank + 1]], H=cfg["H"], Hq=cfg["Hq"], head0=0)


# ------------------------------------------------------------------------- workload
def _outliers(k, g, frac: float = 0.01, factor: float = 8.0):
    """Scale a seeded 1% of the key channels of every head by 8 (in place), k [.., H, n, D]."""
    import torch

    D = k.shape[-1]
    nout = max(1, int(D * frac))
    for h in range(k.shape[-3]):
        ch = torch.randperm(D, generator=g, device=k.device)[:nout]
        k[..., h, :, ch] *= factor


class Workload:
    """Seeded synthetic inputs of one rank's share, resident on the device."""

    def __init__(self, cfg: dict, device, seed: int, share: dict, world: int = 1):
        import torch
        from maskahead_b200.layouts import Prefix, key_divisor, pack_prefix, quantize_tokens

        c = cfg
        g = torch.Generator(device=device).manual_seed(seed)
        bf = torch.bfloat16
        L, D, T, S, P = c["L"], c["D"], c["T"], c["substeps"], c["probe_blocks"]
        lens = share["lens"]
        B, H, Hq = len(lens), share["H"], share["Hq"]
        n = max(lens)
        self.cfg, self.device, self.world = c, device, world
        self.lens, self.B, self.H, self.Hq, self.n = lens, B, H, Hq, n

        def randn(*shape):
            return torch.randn(*shape, generator=g, device=device, dtype=torch.float32).to(bf)

        self.Q = randn(L, S, B, Hq, T, D)
        self.KC = randn(L, S, B, H, T, D)
        self.VC = randn(L, S, B, H, T, D)
        if c["retention"]:
            self.QP = randn(L, B, Hq, T * (1 + P), D)
            self.KCP = randn(L, B, H, T * (1 + P), D)
            self.VCP = randn(L, B, H, T * (1 + P), D)
            self.pos = torch.arange(n, device=device, dtype=torch.int32).expand(L, B, H, n).contiguous()
        self.rows = torch.arange(T, device=device, dtype=torch.int32)
        self.probe_rows = torch.arange(T, T * (1 + P), device=device, dtype=torch.int32)
        self.scale = D ** -0.5
        self.K = self.V = None
        self.prefixes = []
        if c["kv"] == "bf16":
            self.K = randn(L, B, H, n, D)
            self.V = randn(L, B, H, n, D)
        elif c["kv"] == "k4v4_token":
            for _ in range(L):
                k = torch.randn(B, H, n, D, generator=g, device=device)
                _outliers(k, g)
                self.prefixes.append(pack_prefix(k.to(bf), randn(B, H, n, D), key_mode="token"))
                del k
        elif c["kv"] == "k4v4_token_paged":
            page = c["page"]
            need = [(x + page - 1) // page for x in lens]
            npages, maxp = sum(need), max(need)
            cg = torch.Generator().manual_seed(seed + 5)
            perm = torch.randperm(npages, generator=cg)
            table = torch.full((B, maxp), -1, dtype=torch.int32)
            owner = torch.empty(npages, dtype=torch.int64)
            at = 0
            for b, m in enumerate(need):
                table[b, :m] = perm[at:at + m].to(torch.int32)
                owner[perm[at:at + m]] = b
                at += m
            self.pages = table.to(device)
            self.lens_t = torch.tensor(lens, dtype=torch.int32, device=device)
            own = owner.to(device)
            for _ in range(L):
                kpool = torch.randn(npages, H, page, D, generator=g, device=device)
                _outliers(kpool, g)
                kpool = kpool.to(bf)
                kdiv = key_divisor(kpool)                            # [pages, H, D], per page
                kchan = torch.zeros(B, H, D, device=device).index_reduce_(0, own, kdiv, "amax",
                                                                          include_self=False)
                kq, ks, kz = quantize_tokens(kpool, kchan[own])
                del kpool, kdiv
                vq, vs, vz = quantize_tokens(randn(npages, H, page, D))
                self.prefixes.append(Prefix(kq=kq, ks=ks, kz=kz, vq=vq, vs=vs, vz=vz, nq=n, kb=4, vb=4, kg=32,
                                            vg=32, kmode=1, kch=kchan, pages=self.pages, page_size=page,
                                            lens=self.lens_t))
        else:
            raise ValueError(c["kv"])
        # each layer's compact cache: the read set's K/V rows, gathered at step 0 and attended
        # by the sub-steps (the session's state.key / state.value)
        self.compact = [(torch.empty(B, H, c["k"], D, device=device, dtype=bf),
                         torch.empty(B, H, c["k"], D, device=device, dtype=bf)) for _ in range(L)]
        torch.cuda.synchronize(device)
        self.outputs = None

    def compact_buffers(self, layer: int):
        return self.compact[layer]

    def prefix(self, layer: int):
        from maskahead_b200.layouts import Prefix

        if self.prefixes:
            return self.prefixes[layer]
        return Prefix.dense(self.K[layer], self.V[layer])

    def gather_heads(self, out):
        """KV-head sharding: the full [B, Hq, T, D] output from every rank's heads (NCCL)."""
        if self.world == 1 or self.cfg["shard"] != "heads":
            return out
        return gather_heads(out, self.world)

    def block_step(self, retain: bool):
        """One block-step over every layer through the public hot-path API."""
        import torch
        from maskahead_b200.hotpath import (compact_attention, fast_step0, lookahead_survivors,
                                            probe_attention, value_score, value_score_prefix)

        c = self.cfg
        outs, idxs, masses = [], [], []
        for layer in range(c["L"]):
            pre = self.prefix(layer)
            # the read set's rows are gathered once into the layer's compact cache (the
            # session's state.key / state.value), which every sub-step attends
            res = fast_step0(self.Q[layer, 0], pre, self.KC[layer, 0], self.VC[layer, 0], query_indices=self.rows,
                             topk=c["k"], value_aware=True, scaling=self.scale, gather=True,
                             compact_out=self.compact_buffers(layer))
            out = self.gather_heads(res.out)
            for s in range(1, c["substeps"]):
                out = self.gather_heads(compact_attention(self.Q[layer, s], res.compact, None, self.KC[layer, s],
                                                          self.VC[layer, s], scaling=self.scale))
            outs.append(out)
            idxs.append(res.indices)
            masses.append(res.mass)
        keep = None
        if retain and c["retention"]:
            probe = []
            for layer in range(c["L"]):
                _, ap = probe_attention(self.QP[layer], self.prefix(layer), self.KCP[layer], self.VCP[layer],
                                        block_size=c["T"], scaling=self.scale, probe_rows=self.probe_rows)
                probe.append(ap)
            a = torch.stack(masses) + torch.stack(probe)
            if self.V is not None:
                score = value_score(a, self.V)
            else:
                score = torch.stack([value_score_prefix(a[layer], self.prefix(layer)) for layer in range(c["L"])])
            keep = lookahead_survivors(self.pos, score, c["C"], recent_window=c["W"], sink_tokens=c["sinks"])
        self.outputs = (outs, idxs, keep)
        return self.outputs


def gather_heads(out, world: int):
    """All-gather of per-rank head outputs [B, Hq/world, T, D] into [B, Hq, T, D]; rank r
    holds query heads [r*Hq/world, (r+1)*Hq/world) (the heads of its KV heads)."""
    import torch
    import torch.distributed as dist

    b = out.shape[0]
    buf = torch.empty((world * b,) + tuple(out.shape[1:]), device=out.device, dtype=out.dtype)
    dist.all_gather_into_tensor(buf, out.contiguous())   # rank-major along dim 0
    return buf.view(world, b, *out.shape[1:]).permute(1, 0, 2, 3, 4).reshape(b, -1, out.shape[2], out.shape[3])


def fused_scores(cfg: dict, share: dict) -> bool:
    """Whether step 0's value score runs inside the (cooperative) mass launch: every CTA
    of the launch must be resident, i.e. B*H <= the SM count."""
    return len(share["lens"]) * share["H"] <= 148


def kernel_launches(cfg: dict, share: dict, retain: bool) -> int:
    """Our kernels in one block-step: step 0 = attention partial + combine + mass (with the
    fused value score, or + value apply) + top-k; each sub-step = partial + combine;
    retention = per layer probe partial + combine + mass, then value centre + apply (once
    for dense values, per layer for packed ones) and the survivors."""
    step0 = 4 if fused_scores(cfg, share) else 5
    n = (step0 + 2 * (cfg["substeps"] - 1)) * cfg["L"]
    if retain and cfg["retention"]:
        n += 3 * cfg["L"] + (2 if cfg["kv"] == "bf16" else 2 * cfg["L"]) + 1
    return n


def graph_kernel_count(g) -> int | None:
    """Kernel nodes of a captured (keep_graph=True) CUDA graph whose function is one of this
    library's kernels (mangled names in namespace ma); None when the driver bindings are
    unavailable."""
    try:
        from cuda.bindings import driver as dr

        graph = g.raw_cuda_graph()
        err, _, count = dr.cuGraphGetNodes(graph, 0)
        err, nodes, count = dr.cuGraphGetNodes(graph, count)
        if err != dr.CUresult.CUDA_SUCCESS:
            return None
        ours = 0
        for node in nodes[:count]:
            err, kind = dr.cuGraphNodeGetType(node)
            if err != dr.CUresult.CUDA_SUCCESS or kind != dr.CUgraphNodeType.CU_GRAPH_NODE_TYPE_KERNEL:
                continue
            err, params = dr.cuGraphKernelNodeGetParams(node)
            if err != dr.CUresult.CUDA_SUCCESS:
                return None
            err, name = dr.cuFuncGetName(params.func)
            if err != dr.CUresult.CUDA_SUCCESS:
                return None
            name = name.decode() if isinstance(name, bytes) else str(name)
            ours += name.startswith("_ZN2ma")
        return ours
    except Exception:
        return None


def token_bytes(cfg: dict) -> int:
    """K+V bytes per token per KV head: bf16 2*D*2, k4v4 token mode 2*(D/2 + 4*D/32)."""
    D = cfg["D"]
    return 2 * D * 2 if cfg["kv"] == "bf16" else 2 * (D // 2 + 4 * (D // 32))


def algorithmic_bytes(cfg: dict, share: dict) -> dict:
    """Bytes each phase must move at least on one rank (K/V counted once per read phase)."""
    L, D, T, k = cfg["L"], cfg["D"], cfg["T"], cfg["k"]
    lens, H, Hq = share["lens"], share["H"], share["Hq"]
    B = len(lens)
    bt = token_bytes(cfg)
    kchan = 0 if cfg["kv"] == "bf16" else B * H * D * 4
    q = B * Hq * T * D * 2
    cur = 2 * B * H * T * D * 2
    step0 = sum(lens) * H * bt + kchan + 2 * q + cur                # prefix K/V, Q, out, current K/V
    gather = B * H * k * (bt + 8 + 2 * D * 2) + kchan               # read set K/V + indices -> compact bf16
    sub = B * H * k * 2 * D * 2 + 2 * q + cur                       # the compact bf16 cache, Q, out, block K/V
    ret = (sum(lens) * H * bt + kchan) if cfg["retention"] else 0   # the probe re-reads the live set
    return dict(step0_layer=step0, gather_layer=gather, substep_layer=sub,
                block_step=L * (step0 + gather + (cfg["substeps"] - 1) * sub), retention=L * ret)


def step0_flops(cfg: dict, share: dict) -> float:
    """Tensor-core FLOPs of the step-0 attention partial kernel per layer: Q.K^T and P.V."""
    return 4.0 * share["Hq"] * cfg["T"] * sum(share["lens"]) * cfg["D"]


# ---------------------------------------------------------------------- CPU baseline
def cpu_block_step_time(cfg: dict, sample_layers: int, threads: int | None = None):
    """The oracle (a restatement of the reference's torch CPU path) timed on the host:
    step 0 (importance, value-aware rescoring, top-k, dense attention) and the sparse
    sub-steps (sdpa over the gathered read set) -- with packed caches dequantized first,
    as the reference's torch path reads them -- plus the retention scoring once per
    interval, for `sample_layers` layers of one sampled sequence; scaled to one
    block-step of the whole job (all layers, all sequences by their lengths).
    Returns (seconds per block-step, threads, sample description)."""
    import torch

    import oracle

    threads = threads or os.cpu_count() or 1
    torch.set_num_threads(threads)
    c = cfg
    g = torch.Generator().manual_seed(c["seed"])
    Hq, H, D, T = c["Hq"], c["H"], c["D"], c["T"]
    lens = sequence_lengths(c)
    n = int(statistics.median(lens))
    bf = torch.bfloat16
    rows = list(range(T))
    scale = D ** -0.5
    packed = c["kv"] != "bf16"

    def one_layer():
        k = torch.randn(1, H, n, D, generator=g)
        v = torch.randn(1, H, n, D, generator=g).to(bf)
        q = torch.randn(1, Hq, T, D, generator=g).to(bf)
        kc = torch.randn(1, H, T, D, generator=g).to(bf)
        vc = torch.randn(1, H, T, D, generator=g).to(bf)
        qp = torch.randn(1, Hq, T * (1 + c["probe_blocks"]), D, generator=g).to(bf)
        if packed:
            kb = k.to(bf)
            kchan = oracle.key_channel_divisor(kb)
            pk = oracle.quantize_keys_token(kb, kchan)
            pv = oracle.quantize_values(v)
        else:
            k = k.to(bf)
        t0 = time.perf_counter()
        if packed:   # the reference's torch path dequantizes the packed view before attending
            k = oracle.dequantize_keys_token(*pk, kchan)
            v = oracle.dequantize_values(*pv)
        imp = oracle.selector_importance(q, k, query_indices=rows, scale=scale)
        score = oracle.rescore_by_value(imp, v)
        idx, _ = oracle.topk_reference_torch(score, c["k"])
        oracle.dense_attention(q, k, v, kc, vc, scale=scale)
        sk = torch.cat([oracle.gather_per_kv_head(k, idx), kc], dim=2)
        sv = torch.cat([oracle.gather_per_kv_head(v, idx), vc], dim=2)
        for _ in range(c["substeps"] - 1):
            oracle.sdpa_compact(q, sk, sv)
        t1 = time.perf_counter()
        if c["retention"]:
            ap = oracle.selector_importance(qp, k, query_indices=list(range(T, qp.shape[2])), scale=scale)
            oracle.lookahead_score(imp, ap, v)
        t2 = time.perf_counter()
        return t1 - t0, t2 - t1

    one_layer()  # warm-up
    step, ret = [], []
    for _ in range(sample_layers):
        a, b = one_layer()
        step.append(a)
        ret.append(b)
    t_surv = 0.0
    if c["retention"]:
        pos = torch.arange(n, dtype=torch.int32).expand(1, 1, H, n).contiguous()
        sc = torch.rand(1, 1, H, n, generator=g)
        t0 = time.perf_counter()
        oracle.survivors_lookahead(pos, sc, c["C"], recent_window=c["W"], sink_tokens=c["sinks"])
        t_surv = (time.perf_counter() - t0) * c["L"]
    scale_seqs = sum(lens) / n            # the job's sequences, by length
    per_block = scale_seqs * (c["L"] * statistics.median(step) +
                              (c["L"] * statistics.median(ret) + t_surv) / c["interval"])
    sample = (f"{sample_layers} layer(s) of one sequence (n={n}): step 0 + {c['substeps'] - 1} sparse sub-steps"
              + (" + retention scoring" if c["retention"] else "")
              + (" with k4v4 dequantization" if packed else "")
              + f" (median), scaled to {c['L']} layers x {len(lens)} sequence(s) by length"
              + (f", retention every {c['interval']} blocks" if c["retention"] else "")
              + f"; torch fp32 CPU, {threads} threads")
    return per_block, threads, sample


def tokens_per_step(cfg: dict) -> int:
    return cfg["T"] * cfg["B"]


def run_reference(args):
    """--impl reference: the reference algorithm's CPU path (the oracle restatement; the
    reference package itself is not shipped to the GPU box) on the host cores."""
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    c = CONFIGS[args.config]
    t_block, threads, sample = cpu_block_step_time(c, max(1, args.cpu_sample_layers))
    steps = []
    for _ in range(max(1, args.steps // 10)):
        t, _, _ = cpu_block_step_time(c, 1, threads)
        steps.append(t)
    t_block = statistics.median(steps + [t_block])
    world = args.gpus if c["scaling"] == "weak" else 1
    tok_s = tokens_per_step(c) * world / t_block
    line = {"impl": "reference", "metric": METRIC, "value": tok_s, "unit": "tokens/s", "n_gpus": args.gpus,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": t_block * 1e3,
            "us_per_block_step": t_block * 1e6, "higher_is_better": True, "scaling": c["scaling"],
            "vs_baseline": None, "dtype": "f32", "data": "synthetic",
            "config": {"workload": c["workload"], "global_batch": c["B"] * world, "seq_len": c["n"],
                       "parallelism": "cpu"},
            "cpu_baseline": {"value": tok_s, "unit": "tokens/s", "cores": threads, "kind": "port",
                             "sample": sample},
            "e2e": {"value": tok_s, "unit": "tokens/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


# ------------------------------------------------------------------------ our arm
def _timed(fn, steps: int, stream):
    """CUDA-event time of `steps` calls of fn(i) on `stream` (ms total)."""
    import torch

    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    start.record(stream)
    for i in range(steps):
        fn(i)
    end.record(stream)
    end.synchronize()
    return start.elapsed_time(end)


def _max_over_ranks(x: float, world: int, dev) -> float:
    if world == 1:
        return x
    import torch
    import torch.distributed as dist

    t = torch.tensor([x], device=dev)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def run_ours(args):
    import torch
    import torch.distributed as dist

    import maskahead_b200
    from maskahead_b200.hotpath import unpacked_prefix
    from maskahead_b200.kernels import splitk_attention

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        import datetime
        dist.init_process_group("nccl", device_id=dev, timeout=datetime.timedelta(seconds=120))
    maskahead_b200.load_library()
    c = dict(CONFIGS[args.config])
    if args.layers > 0:
        c["L"] = args.layers
    share = rank_share(c, rank, world)
    seed = c["seed"] + (rank if c["scaling"] == "weak" else 0) * 1000 + share["head0"]
    wl = Workload(c, dev, seed, share, world)
    stream = torch.cuda.current_stream(dev)
    retain_at = lambda i: c["retention"] and (i % c["interval"]) == c["interval"] - 1  # noqa: E731

    # eager warm-up (sizes the workspaces), then one CUDA graph per step kind
    for i in range(max(1, args.warmup)):
        wl.block_step(retain=retain_at(i))
    torch.cuda.synchronize()
    graphs, graph_outputs, graph_launches = {}, {}, {}
    side = torch.cuda.Stream(dev)
    timing = "CUDA-graph replay, CUDA events"
    try:
        if args.eager:
            raise RuntimeError("eager steps requested")
        side.wait_stream(stream)
        with torch.cuda.stream(side):
            for retain in sorted({retain_at(i) for i in range(c["interval"])}):
                g = torch.cuda.CUDAGraph(keep_graph=True)
                with torch.cuda.graph(g, stream=side):
                    graph_outputs[retain] = wl.block_step(retain)
                graph_launches[retain] = graph_kernel_count(g)
                g.instantiate()
                graphs[retain] = g
        stream.wait_stream(side)
        torch.cuda.synchronize()

        def step(i):
            graphs[retain_at(i)].replay()
    except Exception as exc:  # a collective that cannot be captured: eager steps
        graphs.clear()
        torch.cuda.synchronize()
        timing = ("eager steps (--eager), CUDA events" if args.eager else
                  f"eager steps (graph capture failed: {type(exc).__name__}), CUDA events")

        def step(i):
            wl.block_step(retain_at(i))

    for i in range(args.warmup):
        step(i)
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    with ClockSampler(local) as clocks:
        ms = _timed(step, args.steps, stream)
    torch.cuda.synchronize()
    ms = _max_over_ranks(ms, world, dev)
    ms_step = ms / args.steps
    # diagnostic: each kind of step on its own (a block-step without / with the retention pass)
    step_kinds = {}
    if graphs:
        for retain, g in sorted(graphs.items()):
            t = _timed(lambda i: g.replay(), 3, stream) / 3
            step_kinds["retention" if retain else "plain"] = _max_over_ranks(t, world, dev)
    seqs_job = c["B"] * (world if c["scaling"] == "weak" else 1)
    tokens = c["T"] * seqs_job
    value = tokens / (ms_step / 1e3)

    # dominant kernel: the step-0 attention (tensor-core partial pass + combine) per layer
    hbm_peak, tf_peak, peak_kind = peaks()
    g0 = torch.cuda.CUDAGraph()
    side.wait_stream(stream)
    def step0_attention(layer):
        # what fast_step0 runs: a packed prefix is unpacked to bf16 first
        pre = wl.prefix(layer)
        if pre.nq > 0:
            pre = unpacked_prefix(pre, wl.B, wl.H, c["D"])
        splitk_attention(wl.Q[layer, 0], pre, wl.KC[layer, 0], wl.VC[layer, 0], scaling=wl.scale, want_prefix=True)

    with torch.cuda.stream(side):
        for layer in range(c["L"]):   # warm the workspaces outside the capture
            step0_attention(layer)
        with torch.cuda.graph(g0, stream=side):
            for layer in range(c["L"]):
                step0_attention(layer)
    stream.wait_stream(side)
    for _ in range(3):
        g0.replay()
    torch.cuda.synchronize()
    reps = max(3, args.steps // 2)
    ms_attn = _timed(lambda i: g0.replay(), reps, stream) / (reps * c["L"])
    ms_attn = _max_over_ranks(ms_attn, world, dev)
    ab = algorithmic_bytes(c, share)
    achieved = ab["step0_layer"] / (ms_attn / 1e3) / 1e9
    tflops = step0_flops(c, share) / (ms_attn / 1e3) / 1e12

    # end to end through the public API with host buffers
    e2e = None
    if not args.no_e2e:
        hq = wl.Q.cpu().pin_memory()
        hkc, hvc = wl.KC.cpu().pin_memory(), wl.VC.cpu().pin_memory()
        hp = [t.cpu().pin_memory() for t in (wl.QP, wl.KCP, wl.VCP)] if c["retention"] else []
        outs_h = torch.empty((c["L"], wl.B, c["Hq"], c["T"], c["D"]), dtype=wl.Q.dtype).pin_memory()
        idx_h = torch.empty((c["L"], wl.B, wl.H, c["k"]), dtype=torch.int64).pin_memory()
        h2d_every = sum(t.numel() * t.element_size() for t in (hq, hkc, hvc))
        h2d_retain = sum(t.numel() * t.element_size() for t in hp)
        d2h = outs_h.numel() * outs_h.element_size() + idx_h.numel() * 8

        # Pipelined across steps when the block-step is a captured graph without a data-path
        # collective: two sets of device inputs (the second captured into its own graphs), the
        # copy stream moves step i+1's inputs in and step i's results out while step i
        # computes. Every step still copies its own inputs in and its results out inside
        # the timed region; the first step's copy-in is not overlapped.
        pipelined = bool(graphs) and (world == 1 or c.get("shard") != "heads")
        names = ("Q", "KC", "VC") + (("QP", "KCP", "VCP") if c["retention"] else ())
        sets, set_graphs, set_outputs = [], [], []
        if pipelined:
            sets.append({nm: getattr(wl, nm) for nm in names})
            set_graphs.append(graphs)
            set_outputs.append(graph_outputs)
            second = {nm: getattr(wl, nm).clone() for nm in names}
            for nm in names:
                setattr(wl, nm, second[nm])
            g2, o2 = {}, {}
            side.wait_stream(stream)
            with torch.cuda.stream(side):
                for retain in sorted(graphs):
                    g = torch.cuda.CUDAGraph()
                    with torch.cuda.graph(g, stream=side):
                        o2[retain] = wl.block_step(retain)
                    g2[retain] = g
            stream.wait_stream(side)
            torch.cuda.synchronize()
            for nm in names:
                setattr(wl, nm, sets[0][nm])
            sets.append(second)
            set_graphs.append(g2)
            set_outputs.append(o2)
        host = {"Q": hq, "KC": hkc, "VC": hvc}
        if c["retention"]:
            host.update(zip(("QP", "KCP", "VCP"), hp))
        copy_stream = torch.cuda.Stream(dev)
        ev_in = [torch.cuda.Event(), torch.cuda.Event()]
        ev_done = [torch.cuda.Event(), torch.cuda.Event()]
        ev_out = [torch.cuda.Event(), torch.cuda.Event()]

        def copy_in(i):
            b = i % 2
            with torch.cuda.stream(copy_stream):
                if i >= 2:
                    copy_stream.wait_event(ev_done[b])   # step i-2 has read this set
                for nm in ("Q", "KC", "VC") + (("QP", "KCP", "VCP") if retain_at(i) else ()):
                    sets[b][nm].copy_(host[nm], non_blocking=True)
                ev_in[b].record(copy_stream)

        def compute_and_copy_out(i):
            b, retain = i % 2, retain_at(i)
            stream.wait_event(ev_in[b])
            if i >= 2:
                stream.wait_event(ev_out[b])             # step i-2's results are out
            set_graphs[b][retain].replay()
            ev_done[b].record(stream)
            outs, idxs, _ = set_outputs[b][retain]
            with torch.cuda.stream(copy_stream):
                copy_stream.wait_event(ev_done[b])
                for layer in range(c["L"]):
                    outs_h[layer].copy_(outs[layer], non_blocking=True)
                    idx_h[layer].copy_(idxs[layer], non_blocking=True)
                ev_out[b].record(copy_stream)

        def run_pipelined(steps):
            copy_stream.wait_stream(stream)   # after the timing start
            copy_in(0)
            for i in range(steps):
                if i + 1 < steps:
                    copy_in(i + 1)
                compute_and_copy_out(i)
            stream.wait_stream(copy_stream)

        # the outputs of the captured step live in the graph's static buffers (wl.outputs
        # holds them after the capture); eager steps produce fresh ones
        def e2e_step(i):
            retain = retain_at(i)
            wl.Q.copy_(hq, non_blocking=True)
            wl.KC.copy_(hkc, non_blocking=True)
            wl.VC.copy_(hvc, non_blocking=True)
            if retain:
                for dst, src in zip((wl.QP, wl.KCP, wl.VCP), hp):
                    dst.copy_(src, non_blocking=True)
            if graphs:
                graphs[retain].replay()
                outs, idxs, _ = graph_outputs[retain]
            else:
                outs, idxs, _ = wl.block_step(retain)
            for layer in range(c["L"]):
                outs_h[layer].copy_(outs[layer], non_blocking=True)
                idx_h[layer].copy_(idxs[layer], non_blocking=True)

        if pipelined:
            run_pipelined(2)
        else:
            for i in range(2):
                e2e_step(i)
        torch.cuda.synchronize()
        if world > 1:
            dist.barrier()
        if pipelined:
            ms_e = _max_over_ranks(_timed(lambda i: run_pipelined(args.steps) if i == 0 else None, 1, stream),
                                   world, dev)
        else:
            ms_e = _max_over_ranks(_timed(e2e_step, args.steps, stream), world, dev)
        e2e = {"value": tokens / (ms_e / args.steps / 1e3), "unit": "tokens/s",
               "h2d_bytes_per_step": int(h2d_every + (h2d_retain / c["interval"] if c["retention"] else 0)),
               "d2h_bytes_per_step": int(d2h), "ms_per_step": ms_e / args.steps,
               "path": ("pinned host -> device copies of the step's queries and block K/V, the block-step "
                        "through the public API (maskahead_b200.hotpath) " +
                        ("as a CUDA-graph replay" if graphs else "eagerly") +
                        ", device -> pinned host copies of every layer's output and read set" +
                        ("; copies on a second stream overlap the neighbouring steps' compute (two input "
                         "sets, the first step's copy-in not overlapped)" if pipelined else ""))}

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        t_block, threads, sample = cpu_block_step_time(c, max(1, args.cpu_sample_layers))
        cpu = {"value": tokens_per_step(c) / t_block, "unit": "tokens/s", "cores": threads, "kind": "port",
               "sample": sample}

    if world > 1:
        dist.barrier()
        for g in list(graphs.values()) + [g0]:
            del g
        graphs.clear()
        del g0
        torch.cuda.synchronize()
        dist.destroy_process_group()
    if rank != 0:
        return
    n_ret = sum(1 for i in range(args.steps) if retain_at(i))
    if graphs and all(graph_launches.get(r) is not None for r in graphs):
        # counted: the kernel nodes of the captured step graphs that run this library's kernels
        launches = sum(graph_launches[retain_at(i)] for i in range(args.steps))
        launches_source = "kernel nodes of the captured block-step graphs in namespace ma"
    else:
        launches = n_ret * kernel_launches(c, share, True) + (args.steps - n_ret) * kernel_launches(c, share, False)
        launches_source = "per-step formula (kernel_launches)"
    if c["scaling"] == "weak":   # every rank runs the same share
        job_ab = {key: world * val for key, val in ab.items()}
    else:                          # the whole job's sequences and heads
        job_ab = algorithmic_bytes(c, dict(lens=sequence_lengths(c), H=c["H"], Hq=c["Hq"]))
    step_bytes = job_ab["block_step"] + job_ab["retention"] / c["interval"]
    parallelism = {"heads": f"kvheads{world} (NCCL all-gather of head outputs)" if world > 1 else "single GPU",
                   "seqs": f"seq{world} (no collective)"}[c["shard"]]
    line = {
        "metric": METRIC, "value": value, "unit": "tokens/s", "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": ms_step, "us_per_block_step": ms_step * 1e3,
        "higher_is_better": True, "scaling": c["scaling"], "vs_baseline": None, "dtype": "bf16",
        "data": "synthetic (seeded N(0,1) K/V/Q, random-init; no model weights)",
        "config": {"workload": c["workload"] + (f" [layers overridden: {c['L']}]" if args.layers > 0 else ""),
                   "global_batch": seqs_job, "seq_len": c["n"],
                   "parallelism": parallelism, "l2": "inputs larger than L2 (the per-step cache exceeds 126 MB)",
                   "timing": timing},
        "roofline": {"kernel": ("step-0 attention per layer: attn_partial_fa (merge fused)" if c["kv"] == "bf16" else
                                "step-0 attention per layer: unpack of the packed prefix + attn_partial_fa"),
                     "bound": "hbm",
                     "achieved": achieved, "peak": hbm_peak, "unit": "GB/s", "frac": achieved / hbm_peak,
                     "traffic": ATTN_TRAFFIC_BYTES.get(c["name"]), "peak_kind": f"{peak_kind} burst",
                     "traffic_source": "ncu dram__bytes_read.sum + dram__bytes_write.sum of attn_partial_fa, "
                                       "profiles/attn_partial_fa_cfg2.md (cfg2), profiles/attn_partial_fa_cfg4_step0.md "
                                       "(cfg4)",
                     "us_per_launch": ms_attn * 1e3, "tensor_tflops": tflops, "tensor_frac": tflops / tf_peak,
                     "bytes_per_launch": ab["step0_layer"]},
        "ms_per_step_kind": step_kinds,
        "algorithmic_bytes_per_step": step_bytes,
        "achieved_step_gbs": step_bytes / (ms_step / 1e3) / 1e9,
        "block_steps_per_s": seqs_job / (ms_step / 1e3),
        "cpu_baseline": cpu, "e2e": e2e, "gpu_launches": launches, "gpu_launches_source": launches_source,
        "clocks": clocks.summary(),
    }
    print(json.dumps(line), flush=True)


def main():
    args = parse_args()
    if args.impl == "reference":
        run_reference(args)
    else:
        run_ours(args)


if __name__ == "__main__":
    main()
