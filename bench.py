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
        gathers the head outputs of every layer step over NVLink (peer stores of this
        library's own kernel into IPC-mapped receive regions, ma_head_gather).
  cfg5  serving batch: 256 sequences of the cfg3 shape, prefix lengths U[4096, 16384],
        k4v4 token mode in a shuffled pool of 64-slot pages; --gpus N shards the
        sequences (strong scaling, no collective). Retention is not part of this step:
        the retention kernel takes one live length for all lanes.

The headline line measures --config (default cfg2); the further configs (--configs,
default cfg3, cfg4 and cfg5) are measured in the same run, each under "configs" with its
own timing, e2e leg and per-kernel rooflines.

One step = one block-step over all layers:
  step 0     score (prefix mass of the 32 mask queries x G query heads), value-aware
             score, top-k read set, dense attention over [prefix | block];
  3 sparse sub-steps: attention over [read set | block];
  retention (every 4th block, interval_blocks = 4): the lookahead probe merged into step 0
             (one launch over [block | probe blocks], block-causal), the probe mass, the
             lookahead value score, survivors.
Synthetic seeded inputs, N(0,1); every cache exceeds L2 (126 MB), so each step reads it
from HBM. `value` = tokens/s (32 tokens per block-step per sequence) over all ranks.

Per kernel family ("rooflines"): one CUDA graph of one call per layer, L2 flushed before
every replay, achieved GB/s on algorithmic bytes against the measured HBM copy peak and
tensor TFLOP/s against the measured bf16 GEMM peaks (burst and sustained).

  python bench.py [--config cfg2] [--configs cfg3,cfg4,cfg5] [--gpus N] [--steps K] [--warmup W]
                  [--impl ours|reference]
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
                          "2 lookahead blocks; KV heads sharded across ranks, head outputs gathered by peer stores over NVLink"),
    "cfg5": dict(_BASE, name="cfg5", B=256, n=16384, n_min=4096, kv="k4v4_token_paged", page=64,
                 scaling="strong", retention=False,
                 workload="cfg5: 256 sequences of the cfg3 shape, prefix U[4096,16384], k4v4 token mode in "
                          "64-slot pages (shuffled pool), sequences sharded across ranks; step 0 + 3 sub-steps"),
}
METRIC = "µs per block-step select+attend; achieved HBM GB/s vs peak; tokens/s at 1/2/4/8 GPU"
# DRAM bytes (read + write) per launch of a kernel family, from the ncu captures summarized in
# profiles/attn_partial_fa_cfg2.md (cfg2 step 0 and sub-step) and
# profiles/attn_partial_fa_cfg4_step0.md (cfg4 step 0)
TRAFFIC_BYTES = {("cfg2", "step0_attention"): 17_142_528, ("cfg4", "step0_attention"): 273_547_264,
                 ("cfg2", "substep_attention"): 2_461_952}


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
    ap.add_argument("--batch", type=int, default=0,
                    help="override the config's number of sequences (profiling captures on a small device "
                         "footprint; the JSON line records it and is not the config's headline number)")
    ap.add_argument("--configs", default="auto",
                    help="further configs measured in the same run, each reported under 'configs' with its own "
                         "timing, e2e and rooflines (comma list; 'auto': cfg3,cfg4,cfg5; '' for none)")
    ap.add_argument("--eager", action="store_true",
                    help="time eager block-steps instead of CUDA-graph replays (for launch lists: under ncu "
                         "the replay of a cooperative kernel node fails to launch)")
    return ap.parse_args()


# --------------------------------------------------------------------------- helpers
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
    """What one rank runs: its sequences (lengths) and KV heads (maskahead_b200.shard)."""
    from maskahead_b200.shard import head_shard, sequence_shard

    lens = sequence_lengths(cfg)
    if cfg["shard"] == "heads":
        try:
            hs = head_shard(cfg["H"], cfg["Hq"], world, rank)
        except ValueError as exc:
            raise SystemExit(f"{cfg['name']}: {exc}")
        return dict(lens=lens, H=hs.H, Hq=hs.Hq, head0=hs.h0)
    if cfg["scaling"] == "weak":
        return dict(lens=lens, H=cfg["H"], Hq=cfg["Hq"], head0=0)
    return dict(lens=sequence_shard(lens, world, rank).lens, H=cfg["H"], Hq=cfg["Hq"], head0=0)


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
        self.K = self.V = self.UK = self.UV = None
        self.prefixes = []
        if c["kv"] == "bf16":
            self.K = randn(L, B, H, n, D)
            self.V = randn(L, B, H, n, D)
            self.prefix_all = Prefix.dense(self.K.flatten(0, 1), self.V.flatten(0, 1))
        elif c["kv"] == "k4v4_token":
            packs = []
            for _ in range(L):
                k = torch.randn(B, H, n, D, generator=g, device=device)
                _outliers(k, g)
                packs.append(pack_prefix(k.to(bf), randn(B, H, n, D), key_mode="token"))
                del k
            # one layer-stacked allocation [L*B, H, n, ...] per field (a cache's layers side
            # by side), each layer's Prefix a view of its slice
            fields = ("kq", "ks", "kz", "vq", "vs", "vz", "kch")
            stacked = {f: torch.cat([getattr(pk, f) for pk in packs]) for f in fields}
            meta = {sl: getattr(packs[0], sl) for sl in Prefix.__slots__
                    if sl not in fields and sl not in ("kf", "vf", "mask", "pages", "lens")}
            del packs
            self.prefixes = [Prefix(**{f: stacked[f][l * B:(l + 1) * B] for f in fields}, **meta) for l in range(L)]
            self.prefix_all = Prefix(**stacked, **meta)
            # each layer's step-0 unpack (the path's bf16 copy of the packed prefix) into its
            # slice of layer-stacked buffers, which the batched selection then reads
            self.UK = torch.empty(L, B, H, n, D, device=device, dtype=bf)
            self.UV = torch.empty_like(self.UK)
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
        # by the sub-steps (the session's state.key / state.value); layer-stacked
        self.CK = torch.empty(L, B, H, c["k"], D, device=device, dtype=bf)
        self.CV = torch.empty_like(self.CK)
        self.compact = [(self.CK[layer], self.CV[layer]) for layer in range(L)]
        # one sequence per rank (cfg2, cfg3, cfg4): a layer's selection is a few CTAs per
        # launch, so step 0 selects for every layer at once after the step-0 attention of
        # all layers (the session's finish_step0), over the layer-stacked cache and the
        # prefix statistics each layer's attention writes into its slice of MP / LP
        self.batched = B == 1 and c["kv"] in ("bf16", "k4v4_token")
        G = Hq // H
        self.MP = torch.empty(L, B, H, G * T, device=device, dtype=torch.float32)
        self.LP = torch.empty_like(self.MP)
        if c["retention"]:
            self.MPR = torch.empty(L, B, H, G * T * (1 + P), device=device, dtype=torch.float32)
            self.LPR = torch.empty_like(self.MPR)
        torch.cuda.synchronize(device)
        self.outputs = None
        from maskahead_b200.shard import HeadGather, PeerHeadGather

        if world > 1 and c["shard"] == "heads":
            import torch.distributed as dist

            # the head outputs of every layer step, by this library's peer-store kernel
            self.head_gather = PeerHeadGather(world, dist.get_rank())
        else:
            self.head_gather = HeadGather(world)

    def compact_buffers(self, layer: int):
        return self.compact[layer]

    def unpack_out(self, layer: int):
        """Where a packed prefix's step-0 unpack goes in the batched block-step: this
        layer's slice of the stacked copy (None: the library's scratch)."""
        return None if self.UK is None else (self.UK[layer], self.UV[layer])

    def prefix_sel(self):
        """The layer-stacked cache the batched selection reads: the bf16 cache, or the
        step's unpacked copies of a packed one (the same bf16 numbers)."""
        from maskahead_b200.layouts import Prefix

        if self.UK is not None:
            return Prefix.dense(self.UK.flatten(0, 1), self.UV.flatten(0, 1))
        return self.prefix_all

    def prefix(self, layer: int):
        from maskahead_b200.layouts import Prefix

        if self.prefixes:
            return self.prefixes[layer]
        return Prefix.dense(self.K[layer], self.V[layer])

    def step0_prefix(self, layer: int):
        """The prefix step 0 of the batched block-step attends: the layer's slice of the
        step's unpacked copy for a packed cache (unpacked at the start of the step), else
        the cache."""
        from maskahead_b200.layouts import Prefix

        if self.UK is not None:
            return Prefix.dense(self.UK[layer], self.UV[layer])
        return self.prefix(layer)

    def gather_heads(self, out):
        """KV-head sharding: the full [B, Hq, T, D] output from every rank's heads (NCCL)."""
        if self.world == 1 or self.cfg["shard"] != "heads":
            return out
        return self.head_gather(out)

    def head_gather_arg(self, rows: int):
        """KV-head sharding: the attention call's head_gather argument -- the exchange of
        its output rows t < rows inside the attention launch, into a new [B, Hq, rows, D]
        tensor -- or None (one rank, or sequences sharded)."""
        import torch

        if self.world == 1 or self.cfg["shard"] != "heads":
            return None
        c = self.cfg
        gout = torch.empty(len(self.lens), c["Hq"], rows, c["D"], device=self.device, dtype=torch.bfloat16)
        return (self.head_gather, gout)

    def block_step(self, retain: bool):
        """One block-step over every layer through the public hot-path API."""
        import torch
        from maskahead_b200.hotpath import (compact_attention, fast_step0, lookahead_survivors, value_score,
                                            value_score_prefix)

        c = self.cfg
        if self.batched:
            return self.block_step_batched(retain)
        # a retention block runs its lookahead probe merged into step 0 (lookahead_merge):
        # one launch over [block | probe blocks] per layer instead of a second pass
        merge = retain and c["retention"]
        outs, idxs, masses, probe = [], [], [], []
        for layer in range(c["L"]):
            pre = self.prefix(layer)
            # the read set's rows are gathered once into the layer's compact cache (the
            # session's state.key / state.value), which every sub-step attends
            if merge:
                res = fast_step0(self.QP[layer], pre, self.KCP[layer], self.VCP[layer], query_indices=self.rows,
                                 topk=c["k"], value_aware=True, scaling=self.scale, gather=True,
                                 compact_out=self.compact_buffers(layer), probe_blocks=c["probe_blocks"],
                                 block_size=c["T"], probe_rows=self.probe_rows)
                out = self.gather_heads(res.out[:, :, :c["T"]])   # the block's rows
                probe.append(res.probe_mass)
            else:
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
            a = torch.stack(masses) + torch.stack(probe)
            if self.V is not None:
                score = value_score(a, self.V)
            else:
                score = torch.stack([value_score_prefix(a[layer], self.prefix(layer)) for layer in range(c["L"])])
            keep = lookahead_survivors(self.pos, score, c["C"], recent_window=c["W"], sink_tokens=c["sinks"])
        self.outputs = (outs, idxs, keep)
        return self.outputs


    def block_step_batched(self, retain: bool):
        """The block-step with step 0's selection run once for every layer: the step-0
        attention of each layer (its prefix statistics into the layer's slice of MP / LP),
        then select_step0 over the layer-stacked queries, cache and statistics (mass, score,
        top-k and the gather into the layer-stacked compact caches -- and, on a retention
        block, the merged probe's mass -- one launch each for all layers), then the
        sub-steps of every layer."""
        import torch
        from maskahead_b200.hotpath import (compact_attention, lookahead_survivors, select_step0,
                                            step0_attention, unpacked_prefix, value_score, value_score_prefix)
        from maskahead_b200.layouts import Prefix

        c = self.cfg
        L, T = c["L"], c["T"]
        merge = retain and c["retention"]
        outs = []
        if self.UK is not None:
            # a packed cache: every layer's prefix unpacked in one launch at the start of the
            # block-step (the cache does not change during it) into the layer-stacked copy
            # that step 0's attention of each layer and the batched selection read
            unpacked_prefix(self.prefix_all, L * self.B, self.H, c["D"],
                            out=(self.UK.flatten(0, 1), self.UV.flatten(0, 1)))
        for layer in range(L):
            hg = self.head_gather_arg(T)   # KV-head sharding: the exchange inside the launch
            if merge:
                out, _ = step0_attention(self.QP[layer], self.step0_prefix(layer), self.KCP[layer], self.VCP[layer],
                                         scaling=self.scale, stats_out=(self.MPR[layer], self.LPR[layer]),
                                         probe_blocks=c["probe_blocks"],
                                         block_size=T, head_gather=hg)
                outs.append(out[:, :, :T] if hg is None else hg[1])
            else:
                out, _ = step0_attention(self.Q[layer, 0], self.step0_prefix(layer), self.KC[layer, 0], self.VC[layer, 0],
                                         scaling=self.scale, stats_out=(self.MP[layer], self.LP[layer]),
                                         head_gather=hg)
                outs.append(out if hg is None else hg[1])
        # B == 1: merging the layer and batch axes of the queries is a view
        if merge:
            q0, st = self.QP.flatten(0, 1), (self.MPR.flatten(0, 1), self.LPR.flatten(0, 1))
        else:
            q0, st = self.Q[:, 0].flatten(0, 1), (self.MP.flatten(0, 1), self.LP.flatten(0, 1))
        res = select_step0(q0, self.prefix_sel(), st, query_indices=self.rows, topk=c["k"], value_aware=True,
                           scaling=self.scale, gather=True, compact_out=(self.CK.flatten(0, 1), self.CV.flatten(0, 1)),
                           probe_blocks=c["probe_blocks"] if merge else 0, block_size=T, probe_rows=self.probe_rows)
        for layer in range(L):
            compact = Prefix.dense(self.CK[layer], self.CV[layer])
            for s in range(1, c["substeps"]):
                hg = self.head_gather_arg(T)
                out = compact_attention(self.Q[layer, s], compact, None, self.KC[layer, s], self.VC[layer, s],
                                        scaling=self.scale, head_gather=hg)
                outs[layer] = out if hg is None else hg[1]
        n = self.prefix_all.n
        idx = res.indices.view(L, self.B, self.H, -1)
        keep = None
        if merge:
            a = res.mass.view(L, self.B, self.H, n) + res.probe_mass.view(L, self.B, self.H, n)
            score = value_score(a, self.V if self.V is not None else self.UV)   # every layer in one call
            keep = lookahead_survivors(self.pos, score, c["C"], recent_window=c["W"], sink_tokens=c["sinks"])
        self.outputs = (outs, [idx[layer] for layer in range(L)], keep)
        return self.outputs


def fused_scores(cfg: dict, share: dict) -> bool:
    """Whether step 0's value score runs inside the (cooperative) mass launch: every CTA
    of the launch must be resident, i.e. B*H <= the SM count."""
    return len(share["lens"]) * share["H"] <= 148


def kernel_launches(cfg: dict, share: dict, retain: bool) -> int:
    """Our kernels in one block-step (an upper bound; the bench counts the captured graph's
    kernel nodes when it can): step 0 = attention partial + combine + mass (with the fused
    value score, or + value apply) + top-k + gather per layer -- with the selection batched
    over the layers (one sequence), the attention per layer and the rest once; each
    sub-step = partial + combine; retention = the merged probe's mass launch (per layer, or
    once batched), then value centre + apply (once for dense values, per layer for packed
    ones unless batched) and the survivors."""
    L = cfg["L"]
    batched = len(share["lens"]) == 1 and cfg["kv"] in ("bf16", "k4v4_token")
    fused = (L * share["H"] <= 148) if batched else fused_scores(cfg, share)
    select = 3 if fused else 4
    n = L * (2 + 2 * (cfg["substeps"] - 1)) + select * (1 if batched else L)
    if retain and cfg["retention"]:
        n += (1 if batched else L) + (2 if cfg["kv"] == "bf16" or batched else 2 * L) + 1
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


# ---------------------------------------------------------------------- CPU baseline
def cpu_model() -> str:
    try:
        for line in Path("/proc/cpuinfo").read_text().splitlines():
            if line.startswith("model name"):
                return line.split(":", 1)[1].strip()
    except OSError:
        pass
    import platform

    return platform.processor() or "unknown"


class CpuBlockStep:
    """The oracle (a restatement of the reference's torch CPU path) for one sequence of
    prefix n on the host: per layer step 0 (importance, value-aware rescoring, top-k,
    dense attention over [prefix | block]) and the sparse sub-steps (sdpa over the gathered
    read set), with a packed cache dequantized first as the reference's torch path reads
    it; the retention scoring (probe importance, lookahead value score, survivors) per layer.
    Inputs of `distinct` layers are generated once (untimed) and used in turn."""

    def __init__(self, cfg: dict, n: int, distinct: int = 4):
        import torch

        import oracle

        c = self.cfg = cfg
        self.n = n
        g = torch.Generator().manual_seed(c["seed"])
        Hq, H, D, T = c["Hq"], c["H"], c["D"], c["T"]
        bf = torch.bfloat16
        self.packed = c["kv"] != "bf16"
        self.layers = []
        for _ in range(max(1, min(distinct, c["L"]))):
            k = torch.randn(1, H, n, D, generator=g).to(bf)
            v = torch.randn(1, H, n, D, generator=g).to(bf)
            d = dict(q=[torch.randn(1, Hq, T, D, generator=g).to(bf) for _ in range(c["substeps"])],
                     kc=torch.randn(1, H, T, D, generator=g).to(bf), vc=torch.randn(1, H, T, D, generator=g).to(bf),
                     qp=torch.randn(1, Hq, T * (1 + c["probe_blocks"]), D, generator=g).to(bf))
            if self.packed:
                kchan = oracle.key_channel_divisor(k)
                d.update(pk=oracle.quantize_keys_token(k, kchan), pv=oracle.quantize_values(v), kchan=kchan)
            else:
                d.update(k=k, v=v)
            self.layers.append(d)
        self.pos = torch.arange(n, dtype=torch.int32).expand(1, 1, H, n).contiguous()
        self.rows = list(range(T))
        self.probe_rows = list(range(T, T * (1 + c["probe_blocks"])))
        self.scale = D ** -0.5

    def _kv(self, d):
        import oracle

        if self.packed:   # the reference's torch path dequantizes the packed view before attending
            return oracle.dequantize_keys_token(*d["pk"], d["kchan"]), oracle.dequantize_values(*d["pv"])
        return d["k"], d["v"]

    def layer(self, i: int, retain: bool) -> float:
        """Seconds of layer i's block-step (and its retention scoring when retain)."""
        import torch

        import oracle

        c, d = self.cfg, self.layers[i % len(self.layers)]
        t0 = time.perf_counter()
        k, v = self._kv(d)
        q = d["q"][0]
        imp = oracle.selector_importance(q, k, query_indices=self.rows, scale=self.scale)
        score = oracle.rescore_by_value(imp, v)
        idx, _ = oracle.topk_reference_torch(score, c["k"])
        oracle.dense_attention(q, k, v, d["kc"], d["vc"], scale=self.scale)
        sk = torch.cat([oracle.gather_per_kv_head(k, idx), d["kc"]], dim=2)
        sv = torch.cat([oracle.gather_per_kv_head(v, idx), d["vc"]], dim=2)
        for s in range(1, c["substeps"]):
            oracle.sdpa_compact(d["q"][s], sk, sv)
        if retain and c["retention"]:
            ap = oracle.selector_importance(d["qp"], k, query_indices=self.probe_rows, scale=self.scale)
            sc = oracle.lookahead_score(imp, ap * c["probe_blocks"], v)
            oracle.survivors_lookahead(self.pos, sc.unsqueeze(0), c["C"], recent_window=c["W"],
                                       sink_tokens=c["sinks"])
        return time.perf_counter() - t0


def cpu_baseline(cfg: dict, budget_s: float = 20.0, threads: int | None = None) -> dict:
    """The oracle timed on the host cores, one sequence (the median length): whole
    block-steps over all layers when three of them fit in budget_s (each the step 0 and
    sub-steps of every layer, the retention scoring on every interval-th), else a sample
    of layers scaled to the block-step; scaled to the job's sequences by length."""
    import torch

    threads = threads or os.cpu_count() or 1
    torch.set_num_threads(threads)
    c = cfg
    lens = sequence_lengths(c)
    n = int(statistics.median(lens))
    step = CpuBlockStep(c, n)
    step.layer(0, True)                      # warm-up (untimed)
    probe = step.layer(1, False)
    L = c["L"]
    if 3 * L * probe <= budget_s:
        reps = max(3, min(c["interval"], int(budget_s // max(L * probe, 1e-6))))
        times = []
        for r in range(reps):
            retain = c["retention"] and (r % c["interval"]) == c["interval"] - 1
            times.append(sum(step.layer(i, retain) for i in range(L)))
        plain = [t for r, t in enumerate(times) if not (c["retention"] and (r % c["interval"]) == c["interval"] - 1)]
        ret = [t for t in times if t not in plain]
        per_block = statistics.mean(plain) if not ret else \
            ((c["interval"] - 1) * statistics.mean(plain) + statistics.mean(ret)) / c["interval"]
        sample = (f"{reps} whole block-steps of one sequence (n={n}, {L} layers: step 0 + {c['substeps'] - 1} "
                  f"sparse sub-steps each" + (f", the retention scoring in every {c['interval']}th" if ret else "")
                  + ")" + ("; k4v4 dequantization included" if step.packed else ""))
        layers_timed, whole_steps = reps * L, reps
    else:
        m = max(2, min(L, int(budget_s // max(probe, 1e-6))))
        plain = [step.layer(i, False) for i in range(m)]
        ret = [step.layer(i, True) - p for i, p in zip(range(min(2, m)), plain)] if c["retention"] else []
        per_block = L * statistics.median(plain) + (L * statistics.median(ret) / c["interval"] if ret else 0.0)
        sample = (f"{m} layer(s) of one sequence (n={n}): step 0 + {c['substeps'] - 1} sparse sub-steps (median), "
                  f"scaled to {L} layers" + (f", retention scoring every {c['interval']} blocks" if ret else "")
                  + ("; k4v4 dequantization included" if step.packed else ""))
        layers_timed, whole_steps = m, 0
    scale_seqs = sum(lens) / n
    if len(lens) > 1:
        sample += f"; scaled to {len(lens)} sequences by length"
    sample += f"; torch fp32 CPU, {threads} threads"
    return dict(seconds=per_block * scale_seqs, threads=threads, sample=sample, layers_timed=layers_timed,
                whole_steps=whole_steps, cpu_model=cpu_model())


def tokens_per_step(cfg: dict) -> int:
    return cfg["T"] * cfg["B"]


def run_reference(args):
    """--impl reference: the reference algorithm's CPU path (the oracle restatement; the
    reference package is pure Python and does not travel to the GPU box) on every host
    core, on the same workload as our arm. For a config whose block-step takes a few
    seconds on the host (cfg2, cfg3) each of the K timed steps is one whole block-step of
    all layers (the retention scoring in every interval-th), after W untimed ones; for the
    larger ones each step is a bounded sample (stated) scaled to the block-step."""
    import torch

    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    c = CONFIGS[args.config]
    threads = os.cpu_count() or 1
    torch.set_num_threads(threads)
    lens = sequence_lengths(c)
    n = int(statistics.median(lens))
    step = CpuBlockStep(c, n)
    step.layer(0, True)
    probe = step.layer(1, False)
    world = args.gpus if c["scaling"] == "weak" else 1
    if len(lens) == 1 and c["L"] * probe <= 3.0:
        retain_at = lambda i: c["retention"] and (i % c["interval"]) == c["interval"] - 1  # noqa: E731
        for i in range(args.warmup):
            for layer in range(c["L"]):
                step.layer(layer, retain_at(i))
        t0 = time.perf_counter()
        for i in range(args.steps):
            for layer in range(c["L"]):
                step.layer(layer, retain_at(i))
        t_block = (time.perf_counter() - t0) / args.steps
        steps, warmup = args.steps, args.warmup
        sample = (f"{args.steps} whole block-steps after {args.warmup} untimed (one sequence, n={n}, {c['L']} layers: "
                  f"step 0 + {c['substeps'] - 1} sparse sub-steps each, the retention scoring in every "
                  f"{c['interval']}th)" + ("; k4v4 dequantization included" if step.packed else ""))
    else:
        base = cpu_baseline(c, budget_s=30.0, threads=threads)
        t_block, steps, warmup, sample = base["seconds"], max(1, base["whole_steps"]), 1, base["sample"]
    tok_s = tokens_per_step(c) * world / t_block
    line = {"impl": "reference", "metric": METRIC, "value": tok_s, "unit": "tokens/s", "n_gpus": args.gpus,
            "steps": steps, "warmup": warmup, "ms_per_step": t_block * 1e3, "us_per_block_step": t_block * 1e6,
            "higher_is_better": True, "scaling": c["scaling"], "vs_baseline": None, "dtype": "f32",
            "data": "synthetic (seeded N(0,1) K/V/Q)",
            "config": {"workload": c["workload"], "global_batch": c["B"] * world, "seq_len": c["n"],
                       "parallelism": "cpu (host cores of rank 0)"},
            "cpu_baseline": {"value": tok_s, "unit": "tokens/s", "cores": threads, "kind": "port",
                             "cpu_model": cpu_model(), "sample": sample},
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


def _capture(fn, side, stream):
    """A CUDA graph of fn() captured on the side stream (kernel nodes kept for counting)."""
    import torch

    g = torch.cuda.CUDAGraph(keep_graph=True)
    side.wait_stream(stream)
    with torch.cuda.stream(side):
        with torch.cuda.graph(g, stream=side):
            out = fn()
    stream.wait_stream(side)
    count = graph_kernel_count(g)
    g.instantiate()
    return g, out, count


def kernel_rooflines(c: dict, wl, share: dict, dev, stream, side, reps: int, world: int) -> dict:
    """Each kernel family of the block-step on its own: a CUDA graph of one call per layer,
    replayed `reps` times with L2 flushed before every replay (the events bracket the replay
    only); per launch: time, algorithmic bytes, GB/s and tensor FLOP/s against the measured
    peaks."""
    import torch

    from maskahead_b200.hotpath import _needs_unpack, compact_attention, gather_read_set, unpacked_prefix
    from maskahead_b200.kernels import prefix_scores, select_topk_indices, splitk_attention

    hbm, tf_burst, tf_sust, kind = peaks_all()
    L, D, T, k = c["L"], c["D"], c["T"], c["k"]
    ab = algorithmic_bytes(c, share)
    B, H, Hq = len(share["lens"]), share["H"], share["Hq"]
    n_sum = sum(share["lens"])
    packed = c["kv"] != "bf16"
    flush = torch.empty(256 << 20, dtype=torch.uint8, device=dev)

    def pre(layer):
        # the prefix as fast_step0 reads it: a packed one unpacked to bf16 first (the step-0
        # family below includes that unpack: it is the path's, once per layer)
        p = wl.prefix(layer)
        return unpacked_prefix(p, B, H, D) if _needs_unpack(p, B, H, D, None) else p

    # the later kernels of step 0 read the same unpacked copy: for them, copies made once
    # (up to 8 GB of them, cycled over the layers; each larger than L2 or all distinct)
    copies = []
    if packed:
        per = B * H * max(share["lens"]) * D * 2 * 2
        for layer in range(max(1, min(L, (8 << 30) // max(per, 1)))):
            u = unpacked_prefix(wl.prefix(layer), B, H, D)
            copies.append(type(u)(**{**{s: getattr(u, s) for s in type(u).__slots__}, "kf": u.kf.clone(),
                                     "vf": u.vf.clone()}))

    def pre_k(layer):
        return copies[layer % len(copies)] if copies else wl.prefix(layer)

    # eager inputs of the later families (outside the graphs)
    stats, scores, idxs = [], [], []
    for layer in range(L):
        _, st = splitk_attention(wl.Q[layer, 0], pre_k(layer), wl.KC[layer, 0], wl.VC[layer, 0], scaling=wl.scale,
                                 want_prefix=True)
        stats.append(st)
        _, sc = prefix_scores(wl.Q[layer, 0], pre_k(layer), st, wl.rows, value=True, scaling=wl.scale)
        scores.append(sc)
        idx, _ = select_topk_indices(sc, min(k, min(share["lens"])), want_values=False,
                                     lens=getattr(wl, "lens_t", None))
        idxs.append(idx)
    compacts = [gather_read_set(pre_k(layer), idxs[layer], out=wl.compact_buffers(layer)) for layer in range(L)]
    if wl.batched:   # the selection's inputs of every layer, stacked as the block-step passes them
        q_all = wl.Q[:, 0].flatten(0, 1)
        sel_prefix = wl.prefix_sel()
        st_all = (torch.cat([st[0] for st in stats]), torch.cat([st[1] for st in stats]), None, sel_prefix)
        sc_all = torch.cat(scores)
        idx_all = torch.cat(idxs)
        ck_all, cv_all = wl.CK.flatten(0, 1), wl.CV.flatten(0, 1)
    torch.cuda.synchronize(dev)

    b_tok = token_bytes(c)
    q_bytes = B * Hq * T * D * 2
    families = {
        "step0_attention": (lambda layer: splitk_attention(wl.Q[layer, 0], pre(layer), wl.KC[layer, 0],
                                                           wl.VC[layer, 0], scaling=wl.scale, want_prefix=True),
                            ab["step0_layer"], 4.0 * Hq * T * n_sum * D,
                            ("unpack of the packed prefix to bf16 + " if packed else "")
                            + "attn_partial_fa (split-K, merge in the launch)"),
        "mass_value_score": (lambda layer: prefix_scores(wl.Q[layer, 0], pre_k(layer), stats[layer], wl.rows,
                                                         value=True, scaling=wl.scale),
                             n_sum * H * (512 if packed else b_tok) + q_bytes + 2 * n_sum * H * 4, 2.0 * Hq * T * n_sum * D,
                             "prefix_mass_fa (mass, centre and value score in one launch)"
                             + (" over the step's unpacked bf16 copy" if packed else "")),
        "select_topk": (lambda layer: select_topk_indices(scores[layer], idxs[layer].shape[2], want_values=False,
                                                          lens=getattr(wl, "lens_t", None)),
                        n_sum * H * 4 + B * H * k * 8, 0.0, "select_topk (radix select, ascending emission)"),
        "gather": (lambda layer: gather_read_set(pre_k(layer), idxs[layer], out=wl.compact_buffers(layer)),
                   ab["gather_layer"] + (B * H * c["k"] * (512 - b_tok) if packed else 0), 0.0,
                   "gather_kv (read set into the compact cache" + (", from the unpacked bf16 copy)" if packed else ")")),
        "substep_attention": (lambda layer: compact_attention(wl.Q[layer, 1], compacts[layer], None, wl.KC[layer, 1],
                                                              wl.VC[layer, 1], scaling=wl.scale),
                              ab["substep_layer"], 4.0 * Hq * T * (B * k + B * T) * D,
                              "attn_partial_fa over the compact cache (merge in the launch)"),
    }
    per_launch = {name: 1 for name in families}
    if wl.batched:
        # the block-step's selection: one launch over every layer (the layer-stacked inputs);
        # the per-launch figures below are then for all L layers
        sel = {
            "mass_value_score": (lambda layer: prefix_scores(q_all, sel_prefix, st_all, wl.rows, value=True,
                                                             scaling=wl.scale),
                                 L * (n_sum * H * (512 if packed else b_tok) + q_bytes + 2 * n_sum * H * 4),
                                 L * 2.0 * Hq * T * n_sum * D,
                                 "prefix_mass_fa over the layer-stacked cache (every layer in one launch)"
                                 + (", the step's unpacked bf16 copies" if packed else "")),
            "select_topk": (lambda layer: select_topk_indices(sc_all, idx_all.shape[2], want_values=False),
                            L * (n_sum * H * 4 + B * H * k * 8), 0.0,
                            "select_topk over every layer's scores in one launch"),
            "gather": (lambda layer: gather_read_set(sel_prefix, idx_all, out=(ck_all, cv_all)),
                       L * (ab["gather_layer"] + (B * H * c["k"] * (512 - b_tok) if packed else 0)), 0.0,
                       "gather_kv of every layer's read set into the layer-stacked compact caches"
                       + (" (from the unpacked bf16 copies)" if packed else "")),
        }
        families.update(sel)
        per_launch.update({name: L for name in sel})
    out = {}
    for name, (fn, nbytes, flops, what) in families.items():
        calls = 1 if per_launch[name] > 1 else L   # one launch covers every layer, or one per layer
        for layer in range(calls):      # workspaces at their final size before the capture
            fn(layer)
        g, _, _ = _capture(lambda: [fn(layer) for layer in range(calls)], side, stream)
        for _ in range(2):
            g.replay()
        total = 0.0
        for _ in range(reps):
            flush.fill_(1)
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record(stream)
            g.replay()
            e1.record(stream)
            e1.synchronize()
            total += e0.elapsed_time(e1)
        us = _max_over_ranks(total / (reps * calls), world, dev) * 1e3
        gbs = nbytes / (us * 1e-6) / 1e9
        row = {"kernel": what, "us_per_launch": us, "bytes_per_launch": int(nbytes), "achieved_gbs": gbs,
               "hbm_frac": gbs / hbm, "layers_per_launch": per_launch[name]}
        if flops:
            tfl = flops / (us * 1e-6) / 1e12
            row.update(tflops=tfl, tensor_frac_burst=tfl / tf_burst, tensor_frac_sustained=tfl / tf_sust)
        out[name] = row
        del g
    out["peaks"] = {"hbm_gbs": hbm, "bf16_tflops_burst": tf_burst, "bf16_tflops_sustained": tf_sust, "kind": kind}
    del flush
    return out


def peaks_all():
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return (float(d["hbm_gbs"]), float(d["bf16_tflops"]), float(d.get("bf16_tflops_sustained", d["bf16_tflops"])),
                "measured")
    return 6650.0, 1590.0, 1400.0, "fallback"


def e2e_leg(c: dict, wl, graphs: dict, graph_outputs: dict, retain_at, args, world: int, dev, stream, side) -> dict:
    """The block-step end to end through the public API with host buffers: every step
    copies its queries and block K/V in from pinned host memory and every layer's output
    and read set out. With captured graphs and no data-path collective the copies of step
    i+1 (in) and i (out) overlap step i's compute on a copy stream (two device input sets,
    each with its own graphs); otherwise the steps run serially."""
    import torch

    L = c["L"]
    names = ("Q", "KC", "VC") + (("QP", "KCP", "VCP") if c["retention"] else ())
    host = {nm: getattr(wl, nm).cpu().pin_memory() for nm in names}
    outs_h = torch.empty((L, wl.B, c["Hq"], c["T"], c["D"]), dtype=wl.Q.dtype).pin_memory()
    idx_h = torch.empty((L, wl.B, wl.H, c["k"]), dtype=torch.int64).pin_memory()
    h2d_every = sum(host[nm].numel() * host[nm].element_size() for nm in ("Q", "KC", "VC"))
    h2d_retain = sum(host[nm].numel() * host[nm].element_size() for nm in names[3:])
    d2h = outs_h.numel() * outs_h.element_size() + idx_h.numel() * 8
    pipelined = bool(graphs) and (world == 1 or c.get("shard") != "heads")
    copy_stream = torch.cuda.Stream(dev)
    if pipelined:
        sets = [{nm: getattr(wl, nm) for nm in names}]
        second = {nm: getattr(wl, nm).clone() for nm in names}
        for nm in names:
            setattr(wl, nm, second[nm])
        g2, o2 = {}, {}
        for retain in sorted(graphs):
            g2[retain], o2[retain], _ = _capture(lambda: wl.block_step(retain), side, stream)
        torch.cuda.synchronize(dev)
        for nm in names:
            setattr(wl, nm, sets[0][nm])
        sets.append(second)
        set_graphs, set_outputs = [graphs, g2], [graph_outputs, o2]
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
                for layer in range(L):
                    outs_h[layer].copy_(outs[layer], non_blocking=True)
                    idx_h[layer].copy_(idxs[layer], non_blocking=True)
                ev_out[b].record(copy_stream)

        def run(steps):
            copy_stream.wait_stream(stream)               # after the timing start
            copy_in(0)
            for i in range(steps):
                if i + 1 < steps:
                    copy_in(i + 1)
                compute_and_copy_out(i)
            stream.wait_stream(copy_stream)
    else:
        def run(steps):
            for i in range(steps):
                retain = retain_at(i)
                for nm in ("Q", "KC", "VC") + (("QP", "KCP", "VCP") if retain else ()):
                    getattr(wl, nm).copy_(host[nm], non_blocking=True)
                if graphs:
                    graphs[retain].replay()
                    outs, idxs, _ = graph_outputs[retain]
                else:
                    outs, idxs, _ = wl.block_step(retain)
                for layer in range(L):
                    outs_h[layer].copy_(outs[layer], non_blocking=True)
                    idx_h[layer].copy_(idxs[layer], non_blocking=True)

    run(2)
    torch.cuda.synchronize(dev)
    if world > 1:
        import torch.distributed as dist

        dist.barrier()
    ms = _max_over_ranks(_timed(lambda i: run(args.steps), 1, stream), world, dev)
    seqs_job = c["B"] * (world if c["scaling"] == "weak" else 1)
    return {"value": c["T"] * seqs_job / (ms / args.steps / 1e3), "unit": "tokens/s",
            "h2d_bytes_per_step": int(h2d_every + (h2d_retain / c["interval"] if c["retention"] else 0)),
            "d2h_bytes_per_step": int(d2h), "ms_per_step": ms / args.steps,
            "path": ("pinned host -> device copies of the step's queries and block K/V, the block-step through the "
                     "public API (maskahead_b200.hotpath) " + ("as a CUDA-graph replay" if graphs else "eagerly") +
                     ", device -> pinned host copies of every layer's output and read set" +
                     ("; copies on a second stream overlap the neighbouring steps' compute (two input sets, the first "
                      "step's copy-in not overlapped)" if pipelined else ""))}


def measure(c: dict, args, world: int, rank: int, dev, headline: bool) -> dict:
    """One config on this rank's share: warm-up, graphs, K timed block-steps (max over
    ranks), the per-kernel rooflines, the e2e leg and (rank 0, one GPU) the CPU baseline."""
    import torch
    import torch.distributed as dist

    share = rank_share(c, rank, world)
    seed = c["seed"] + (rank if c["scaling"] == "weak" else 0) * 1000 + share["head0"]
    wl = Workload(c, dev, seed, share, world)
    stream = torch.cuda.current_stream(dev)
    side = torch.cuda.Stream(dev)
    retain_at = lambda i: c["retention"] and (i % c["interval"]) == c["interval"] - 1  # noqa: E731
    kinds = sorted({retain_at(i) for i in range(c["interval"])})
    # eager warm-up; every kind of step runs before any capture, so the library's grow-only
    # workspaces reach their final size first and every graph addresses the same buffers
    for i in range(max(1, args.warmup)):
        wl.block_step(retain=retain_at(i))
    for retain in kinds:
        wl.block_step(retain=retain)
    torch.cuda.synchronize(dev)
    graphs, graph_outputs, graph_launches = {}, {}, {}
    timing = "CUDA-graph replay, CUDA events"
    try:
        if args.eager:
            raise RuntimeError("eager steps requested")
        for retain in kinds:
            graphs[retain], graph_outputs[retain], graph_launches[retain] = _capture(
                lambda: wl.block_step(retain), side, stream)
        torch.cuda.synchronize(dev)

        def step(i):
            graphs[retain_at(i)].replay()
    except Exception as exc:   # a collective that cannot be captured: eager steps
        graphs.clear()
        torch.cuda.synchronize(dev)
        timing = ("eager steps (--eager), CUDA events" if args.eager else
                  f"eager steps (graph capture failed: {type(exc).__name__}), CUDA events")

        def step(i):
            wl.block_step(retain_at(i))

    for i in range(args.warmup):
        step(i)
    torch.cuda.synchronize(dev)
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize(dev)
    with ClockSampler(int(os.environ.get("LOCAL_RANK", "0"))) as clocks:
        ms = _timed(step, args.steps, stream)
    torch.cuda.synchronize(dev)
    ms = _max_over_ranks(ms, world, dev)
    ms_step = ms / args.steps
    step_kinds = {}
    if graphs:
        for retain, g in sorted(graphs.items()):
            t = _timed(lambda i, g=g: g.replay(), 3, stream) / 3
            step_kinds["retention" if retain else "plain"] = _max_over_ranks(t, world, dev)
    seqs_job = c["B"] * (world if c["scaling"] == "weak" else 1)
    value = c["T"] * seqs_job / (ms_step / 1e3)

    rooflines = kernel_rooflines(c, wl, share, dev, stream, side, max(3, min(10, args.steps // 2)), world)
    e2e = None if args.no_e2e else e2e_leg(c, wl, graphs, graph_outputs, retain_at, args, world, dev, stream, side)
    from maskahead_b200 import MaError, device_status

    try:
        device_status(dev)
        status = "ok (no bounded device wait gave up)"
    except MaError as exc:   # the numbers above then include timed-out waits: flagged, not hidden
        status = f"TIMEOUT: {exc}"

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        base = cpu_baseline(c, budget_s=20.0 if headline else 8.0)
        cpu = {"value": tokens_per_step(c) / base["seconds"], "unit": "tokens/s", "cores": base["threads"],
               "kind": "port", "cpu_model": base["cpu_model"], "sample": base["sample"]}
    n_ret = sum(1 for i in range(args.steps) if retain_at(i))
    if graphs and all(graph_launches.get(r) is not None for r in graphs):
        launches = sum(graph_launches[retain_at(i)] for i in range(args.steps))
        launches_source = "kernel nodes of the captured block-step graphs in namespace ma"
    else:
        launches = n_ret * kernel_launches(c, share, True) + (args.steps - n_ret) * kernel_launches(c, share, False)
        launches_source = "per-step formula (kernel_launches)"
    ab = algorithmic_bytes(c, share)
    if c["scaling"] == "weak":
        job_ab = {key: world * val for key, val in ab.items()}
    else:
        job_ab = algorithmic_bytes(c, dict(lens=sequence_lengths(c), H=c["H"], Hq=c["Hq"]))
    step_bytes = job_ab["block_step"] + job_ab["retention"] / c["interval"]
    parallelism = {"heads": f"kvheads{world} (head outputs gathered by peer stores over NVLink)" if world > 1
                   else "single GPU",
                   "seqs": f"seq{world} (no collective)"}[c["shard"]]
    # the dominant kernel: the family with the largest share of a plain block-step (its time
    # per launch x its launches per step); bound by the tensor pipe when its arithmetic
    # intensity is above the measured ridge, else by HBM
    peaks = rooflines["peaks"]
    fams = {k: v for k, v in rooflines.items() if isinstance(v, dict) and "us_per_launch" in v}
    for name, v in fams.items():
        mult = c["substeps"] - 1 if name == "substep_attention" else 1
        v["launches_per_step"] = c["L"] // v["layers_per_launch"] * mult
        v["us_per_step"] = v["us_per_launch"] * v["launches_per_step"]
    total_us = sum(v["us_per_step"] for v in fams.values())
    for v in fams.values():
        v["share"] = v["us_per_step"] / total_us
    top = max(fams, key=lambda k: fams[k]["us_per_step"])
    s0 = fams[top]
    ai = s0["tflops"] * 1e12 / (s0["achieved_gbs"] * 1e9) if s0.get("tflops") else 0.0
    tensor = ai * peaks["hbm_gbs"] > peaks["bf16_tflops_burst"] * 1e3
    traffic = TRAFFIC_BYTES.get((c["name"], top)) if world == 1 and not args.layers and not args.batch else None
    roofline = {"kernel": f"{top}: {s0['kernel']} ({s0['share']:.0%} of the kernel time of a plain block-step)",
                "bound": "tensor" if tensor else "hbm",
                "achieved": s0["tflops"] if tensor else s0["achieved_gbs"],
                "peak": peaks["bf16_tflops_burst"] if tensor else peaks["hbm_gbs"],
                "unit": "TFLOP/s" if tensor else "GB/s",
                "frac": s0["tensor_frac_burst"] if tensor else s0["hbm_frac"],
                "traffic": traffic, "peak_kind": f"{peaks['kind']} burst",
                "traffic_source": "ncu dram__bytes_read.sum + dram__bytes_write.sum of one launch "
                                  "(profiles/attn_partial_fa_cfg2.md, profiles/attn_partial_fa_cfg4_step0.md); "
                                  "null where no capture of this family at this config is committed",
                "us_per_launch": s0["us_per_launch"], "bytes_per_launch": s0["bytes_per_launch"],
                "arithmetic_intensity_flop_per_byte": ai, "hbm_frac": s0["hbm_frac"],
                "tensor_tflops": s0.get("tflops"), "tensor_frac": s0.get("tensor_frac_burst"),
                "tensor_frac_sustained": s0.get("tensor_frac_sustained")}
    res = {
        "value": value, "unit": "tokens/s", "ms_per_step": ms_step, "us_per_block_step": ms_step * 1e3,
        "scaling": c["scaling"], "steps": args.steps, "warmup": args.warmup,
        "config": {"workload": c["workload"] + (f" [layers overridden: {c['L']}]" if args.layers > 0 else "")
                   + (f" [sequences overridden: {c['B']}]" if args.batch > 0 else ""),
                   "global_batch": seqs_job, "seq_len": c["n"], "parallelism": parallelism,
                   "l2": "inputs larger than L2 (the per-step cache exceeds 126 MB); the per-kernel timings flush "
                         "L2 (a 256 MB write) before every replay", "timing": timing},
        "roofline": roofline, "rooflines": rooflines, "ms_per_step_kind": step_kinds,
        "algorithmic_bytes_per_step": step_bytes, "achieved_step_gbs": step_bytes / (ms_step / 1e3) / 1e9,
        "block_steps_per_s": seqs_job / (ms_step / 1e3), "cpu_baseline": cpu, "e2e": e2e,
        "gpu_launches": launches, "gpu_launches_source": launches_source, "clocks": clocks.summary(),
        "device_status": status,
    }
    if world > 1:
        dist.barrier()
    graphs.clear()
    graph_outputs.clear()
    del wl
    torch.cuda.synchronize(dev)
    torch.cuda.empty_cache()
    return res


def run_ours(args):
    import torch
    import torch.distributed as dist

    import maskahead_b200

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        import datetime

        dist.init_process_group("nccl", device_id=dev, timeout=datetime.timedelta(seconds=120))
    maskahead_b200.load_library()

    def cfg_of(name):
        c = dict(CONFIGS[name])
        if args.layers > 0:
            c["L"] = args.layers
        if args.batch > 0:
            c["B"] = args.batch
        return c

    if args.configs == "auto":
        args.configs = "cfg3,cfg4,cfg5"
    head = measure(cfg_of(args.config), args, world, rank, dev, headline=True)
    extra = {}
    names = [x for x in (args.configs.split(",") if args.configs else []) if x and x != args.config]
    for name in names:
        if name not in CONFIGS:
            raise SystemExit(f"unknown config {name}")
        c = cfg_of(name)
        if c["shard"] == "heads" and c["H"] % world:
            extra[name] = {"skipped": f"{c['H']} KV heads do not split over {world} ranks"}
            continue
        extra[name] = measure(c, args, world, rank, dev, headline=False)
    if world > 1:
        dist.barrier()
        torch.cuda.synchronize()
        dist.destroy_process_group()
    if rank != 0:
        return
    line = {"metric": METRIC, "value": head["value"], "unit": "tokens/s", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": head["ms_per_step"], "us_per_block_step": head["us_per_block_step"],
            "higher_is_better": True, "scaling": head["scaling"], "vs_baseline": None, "dtype": "bf16",
            "data": "synthetic (seeded N(0,1) K/V/Q, random-init; no model weights)", "config": head["config"]}
    for key in ("roofline", "rooflines", "ms_per_step_kind", "algorithmic_bytes_per_step", "achieved_step_gbs",
                "block_steps_per_s", "cpu_baseline", "e2e", "gpu_launches", "gpu_launches_source", "clocks",
                "device_status"):
        line[key] = head[key]
    line["configs"] = extra
    print(json.dumps(line), flush=True)


def main():
    args = parse_args()
    if args.impl == "reference":
        run_reference(args)
    else:
        run_ours(args)


if __name__ == "__main__":
    main()
