#!/usr/bin/env python
"""Benchmark of the MaskAhead select + attend block-step on B200.

Workload (Qwen2.5-7B-shaped layer stack): 28 layers, batch 1,
28 query / 4 KV heads, head_dim 128, bf16 K/V, prefix 8192, a 32-token mask block
denoised in 4 sub-steps, read budget 1024, retain budget 2048, one lookahead block.

One step = one block-step over all 28 layers:
  step 0     score (prefix mass of the 32 mask queries x 7 query heads), value-aware
             score, top-1024 read set, dense attention over [prefix | block];
  3 sparse sub-steps: attention over [read set | block];
  retention (every 4th block, interval_blocks = 4): probe attention of the next mask
             block, probe mass, lookahead value score, survivors (W 64, 4 sinks, C 2048).
Synthetic seeded inputs, N(0,1); the K/V cache (470 MB) exceeds L2, so every step reads
it from HBM. `value` = tokens/s (32 tokens per block-step per sequence) over all ranks;
each rank runs its own sequence (weak scaling, no collective).

  python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
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

CFG = dict(name="cfg2", L=28, B=1, Hq=28, H=4, D=128, T=32, n=8192, k=1024, C=2048, substeps=4,
           probe_blocks=1, interval=4, W=64, sinks=4, seed=1234)
METRIC = "µs per block-step select+attend; achieved HBM GB/s vs peak; tokens/s at 1/2/4/8 GPU"
# DRAM bytes per launch of the step-0 attention partial pass at this workload, from the
# ncu capture summarized in profiles/attn_partial_mma_cfg2_step0.md (re-taken per kernel change)
ATTN_TRAFFIC_BYTES = 17_129_984


def parse_args():
    ap = argparse.ArgumentParser(description="MaskAhead select+attend block-step benchmark (B200)")
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=4)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--cpu-sample-layers", type=int, default=2)
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


# ------------------------------------------------------------------------- workload
class Workload:
    """Seeded synthetic inputs of one sequence, resident on the device."""

    def __init__(self, cfg: dict, device, seed: int):
        import torch

        c = cfg
        g = torch.Generator(device=device).manual_seed(seed)
        bf = torch.bfloat16
        L, B, Hq, H, D, T, n, S = c["L"], c["B"], c["Hq"], c["H"], c["D"], c["T"], c["n"], c["substeps"]
        P = c["probe_blocks"]
        self.cfg, self.device = c, device

        def randn(*shape):
            return torch.randn(*shape, generator=g, device=device, dtype=torch.float32).to(bf)

        self.K = randn(L, B, H, n, D)
        self.V = randn(L, B, H, n, D)
        self.Q = randn(L, S, B, Hq, T, D)
        self.KC = randn(L, S, B, H, T, D)
        self.VC = randn(L, S, B, H, T, D)
        self.QP = randn(L, B, Hq, T * (1 + P), D)
        self.KCP = randn(L, B, H, T * (1 + P), D)
        self.VCP = randn(L, B, H, T * (1 + P), D)
        self.rows = torch.arange(T, device=device, dtype=torch.int32)
        self.probe_rows = torch.arange(T, T * (1 + P), device=device, dtype=torch.int32)
        self.pos = torch.arange(n, device=device, dtype=torch.int32).expand(L, B, H, n).contiguous()
        self.scale = D ** -0.5
        self.outputs = None

    def prefix(self, layer: int):
        from maskahead_b200.layouts import Prefix

        return Prefix.dense(self.K[layer], self.V[layer])

    def block_step(self, retain: bool):
        """One block-step over every layer through the public hot-path API."""
        import torch
        from maskahead_b200.hotpath import (compact_attention, fast_step0, lookahead_survivors,
                                            probe_attention, value_score)

        c = self.cfg
        outs, idxs, masses = [], [], []
        for layer in range(c["L"]):
            pre = self.prefix(layer)
            res = fast_step0(self.Q[layer, 0], pre, self.KC[layer, 0], self.VC[layer, 0], query_indices=self.rows,
                             topk=c["k"], value_aware=True, scaling=self.scale)
            out = res.out
            for s in range(1, c["substeps"]):
                out = compact_attention(self.Q[layer, s], pre, res.indices, self.KC[layer, s], self.VC[layer, s],
                                        scaling=self.scale)
            outs.append(out)
            idxs.append(res.indices)
            masses.append(res.mass)
        keep = None
        if retain:
            probe = []
            for layer in range(c["L"]):
                _, ap = probe_attention(self.QP[layer], self.prefix(layer), self.KCP[layer], self.VCP[layer],
                                        block_size=c["T"], scaling=self.scale, probe_rows=self.probe_rows)
                probe.append(ap)
            a = torch.stack(masses) + torch.stack(probe)
            score = value_score(a, self.V)
            keep = lookahead_survivors(self.pos, score, c["C"], recent_window=c["W"], sink_tokens=c["sinks"])
        self.outputs = (outs, idxs, keep)
        return self.outputs


def kernel_launches(cfg: dict, retain: bool) -> int:
    """Kernels of one block-step: step 0 = attention partial + combine + mass (with the
    value centre) + value apply + top-k (5); each sub-step = partial + combine (2);
    retention = per layer probe partial + combine + mass (3), then value centre + apply +
    survivors."""
    per_layer = 5 + 2 * (cfg["substeps"] - 1)
    n = per_layer * cfg["L"]
    if retain:
        n += 3 * cfg["L"] + 3
    return n


def algorithmic_bytes(cfg: dict) -> dict:
    """Bytes each phase must move at least (K/V counted once per read phase)."""
    L, B, Hq, H, D, T, n, k = (cfg[x] for x in ("L", "B", "Hq", "H", "D", "T", "n", "k"))
    bt = 2 * D * 2                      # bf16 K+V bytes per token per head
    q = B * Hq * T * D * 2
    cur = 2 * B * H * T * D * 2
    step0 = B * H * n * bt + 2 * q + cur                    # prefix K/V, Q, out, current K/V
    sub = B * H * k * bt + B * H * k * 8 + 2 * q + cur      # read set K/V + indices
    return dict(step0_layer=step0, substep_layer=sub,
                block_step=L * (step0 + (cfg["substeps"] - 1) * sub),
                retention=L * (B * H * n * bt))             # the probe re-reads the live set


def step0_flops(cfg: dict) -> float:
    """Tensor-core FLOPs of the step-0 attention partial kernel per layer: Q.K^T and P.V."""
    B, Hq, D, T, n = (cfg[x] for x in ("B", "Hq", "D", "T", "n"))
    return 4.0 * B * Hq * T * n * D


# ---------------------------------------------------------------------- CPU baseline
def cpu_block_step_time(cfg: dict, sample_layers: int, threads: int | None = None):
    """The oracle (a restatement of the reference's torch CPU path) timed on the host:
    step 0 (importance, value-aware rescoring, top-k, dense attention) and the three
    sparse sub-steps (sdpa over the gathered read set) for `sample_layers` layers, plus
    the retention pass once per interval; scaled to one 28-layer block-step.
    Returns (seconds per block-step, threads, sample description)."""
    import torch

    import oracle

    threads = threads or os.cpu_count() or 1
    torch.set_num_threads(threads)
    c = cfg
    g = torch.Generator().manual_seed(c["seed"])
    B, Hq, H, D, T, n = c["B"], c["Hq"], c["H"], c["D"], c["T"], c["n"]
    bf = torch.bfloat16
    rows = list(range(T))
    scale = D ** -0.5

    def one_layer():
        k = torch.randn(B, H, n, D, generator=g).to(bf)
        v = torch.randn(B, H, n, D, generator=g).to(bf)
        q = torch.randn(B, Hq, T, D, generator=g).to(bf)
        kc = torch.randn(B, H, T, D, generator=g).to(bf)
        vc = torch.randn(B, H, T, D, generator=g).to(bf)
        qp = torch.randn(B, Hq, 2 * T, D, generator=g).to(bf)
        t0 = time.perf_counter()
        imp = oracle.selector_importance(q, k, query_indices=rows, scale=scale)
        score = oracle.rescore_by_value(imp, v)
        idx, _ = oracle.topk_reference_torch(score, c["k"])
        oracle.dense_attention(q, k, v, kc, vc, scale=scale)
        sk = torch.cat([oracle.gather_per_kv_head(k, idx), kc], dim=2)
        sv = torch.cat([oracle.gather_per_kv_head(v, idx), vc], dim=2)
        for _ in range(c["substeps"] - 1):
            oracle.sdpa_compact(q, sk, sv)
        t1 = time.perf_counter()
        # retention: probe importance + lookahead score (survivors timed separately below)
        ap = oracle.selector_importance(qp, k, query_indices=list(range(T, 2 * T)), scale=scale)
        oracle.lookahead_score(imp, ap, v)
        t2 = time.perf_counter()
        return t1 - t0, t2 - t1

    one_layer()  # warm-up
    step, ret = [], []
    for _ in range(sample_layers):
        a, b = one_layer()
        step.append(a)
        ret.append(b)
    pos = torch.arange(n, dtype=torch.int32).expand(c["L"], B, H, n).contiguous()
    sc = torch.rand(c["L"], B, H, n, generator=g)
    t0 = time.perf_counter()
    oracle.survivors_lookahead(pos, sc, c["C"], recent_window=c["W"], sink_tokens=c["sinks"])
    t_surv = time.perf_counter() - t0
    per_block = c["L"] * statistics.median(step) + (c["L"] * statistics.median(ret) + t_surv) / c["interval"]
    sample = (f"{sample_layers} layers of step 0 + {c['substeps'] - 1} sparse sub-steps + retention scoring "
              f"(median), survivors over all {c['L']} layers once, scaled to {c['L']} layers with retention "
              f"every {c['interval']} blocks; torch fp32 CPU, {threads} threads")
    return per_block, threads, sample


def run_reference(args):
    """--impl reference: the reference algorithm's CPU path (the oracle restatement; the
    reference package itself is not shipped to the GPU box) on the host cores."""
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    t_block, threads, sample = cpu_block_step_time(CFG, max(1, args.cpu_sample_layers))
    steps = []
    for _ in range(max(1, args.steps // 10)):
        t, _, _ = cpu_block_step_time(CFG, 1, threads)
        steps.append(t)
    t_block = statistics.median(steps + [t_block])
    tok_s = CFG["T"] * CFG["B"] / t_block
    line = {"impl": "reference", "metric": METRIC, "value": tok_s, "unit": "tokens/s", "n_gpus": args.gpus,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": t_block * 1e3,
            "us_per_block_step": t_block * 1e6, "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "f32", "data": "synthetic",
            "config": {"workload": "cfg2: 28 layers, 28q/4kv heads, d128, bf16 K/V, prefix 8192, "
                                   "block 32 x 4 sub-steps, k_r 1024, C 2048, 1 lookahead block",
                       "global_batch": CFG["B"], "seq_len": CFG["n"], "parallelism": "cpu"},
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


def run_ours(args):
    import torch
    import torch.distributed as dist

    import maskahead_b200
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
    c = CFG
    wl = Workload(c, dev, c["seed"] + rank)
    stream = torch.cuda.current_stream(dev)

    # eager warm-up (sizes the workspaces), then one CUDA graph per step kind
    for i in range(max(1, args.warmup)):
        wl.block_step(retain=(i % c["interval"]) == c["interval"] - 1)
    torch.cuda.synchronize()
    graphs = {}
    side = torch.cuda.Stream(dev)
    side.wait_stream(stream)
    with torch.cuda.stream(side):
        for retain in (False, True):
            g = torch.cuda.CUDAGraph()
            with torch.cuda.graph(g, stream=side):
                wl.block_step(retain)
            graphs[retain] = g
    stream.wait_stream(side)
    torch.cuda.synchronize()

    def replay(i):
        graphs[(i % c["interval"]) == c["interval"] - 1].replay()

    for i in range(args.warmup):
        replay(i)
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    with ClockSampler(local) as clocks:
        ms = _timed(replay, args.steps, stream)
    torch.cuda.synchronize()
    if world > 1:
        t = torch.tensor([ms], device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms = float(t.item())
    ms_step = ms / args.steps
    tokens = c["T"] * c["B"] * world
    value = tokens / (ms_step / 1e3)

    # dominant kernel: the step-0 attention (tensor-core partial pass + combine) per layer
    hbm_peak, tf_peak, peak_kind = peaks()
    g0 = torch.cuda.CUDAGraph()
    with torch.cuda.stream(side):
        with torch.cuda.graph(g0, stream=side):
            for layer in range(c["L"]):
                splitk_attention(wl.Q[layer, 0], wl.prefix(layer), wl.KC[layer, 0], wl.VC[layer, 0],
                                 scaling=wl.scale, want_prefix=True)
    stream.wait_stream(side)
    for _ in range(3):
        g0.replay()
    torch.cuda.synchronize()
    reps = max(3, args.steps // 2)
    ms_attn = _timed(lambda i: g0.replay(), reps, stream) / (reps * c["L"])
    ab = algorithmic_bytes(c)
    achieved = ab["step0_layer"] / (ms_attn / 1e3) / 1e9
    tflops = step0_flops(c) / (ms_attn / 1e3) / 1e12

    # end to end through the public API with host buffers
    e2e = None
    if not args.no_e2e:
        hq = wl.Q.cpu().pin_memory()
        hkc, hvc = wl.KC.cpu().pin_memory(), wl.VC.cpu().pin_memory()
        hqp, hkcp, hvcp = wl.QP.cpu().pin_memory(), wl.KCP.cpu().pin_memory(), wl.VCP.cpu().pin_memory()
        outs_h = torch.empty((c["L"],) + tuple(wl.Q.shape[2:]), dtype=wl.Q.dtype).pin_memory()
        idx_h = torch.empty((c["L"], c["B"], c["H"], c["k"]), dtype=torch.int64).pin_memory()
        h2d_every = sum(t.numel() * t.element_size() for t in (hq, hkc, hvc))      # every block-step
        h2d_retain = sum(t.numel() * t.element_size() for t in (hqp, hkcp, hvcp))  # retention steps
        d2h = outs_h.numel() * outs_h.element_size() + idx_h.numel() * 8

        def e2e_step(i):
            retain = (i % c["interval"]) == c["interval"] - 1
            wl.Q.copy_(hq, non_blocking=True)
            wl.KC.copy_(hkc, non_blocking=True)
            wl.VC.copy_(hvc, non_blocking=True)
            if retain:
                wl.QP.copy_(hqp, non_blocking=True)
                wl.KCP.copy_(hkcp, non_blocking=True)
                wl.VCP.copy_(hvcp, non_blocking=True)
            outs, idxs, _ = wl.block_step(retain)
            outs_h.copy_(torch.stack(outs), non_blocking=True)
            idx_h.copy_(torch.stack(idxs), non_blocking=True)

        for i in range(2):
            e2e_step(i)
        torch.cuda.synchronize()
        if world > 1:
            dist.barrier()
        ms_e = _timed(e2e_step, args.steps, stream)
        if world > 1:
            t = torch.tensor([ms_e], device=dev)
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
            ms_e = float(t.item())
        e2e = {"value": tokens / (ms_e / args.steps / 1e3), "unit": "tokens/s",
               "h2d_bytes_per_step": int(h2d_every + h2d_retain / c["interval"]),
               "d2h_bytes_per_step": int(d2h), "ms_per_step": ms_e / args.steps,
               "path": "eager public API (maskahead_b200.hotpath) per layer, pinned host copies in and out"}

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        t_block, threads, sample = cpu_block_step_time(c, max(1, args.cpu_sample_layers))
        cpu = {"value": c["T"] * c["B"] / t_block, "unit": "tokens/s", "cores": threads, "kind": "port",
               "sample": sample}

    if world > 1:
        dist.barrier()
        for g in list(graphs.values()) + [g0]:
            del g
        graphs.clear()
        dist.destroy_process_group()
    if rank != 0:
        return
    launches = (args.steps // c["interval"]) * kernel_launches(c, True) + \
        (args.steps - args.steps // c["interval"]) * kernel_launches(c, False)
    line = {
        "metric": METRIC, "value": value, "unit": "tokens/s", "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": ms_step, "us_per_block_step": ms_step * 1e3,
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "bf16",
        "data": "synthetic (seeded N(0,1) K/V/Q, random-init; no model weights)",
        "config": {"workload": "cfg2: 28 layers, 28q/4kv heads, d128, bf16 K/V, prefix 8192, block 32 x 4 "
                               "sub-steps, k_r 1024, C 2048, 1 lookahead block, retention every 4 blocks",
                   "global_batch": c["B"] * world, "seq_len": c["n"], "parallelism": f"seq{world} (no collective)",
                   "l2": "inputs larger than L2 (470 MB K/V per step)", "timing": "CUDA-graph replay, CUDA events"},
        "roofline": {"kernel": "step-0 attention (attn_partial_mma + attn_combine) per layer", "bound": "hbm",
                     "achieved": achieved, "peak": hbm_peak, "unit": "GB/s", "frac": achieved / hbm_peak,
                     "traffic": ATTN_TRAFFIC_BYTES, "peak_kind": f"{peak_kind} burst",
                     "traffic_source": "ncu dram__bytes_read.sum + dram__bytes_write.sum of attn_partial_mma, "
                                       "profiles/attn_partial_mma_cfg2_step0.md",
                     "us_per_launch": ms_attn * 1e3,
                     "tensor_tflops": tflops, "tensor_frac": tflops / tf_peak,
                     "bytes_per_launch": ab["step0_layer"]},
        "algorithmic_bytes_per_step": ab["block_step"] + ab["retention"] / c["interval"],
        "achieved_step_gbs": (ab["block_step"] + ab["retention"] / c["interval"]) / (ms_step / 1e3) / 1e9,
        "cpu_baseline": cpu, "e2e": e2e, "gpu_launches": launches, "clocks": clocks.summary(),
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
