"""Seeded synthetic inputs shared by the golden-fixture generator, the tests and the bench.

Every tensor comes from a CPU ``torch.Generator`` with a fixed seed, so the same case
regenerates bit-identically on any machine; fixtures store a SHA-256 of the inputs to
prove it. Distributions follow the benchmark configurations: K, V, Q ~ N(0, 1); in
packed (k4v4) cases 1% of the key channels of every (layer, head) are scaled x8 as
outliers before quantization.
"""

from __future__ import annotations

import hashlib

import numpy as np
import torch

CASES = {
    # the CPU-runnable configuration: 28 q / 4 KV heads, d 128, fp32, prefix 2048
    "cfg1": dict(B=1, Hq=28, H=4, D=128, T=32, n=2048, dtype="float32", k=256, C=512, seed=1234),
    "small_bf16": dict(B=1, Hq=8, H=2, D=128, T=32, n=448, dtype="bfloat16", k=64, C=128, seed=7),
    "small_bf16_live": dict(B=1, Hq=8, H=2, D=128, T=32, n=448, dtype="bfloat16", k=64, C=128, seed=8,
                            live_frac=0.7),
    "small_bf16_rows": dict(B=1, Hq=8, H=2, D=128, T=32, n=300, dtype="bfloat16", k=50, C=100, seed=13,
                            rows=[0, 3, 4, 9, 10, 11, 17, 20, 21, 28, 31]),
    "batch2_bf16": dict(B=2, Hq=12, H=3, D=128, T=32, n=256, dtype="bfloat16", k=40, C=80, seed=11),
    "small_k4v4_token": dict(B=1, Hq=8, H=2, D=128, T=32, n=320, dtype="bfloat16", k=64, C=128, seed=9,
                             packed="token"),
    "small_k4v4_channel": dict(B=1, Hq=8, H=2, D=128, T=32, n=320, dtype="bfloat16", k=64, C=128, seed=10,
                               packed="channel"),
    # one layer of the benchmarked configurations: cfg2 (bf16 K/V, prefix 8192, read budget
    # 1024) and cfg3 (the same shape in k4v4 token mode, 1% of the key channels x8)
    "cfg2_layer": dict(B=1, Hq=28, H=4, D=128, T=32, n=8192, dtype="bfloat16", k=1024, C=2048, seed=1236),
    "cfg3_layer": dict(B=1, Hq=28, H=4, D=128, T=32, n=8192, dtype="bfloat16", k=1024, C=2048, seed=1237,
                       packed="token"),
}

# cases whose packed payloads are too large to store: the fixture's input digest (which
# covers the payloads) pins them instead
LARGE = {"cfg2_layer", "cfg3_layer"}


def _dt(name: str) -> torch.dtype:
    return {"float32": torch.float32, "bfloat16": torch.bfloat16, "float16": torch.float16}[name]


def make_case(name: str, **override) -> dict:
    """Inputs of one case: query, prefix key/value (compute dtype), current key/value,
    optional live mask and packed payloads, selection rows."""
    spec = dict(CASES[name]) if name in CASES else {}
    spec.update(override)
    g = torch.Generator().manual_seed(spec["seed"])
    B, Hq, H, D, T, n = (spec[x] for x in ("B", "Hq", "H", "D", "T", "n"))
    dt = _dt(spec["dtype"])
    q = torch.randn(B, Hq, T, D, generator=g).to(dt)
    k = torch.randn(B, H, n, D, generator=g)
    v = torch.randn(B, H, n, D, generator=g)
    kc = torch.randn(B, H, T, D, generator=g).to(dt)
    vc = torch.randn(B, H, T, D, generator=g).to(dt)
    out = dict(spec=spec, query=q, current_key=kc, current_value=vc,
               rows=list(spec.get("rows", range(T))))
    packed = spec.get("packed")
    if packed:
        # 1% of the key channels of each head are outliers (x8)
        nout = max(1, D // 100)
        for b in range(B):
            for h in range(H):
                ch = torch.randperm(D, generator=g)[:nout]
                k[b, h, :, ch] *= 8.0
        out["key_fp"] = k.to(dt)
        out["value_fp"] = v.to(dt)
    else:
        out["key"] = k.to(dt)
        out["value"] = v.to(dt)
    if "live_frac" in spec:
        # the same live count in every (batch, head), as the eviction state keeps it
        n_live = int(round(spec["live_frac"] * n))
        live = torch.zeros(B, H, n, dtype=torch.bool)
        for b in range(B):
            for h in range(H):
                pick = torch.randperm(n - 4, generator=g)[: n_live - 4] + 4
                live[b, h, :4] = True
                live[b, h, pick] = True
        out["live_mask"] = live
    return out


def make_retain_case(seed: int = 12, L: int = 2, B: int = 1, H: int = 2, live: int = 600,
                     D: int = 128, C: int = 256, W: int = 64, sinks: int = 4) -> dict:
    """Inputs of the lookahead retention: step-0 mass a1, probe mass, live values and
    positions (distinct, increasing along the live axis, with the sinks present)."""
    g = torch.Generator().manual_seed(seed)
    a1 = torch.softmax(torch.randn(L, B, H, live, generator=g) * 2.0, dim=-1)
    ap = torch.softmax(torch.randn(L, B, H, live, generator=g) * 2.0, dim=-1)
    v = torch.randn(L, B, H, live, D, generator=g).to(torch.bfloat16)
    pos = torch.empty(L, B, H, live, dtype=torch.int32)
    for i in range(L * B * H):
        extra = torch.randperm(3 * live, generator=g)[: live - sinks] + sinks
        p = torch.cat([torch.arange(sinks), extra.sort().values])
        pos.view(-1, live)[i] = p.to(torch.int32)
    return dict(a1=a1, a_probe=ap, v_live=v, pos=pos, C=C, W=W, sinks=sinks)


def digest(tensors: dict) -> str:
    """SHA-256 over the raw bytes of the tensors of a case, in sorted key order."""
    h = hashlib.sha256()
    for key in sorted(tensors):
        t = tensors[key]
        if isinstance(t, torch.Tensor):
            x = t.detach().contiguous()
            if x.dtype == torch.bfloat16:
                x = x.view(torch.int16)
            h.update(key.encode())
            h.update(np.ascontiguousarray(x.numpy()).tobytes())
    return h.hexdigest()
