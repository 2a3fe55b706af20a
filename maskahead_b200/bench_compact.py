"""Time the cache compaction after an eviction (ma_compact_tokens) on one GPU.

    python -m maskahead_b200.bench_compact [--layout token|bf16] [--lanes N] [--n SLOTS]
                                           [--keep C] [--iters K]

Every layer of a serving batch compacts in one launch: lanes = layers x sequences x KV
heads. The source arrays are filled with random bytes (the compaction moves codes and
never reads them as numbers). Algorithmic bytes per launch = lanes x C x bytes per slot
x 2 (each kept slot read once and written once; 160 B per slot for token-mode k4v4,
512 B for bf16 at D = 128). Both the source and the destination are larger than L2, so
no flush is needed between launches. Prints one JSON line: the mean launch time over
K launches (CUDA events on the launching stream, after 3 warm-up launches) and the
achieved HBM bandwidth against the measured copy peak.
"""

from __future__ import annotations

import argparse
import json
from pathlib import Path

import torch

from .layouts import Prefix, compact_tokens


def _peak_gbs() -> tuple[float, str]:
    p = Path(__file__).resolve().parents[1] / "MEASURED_PEAKS.json"
    if p.exists():
        return float(json.loads(p.read_text())["hbm_gbs"]), "measured"
    return 6650.0, "fallback"


def main() -> None:
    ap = argparse.ArgumentParser(description=__doc__.splitlines()[0])
    ap.add_argument("--layout", choices=("token", "bf16"), default="token")
    ap.add_argument("--lanes", type=int, default=28 * 64 * 4, help="layers x sequences x KV heads")
    ap.add_argument("--n", type=int, default=8192, help="slots before the compaction")
    ap.add_argument("--keep", type=int, default=2048, help="slots kept (C)")
    ap.add_argument("--iters", type=int, default=20)
    args = ap.parse_args()
    dev = torch.device("cuda")
    H = 4
    B = args.lanes // H
    n, C, D = args.n, args.keep, 128
    gen = torch.Generator(device=dev).manual_seed(7)

    def rnd_u8(*shape):
        return torch.randint(0, 256, shape, dtype=torch.uint8, device=dev, generator=gen)

    if args.layout == "token":
        def arrays(slots):
            return dict(kq=rnd_u8(B, H, slots, D // 32, 16), ks=rnd_u8(B, H, slots, D // 32, 2).view(torch.float16)[..., 0],
                        kz=rnd_u8(B, H, slots, D // 32, 2).view(torch.float16)[..., 0],
                        vq=rnd_u8(B, H, slots, D // 32, 16), vs=rnd_u8(B, H, slots, D // 32, 2).view(torch.float16)[..., 0],
                        vz=rnd_u8(B, H, slots, D // 32, 2).view(torch.float16)[..., 0])
        kch = torch.ones(B, H, D, device=dev)
        src = Prefix(**arrays(n), nq=n, kb=4, vb=4, kmode=1, kch=kch)
        dst = Prefix(**arrays(C), nq=C, kb=4, vb=4, kmode=1, kch=kch)
        slot_bytes = 2 * (D // 2 + 2 * 2 * (D // 32))
    else:
        def dense(slots):
            return rnd_u8(B, H, slots, D * 2).view(torch.bfloat16)
        src = Prefix.dense(dense(n), dense(n))
        dst = Prefix.dense(dense(C), dense(C))
        slot_bytes = 2 * D * 2
    # an ascending random subset of the slots per lane, as the eviction keeps them
    keep = torch.rand(B, H, n, device=dev, generator=gen).argsort(-1)[..., :C].sort(-1).values.contiguous()
    stream = torch.cuda.current_stream()
    for _ in range(3):
        compact_tokens(src, keep, out=dst)
    torch.cuda.synchronize()
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    start.record(stream)
    for _ in range(args.iters):
        compact_tokens(src, keep, out=dst)
    end.record(stream)
    torch.cuda.synchronize()
    us = start.elapsed_time(end) * 1e3 / args.iters
    alg = args.lanes * C * slot_bytes * 2
    peak, kind = _peak_gbs()
    gbs = alg / (us * 1e-6) / 1e9
    print(json.dumps({"kernel": "compact_kernel", "layout": args.layout, "lanes": args.lanes, "n": n, "keep": C,
                      "us_per_launch": round(us, 2), "algorithmic_bytes": alg, "achieved_gbs": round(gbs, 1),
                      "peak_gbs": peak, "peak_kind": kind, "frac": round(gbs / peak, 3)}))


if __name__ == "__main__":
    main()
