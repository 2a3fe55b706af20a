"""Time the cache compaction after an eviction (ma_compact_tokens) on one GPU.

    python bench_compact.py [--layout token|bf16|channel] [--lanes N] [--n SLOTS]
                            [--keep C] [--iters K]

Every layer of a serving batch compacts in one launch: lanes = layers x sequences x KV
heads. The source arrays are filled with random bytes (the compaction moves codes and
never reads them as numbers). Algorithmic bytes per launch = lanes x C x bytes per slot
x 2 (each kept slot read once and written once; 160 B per slot for token-mode k4v4,
512 B for bf16 at D = 128). Both the source and the destination are larger than L2, so
no flush is needed between launches. Prints one JSON line: the mean launch time over
K launches (CUDA events on the launching stream, after 3 warm-up launches) and the
achieved HBM bandwidth against the measured copy peak.

--layout channel times the whole group-preserving rebuild of a KIVI channel-mode cache
(`layouts.rebuild`: every launch and device-side index operation of one call) with
C / 32 kept key groups per lane (the first half of the groups, every other one, and
groups from the second half), the survivors of 8 further groups re-encoded (a third of
their slots) and 64 slots staged; its bytes count the kept groups moved (160 B per slot,
read and written) and the re-encoded and staged slots (read packed, written once).
"""

from __future__ import annotations

import argparse
import json
import sys
from pathlib import Path

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

import torch  # noqa: E402

from maskahead_b200.layouts import Prefix, compact_tokens  # noqa: E402


def _peak_gbs() -> tuple[float, str]:
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        return float(json.loads(p.read_text())["hbm_gbs"]), "measured"
    return 6650.0, "fallback"


def _time_rebuild(args, B, H, n, C, D, gen, rnd_u8, dev) -> None:
    from maskahead_b200.layouts import rebuild

    gk, rl = 32, 64
    ng = n // gk

    def scales(*shape):
        # finite fp16 scales/zeros in [0.5, 1): random bytes could hold NaN/Inf patterns
        return (torch.rand(*shape, device=dev, generator=gen) * 0.5 + 0.5).to(torch.float16)

    src = Prefix(kq=rnd_u8(B, H, ng, D, gk // 2), ks=scales(B, H, ng, D), kz=scales(B, H, ng, D),
                 vq=rnd_u8(B, H, n, D // 32, 16), vs=scales(B, H, n, D // 32), vz=scales(B, H, n, D // 32),
                 kf=torch.randn(B, H, rl, D, device=dev, generator=gen).to(torch.bfloat16),
                 vf=torch.randn(B, H, rl, D, device=dev, generator=gen).to(torch.bfloat16),
                 nq=n, nf=rl, kb=4, vb=4, kmode=0)
    g1 = C // gk
    kept = torch.arange(0, 2 * g1, 2, device=dev)[:g1].clamp_max(ng - 10)
    groups_before = kept.expand(B, H, g1).contiguous()
    sparse = torch.arange(ng - 9, ng - 1, device=dev)
    slots = (sparse.view(-1, 1) * gk + torch.arange(0, gk, 3, device=dev)).reshape(-1)
    encode = slots.expand(B, H, slots.numel()).contiguous()
    groups_after = torch.full((B, H, 1), ng - 1, device=dev, dtype=torch.int64)
    stage = (torch.arange(rl, device=dev) + n).expand(B, H, rl).contiguous()
    for _ in range(3):
        rebuild(src, groups_before, encode, groups_after, stage)
    torch.cuda.synchronize()
    stream = torch.cuda.current_stream()
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    start.record(stream)
    for _ in range(args.iters):
        rebuild(src, groups_before, encode, groups_after, stage)
    end.record(stream)
    torch.cuda.synchronize()
    us = start.elapsed_time(end) * 1e3 / args.iters
    lanes = B * H
    moved = (g1 + 1) * gk * 160 * 2 + encode.shape[-1] * 160 * 2 + rl * 512 * 2
    alg = lanes * moved
    peak, kind = _peak_gbs()
    gbs = alg / (us * 1e-6) / 1e9
    print(json.dumps({"kernel": "rebuild (channel-mode)", "lanes": lanes, "n": n, "kept_groups": g1 + 1,
                      "encoded": encode.shape[-1], "staged": rl, "us_per_call": round(us, 2),
                      "algorithmic_bytes": alg, "achieved_gbs": round(gbs, 1), "peak_gbs": peak,
                      "peak_kind": kind, "frac": round(gbs / peak, 3)}))


def main() -> None:
    ap = argparse.ArgumentParser(description=__doc__.splitlines()[0])
    ap.add_argument("--layout", choices=("token", "bf16", "channel"), default="token")
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

    if args.layout == "channel":
        _time_rebuild(args, B, H, n, C, D, gen, rnd_u8, dev)
        return
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
