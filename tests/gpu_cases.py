"""Shared helpers of the GPU tests: device copies of the seeded cases in the hot path's
layouts, and the oracle's view of the same inputs (dequantized as the reference reads
them). Only test code imports this module."""

from __future__ import annotations

import numpy as np
import torch

import oracle
from gen_inputs import make_case
from maskahead_b200.layouts import Prefix


def oracle_kv(case):
    """(K, V, packed tensors) of a case: the prefix exactly as the reference attends it."""
    spec = case["spec"]
    packed = spec.get("packed")
    if not packed:
        return case["key"], case["value"], {}
    kf, vf = case["key_fp"], case["value_fp"]
    vq, vs, vz = oracle.quantize_values(vf)
    v = oracle.dequantize_values(vq, vs, vz)
    extra = dict(vq=vq, vs=vs, vz=vz)
    if packed == "channel":
        kq, ks, kz = oracle.quantize_keys(kf)
        k = oracle.dequantize_keys(kq, ks, kz)
    else:
        kchan = oracle.key_channel_divisor(kf)
        kq, ks, kz = oracle.quantize_keys_token(kf, kchan)
        k = oracle.dequantize_keys_token(kq, ks, kz, kchan)
        extra["kchan"] = kchan
    extra.update(kq=kq, ks=ks, kz=kz)
    return k, v, extra


def device_prefix(case, k, v, extra, dev="cuda", mask=True) -> Prefix:
    spec = case["spec"]
    live = case.get("live_mask") if mask else None
    live = None if live is None else live.to(dev)
    packed = spec.get("packed")
    if not packed:
        return Prefix.dense(k.to(dev), v.to(dev), mask=live)
    n = spec["n"]
    d = {key: t.to(dev) for key, t in extra.items()}
    return Prefix(kq=d["kq"], ks=d["ks"], kz=d["kz"], vq=d["vq"], vs=d["vs"], vz=d["vz"], nq=n, nf=0,
                  kb=4, vb=4, kg=32, vg=32, mask=live, kmode=1 if packed == "token" else 0,
                  kch=d.get("kchan"))


def load_case(name):
    case = make_case(name)
    k, v, extra = oracle_kv(case)
    return case, k, v, extra


def band_equal(got: np.ndarray, want: np.ndarray, score: np.ndarray, k: int, rel: float = 1e-5):
    """Per row, the selected sets agree except on entries whose oracle score lies within
    `rel` (relative) of the row's k-th score -- there the fp32 rounding of two
    different summation orders may legitimately flip the order. Returns the number of
    rows compared and the number of entries that differed inside the band."""
    flips = 0
    rows = got.reshape(-1, got.shape[-1])
    ref = want.reshape(-1, want.shape[-1])
    sc = score.reshape(-1, score.shape[-1])
    for i in range(rows.shape[0]):
        a, b = set(rows[i].tolist()), set(ref[i].tolist())
        if a == b:
            continue
        kth = np.sort(sc[i])[::-1][k - 1]
        band = rel * max(abs(float(kth)), 1e-30)
        for j in a ^ b:
            assert abs(float(sc[i][j]) - float(kth)) <= band, (
                f"row {i}: slot {j} (score {sc[i][j]!r}, k-th {kth!r}) differs outside the tie band")
            flips += 1
    return rows.shape[0], flips
