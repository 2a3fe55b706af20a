"""GPU parity of the cache compaction after an eviction (ma_compact_tokens).

* On the reference's own caches (fixtures recorded by running PackedKVCache.compact_tokens
  on a token-mode k4v4 cache and PackedKVCache.compact on a bf16 cache,
  tests/golden/make_golden.py) the device compaction must give the reference's arrays
  bit for bit, every layer in one call (the layer axis merged into the batch axis).
* On larger random caches it must equal the oracle's compaction bit for bit for any keep
  order, out-of-range keep entries (zero rows), strided sources and a destination with
  more slots than kept (slots past C untouched).
"""

from __future__ import annotations

import pytest
import torch

import oracle
from test_oracle_golden import load_compact

pytestmark = pytest.mark.gpu

DEV = "cuda"


def _merge_layers(t: torch.Tensor) -> torch.Tensor:
    """[L, B, H, ...] -> [L*B, H, ...] (the C ABI's batch axis covers every layer)."""
    return t.reshape(t.shape[0] * t.shape[1], *t.shape[2:])


def _bytes(t: torch.Tensor) -> torch.Tensor:
    return t.contiguous().view(torch.uint8)


def test_token_mode_matches_reference_compact_tokens():
    from maskahead_b200.layouts import Prefix, compact_tokens

    f = load_compact("compact_token")
    dev = {k: _merge_layers(v).to(DEV) for k, v in f.items()}
    n = dev["before_k_q"].shape[2]
    src = Prefix(kq=dev["before_k_q"], ks=dev["before_k_scale"], kz=dev["before_k_zero"],
                 vq=dev["before_v_q"], vs=dev["before_v_scale"], vz=dev["before_v_zero"], nq=n, kb=4, vb=4,
                 kmode=1, kch=dev["k_chan"])
    out = compact_tokens(src, dev["keep"])
    torch.cuda.synchronize()
    for ours, name in ((out.kq, "k_q"), (out.ks, "k_scale"), (out.kz, "k_zero"), (out.vq, "v_q"),
                       (out.vs, "v_scale"), (out.vz, "v_zero")):
        want = _merge_layers(f[f"after_{name}"])
        assert torch.equal(_bytes(ours.cpu()), _bytes(want)), name
    assert out.nq == f["keep"].shape[-1]


def test_bf16_matches_reference_compact():
    from maskahead_b200.layouts import Prefix, compact_tokens

    f = load_compact("compact_bf16")
    kf, vf = _merge_layers(f["before_k_fp"]).to(DEV), _merge_layers(f["before_v_fp"]).to(DEV)
    out = compact_tokens(Prefix.dense(kf, vf), _merge_layers(f["keep"]).to(DEV))
    torch.cuda.synchronize()
    assert torch.equal(_bytes(out.kf.cpu()), _bytes(_merge_layers(f["after_k_fp"])))
    assert torch.equal(_bytes(out.vf.cpu()), _bytes(_merge_layers(f["after_v_fp"])))


def _random_keep(B, H, n, C, gen, *, sorted_=True, bad=0):
    keep = torch.stack([torch.randperm(n, generator=gen)[:C] for _ in range(B * H)]).view(B, H, C)
    if sorted_:
        keep = keep.sort(-1).values
    if bad:
        flat = keep.view(-1)
        pos = torch.randperm(flat.numel(), generator=gen)[:bad]
        flat[pos[: bad // 2]] = -1
        flat[pos[bad // 2:]] = n + 7
    return keep


@pytest.mark.parametrize("sorted_,bad", [(True, 0), (False, 64)])
def test_token_mode_random_matches_oracle(sorted_, bad):
    from maskahead_b200.layouts import Prefix, compact_tokens, pack_prefix

    gen = torch.Generator().manual_seed(31)
    B, H, n, D, C, cap = 2, 4, 20000, 128, 4096, 5000
    k = torch.randn(B, H, n, D, generator=gen).to(torch.bfloat16).to(DEV)
    v = torch.randn(B, H, n, D, generator=gen).to(torch.bfloat16).to(DEV)
    src = pack_prefix(k, v, key_mode="token")
    keep = _random_keep(B, H, n, C, gen, sorted_=sorted_, bad=bad)
    # destination with more slots than kept: slots >= C keep their sentinel
    dst = Prefix(kq=torch.full((B, H, cap, D // 32, 16), 0xA5, dtype=torch.uint8, device=DEV),
                 ks=torch.full((B, H, cap, D // 32), 3.0, dtype=torch.float16, device=DEV),
                 kz=torch.full((B, H, cap, D // 32), 3.0, dtype=torch.float16, device=DEV),
                 vq=torch.full((B, H, cap, D // 32, 16), 0xA5, dtype=torch.uint8, device=DEV),
                 vs=torch.full((B, H, cap, D // 32), 3.0, dtype=torch.float16, device=DEV),
                 vz=torch.full((B, H, cap, D // 32), 3.0, dtype=torch.float16, device=DEV),
                 nq=cap, kb=4, vb=4, kmode=1, kch=src.kch)
    before = {name: getattr(dst, name).cpu() for name in ("kq", "ks", "kz", "vq", "vs", "vz")}
    out = compact_tokens(src, keep.to(DEV), out=dst)
    torch.cuda.synchronize()
    assert out is dst and out.nq == C
    for name in ("kq", "ks", "kz", "vq", "vs", "vz"):
        want = oracle.compact_slots(getattr(src, name).cpu(), keep)
        got = getattr(out, name).cpu()
        assert torch.equal(_bytes(got[:, :, :C]), _bytes(want)), name
        assert torch.equal(_bytes(got[:, :, C:]), _bytes(before[name][:, :, C:])), f"{name}: slots past C written"


@pytest.mark.parametrize("dtype,D", [(torch.bfloat16, 128), (torch.float32, 64)])
def test_dense_strided_source_matches_oracle(dtype, D):
    from maskahead_b200.layouts import Prefix, compact_tokens

    gen = torch.Generator().manual_seed(32)
    B, H, n, cap, C = 3, 2, 3000, 3500, 1000
    kbuf = torch.randn(B, H, cap, D, generator=gen).to(dtype).to(DEV)
    vbuf = torch.randn(B, H, cap, D, generator=gen).to(dtype).to(DEV)
    src = Prefix.dense(kbuf[:, :, :n], vbuf[:, :, :n])          # strided: capacity > live
    keep = _random_keep(B, H, n, C, gen, sorted_=False, bad=10)
    out = compact_tokens(src, keep.to(DEV))
    torch.cuda.synchronize()
    assert torch.equal(out.kf.cpu(), oracle.compact_slots(kbuf[:, :, :n].cpu(), keep))
    assert torch.equal(out.vf.cpu(), oracle.compact_slots(vbuf[:, :, :n].cpu(), keep))


def test_rejected_requests():
    from maskahead_b200._lib import MaError
    from maskahead_b200.layouts import Prefix, compact_tokens, pack_prefix

    k = torch.randn(1, 2, 256, 128, device=DEV).to(torch.bfloat16)
    v = torch.randn(1, 2, 256, 128, device=DEV).to(torch.bfloat16)
    keep = torch.arange(64, device=DEV).expand(1, 2, 64).contiguous()
    with pytest.raises(NotImplementedError):
        compact_tokens(pack_prefix(k, v, key_mode="channel"), keep)
    with pytest.raises(ValueError):
        compact_tokens(Prefix.dense(k[:, :, :32], v[:, :, :32]), keep)
    src = Prefix.dense(k, v)
    with pytest.raises(MaError):
        compact_tokens(src, keep, out=src)                       # in place is refused
    empty = compact_tokens(src, keep[:, :, :0])
    assert empty.nf == 0
