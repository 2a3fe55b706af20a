// Staging of packed (k4v4) prefix rows into the bf16 shared-memory tiles the tensor-core
// kernels read, with the dequantization fused in (cache.py:142-189 layouts; dequantize
// as reference.py:168-179, 259-268 and, for token-mode keys, splitk.py:389-395).
//
// Work items are wide so every global load is 16 bytes (or a 2-byte parameter) and all of
// an item's loads are issued before any arithmetic:
//   * token-mode K and every V: one item = (row, 32-channel group): 16 payload bytes,
//     the group's fp16 scale and zero; keys are multiplied by the per-channel divisor
//     (staged once per CTA in shared memory);
//   * KIVI channel-mode K: one item = (channel, 32-token group): 16 payload bytes holding
//     the channel's 32 tokens, its scale and zero.
// Values are fmaf(code, scale, zero) in fp32 (times the divisor for token-mode keys),
// rounded once to bf16 -- exactly kv_read8 (ma_common.cuh). Rows that are dead, missing
// or past the tile's end are zero; rows in the dense tail (slot >= nq) are copied as
// bf16 with cp.async.
#pragma once

#include "ma_common.cuh"
#include "ma_cp_async.cuh"
#include "ma_tcgen05.cuh"

namespace ma {
namespace stage {

constexpr int kGroupCh = 32;   // channels per token-mode group (the vgroup every layout here uses)

// 32 codes of a 16-byte payload -> 32 floats, code*scale + zero (element 2i: low nibble)
__device__ __forceinline__ void dequant32(const uint4& p, float s, float z, float* f) {
  const uint32_t w[4] = {p.x, p.y, p.z, p.w};
#pragma unroll
  for (int i = 0; i < 32; ++i) f[i] = fmaf((float)((w[i >> 3] >> (4 * (i & 7))) & 0xFu), s, z);
}

__device__ __forceinline__ uint4 bf16x8(const float* f) { return float8_to_bf16x8(f); }

// Byte offset of (row, 16-byte chunk) in a tile: the MMA's K-major 128-byte-swizzled
// layout, or plain row-major 256-byte rows.
template <bool SWZ>
__device__ __forceinline__ uint32_t tile_off(int row, int chunk, int rows) {
  return SWZ ? tc::kmajor_off(row, chunk, rows) : (uint32_t)(row * 256 + chunk * 16);
}

// Resolve slot `j` of the tile (read set index, liveness, storage coordinates).
struct Row {
  bool ok;      // a live prefix slot
  bool tail;    // in the dense tail (slot >= nq)
  int sb, sj;   // storage coordinates of the packed part (page or sequence, position)
  int slot;
};
__device__ __forceinline__ Row resolve(const ma_kv& kv, int H, int b, int h, int j, int end, const int64_t* idx,
                                       int64_t si0, int64_t si1) {
  Row r;
  r.slot = j;
  r.ok = j < end;
  if (r.ok && idx) r.slot = (int)idx[(int64_t)b * si0 + (int64_t)h * si1 + j];
  r.ok = r.ok && kv_live(kv, H, b, h, r.slot);
  r.tail = r.ok && r.slot >= kv.nq;
  r.sb = b;
  r.sj = r.slot;
  if (r.ok && !r.tail && kv_paged(kv, r.slot)) kv_page(kv, b, r.slot, r.sb, r.sj);
  return r;
}

// Stage `rows` slots [j0, j0+rows) (or their read-set entries) of one (b, h) with
// `nthreads` threads (thread id `tid`): K always into the swizzled K-major tile sK, V into
// sV (swizzled when VSWZ, else row-major), validity bytes into sOk. kchan_s: the
// CTA's token-mode key divisor [D] in shared memory (token layout only).
template <int ROWS, bool VSWZ, bool WANT_V>
__device__ __forceinline__ void packed_tile(const ma_kv& kv, int H, int b, int h, int j0, int end, const int64_t* idx,
                                            int64_t si0, int64_t si1, uint8_t* sK, uint8_t* sV, uint8_t* sOk,
                                            const float* kchan_s, int tid, int nthreads) {
  constexpr int kD = 128;
  constexpr int kGroups = kD / kGroupCh;                      // 4
  const bool tokk = kv.layout == MA_KV_PACKED_TOKEN;
  const __nv_bfloat16* kf = reinterpret_cast<const __nv_bfloat16*>(kv.kf);
  const __nv_bfloat16* vf = reinterpret_cast<const __nv_bfloat16*>(kv.vf);
  // (row, channel group) items: V always, K in token mode
  for (int it = tid; it < ROWS * kGroups; it += nthreads) {
    const int jj = it >> 2, g = it & 3;
    const Row r = resolve(kv, H, b, h, j0 + jj, end, idx, si0, si1);
    if (r.ok && !r.tail) {
      uint4 pv = make_uint4(0, 0, 0, 0);
      uint16_t vs = 0, vz = 0;
      if (WANT_V) {
        const int64_t vo = (int64_t)r.sb * kv.svq[0] + (int64_t)h * kv.svq[1] + (int64_t)r.sj * kv.svq[2] + g * 16;
        const int64_t vso = (int64_t)r.sb * kv.svs[0] + (int64_t)h * kv.svs[1] + (int64_t)r.sj * kv.svs[2] + g;
        pv = *reinterpret_cast<const uint4*>(kv.vq + vo);
        vs = kv.vs[vso];
        vz = kv.vz[vso];
      }
      uint4 pk = make_uint4(0, 0, 0, 0);
      uint16_t ks = 0, kz = 0;
      if (tokk) {
        const int64_t ko = (int64_t)r.sb * kv.skq[0] + (int64_t)h * kv.skq[1] + (int64_t)r.sj * kv.skq[2] + g * 16;
        const int64_t kso = (int64_t)r.sb * kv.sks[0] + (int64_t)h * kv.sks[1] + (int64_t)r.sj * kv.sks[2] + g;
        pk = *reinterpret_cast<const uint4*>(kv.kq + ko);
        ks = kv.ks[kso];
        kz = kv.kz[kso];
      }
      float f[32];
      if (WANT_V) {
        dequant32(pv, half_bits_to_float(vs), half_bits_to_float(vz), f);
#pragma unroll
        for (int c = 0; c < 4; ++c) {
          float t[8];
#pragma unroll
          for (int i = 0; i < 8; ++i) t[i] = bf16_round(f[8 * c + i]);
          *reinterpret_cast<uint4*>(sV + tile_off<VSWZ>(jj, g * 4 + c, ROWS)) = bf16x8(t);
        }
      }
      if (tokk) {
        dequant32(pk, half_bits_to_float(ks), half_bits_to_float(kz), f);
#pragma unroll
        for (int c = 0; c < 4; ++c) {
          float t[8];
#pragma unroll
          for (int i = 0; i < 8; ++i) t[i] = f[8 * c + i] * kchan_s[g * kGroupCh + 8 * c + i];
          *reinterpret_cast<uint4*>(sK + tile_off<true>(jj, g * 4 + c, ROWS)) = bf16x8(t);
        }
      }
    } else if (r.tail) {   // dense bf16 tail: 4 chunks of 16 bytes per group, by cp.async
      const int row = r.slot - kv.nq;
#pragma unroll
      for (int c = 0; c < 4; ++c) {
        const int ch = g * 4 + c;
        if (WANT_V)
          cp_async16(tc::smem_addr(sV + tile_off<VSWZ>(jj, ch, ROWS)),
                     vf + (int64_t)b * kv.svf[0] + (int64_t)h * kv.svf[1] + (int64_t)row * kv.svf[2] + ch * 8, true);
        cp_async16(tc::smem_addr(sK + tile_off<true>(jj, ch, ROWS)),
                   kf + (int64_t)b * kv.skf[0] + (int64_t)h * kv.skf[1] + (int64_t)row * kv.skf[2] + ch * 8, true);
      }
    } else {               // dead or missing: exact zeros
#pragma unroll
      for (int c = 0; c < 4; ++c) {
        if (WANT_V) *reinterpret_cast<uint4*>(sV + tile_off<VSWZ>(jj, g * 4 + c, ROWS)) = make_uint4(0, 0, 0, 0);
        *reinterpret_cast<uint4*>(sK + tile_off<true>(jj, g * 4 + c, ROWS)) = make_uint4(0, 0, 0, 0);
      }
    }
    if (g == 0) sOk[jj] = r.ok ? 1 : 0;
  }
  if (tokk) return;
  // KIVI keys: (channel, 32-token group) items; the tile's rows in a group share the
  // group's payload. Rows of a group resolve to consecutive slots only without a read
  // set, so read sets (and tails) take the per-row path.
  for (int it = tid; it < (ROWS / 32) * kD; it += nthreads) {
    const int tg = it / kD, d = it - (it / kD) * kD;
    const int jr0 = tg * 32;
    if (!idx && j0 % 32 == 0 && j0 + jr0 + 32 <= kv.nq) {
      // 32 consecutive packed slots = one token group of one page (page_size % kgroup == 0)
      const Row r0 = resolve(kv, H, b, h, j0 + jr0, end, nullptr, 0, 0);
      int sb = b, sj = j0 + jr0;
      if (kv_paged(kv, sj)) kv_page(kv, b, sj, sb, sj);
      const bool page_ok = sb >= 0;
      const int gi = sj / kv.kgroup;
      uint4 p = make_uint4(0, 0, 0, 0);
      uint16_t s = 0, z = 0;
      if (page_ok) {
        const int64_t base = (int64_t)sb * kv.skq[0] + (int64_t)h * kv.skq[1] + (int64_t)gi * kv.skq[2] + d * 16;
        const int64_t so = (int64_t)sb * kv.sks[0] + (int64_t)h * kv.sks[1] + (int64_t)gi * kv.sks[2] + d;
        p = *reinterpret_cast<const uint4*>(kv.kq + base);
        s = kv.ks[so];
        z = kv.kz[so];
      }
      (void)r0;
      float f[32];
      dequant32(p, half_bits_to_float(s), half_bits_to_float(z), f);
      // column d of rows jr0..jr0+31: 2-byte stores (the validity bytes zero dead rows below)
      const int chunk = d >> 3, within = d & 7;
#pragma unroll
      for (int i = 0; i < 32; ++i) {
        const int jj = jr0 + i;
        const bool live = page_ok && kv_live(kv, H, b, h, j0 + jj) && j0 + jj < end;
        reinterpret_cast<__nv_bfloat16*>(sK + tile_off<true>(jj, chunk, ROWS))[within] =
            __float2bfloat16_rn(live ? f[i] : 0.f);
      }
    } else {
      // general path: per row (read sets, tails, partial groups)
#pragma unroll 4
      for (int i = 0; i < 32; ++i) {
        const int jj = jr0 + i;
        const Row r = resolve(kv, H, b, h, j0 + jj, end, idx, si0, si1);
        float v = 0.f;
        if (r.ok && !r.tail) {
          const int gi = r.sj / kv.kgroup, ti = r.sj - gi * kv.kgroup;
          const uint8_t* base = kv.kq + (int64_t)r.sb * kv.skq[0] + (int64_t)h * kv.skq[1] + (int64_t)gi * kv.skq[2];
          const int64_t so = (int64_t)r.sb * kv.sks[0] + (int64_t)h * kv.sks[1] + (int64_t)gi * kv.sks[2] + d;
          const uint32_t byte = base[(int64_t)d * (kv.kgroup / 2) + ti / 2];
          const uint32_t code = (ti & 1) ? (byte >> 4) : (byte & 0xFu);
          v = fmaf((float)code, half_bits_to_float(kv.ks[so]), half_bits_to_float(kv.kz[so]));
        } else if (r.tail) {
          continue;   // the tail row's keys came by cp.async above
        }
        reinterpret_cast<__nv_bfloat16*>(sK + tile_off<true>(jj, d >> 3, ROWS))[d & 7] = __float2bfloat16_rn(v);
      }
    }
  }
}

// ---------------------------------------------------------------------------------
// Register pipeline of the token-mode staging: ONE (row, 32-channel group) item per
// thread and tile (64 rows x 4 groups = 256 threads). Its dependent loads are spread over
// the four iterations before the item is needed --
//   tok_slot    the read-set index (or the contiguous slot),
//   tok_locate  liveness (lens, page table, mask) and storage coordinates,
//   tok_fetch   the 16-byte K and V payloads and their scale/zero,
//   tok_store   dequantization into the bf16 tile (the only step that waits),
// so every global load has a whole tile of work to land.
struct TokItem {
  int slot;          // logical slot (-1: none)
  int sb, sj;        // storage coordinates of the packed part
  bool ok, tail;     // live; in the dense tail
  uint4 pk, pv;      // payloads
  uint16_t ks, kz, vs, vz;
};

__device__ __forceinline__ int tok_slot(int b, int h, int j, int end, const int64_t* idx, int64_t si0, int64_t si1) {
  if (j >= end) return -1;
  return idx ? (int)idx[(int64_t)b * si0 + (int64_t)h * si1 + j] : j;
}

__device__ __forceinline__ void tok_locate(const ma_kv& kv, int H, int b, int h, int slot, TokItem& it) {
  it.slot = slot;
  it.ok = slot >= 0 && kv_live(kv, H, b, h, slot);
  it.tail = it.ok && slot >= kv.nq;
  it.sb = b;
  it.sj = slot;
  if (it.ok && !it.tail && kv_paged(kv, slot)) kv_page(kv, b, slot, it.sb, it.sj);
}

__device__ __forceinline__ void tok_fetch(const ma_kv& kv, int h, int g, TokItem& it) {
  if (!it.ok || it.tail) return;
  const int64_t vo = (int64_t)it.sb * kv.svq[0] + (int64_t)h * kv.svq[1] + (int64_t)it.sj * kv.svq[2] + g * 16;
  const int64_t vso = (int64_t)it.sb * kv.svs[0] + (int64_t)h * kv.svs[1] + (int64_t)it.sj * kv.svs[2] + g;
  const int64_t ko = (int64_t)it.sb * kv.skq[0] + (int64_t)h * kv.skq[1] + (int64_t)it.sj * kv.skq[2] + g * 16;
  const int64_t kso = (int64_t)it.sb * kv.sks[0] + (int64_t)h * kv.sks[1] + (int64_t)it.sj * kv.sks[2] + g;
  it.pv = *reinterpret_cast<const uint4*>(kv.vq + vo);
  it.pk = *reinterpret_cast<const uint4*>(kv.kq + ko);
  it.vs = kv.vs[vso];
  it.vz = kv.vz[vso];
  it.ks = kv.ks[kso];
  it.kz = kv.kz[kso];
}

// Item -> row jj, channels [32g, 32g+32) of the swizzled bf16 K and V tiles (ROWS rows).
template <int ROWS>
__device__ __forceinline__ void tok_store(const ma_kv& kv, int b, int h, int jj, int g, const TokItem& it, uint8_t* sK,
                                          uint8_t* sV, uint8_t* sOk, const float* kchan_s) {
  if (it.ok && !it.tail) {
    float f[32];
    dequant32(it.pv, half_bits_to_float(it.vs), half_bits_to_float(it.vz), f);
#pragma unroll
    for (int c = 0; c < 4; ++c) {
      float t[8];
#pragma unroll
      for (int i = 0; i < 8; ++i) t[i] = bf16_round(f[8 * c + i]);
      *reinterpret_cast<uint4*>(sV + tc::kmajor_off(jj, g * 4 + c, ROWS)) = bf16x8(t);
    }
    dequant32(it.pk, half_bits_to_float(it.ks), half_bits_to_float(it.kz), f);
#pragma unroll
    for (int c = 0; c < 4; ++c) {
      float t[8];
#pragma unroll
      for (int i = 0; i < 8; ++i) t[i] = f[8 * c + i] * kchan_s[g * kGroupCh + 8 * c + i];
      *reinterpret_cast<uint4*>(sK + tc::kmajor_off(jj, g * 4 + c, ROWS)) = bf16x8(t);
    }
  } else if (it.tail) {   // a dense bf16 tail row (rare): plain 16-byte loads
    const int row = it.slot - kv.nq;
    const __nv_bfloat16* kf = reinterpret_cast<const __nv_bfloat16*>(kv.kf);
    const __nv_bfloat16* vf = reinterpret_cast<const __nv_bfloat16*>(kv.vf);
#pragma unroll
    for (int c = 0; c < 4; ++c) {
      const int ch = g * 4 + c;
      const uint4 kk = *reinterpret_cast<const uint4*>(kf + (int64_t)b * kv.skf[0] + (int64_t)h * kv.skf[1] + (int64_t)row * kv.skf[2] + ch * 8);
      const uint4 vv = *reinterpret_cast<const uint4*>(vf + (int64_t)b * kv.svf[0] + (int64_t)h * kv.svf[1] + (int64_t)row * kv.svf[2] + ch * 8);
      *reinterpret_cast<uint4*>(sK + tc::kmajor_off(jj, ch, ROWS)) = kk;
      *reinterpret_cast<uint4*>(sV + tc::kmajor_off(jj, ch, ROWS)) = vv;
    }
  } else {
#pragma unroll
    for (int c = 0; c < 4; ++c) {
      *reinterpret_cast<uint4*>(sV + tc::kmajor_off(jj, g * 4 + c, ROWS)) = make_uint4(0, 0, 0, 0);
      *reinterpret_cast<uint4*>(sK + tc::kmajor_off(jj, g * 4 + c, ROWS)) = make_uint4(0, 0, 0, 0);
    }
  }
  if (g == 0) sOk[jj] = it.ok ? 1 : 0;
}

}  // namespace stage
}  // namespace ma
