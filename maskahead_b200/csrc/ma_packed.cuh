// Dequantizing producers of the TMA-pipelined kernels for token-mode k4v4 prefixes.
//
// A token-mode packed prefix (cache.py:146-152, 172-189) stores per slot and KV head a
// 64-byte payload (128 4-bit codes, element 2i in the low nibble of byte i,
// reference.py:41-45) and per 32-channel group an fp16 scale and zero, for K and V alike;
// keys are multiplied by the per-channel divisor kchan after dequantization
// (splitk.py:389-395). The pipelined kernels read K and V tiles as bf16 [128 slots][128
// channels] in the 128-byte-swizzled layout a TMA box writes (two 16 KB column blocks,
// 16-byte chunk q of row r at q ^ (r & 7)). Here producer warps build those tiles straight
// from the packed bytes, so a step reads 160 B per slot and head instead of an unpacked
// bf16 copy's 512 (plus the unpack's own 160 + 512):
//
//   * one thread per slot row: the row's 64 payload bytes (four 16-byte loads) and its
//     scale/zero words (8 bytes each) for K and V, a warp reading 32 consecutive rows
//     (2 KB contiguous);
//   * value = fma(code, scale, zero) in fp32 (times kchan for keys), one rounding to bf16:
//     the arithmetic of every other reader of this layout (ma_common.cuh kv_read8, the
//     unpack kernel), so tiles are bit-identical to an unpack followed by a TMA load;
//   * codes become floats exactly through the exponent trick: prmt places a code byte
//     under the bit pattern of 2^23, and 2^23 + code - 2^23 is exact; pairs of values go
//     through the packed fp32 pipe (fma.rn.f32x2, mul.rn.f32x2), one cvt per bf16 pair;
//   * rows past the sequence's end (or on a page outside the pool) are written as zeros.
//
// Raw rows reach shared memory by bulk copies (cp.async.bulk, completion on an mbarrier)
// that one thread issues a few tiles ahead into a staging ring (stage_tile, the page-table
// entries of the CTA's range read once into shared memory: PageCache); the producer warps
// then turn a staged tile into bf16 tiles (dequant_item). Kernels that keep raw rows
// in registers instead (the value pass of the mass kernel) read them with load_row.
#pragma once

#include "ma_common.cuh"
#include "ma_tcgen05.cuh"

namespace ma {
namespace packed {

constexpr int kTileRows = 128;
constexpr int kRowBytes = 64;        // 128 channels x 4 bits
constexpr int kBlockBytes = 128 * 128;   // one 64-channel column block of a bf16 tile

// Host-side eligibility: token-mode packed prefix without a dense tail or mask, 128
// channels in groups of 32, every slot's payload and scale/zero rows contiguous and every
// range the prefetch and the loads touch 16-byte aligned.
inline bool eligible(const ma_kv& kv) {
  auto a16 = [](const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; };
  if (kv.layout != MA_KV_PACKED_TOKEN || kv.nq <= 0 || kv.nf != 0 || kv.mask || kv.vgroup != 32 || !kv.kchan)
    return false;
  if (!a16(kv.kq) || !a16(kv.vq) || !a16(kv.ks) || !a16(kv.kz) || !a16(kv.vs) || !a16(kv.vz)) return false;
  if (kv.skq[2] != kRowBytes || kv.svq[2] != kRowBytes || kv.sks[2] != 4 || kv.svs[2] != 4) return false;
  for (int i = 0; i < 2; ++i)
    if ((kv.skq[i] & 15) || (kv.svq[i] & 15) || (kv.sks[i] & 7) || (kv.svs[i] & 7)) return false;
  if (kv.pages) return kv.page_size >= 2 && (kv.page_size & 1) == 0;
  return (kv.nq & 1) == 0;
}

// Storage coordinates of slot j of sequence b: (sequence or page, position); false when
// the slot's page lies outside the pool.
__device__ __forceinline__ bool locate(const ma_kv& kv, int b, int j, int& sb, int& sj) {
  if (kv.pages == nullptr) {
    sb = b;
    sj = j;
    return true;
  }
  kv_page(kv, b, j, sb, sj);
  return sb >= 0;
}

__device__ __forceinline__ void prefetch_l2(const void* p, uint32_t bytes) {
  bytes &= ~15u;
  if (bytes) asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;\n" ::"l"(p), "r"(bytes) : "memory");
}

// L2 prefetch of the K and V rows [j0, j1) of head h of sequence b (every storage
// segment: one per page crossed).
__device__ __forceinline__ void prefetch_rows(const ma_kv& kv, int b, int h, int j0, int j1) {
  for (int j = j0; j < j1;) {
    int sb, sj;
    const int seg_end = kv.pages ? min(j1, (j / kv.page_size + 1) * kv.page_size) : j1;
    const int cnt = seg_end - j;
    if (locate(kv, b, j, sb, sj)) {
      const int64_t q = (int64_t)sb * kv.skq[0] + (int64_t)h * kv.skq[1] + (int64_t)sj * kRowBytes;
      const int64_t qv = (int64_t)sb * kv.svq[0] + (int64_t)h * kv.svq[1] + (int64_t)sj * kRowBytes;
      const int64_t s = (int64_t)sb * kv.sks[0] + (int64_t)h * kv.sks[1] + (int64_t)sj * 4;
      const int64_t sv = (int64_t)sb * kv.svs[0] + (int64_t)h * kv.svs[1] + (int64_t)sj * 4;
      prefetch_l2(kv.kq + q, (uint32_t)cnt * kRowBytes);
      prefetch_l2(kv.vq + qv, (uint32_t)cnt * kRowBytes);
      prefetch_l2(kv.ks + s, (uint32_t)cnt * 8);
      prefetch_l2(kv.kz + s, (uint32_t)cnt * 8);
      prefetch_l2(kv.vs + sv, (uint32_t)cnt * 8);
      prefetch_l2(kv.vz + sv, (uint32_t)cnt * 8);
    }
    j = seg_end;
  }
}

// One slot row of one array: 64 payload bytes, 4 scales and 4 zeros (fp16 bits).
struct Raw {
  uint4 p[4];
  uint2 s, z;
};

__device__ __forceinline__ void load_raw(const uint8_t* q, const uint16_t* s, const uint16_t* z, int64_t qoff,
                                         int64_t soff, Raw& r) {
  const uint4* pq = reinterpret_cast<const uint4*>(q + qoff);
#pragma unroll
  for (int i = 0; i < 4; ++i) r.p[i] = __ldg(pq + i);
  r.s = __ldg(reinterpret_cast<const uint2*>(s + soff));
  r.z = __ldg(reinterpret_cast<const uint2*>(z + soff));
}

// The arrays of slot j (sequence b, head h) a kernel needs (keys, values); ok = false for
// a row outside the sequence (j >= end) or on a missing page: nothing is loaded.
struct RawRow {
  Raw k, v;
  bool ok;
};
__device__ __forceinline__ void load_row(const ma_kv& kv, int b, int h, int j, int end, RawRow& r,
                                         bool want_k = true, bool want_v = true) {
  int sb = 0, sj = 0;
  r.ok = j < end && locate(kv, b, j, sb, sj);
  if (!r.ok) return;
  if (want_k)
    load_raw(kv.kq, kv.ks, kv.kz, (int64_t)sb * kv.skq[0] + (int64_t)h * kv.skq[1] + (int64_t)sj * kRowBytes,
             (int64_t)sb * kv.sks[0] + (int64_t)h * kv.sks[1] + (int64_t)sj * 4, r.k);
  if (want_v)
    load_raw(kv.vq, kv.vs, kv.vz, (int64_t)sb * kv.svq[0] + (int64_t)h * kv.svq[1] + (int64_t)sj * kRowBytes,
             (int64_t)sb * kv.svs[0] + (int64_t)h * kv.svs[1] + (int64_t)sj * 4, r.v);
}

// ------------------------------------------------------------------- staging ring
// One staged tile: the 128 rows' payloads (row r at r*64) of K and V, then their
// scale/zero words (row r at r*8) -- 160 bytes per row.
constexpr int kStageBytes = kTileRows * (2 * kRowBytes + 4 * 8);   // 20 KB
constexpr int kStgKq = 0, kStgVq = kTileRows * kRowBytes, kStgKs = 2 * kTileRows * kRowBytes;
constexpr int kStgKz = kStgKs + kTileRows * 8, kStgVs = kStgKz + kTileRows * 8, kStgVz = kStgVs + kTileRows * 8;

__device__ __forceinline__ void bulk_copy(void* dst, const void* src, uint32_t bytes, uint64_t* bar) {
  asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];\n" ::"r"(
                   tc::smem_addr(dst)),
               "l"(src), "r"(bytes), "r"(tc::smem_addr(bar))
               : "memory");
}

// The page-table entries of a CTA's key range, copied to shared memory once: pages
// p0 .. p0 + n - 1 of the CTA's sequence (n = 0: none cached). A lookup outside them reads
// the global table.
struct PageCache {
  const int* s;
  int p0, n;
};
__device__ __forceinline__ bool locate(const ma_kv& kv, int b, int j, int& sb, int& sj, const PageCache& pc) {
  if (kv.pages != nullptr) {
    const int pi = j / kv.page_size;
    const int k = pi - pc.p0;
    if (k >= 0 && k < pc.n) {
      const int p = pc.s[k];
      sb = (p >= 0 && p < kv.num_pages) ? p : -1;
      sj = j - pi * kv.page_size;
      return sb >= 0;
    }
  }
  return locate(kv, b, j, sb, sj);
}

// The copies of rows [j0, j1) of head h of sequence b into a staging stage: one set of six
// (K and V payloads, scales, zeros) per storage segment (one per page crossed), each
// segment's row count rounded up to even so every scale/zero copy is a multiple of 16 bytes
// (the extra row exists: nq and page sizes are even, segments start at even slots); a
// segment on a page outside the pool is not copied. Returns the bytes they move; with ISSUE
// the copies are issued, completing on `bar` (whose transaction count the caller set).
template <bool ISSUE>
__device__ __forceinline__ uint32_t stage_copies(const ma_kv& kv, int b, int h, int j0, int j1, uint8_t* stg,
                                                 uint64_t* bar, const PageCache& pc) {
  uint32_t total = 0;
  for (int j = j0; j < j1;) {
    const int seg_end = kv.pages ? min(j1, (j / kv.page_size + 1) * kv.page_size) : j1;
    int sb, sj;
    if (locate(kv, b, j, sb, sj, pc)) {
      int cnt = seg_end - j;
      const int avail = kv.pages ? kv.page_size - sj : kv.nq - j;
      cnt = min(cnt + (cnt & 1), avail);
      if (ISSUE) {
        const int r0 = j - j0;
        const int64_t q = (int64_t)sb * kv.skq[0] + (int64_t)h * kv.skq[1] + (int64_t)sj * kRowBytes;
        const int64_t qv = (int64_t)sb * kv.svq[0] + (int64_t)h * kv.svq[1] + (int64_t)sj * kRowBytes;
        const int64_t s = (int64_t)sb * kv.sks[0] + (int64_t)h * kv.sks[1] + (int64_t)sj * 4;
        const int64_t sv = (int64_t)sb * kv.svs[0] + (int64_t)h * kv.svs[1] + (int64_t)sj * 4;
        bulk_copy(stg + kStgKq + r0 * kRowBytes, kv.kq + q, (uint32_t)cnt * kRowBytes, bar);
        bulk_copy(stg + kStgVq + r0 * kRowBytes, kv.vq + qv, (uint32_t)cnt * kRowBytes, bar);
        bulk_copy(stg + kStgKs + r0 * 8, kv.ks + s, (uint32_t)cnt * 8, bar);
        bulk_copy(stg + kStgKz + r0 * 8, kv.kz + s, (uint32_t)cnt * 8, bar);
        bulk_copy(stg + kStgVs + r0 * 8, kv.vs + sv, (uint32_t)cnt * 8, bar);
        bulk_copy(stg + kStgVz + r0 * 8, kv.vz + sv, (uint32_t)cnt * 8, bar);
      }
      total += (uint32_t)cnt * (2 * kRowBytes + 32);
    }
    j = seg_end;
  }
  return total;
}

// Stage rows [j0, j1): the transaction count, then the copies (one issuing thread).
__device__ __forceinline__ void stage_tile(const ma_kv& kv, int b, int h, int j0, int j1, uint8_t* stg,
                                           uint64_t* bar, const PageCache& pc) {
  const uint32_t bytes = stage_copies<false>(kv, b, h, j0, j1, stg, bar, pc);
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%1], %0;\n" ::"r"(bytes), "r"(tc::smem_addr(bar))
               : "memory");
  stage_copies<true>(kv, b, h, j0, j1, stg, bar, pc);
}

// Whether slot j of sequence b holds a row the tiles must carry (below end, on a page of
// the pool); the others are written as zeros.
__device__ __forceinline__ bool row_ok(const ma_kv& kv, int b, int j, int end, const PageCache& pc) {
  int sb, sj;
  return j < end && locate(kv, b, j, sb, sj, pc);
}

__device__ __forceinline__ float2 fmul2(float2 a, float2 b) {
  uint64_t d;
  asm("mul.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(tc::f2_bits(a)), "l"(tc::f2_bits(b)));
  return tc::bits_f2(d);
}
// 2^23 + byte i of x (a code 0..15 in the low nibble), as a float
__device__ __forceinline__ float magic(uint32_t x, uint32_t sel) {
  uint32_t d;
  asm("prmt.b32 %0, %1, %2, %3;" : "=r"(d) : "r"(x), "r"(0x4B000000u), "r"(sel));
  return __uint_as_float(d);
}
__device__ __forceinline__ uint32_t half_word(uint2 w, int g) {
  return ((g & 2) ? w.y : w.x) >> (16 * (g & 1));
}

// 8 codes of payload word w (element 2i in the low nibble of byte i) -> bf16 x 8:
// fma(code, s, z) in fp32, times the divisor kch8[0..7] for keys, one rounding.
template <bool KEY>
__device__ __forceinline__ uint4 chunk_core(uint32_t w, float s, float z, const float* kch8) {
  const uint32_t lo = w & 0x0F0F0F0Fu, hi = (w >> 4) & 0x0F0F0F0Fu;
  const float2 bias = make_float2(-8388608.f, -8388608.f), s2 = make_float2(s, s), z2 = make_float2(z, z);
  uint4 out;
  uint32_t* o = &out.x;
#pragma unroll
  for (int i = 0; i < 4; ++i) {   // elements 2i (low nibble of byte i) and 2i + 1
    const uint32_t sel = (uint32_t)i | 0x7540u;
    float2 x = tc::fadd2(make_float2(magic(lo, sel), magic(hi, sel)), bias);
    x = tc::ffma2(x, s2, z2);
    if (KEY) x = fmul2(x, *reinterpret_cast<const float2*>(kch8 + 2 * i));
    __nv_bfloat162 v = __floats2bfloat162_rn(x.x, x.y);
    o[i] = *reinterpret_cast<uint32_t*>(&v);
  }
  return out;
}

// Chunk c (channels 8c..8c+7) of a raw row.
template <bool KEY>
__device__ __forceinline__ uint4 chunk(const Raw& r, int c, const float* kchan_s) {
  const uint32_t w = (&r.p[c >> 2].x)[c & 3];
  const int g = c >> 2;   // 32-channel group
  const float s = __half2float(__ushort_as_half((uint16_t)half_word(r.s, g)));
  const float z = __half2float(__ushort_as_half((uint16_t)half_word(r.z, g)));
  return chunk_core<KEY>(w, s, z, KEY ? kchan_s + 8 * c : nullptr);
}

// Item (row, group g) of a staged tile: the group's 32 values of K (KEY, times kchan) or V
// dequantized into chunks 4g..4g+3 of the tile's row (zeros if !ok).
template <bool KEY>
__device__ __forceinline__ void dequant_item(const uint8_t* stg, int row, int g, bool ok, uint8_t* tile,
                                             const float* kchan_s) {
  uint8_t* line = tile + (g >> 1) * kBlockBytes + row * 128;
  if (!ok) {
#pragma unroll
    for (int i = 0; i < 4; ++i)
      *reinterpret_cast<uint4*>(line + ((((4 * g + i) & 7) ^ (row & 7)) << 4)) = make_uint4(0, 0, 0, 0);
    return;
  }
  const uint4 p = *reinterpret_cast<const uint4*>(stg + (KEY ? kStgKq : kStgVq) + row * kRowBytes + g * 16);
  const float s = __half2float(*reinterpret_cast<const __half*>(stg + (KEY ? kStgKs : kStgVs) + row * 8 + g * 2));
  const float z = __half2float(*reinterpret_cast<const __half*>(stg + (KEY ? kStgKz : kStgVz) + row * 8 + g * 2));
  const uint32_t w[4] = {p.x, p.y, p.z, p.w};
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const int c = 4 * g + i;
    *reinterpret_cast<uint4*>(line + (((c & 7) ^ (row & 7)) << 4)) =
        chunk_core<KEY>(w[i], s, z, KEY ? kchan_s + 8 * c : nullptr);
  }
}

// Row `row` of a bf16 SW128 tile (two 64-channel blocks) from a raw row (zeros if !ok).
template <bool KEY>
__device__ __forceinline__ void store_row(const Raw& r, bool ok, uint8_t* tile, int row, const float* kchan_s) {
  uint8_t* line = tile + row * 128;
#pragma unroll
  for (int c = 0; c < 16; ++c) {
    const uint4 v = ok ? chunk<KEY>(r, c, kchan_s) : make_uint4(0, 0, 0, 0);
    *reinterpret_cast<uint4*>(line + (c >> 3) * kBlockBytes + (((c & 7) ^ (row & 7)) << 4)) = v;
  }
}

}  // namespace packed
}  // namespace ma
