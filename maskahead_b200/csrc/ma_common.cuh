// Shared device code of the maskahead_b200 kernels: KV-layout readers, partial-result
// layout, warp/block helpers. All kernels are written for sm_100a (B200).
#pragma once

#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <utility>

#include "../../include/maskahead_b200.h"

namespace ma {

constexpr int kMaxD = 128;

// ----------------------------------------------------------------------------------
// Element conversion
// ----------------------------------------------------------------------------------
__device__ __forceinline__ float bf16_round(float x) {
  return __bfloat162float(__float2bfloat16_rn(x));
}
__device__ __forceinline__ float half_bits_to_float(uint16_t h) {
  return __half2float(__ushort_as_half(h));
}
__device__ __forceinline__ void bf16x8_to_float(const uint4& u, float f[8]) {
  const __nv_bfloat162* p = reinterpret_cast<const __nv_bfloat162*>(&u);
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    float2 t = __bfloat1622float2(p[i]);
    f[2 * i] = t.x;
    f[2 * i + 1] = t.y;
  }
}
__device__ __forceinline__ uint4 float8_to_bf16x8(const float f[8]) {
  uint4 u;
  __nv_bfloat162* p = reinterpret_cast<__nv_bfloat162*>(&u);
#pragma unroll
  for (int i = 0; i < 4; ++i) p[i] = __floats2bfloat162_rn(f[2 * i], f[2 * i + 1]);
  return u;
}

// ----------------------------------------------------------------------------------
// Query / output element access ([B,Hq,T,D] with strides over b, hq, t)
// ----------------------------------------------------------------------------------
template <typename T>
__device__ __forceinline__ void load8(const T* p, float f[8]);
template <>
__device__ __forceinline__ void load8<float>(const float* p, float f[8]) {
  float4 a = *reinterpret_cast<const float4*>(p);
  float4 b = *reinterpret_cast<const float4*>(p + 4);
  f[0] = a.x; f[1] = a.y; f[2] = a.z; f[3] = a.w;
  f[4] = b.x; f[5] = b.y; f[6] = b.z; f[7] = b.w;
}
template <>
__device__ __forceinline__ void load8<__nv_bfloat16>(const __nv_bfloat16* p, float f[8]) {
  bf16x8_to_float(*reinterpret_cast<const uint4*>(p), f);
}

template <typename T>
__device__ __forceinline__ void store4(T* p, float a, float b, float c, float d);
template <>
__device__ __forceinline__ void store4<float>(float* p, float a, float b, float c, float d) {
  *reinterpret_cast<float4*>(p) = make_float4(a, b, c, d);
}
template <>
__device__ __forceinline__ void store4<__nv_bfloat16>(__nv_bfloat16* p, float a, float b, float c,
                                                      float d) {
  __nv_bfloat162 x = __floats2bfloat162_rn(a, b);
  __nv_bfloat162 y = __floats2bfloat162_rn(c, d);
  uint2 u;
  u.x = *reinterpret_cast<uint32_t*>(&x);
  u.y = *reinterpret_cast<uint32_t*>(&y);
  *reinterpret_cast<uint2*>(p) = u;
}

// ----------------------------------------------------------------------------------
// KV reader: 8 consecutive channels [8*c8, 8*c8+8) of slot j of (b, h), dequantized.
// Packed codes are rounded to the tail dtype (bf16 in every shipped configuration), as
// the reference dequantizes the cache to its compute dtype before attending.
// ----------------------------------------------------------------------------------
// Storage coordinates of position j of sequence b's paged part: (page, position) with a
// page table, else (b, j). The page is -1 when the table entry is out of range.
__device__ __forceinline__ void kv_page(const ma_kv& kv, int b, int j, int& sb, int& sj) {
  if (kv.pages == nullptr) {
    sb = b;
    sj = j;
    return;
  }
  const int pi = j / kv.page_size;
  const int p = kv.pages[(int64_t)b * kv.spg + pi];
  sb = (p >= 0 && p < kv.num_pages) ? p : -1;
  sj = j - pi * kv.page_size;
}
// Whether slot j of sequence b sits in the paged part of the layout.
__device__ __forceinline__ bool kv_paged(const ma_kv& kv, int j) {
  return kv.pages != nullptr && (kv.layout == MA_KV_DENSE || j < kv.nq);
}

// Slot j exists: inside the prefix, below lens[b], its page (if paged) in range.
__device__ __forceinline__ bool kv_exists(const ma_kv& kv, int b, int j) {
  if (j < 0 || (int64_t)j >= (int64_t)kv.nq + kv.nf) return false;
  if (kv.lens != nullptr && j >= kv.lens[b]) return false;
  if (kv_paged(kv, j)) {
    const int p = kv.pages[(int64_t)b * kv.spg + j / kv.page_size];
    if (p < 0 || p >= kv.num_pages) return false;
  }
  return true;
}

// Slot j exists (0 <= j < nq + nf, below lens[b]) and is live (mask, page table). Slots
// outside the prefix (a bad index in a caller's read set) read as dead, so no kernel
// ever addresses outside the cache.
__device__ __forceinline__ bool kv_live(const ma_kv& kv, int H, int b, int h, int j) {
  const int64_t n = (int64_t)kv.nq + kv.nf;
  if (j < 0 || j >= n) return false;
  if (kv.lens != nullptr && j >= kv.lens[b]) return false;
  if (kv_paged(kv, j)) {
    const int p = kv.pages[(int64_t)b * kv.spg + j / kv.page_size];
    if (p < 0 || p >= kv.num_pages) return false;
  }
  if (kv.mask == nullptr) return true;
  return kv.mask[((int64_t)b * H + h) * n + j] != 0;
}

__device__ __forceinline__ void dequant8_token(const uint8_t* payload, uint16_t scale_bits,
                                               uint16_t zero_bits, float f[8]) {
  // 4 bytes = 8 codes; element 2i is the low nibble of byte i (reference.py:41-45)
  const uint32_t w = *reinterpret_cast<const uint32_t*>(payload);
  const float s = half_bits_to_float(scale_bits);
  const float z = half_bits_to_float(zero_bits);
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    const uint32_t code = (w >> (4 * i)) & 0xFu;
    f[i] = fmaf((float)code, s, z);
  }
}

// Callers read live slots only (kv_live), so a paged slot's page is in range.
template <bool KEY>
__device__ __forceinline__ void kv_read8(const ma_kv& kv, int b, int h, int j, int c8, float f[8]) {
  const int d0 = 8 * c8;
  const int seq = b;                               // the divisor k_chan is per sequence
  if (kv_paged(kv, j)) kv_page(kv, seq, j, b, j);  // from here on (b, j) address the storage
  if (j >= kv.nq) {  // dense slot (the whole prefix for MA_KV_DENSE, else the tail)
    const int jt = j - kv.nq;
    const int64_t* s = KEY ? kv.skf : kv.svf;
    const int64_t off = (int64_t)b * s[0] + (int64_t)h * s[1] + (int64_t)jt * s[2] + d0;
    if (kv.dtype == MA_BF16) {
      load8(reinterpret_cast<const __nv_bfloat16*>(KEY ? kv.kf : kv.vf) + off, f);
    } else {
      load8(reinterpret_cast<const float*>(KEY ? kv.kf : kv.vf) + off, f);
    }
    return;
  }
  const bool round_bf16 = kv.dtype == MA_BF16;
  if (!KEY || kv.layout == MA_KV_PACKED_TOKEN) {
    const uint8_t* q = KEY ? kv.kq : kv.vq;
    const uint16_t* sc = KEY ? kv.ks : kv.vs;
    const uint16_t* zp = KEY ? kv.kz : kv.vz;
    const int64_t* sq = KEY ? kv.skq : kv.svq;
    const int64_t* ss = KEY ? kv.sks : kv.svs;
    const int g = d0 / kv.vgroup;
    const int64_t qo = (int64_t)b * sq[0] + (int64_t)h * sq[1] + (int64_t)j * sq[2] + d0 / 2;
    const int64_t so = (int64_t)b * ss[0] + (int64_t)h * ss[1] + (int64_t)j * ss[2] + g;
    dequant8_token(q + qo, sc[so], zp[so], f);
    if (KEY) {
      const float* kc = kv.kchan + (int64_t)seq * kv.skc[0] + (int64_t)h * kv.skc[1] + d0;
#pragma unroll
      for (int i = 0; i < 8; ++i) f[i] *= kc[i];
    }
  } else {  // KIVI channel-mode keys: one scale/zero per (token group, channel)
    const int gi = j / kv.kgroup;
    const int ti = j - gi * kv.kgroup;
    const int bytes_per_ch = kv.kgroup / 2;
    const uint8_t* base = kv.kq + (int64_t)b * kv.skq[0] + (int64_t)h * kv.skq[1] +
                          (int64_t)gi * kv.skq[2];
    const int64_t so = (int64_t)b * kv.sks[0] + (int64_t)h * kv.sks[1] + (int64_t)gi * kv.sks[2];
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const int d = d0 + i;
      const uint32_t byte = base[(int64_t)d * bytes_per_ch + ti / 2];
      const uint32_t code = (ti & 1) ? (byte >> 4) : (byte & 0xFu);
      f[i] = fmaf((float)code, half_bits_to_float(kv.ks[so + d]), half_bits_to_float(kv.kz[so + d]));
    }
  }
  if (round_bf16) {
#pragma unroll
    for (int i = 0; i < 8; ++i) f[i] = bf16_round(f[i]);
  }
}

// ----------------------------------------------------------------------------------
// Split-K partial results: per (b*H + h, split, row) the pair (m, l) -- the split's
// row max and its softmax sum under that max -- and the split's normalized output
// o = acc / l over D channels (0 for a row without a visible key). The CUDA-core kernel
// writes o in fp32, the tensor-core kernel in bf16 (the combine weights each split by
// l * exp(m - M), so normalized outputs lose nothing to the split's scale).
// ----------------------------------------------------------------------------------
// The fused head gather of a KV-head-sharded attention call: the merge stores every final
// row (t < Tg) of this rank's query heads into slot `calls & 1` of every rank's receive
// region ([slot 0: B Hq Tg D bf16][slot 1][counters: world u32], Hq = world * Hl; mapped
// here through CUDA IPC), then the launch's CTAs arrive on every rank's counter of this
// rank and wait for every rank's CTAs before copying the slot into `out` [B, Hq, Tg, D].
struct PeerOut {
  char* base[8];        // every rank's region as mapped here (this rank's own is local)
  uint32_t* ws;         // [0] error, [1] CTA arrivals, [2] calls done, [3] copy arrivals,
                        // [4] CTAs of every rank's calls so far (per rank)
  int64_t slot_bytes;
  void* out;            // the gathered rows [B, Hq, Tg, D] bf16, strides so
  int64_t so[3];
  int world, rank, Hl, Tg;
};
constexpr int kPeerMaxWorld = 8;

struct Partials {
  float2* ml;   // [BH][S][Rp]
  void* o;      // [BH][S][Rp][D], fp32 or bf16 (o_bf16)
  int o_bf16;   // 1: o holds bf16
  int S;        // splits (the current block, when present, is the last one)
  int Rp;       // padded rows
};

__host__ __device__ inline size_t partials_bytes(int BH, int S, int Rp, int D, bool o_bf16) {
  return (size_t)BH * S * Rp * (sizeof(float2) + (o_bf16 ? 2 : 4) * (size_t)D);
}

// ----------------------------------------------------------------------------------
// Warp / block helpers
// ----------------------------------------------------------------------------------
// ------------------------------------------------------------- thread-block clusters
// Rank within the cluster, the cluster-wide barrier (release / acquire), and distributed
// shared memory: the address of a shared variable in CTA `rank` of the cluster, and
// 32-bit atomics, loads and stores through it.
__device__ __forceinline__ uint32_t cluster_rank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;\n" : "=r"(r));
  return r;
}
__device__ __forceinline__ void cluster_sync() {
  asm volatile("barrier.cluster.arrive.release.aligned;\nbarrier.cluster.wait.acquire.aligned;\n" ::: "memory");
}
// the two halves of the cluster barrier, for work between the arrival and the wait (every
// thread of every CTA in the cluster arrives once per phase, warp-converged)
__device__ __forceinline__ void cluster_arrive_relaxed() {
  asm volatile("barrier.cluster.arrive.relaxed.aligned;\n" ::: "memory");
}
__device__ __forceinline__ void cluster_wait() {
  asm volatile("barrier.cluster.wait.acquire.aligned;\n" ::: "memory");
}
// A bulk copy (the copy engine; `bytes` a multiple of 16, both addresses 16-byte aligned)
// from this CTA's shared memory into another CTA's, counted on that CTA's mbarrier
// (complete_tx): the receiver learns that the data is there by waiting on its own barrier.
// dst and mbar are shared::cluster addresses of the same CTA (peer_addr), src a
// shared::cta address of this one, whose bytes must stay unchanged until the copy is done.
__device__ __forceinline__ void bulk_copy_to_peer(uint32_t dst, uint32_t src, uint32_t bytes, uint32_t mbar) {
  asm volatile("cp.async.bulk.shared::cluster.shared::cta.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];\n"
               ::"r"(dst), "r"(src), "r"(bytes), "r"(mbar) : "memory");
}
// address of this shared variable in CTA `rank` of the cluster
__device__ __forceinline__ uint32_t peer_addr(const void* p, uint32_t rank) {
  uint32_t a;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;\n" : "=r"(a) : "r"(static_cast<uint32_t>(__cvta_generic_to_shared(p))), "r"(rank));
  return a;
}
__device__ __forceinline__ void peer_add(uint32_t addr, uint32_t v) {
  asm volatile("red.shared::cluster.add.u32 [%0], %1;\n" ::"r"(addr), "r"(v) : "memory");
}
__device__ __forceinline__ uint32_t peer_ld(uint32_t addr) {
  uint32_t v;
  asm volatile("ld.shared::cluster.u32 %0, [%1];\n" : "=r"(v) : "r"(addr) : "memory");
  return v;
}
__device__ __forceinline__ void peer_st(uint32_t addr, uint32_t v) {
  asm volatile("st.shared::cluster.u32 [%0], %1;\n" ::"r"(addr), "r"(v) : "memory");
}

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}
__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}

// Programmatic dependent launch: a kernel launched by launch_pdl may start while the
// kernel before it in the stream is still finishing (its prologue overlaps that tail); it
// executes pdl_wait() -- griddepcontrol.wait, which returns once every prerequisite grid
// has completed and its memory is visible -- before it touches anything an earlier
// kernel writes or reads, and before it ends.
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;\n" ::: "memory"); }
// Lets the next kernel in the stream, if launched by launch_pdl, start its CTAs (on SMs this
// grid leaves free) once every CTA of this grid has executed it or exited; the dependent
// still waits in pdl_wait() for this grid to complete before it touches its data.
__device__ __forceinline__ void pdl_launch_dependents() {
  asm volatile("griddepcontrol.launch_dependents;\n" ::: "memory");
}

template <typename... KArgs, typename... Args>
inline cudaError_t launch_pdl(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t st,
                              Args&&... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, kernel, std::forward<Args>(args)...);
}

// gpu-scope acquire load (a flag another CTA publishes with a fence + atomic)
__device__ __forceinline__ unsigned ld_acquire_u32(const unsigned* p) {
  unsigned v;
  asm volatile("ld.acquire.gpu.global.u32 %0, [%1];\n" : "=r"(v) : "l"(p) : "memory");
  return v;
}

// fp32 -> uint32 with the same order (-inf < ... < +inf); dead slots use key 0.
__device__ __forceinline__ uint32_t order_key(float x) {
  uint32_t u = __float_as_uint(x);
  return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}

}  // namespace ma
