// One row of the split-K merge: prefix splits first (giving the prefix-only softmax
// statistics M_p, L_p and O_p that the mass pass needs), then the current block.
// Follows the reference's combine (src/maskahead/kernels/splitk.py:271-318), with the
// row order r = g*T + t of every KV head. Used by the combine kernel and by the
// attention kernel's fused (cooperative) merge.
#pragma once

#include "ma_common.cuh"

namespace ma {

constexpr int kCombineMaxSplits = 256;   // partial slots per row (the planner never exceeds this)
constexpr int kCombineChunk = 16;

// The fused head gather's peer stores of one finished row's channels [d0, d0 + N) (bf16):
// row (b, query head hq of this rank, t) goes to slot `slot` of every rank's region, as
// global query head rank * Hl + hq (plain 8- or 16-byte stores over NVLink).
template <int N>
__device__ __forceinline__ void peer_store_row(const PeerOut* po, uint32_t slot, int b, int hq, int t, int d0,
                                               const float* v) {
  if (po == nullptr || t >= po->Tg) return;
  const int Hq = po->Hl * po->world;
  const int64_t off = (int64_t)slot * po->slot_bytes +
                      ((((int64_t)b * Hq + (int64_t)po->rank * po->Hl + hq) * po->Tg + t) * 128 + d0) * 2;
  uint32_t w[N / 2];
#pragma unroll
  for (int i = 0; i < N / 2; ++i) {
    __nv_bfloat162 x = __floats2bfloat162_rn(v[2 * i], v[2 * i + 1]);
    w[i] = *reinterpret_cast<uint32_t*>(&x);
  }
  for (int p = 0; p < po->world; ++p) {
    if constexpr (N == 8) *reinterpret_cast<uint4*>(po->base[p] + off) = make_uint4(w[0], w[1], w[2], w[3]);
    else *reinterpret_cast<uint2*>(po->base[p] + off) = make_uint2(w[0], w[1]);
  }
}

// Four channels of a partial row, fp32 or bf16.
__device__ __forceinline__ float4 load_o4(const float* p) { return __ldcg(reinterpret_cast<const float4*>(p)); }
__device__ __forceinline__ float4 load_o4(const __nv_bfloat16* p) {
  const uint2 u = __ldcg(reinterpret_cast<const uint2*>(p));
  const float2 a = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&u.x));
  const float2 b = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&u.y));
  return make_float4(a.x, a.y, b.x, b.y);
}

// One warp merges row r of KV head bh. The first kCombineChunk splits' partial outputs
// are requested before the (m, l) pairs are reduced, so the two global round trips
// overlap; lanes hold the pairs of splits lane, lane+32, ... in registers, form the
// weights w_s = l_s * exp(m_s - M) once (into sWw, this warp's kCombineMaxSplits floats),
// and every lane accumulates its 4 channels over the splits.
template <typename QT, typename OT>
__device__ __forceinline__ void combine_row(const ma_rows& q, int H, const Partials& P, int nsplit, bool has_cur,
                                            QT* __restrict__ out, int64_t so0, int64_t so1, int64_t so2,
                                            float* __restrict__ m_p, float* __restrict__ l_p, float* __restrict__ o_p,
                                            int bh, int r, float* __restrict__ sWw, const PeerOut* po = nullptr,
                                            uint32_t slot = 0) {
  const int D = q.D;
  const int G = q.Hq / H;
  const int R = G * q.T;
  const int lane = threadIdx.x & 31;
  const int d0 = 4 * lane;
  const bool active = d0 < D;
  const int64_t row0 = (int64_t)bh * P.S * P.Rp + r;   // partial row of split 0; split s adds s*Rp
  const OT* o = reinterpret_cast<const OT*>(P.o);
  const OT* base = o + row0 * D + d0;
  const int64_t step = (int64_t)P.Rp * D;

  // the first chunk of partial outputs and the current block's row, in flight early
  float4 buf[kCombineChunk];
#pragma unroll
  for (int i = 0; i < kCombineChunk; ++i)
    buf[i] = (active && i < nsplit) ? load_o4(base + i * step) : make_float4(0.f, 0.f, 0.f, 0.f);
  const int64_t crow = row0 + (int64_t)nsplit * P.Rp;
  float2 mlc = make_float2(-INFINITY, 0.f);
  float4 oc = make_float4(0.f, 0.f, 0.f, 0.f);
  if (has_cur) {
    mlc = __ldcg(&P.ml[crow]);
    if (active) oc = load_o4(o + crow * D + d0);
  }
  // prefix splits: (m, l) pairs in registers, global max, weights, sum
  float2 ml[kCombineMaxSplits / 32];
#pragma unroll
  for (int i = 0; i < kCombineMaxSplits / 32; ++i) {
    const int sidx = lane + 32 * i;
    ml[i] = sidx < nsplit ? __ldcg(&P.ml[row0 + (int64_t)sidx * P.Rp]) : make_float2(-INFINITY, 0.f);
  }
  float M = -INFINITY;
#pragma unroll
  for (int i = 0; i < kCombineMaxSplits / 32; ++i) M = fmaxf(M, ml[i].x);
  M = warp_max(M);
  const float Ms = (M == -INFINITY) ? 0.f : M;
  float L = 0.f;
#pragma unroll
  for (int i = 0; i < kCombineMaxSplits / 32; ++i) {
    const int sidx = lane + 32 * i;
    if (sidx < nsplit) {
      const float w = ml[i].y * expf(ml[i].x - Ms);
      sWw[sidx] = w;
      L += w;
    }
  }
  L = warp_sum(L);
  __syncwarp();
  float4 A = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
  for (int i = 0; i < kCombineChunk; ++i) {
    if (i < nsplit) {
      const float w = sWw[i];
      A.x = fmaf(buf[i].x, w, A.x);
      A.y = fmaf(buf[i].y, w, A.y);
      A.z = fmaf(buf[i].z, w, A.z);
      A.w = fmaf(buf[i].w, w, A.w);
    }
  }
  for (int s0 = kCombineChunk; s0 < nsplit; s0 += kCombineChunk) {
#pragma unroll
    for (int i = 0; i < kCombineChunk; ++i)
      buf[i] = (active && s0 + i < nsplit) ? load_o4(base + (s0 + i) * step) : make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
    for (int i = 0; i < kCombineChunk; ++i) {
      if (s0 + i < nsplit) {
        const float w = sWw[s0 + i];
        A.x = fmaf(buf[i].x, w, A.x);
        A.y = fmaf(buf[i].y, w, A.y);
        A.z = fmaf(buf[i].z, w, A.z);
        A.w = fmaf(buf[i].w, w, A.w);
      }
    }
  }
  const int64_t srow = (int64_t)bh * R + r;
  if (m_p != nullptr && lane == 0) {
    m_p[srow] = M;
    l_p[srow] = L;
  }
  if (o_p != nullptr && active) {
    const float inv = 1.f / (L > 0.f ? L : 1.f);
    *reinterpret_cast<float4*>(o_p + srow * D + d0) = make_float4(A.x * inv, A.y * inv, A.z * inv, A.w * inv);
  }
  if (has_cur) {
    const float mn = fmaxf(M, mlc.x);
    const float ms = (mn == -INFINITY) ? 0.f : mn;
    const float ea = expf(M - ms), eb = mlc.y * expf(mlc.x - ms);
    L = L * ea + eb;
    A.x = A.x * ea + oc.x * eb;
    A.y = A.y * ea + oc.y * eb;
    A.z = A.z * ea + oc.z * eb;
    A.w = A.w * ea + oc.w * eb;
  }
  if (active) {
    const float inv = 1.f / (L > 0.f ? L : 1.f);
    const int b = bh / H, h = bh - (bh / H) * H;
    const int g = r / q.T, t = r - (r / q.T) * q.T;
    QT* dst = out + (int64_t)b * so0 + (int64_t)(h * G + g) * so1 + (int64_t)t * so2 + d0;
    store4(dst, A.x * inv, A.y * inv, A.z * inv, A.w * inv);
    const float v[4] = {A.x * inv, A.y * inv, A.z * inv, A.w * inv};
    peer_store_row<4>(po, slot, b, h * G + g, t, d0, v);
  }
}

// A half warp (16 lanes) merges row r when there are at most 16 prefix splits, for bf16
// partials of D = 128: lane l of the half holds channels 8l..8l+7, so a warp merges two
// rows at once (row r of the upper half ignored when !valid). The arithmetic is
// combine_row's: w_s = l_s exp(m_s - M), prefix statistics, then the current block. Every
// lane loads all splits' rows and (m, l) pairs at once (or, for a source with kLaneMl,
// lane i the pair of split i, shared by shuffles; every lane of the warp must then call)
// and derives the weights itself: the merge is one round trip to wherever the partials are,
// with no reduction chain after it. src.o(s) gives this lane's 8 channels of split s's row
// (bf16), src.ml(s) its (m, l); split nsplit is the current block. NS (nsplit <= NS <= 16)
// bounds the unrolled loops: a launch that merges few splits keeps few registers.
template <typename QT, typename Src, int NS = 16>
__device__ __forceinline__ void combine_row16_from(const ma_rows& q, int H, int nsplit, bool has_cur,
                                                   QT* __restrict__ out, int64_t so0, int64_t so1, int64_t so2,
                                                   float* __restrict__ m_p, float* __restrict__ l_p,
                                                   float* __restrict__ o_p, int bh, int r, bool valid, const Src& src,
                                                   const PeerOut* po = nullptr, uint32_t slot = 0) {
  constexpr int D = 128;
  const int G = q.Hq / H;
  const int R = G * q.T;
  const int l16 = threadIdx.x & 15;
  const int d0 = 8 * l16;
  static_assert(NS >= 1 && NS <= 16, "at most 16 prefix splits");
  uint4 buf[NS];
  float2 ml[NS];
#pragma unroll
  for (int i = 0; i < NS; ++i) buf[i] = (valid && i < nsplit) ? src.o(i) : make_uint4(0u, 0u, 0u, 0u);
  if constexpr (Src::kLaneMl) {   // lane i loads split i's pair, the half warp shares them
    const float2 mine = (valid && l16 < nsplit) ? src.ml(l16) : make_float2(-INFINITY, 0.f);
    const int half = threadIdx.x & 16;
#pragma unroll
    for (int i = 0; i < NS; ++i)
      ml[i] = make_float2(__shfl_sync(0xffffffffu, mine.x, half | i), __shfl_sync(0xffffffffu, mine.y, half | i));
  } else {
#pragma unroll
    for (int i = 0; i < NS; ++i) ml[i] = (valid && i < nsplit) ? src.ml(i) : make_float2(-INFINITY, 0.f);
  }
  float2 mlc = make_float2(-INFINITY, 0.f);
  uint4 oc = make_uint4(0u, 0u, 0u, 0u);
  if (valid && has_cur) {
    mlc = src.ml(nsplit);
    oc = src.o(nsplit);
  }
  float M = -INFINITY;
#pragma unroll
  for (int i = 0; i < NS; ++i) M = fmaxf(M, ml[i].x);
  const float Ms = (M == -INFINITY) ? 0.f : M;
  float L = 0.f;
  float A[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
#pragma unroll
  for (int i = 0; i < NS; ++i) {
    if (i < nsplit) {
      const float wi = ml[i].y * expf(ml[i].x - Ms);
      L += wi;
      float f[8];
      bf16x8_to_float(buf[i], f);
#pragma unroll
      for (int e = 0; e < 8; ++e) A[e] = fmaf(f[e], wi, A[e]);
    }
  }
  if (!valid) return;
  const int64_t srow = (int64_t)bh * R + r;
  if (m_p != nullptr && l16 == 0) {
    m_p[srow] = M;
    l_p[srow] = L;
  }
  if (o_p != nullptr) {
    const float inv = 1.f / (L > 0.f ? L : 1.f);
    float4* dp = reinterpret_cast<float4*>(o_p + srow * D + d0);
    dp[0] = make_float4(A[0] * inv, A[1] * inv, A[2] * inv, A[3] * inv);
    dp[1] = make_float4(A[4] * inv, A[5] * inv, A[6] * inv, A[7] * inv);
  }
  if (has_cur) {
    const float mn = fmaxf(M, mlc.x);
    const float ms = (mn == -INFINITY) ? 0.f : mn;
    const float ea = expf(M - ms), eb = mlc.y * expf(mlc.x - ms);
    L = L * ea + eb;
    float f[8];
    bf16x8_to_float(oc, f);
#pragma unroll
    for (int e = 0; e < 8; ++e) A[e] = A[e] * ea + f[e] * eb;
  }
  const float inv = 1.f / (L > 0.f ? L : 1.f);
  const int b = bh / H, h = bh - (bh / H) * H;
  const int g = r / q.T, t = r - (r / q.T) * q.T;
  QT* dst = out + (int64_t)b * so0 + (int64_t)(h * G + g) * so1 + (int64_t)t * so2 + d0;
  store4(dst, A[0] * inv, A[1] * inv, A[2] * inv, A[3] * inv);
  store4(dst + 4, A[4] * inv, A[5] * inv, A[6] * inv, A[7] * inv);
  const float v[8] = {A[0] * inv, A[1] * inv, A[2] * inv, A[3] * inv, A[4] * inv, A[5] * inv, A[6] * inv, A[7] * inv};
  peer_store_row<8>(po, slot, b, h * G + g, t, d0, v);
}

// The partial rows of the global split buffers (bf16, split s of row r at row0 + s*Rp).
struct GlobalPartials {
  static constexpr bool kLaneMl = false;
  const __nv_bfloat16* po;
  const float2* pml;
  int64_t row0, step;
  int d0;
  __device__ __forceinline__ uint4 o(int s) const {
    return __ldcg(reinterpret_cast<const uint4*>(po + (row0 + (int64_t)s * step) * 128 + d0));
  }
  __device__ __forceinline__ float2 ml(int s) const { return __ldcg(&pml[row0 + (int64_t)s * step]); }
};

template <typename QT, int NS = 16>
__device__ __forceinline__ void combine_row16(const ma_rows& q, int H, const Partials& P, int nsplit, bool has_cur,
                                              QT* __restrict__ out, int64_t so0, int64_t so1, int64_t so2,
                                              float* __restrict__ m_p, float* __restrict__ l_p,
                                              float* __restrict__ o_p, int bh, int r, bool valid,
                                              const PeerOut* po = nullptr, uint32_t slot = 0) {
  GlobalPartials src;
  src.po = reinterpret_cast<const __nv_bfloat16*>(P.o);
  src.pml = P.ml;
  src.row0 = (int64_t)bh * P.S * P.Rp + r;
  src.step = P.Rp;
  src.d0 = 8 * (threadIdx.x & 15);
  combine_row16_from<QT, GlobalPartials, NS>(q, H, nsplit, has_cur, out, so0, so1, so2, m_p, l_p, o_p, bh, r, valid,
                                              src, po, slot);
}

}  // namespace ma
