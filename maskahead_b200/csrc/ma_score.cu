// Scoring kernels of step 0:
//   prefix mass   a_j = mean over the selection rows of exp(s_rj - M_p,r) / L_p,r
//                 (src/maskahead/kernels/splitk.py:320-359; reference.py:318-366)
//   value score   c = sum_j a_j v_j / max(sum_j a_j, 1e-12), score_j = a_j ||v_j - c||
//                 (src/maskahead/runtime/session.py:27-40 fp32 centre, 870-899)
// The mass kernel here runs on CUDA cores in fp32 for every cache type; it is exact
// to fp32 rounding, which the read-set selection needs.
#include "ma_kernels.cuh"

namespace ma {

namespace {

constexpr int kMassTok = 64;    // keys per CTA
constexpr int kMassRows = 16;   // query rows staged at a time
constexpr int kThreads = 256;

template <typename QT>
__global__ void __launch_bounds__(kThreads)
prefix_mass_simt(ma_rows q, ma_kv kv, int H, const int32_t* __restrict__ q_rows, int T2,
                 const float* __restrict__ m_p, const float* __restrict__ l_p, float scale,
                 float* __restrict__ mass, int64_t sm0, int64_t sm1) {
  const int D = q.D;
  const int n = kv.nq + kv.nf;
  const int bh = blockIdx.y;
  const int b = bh / H, h = bh - (bh / H) * H;
  const int G = q.Hq / H;
  const int R = G * q.T;
  const int R2 = G * T2;
  const int j0 = blockIdx.x * kMassTok;
  const int tid = threadIdx.x;

  __shared__ float sK[kMassTok][kMaxD + 1];
  __shared__ float sQ[kMassRows][kMaxD];
  __shared__ float sM[kMassRows], sL[kMassRows];
  __shared__ float sAcc[kThreads / kMassTok][kMassTok];
  __shared__ unsigned char sLive[kMassTok];

  const int chunks = D / 8;
  for (int c = tid; c < kMassTok * chunks; c += kThreads) {
    const int jj = c / chunks, c8 = c - (c / chunks) * chunks;
    const int j = j0 + jj;
    float f[8];
    const bool ok = j < n && kv_live(kv, H, b, h, j);
    if (ok) {
      kv_read8<true>(kv, b, h, j, c8, f);
    } else {
#pragma unroll
      for (int i = 0; i < 8; ++i) f[i] = 0.f;
    }
#pragma unroll
    for (int i = 0; i < 8; ++i) sK[jj][8 * c8 + i] = f[i];
    if (c8 == 0) sLive[jj] = ok ? 1 : 0;
  }

  const int jj = tid % kMassTok;
  const int rg = tid / kMassTok;                       // 4 row groups
  constexpr int kPerThread = kMassRows / (kThreads / kMassTok);
  const QT* qp = reinterpret_cast<const QT*>(q.q);
  float acc = 0.f;
  for (int rc = 0; rc < R2; rc += kMassRows) {
    __syncthreads();
    for (int c = tid; c < kMassRows * chunks; c += kThreads) {
      const int rr = c / chunks, c8 = c - (c / chunks) * chunks;
      const int r2 = rc + rr;
      float f[8];
      const int g = r2 / T2;
      const int t = r2 < R2 ? q_rows[r2 - g * T2] : -1;
      if (t >= 0 && t < q.T) {  // a row position outside the block is ignored
        load8(qp + (int64_t)b * q.sq[0] + (int64_t)(h * G + g) * q.sq[1] + (int64_t)t * q.sq[2] + 8 * c8, f);
        if (c8 == 0) {
          sM[rr] = m_p[(int64_t)bh * R + g * q.T + t];
          sL[rr] = l_p[(int64_t)bh * R + g * q.T + t];
        }
      } else {
#pragma unroll
        for (int i = 0; i < 8; ++i) f[i] = 0.f;
        if (c8 == 0) {
          sM[rr] = 0.f;
          sL[rr] = 0.f;
        }
      }
#pragma unroll
      for (int i = 0; i < 8; ++i) sQ[rr][8 * c8 + i] = f[i];
    }
    __syncthreads();
#pragma unroll
    for (int i = 0; i < kPerThread; ++i) {
      const int rr = rg * kPerThread + i;
      float s = 0.f;
      for (int d = 0; d < D; ++d) s = fmaf(sQ[rr][d], sK[jj][d], s);
      s *= scale;
      const float L = sL[rr];
      if (L > 0.f) acc += expf(s - sM[rr]) / L;
    }
  }
  sAcc[rg][jj] = acc;
  __syncthreads();
  if (tid < kMassTok) {
    const int j = j0 + tid;
    if (j < n) {
      float a = 0.f;
#pragma unroll
      for (int g = 0; g < kThreads / kMassTok; ++g) a += sAcc[g][tid];
      a = sLive[tid] ? a / (float)R2 : 0.f;
      mass[(int64_t)b * sm0 + (int64_t)h * sm1 + j] = a;
    }
  }
}

// ---------------------------------------------------------------- value-aware score
constexpr int kVTok = 64;  // keys per CTA

// Stage the values of keys [j0, j0+kVTok) into sV (fp32, dead or out-of-range rows are
// zero) with their weights a_j (0 when dead).
__device__ __forceinline__ void stage_values(const ma_kv& kv, int H, int D, int b, int h, int j0,
                                             int n, const float* a, int64_t sa0, int64_t sa1,
                                             float (*sV)[kMaxD], float* sA) {
  const int chunks = D / 8;
  for (int c = threadIdx.x; c < kVTok * chunks; c += blockDim.x) {
    const int jj = c / chunks, c8 = c - (c / chunks) * chunks;
    const int j = j0 + jj;
    float f[8];
    const bool ok = j < n && kv_live(kv, H, b, h, j);
    if (ok) {
      kv_read8<false>(kv, b, h, j, c8, f);
    } else {
#pragma unroll
      for (int i = 0; i < 8; ++i) f[i] = 0.f;
    }
#pragma unroll
    for (int i = 0; i < 8; ++i) sV[jj][8 * c8 + i] = f[i];
    if (c8 == 0) sA[jj] = ok ? a[(int64_t)b * sa0 + (int64_t)h * sa1 + j] : 0.f;
  }
}

__global__ void __launch_bounds__(kThreads)
value_centre_kernel(ma_kv kv, int H, int D, const float* __restrict__ a, int64_t sa0, int64_t sa1,
                    int ntile, float* __restrict__ part, uint2* __restrict__ sync,
                    float* __restrict__ centre) {
  const int n = kv.nq + kv.nf;
  const int bh = blockIdx.y;
  const int b = bh / H, h = bh - (bh / H) * H;
  const int tile = blockIdx.x;
  __shared__ float sV[kVTok][kMaxD];
  __shared__ float sA[kVTok];
  __shared__ float sRed[kThreads];
  __shared__ float sRedA[kThreads];
  __shared__ bool sLast;
  stage_values(kv, H, D, b, h, tile * kVTok, n, a, sa0, sa1, sV, sA);
  __syncthreads();
  const int ngrp = kThreads / D;              // 2 (D=128) or 4 (D=64)
  const int d = threadIdx.x % D;
  const int grp = threadIdx.x / D;
  const int per = kVTok / ngrp;
  float s = 0.f, sa = 0.f;
  for (int i = 0; i < per; ++i) {
    const int jj = grp * per + i;
    s = fmaf(sA[jj], sV[jj][d], s);
    sa += sA[jj];
  }
  sRed[threadIdx.x] = s;
  sRedA[threadIdx.x] = sa;
  __syncthreads();
  float* mine = part + ((int64_t)bh * ntile + tile) * (D + 1);
  if (threadIdx.x < D) {
    float tot = 0.f;
    for (int g = 0; g < ngrp; ++g) tot += sRed[g * D + threadIdx.x];
    mine[threadIdx.x] = tot;
  }
  if (threadIdx.x == 0) {
    float tot = 0.f;
    for (int g = 0; g < ngrp; ++g) tot += sRedA[g * D];
    mine[D] = tot;
  }
  // the last CTA of this (b, h) reduces the per-tile partials in tile order
  __threadfence();
  __syncthreads();
  if (threadIdx.x == 0) {
    const unsigned prev = atomicAdd(&sync[bh].x, 1u);
    sLast = prev == (unsigned)(ntile - 1);
  }
  __syncthreads();
  if (!sLast) return;
  __threadfence();
  const float* base = part + (int64_t)bh * ntile * (D + 1);
  if (threadIdx.x <= D) {
    float tot = 0.f;
    for (int t = 0; t < ntile; ++t) tot += __ldcg(base + (int64_t)t * (D + 1) + threadIdx.x);
    sRed[threadIdx.x] = tot;
  }
  __syncthreads();
  if (threadIdx.x < D) centre[(int64_t)bh * D + threadIdx.x] = sRed[threadIdx.x] / fmaxf(sRed[D], 1e-12f);
  if (threadIdx.x == 0) sync[bh].x = 0u;   // ready for the next call
}

// a_j * ||v_j - c||: one group of D/8 lanes (a half-warp for D = 128) per key, each lane
// holding 8 channels of the row (one 16-byte load of a bf16 row) and the same 8 channels
// of the centre in registers; every group takes kApplyKeys keys with all loads issued
// before the first reduction. Dead slots score 0.
constexpr int kApplyKeys = 4;
constexpr int kApplyTok = (kThreads / 16) * kApplyKeys;   // keys per CTA

__global__ void __launch_bounds__(kThreads)
value_apply_kernel(ma_kv kv, int H, int D, const float* __restrict__ a, int64_t sa0, int64_t sa1,
                   const float* __restrict__ centre, float* __restrict__ score, int64_t ss0,
                   int64_t ss1) {
  const int n = kv.nq + kv.nf;
  const int bh = blockIdx.y;
  const int b = bh / H, h = bh - (bh / H) * H;
  pdl_wait();   // the mass and centre of the kernels before
  const int grp = threadIdx.x >> 4, l16 = threadIdx.x & 15;
  const bool lane_on = l16 < D / 8;
  float cc[8];
#pragma unroll
  for (int i = 0; i < 8; ++i) cc[i] = lane_on ? __ldcg(centre + (int64_t)bh * D + 8 * l16 + i) : 0.f;
  float f[kApplyKeys][8];
  bool live[kApplyKeys];
#pragma unroll
  for (int u = 0; u < kApplyKeys; ++u) {
    const int j = blockIdx.x * kApplyTok + u * (kThreads / 16) + grp;
    live[u] = j < n && kv_live(kv, H, b, h, j);
    if (live[u] && lane_on) {
      kv_read8<false>(kv, b, h, j, l16, f[u]);
    } else {
#pragma unroll
      for (int i = 0; i < 8; ++i) f[u][i] = cc[i];
    }
  }
#pragma unroll
  for (int u = 0; u < kApplyKeys; ++u) {
    float s2 = 0.f;
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const float x = f[u][i] - cc[i];
      s2 = fmaf(x, x, s2);
    }
#pragma unroll
    for (int o = 8; o > 0; o >>= 1) s2 += __shfl_xor_sync(0xffffffffu, s2, o);
    const int j = blockIdx.x * kApplyTok + u * (kThreads / 16) + grp;
    if (l16 == 0 && j < n) {
      const float aj = live[u] ? a[(int64_t)b * sa0 + (int64_t)h * sa1 + j] : 0.f;
      score[(int64_t)b * ss0 + (int64_t)h * ss1 + j] = aj * sqrtf(s2);
    }
  }
}

}  // namespace

int launch_prefix_mass(const ma_rows& q, const ma_kv& kv, int H, const int32_t* q_rows, int T2,
                       const float* m_p, const float* l_p, float scale, float* mass,
                       int64_t sm0, int64_t sm1, cudaStream_t st) {
  const int n = kv.nq + kv.nf;
  if (n == 0) return MA_OK;
  dim3 grid((n + kMassTok - 1) / kMassTok, q.B * H);
  if (q.dtype == MA_F32) {
    prefix_mass_simt<float><<<grid, kThreads, 0, st>>>(q, kv, H, q_rows, T2, m_p, l_p, scale, mass, sm0, sm1);
  } else {
    prefix_mass_simt<__nv_bfloat16><<<grid, kThreads, 0, st>>>(q, kv, H, q_rows, T2, m_p, l_p, scale,
                                                                mass, sm0, sm1);
  }
  return cudaGetLastError() == cudaSuccess ? MA_OK : MA_ERR_CUDA;
}

// workspace: the error word and the per-head (counter, generation) pairs (one 256-byte
// aligned block), centre [BH][D], partials [BH][ntile][D+1]
// The error word and the per-head (arrival counter, centre generation) pairs: a block of
// fixed size at the front of the workspace, so a head's counter is the same word in every
// call. Calls with other head counts share the workspace (a mass call of a few heads, then
// a value score over every layer's heads); a block that grew with the head count would let
// one call's centres land on another's counters, which must read zero when a call starts.
constexpr size_t kValueSyncSlots = size_t(1) << 16;
size_t value_sync_bytes(int BH) {
  (void)BH;
  return ((8 + kValueSyncSlots * sizeof(uint2) + 255) / 256) * 256;
}
int value_sync_slots() { return (int)kValueSyncSlots; }

size_t value_score_ws_bytes(int B, int H, int n, int D) {
  const size_t BH = (size_t)B * H;
  const size_t ntile = (size_t)(n + kVTok - 1) / kVTok;
  const size_t cnt = value_sync_bytes((int)BH);
  const size_t cen = ((BH * D * sizeof(float) + 255) / 256) * 256;
  return cnt + cen + BH * (ntile > 0 ? ntile : 1) * (D + 1) * sizeof(float);
}

ValueWs carve_value_ws(void* ws, int BH, int D) {
  ValueWs w;
  char* p = reinterpret_cast<char*>(ws);
  w.err = reinterpret_cast<int*>(p);
  w.sync = reinterpret_cast<uint2*>(p + 8);
  p += value_sync_bytes(BH);
  w.centre = reinterpret_cast<float*>(p);
  p += (((size_t)BH * D * sizeof(float) + 255) / 256) * 256;
  w.part = reinterpret_cast<float*>(p);
  return w;
}

int launch_value_apply(const ma_kv& kv, int B, int H, int D, const float* a, int64_t sa0, int64_t sa1,
                       const float* centre, float* score, int64_t ss0, int64_t ss1, cudaStream_t st) {
  const int n = kv.nq + kv.nf;
  if (n == 0) return MA_OK;
  dim3 grid((n + kApplyTok - 1) / kApplyTok, B * H);
  launch_pdl(value_apply_kernel, grid, dim3(kThreads), 0, st, kv, H, D, a, sa0, sa1, centre, score, ss0, ss1);
  return cudaGetLastError() == cudaSuccess ? MA_OK : MA_ERR_CUDA;
}

int launch_value_score(const ma_kv& kv, int B, int H, int D, const float* a, int64_t sa0,
                       int64_t sa1, float* score, int64_t ss0, int64_t ss1, void* ws,
                       cudaStream_t st) {
  const int n = kv.nq + kv.nf;
  if (n == 0) return MA_OK;
  const int ntile = (n + kVTok - 1) / kVTok;
  const ValueWs w = carve_value_ws(ws, B * H, D);
  dim3 grid(ntile, B * H);
  value_centre_kernel<<<grid, kThreads, 0, st>>>(kv, H, D, a, sa0, sa1, ntile, w.part, w.sync, w.centre);
  if (cudaGetLastError() != cudaSuccess) return MA_ERR_CUDA;
  return launch_value_apply(kv, B, H, D, a, sa0, sa1, w.centre, score, ss0, ss1, st);
}

}  // namespace ma
