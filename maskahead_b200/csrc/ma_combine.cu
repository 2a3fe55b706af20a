// Merge of the split-K partials: prefix splits first (giving the prefix-only softmax
// statistics M_p, L_p and O_p that the mass pass needs), then the current block.
// Follows the reference's combine (src/maskahead/kernels/splitk.py:271-318), with the
// row order r = g*T + t of every KV head.
#include "ma_kernels.cuh"

namespace ma {

namespace {

constexpr int kWarps = 8;       // one warp per row
constexpr int kMaxSplits = 256;  // partial slots per row (the planner never exceeds this)

// One warp per row. Lanes read the per-split (m, l) in parallel, reduce the global max
// and the weights exp(m_s - M) once, then every lane accumulates its 4 channels over
// the splits with independent loads (no serial dependency through the running max).
template <typename QT>
__global__ void __launch_bounds__(kWarps * 32)
attn_combine_kernel(ma_rows q, int H, Partials P, int nsplit, int has_cur, QT* __restrict__ out,
                    int64_t so0, int64_t so1, int64_t so2, float* __restrict__ m_p,
                    float* __restrict__ l_p, float* __restrict__ o_p) {
  __shared__ float sW[kWarps][kMaxSplits];
  const int D = q.D;
  const int G = q.Hq / H;
  const int R = G * q.T;
  const int bh = blockIdx.y;
  const int warp = threadIdx.x >> 5;
  const int r = blockIdx.x * kWarps + warp;
  const int lane = threadIdx.x & 31;
  if (r >= R) return;
  const int d0 = 4 * lane;
  const bool active = d0 < D;
  const int64_t row0 = (int64_t)bh * P.S * P.Rp + r;   // partial row of split 0; split s adds s*Rp

  // prefix splits: global max, weights, sum
  float M = -INFINITY;
  for (int s = lane; s < nsplit; s += 32) M = fmaxf(M, __ldcg(&P.ml[row0 + (int64_t)s * P.Rp].x));
  M = warp_max(M);
  const float Ms = (M == -INFINITY) ? 0.f : M;
  float L = 0.f;
  for (int s = lane; s < nsplit; s += 32) {
    const float2 ml = __ldcg(&P.ml[row0 + (int64_t)s * P.Rp]);
    const float w = expf(ml.x - Ms);
    sW[warp][s] = w;
    L = fmaf(ml.y, w, L);
  }
  L = warp_sum(L);
  __syncwarp();
  float4 A = make_float4(0.f, 0.f, 0.f, 0.f);
  if (active) {
    const float* base = P.acc + row0 * D + d0;
    const int64_t step = (int64_t)P.Rp * D;
#pragma unroll 16
    for (int s = 0; s < nsplit; ++s) {
      const float w = sW[warp][s];
      const float4 a = __ldcg(reinterpret_cast<const float4*>(base + s * step));
      A.x = fmaf(a.x, w, A.x);
      A.y = fmaf(a.y, w, A.y);
      A.z = fmaf(a.z, w, A.z);
      A.w = fmaf(a.w, w, A.w);
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
    const int64_t crow = row0 + (int64_t)nsplit * P.Rp;
    const float2 ml = __ldcg(&P.ml[crow]);
    const float mn = fmaxf(M, ml.x);
    const float ms = (mn == -INFINITY) ? 0.f : mn;
    const float ea = expf(M - ms), eb = expf(ml.x - ms);
    L = L * ea + ml.y * eb;
    if (active) {
      const float4 a = __ldcg(reinterpret_cast<const float4*>(P.acc + crow * D + d0));
      A.x = A.x * ea + a.x * eb;
      A.y = A.y * ea + a.y * eb;
      A.z = A.z * ea + a.z * eb;
      A.w = A.w * ea + a.w * eb;
    }
  }
  if (active) {
    const float inv = 1.f / (L > 0.f ? L : 1.f);
    const int b = bh / H, h = bh - (bh / H) * H;
    const int g = r / q.T, t = r - (r / q.T) * q.T;
    QT* dst = out + (int64_t)b * so0 + (int64_t)(h * G + g) * so1 + (int64_t)t * so2 + d0;
    store4(dst, A.x * inv, A.y * inv, A.z * inv, A.w * inv);
  }
}

}  // namespace

int launch_attn_combine(const ma_rows& q, int H, const Partials& P, int nsplit, bool has_cur,
                        void* out, const int64_t so[3], float* m_p, float* l_p, float* o_p,
                        cudaStream_t st) {
  const int G = q.Hq / H;
  const int R = G * q.T;
  dim3 grid((R + kWarps - 1) / kWarps, q.B * H);
  if (q.dtype == MA_F32) {
    attn_combine_kernel<float><<<grid, kWarps * 32, 0, st>>>(
        q, H, P, nsplit, has_cur ? 1 : 0, reinterpret_cast<float*>(out), so[0], so[1], so[2], m_p, l_p, o_p);
  } else {
    attn_combine_kernel<__nv_bfloat16><<<grid, kWarps * 32, 0, st>>>(
        q, H, P, nsplit, has_cur ? 1 : 0, reinterpret_cast<__nv_bfloat16*>(out), so[0], so[1], so[2],
        m_p, l_p, o_p);
  }
  return cudaGetLastError() == cudaSuccess ? MA_OK : MA_ERR_CUDA;
}

}  // namespace ma
