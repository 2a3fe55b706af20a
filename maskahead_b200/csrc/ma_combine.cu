// Merge of the split-K partials: prefix splits first (giving the prefix-only softmax
// statistics M_p, L_p and O_p that the mass pass needs), then the current block.
// Follows the reference's combine (src/maskahead/kernels/splitk.py:271-318), with the
// row order r = g*T + t of every KV head.
#include <type_traits>

#include "ma_combine.cuh"
#include "ma_kernels.cuh"

namespace ma {

namespace {

constexpr int kWarps = 8;       // one warp per row

template <typename QT, typename OT>
__global__ void __launch_bounds__(kWarps * 32)
attn_combine_kernel(ma_rows q, int H, Partials P, int nsplit, int has_cur, QT* __restrict__ out,
                    int64_t so0, int64_t so1, int64_t so2, float* __restrict__ m_p,
                    float* __restrict__ l_p, float* __restrict__ o_p) {
  __shared__ float sW[kWarps][kCombineMaxSplits];
  pdl_wait();   // the partials of the attention kernel before
  const int G = q.Hq / H;
  const int R = G * q.T;
  const int warp = threadIdx.x >> 5;
  const int r = blockIdx.x * kWarps + warp;
  if (r >= R) return;
  combine_row<QT, OT>(q, H, P, nsplit, has_cur != 0, out, so0, so1, so2, m_p, l_p, o_p, blockIdx.y, r, sW[warp]);
}

// bf16 partials of D = 128 with at most NS prefix splits: a half warp per row (every
// split's row in flight at once), two rows per warp
template <typename QT, int NS>
__global__ void __launch_bounds__(kWarps * 32)
attn_combine16_kernel(ma_rows q, int H, Partials P, int nsplit, int has_cur, QT* __restrict__ out,
                      int64_t so0, int64_t so1, int64_t so2, float* __restrict__ m_p,
                      float* __restrict__ l_p, float* __restrict__ o_p) {
  pdl_wait();   // the partials of the attention kernel before
  const int R = (q.Hq / H) * q.T;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int r0 = (blockIdx.x * kWarps + warp) * 2;
  if (r0 >= R) return;   // warp-uniform
  const int r = r0 + (lane >> 4);
  combine_row16<QT, NS>(q, H, P, nsplit, has_cur != 0, out, so0, so1, so2, m_p, l_p, o_p, blockIdx.y,
                        r < R ? r : r0, r < R);
}

}  // namespace

int launch_attn_combine(const ma_rows& q, int H, const Partials& P, int nsplit, bool has_cur,
                        void* out, const int64_t so[3], float* m_p, float* l_p, float* o_p,
                        cudaStream_t st) {
  const int G = q.Hq / H;
  const int R = G * q.T;
  if (P.o_bf16 && q.D == 128 && nsplit <= 16) {   // half warps per row
    dim3 grid16((R + 2 * kWarps - 1) / (2 * kWarps), q.B * H);
    auto go16 = [&](auto qt, auto ns) {
      using QT = decltype(qt);
      launch_pdl(attn_combine16_kernel<QT, decltype(ns)::value>, grid16, dim3(kWarps * 32), 0, st, q, H, P, nsplit,
                 has_cur ? 1 : 0, reinterpret_cast<QT*>(out), so[0], so[1], so[2], m_p, l_p, o_p);
    };
    auto pick = [&](auto qt) {   // the unrolled width: the smallest power of two >= nsplit
      if (nsplit <= 2) go16(qt, std::integral_constant<int, 2>());
      else if (nsplit <= 4) go16(qt, std::integral_constant<int, 4>());
      else if (nsplit <= 8) go16(qt, std::integral_constant<int, 8>());
      else go16(qt, std::integral_constant<int, 16>());
    };
    if (q.dtype == MA_F32) pick(float());
    else pick(__nv_bfloat16());
    return cudaGetLastError() == cudaSuccess ? MA_OK : MA_ERR_CUDA;
  }
  dim3 grid((R + kWarps - 1) / kWarps, q.B * H);
  auto go = [&](auto qt, auto ot) {
    using QT = decltype(qt);
    using OT = decltype(ot);
    launch_pdl(attn_combine_kernel<QT, OT>, grid, dim3(kWarps * 32), 0, st, q, H, P, nsplit, has_cur ? 1 : 0,
               reinterpret_cast<QT*>(out), so[0], so[1], so[2], m_p, l_p, o_p);
  };
  if (q.dtype == MA_F32) {
    if (P.o_bf16) go(float(), __nv_bfloat16());
    else go(float(), float());
  } else {
    if (P.o_bf16) go(__nv_bfloat16(), __nv_bfloat16());
    else go(__nv_bfloat16(), float());
  }
  return cudaGetLastError() == cudaSuccess ? MA_OK : MA_ERR_CUDA;
}

}  // namespace ma
