// Prefix mass on the tensor cores, with the value-score centre fused in.
//
// For bf16 queries over a bf16 (or dequantized packed) prefix: every CTA owns a range
// of prefix slots of one KV head, stages all selection rows of that head once (up to
// 256 rows = the G query heads x the block's mask positions), and streams its slots in
// tiles of 64 through shared memory. S = Q K^T runs as m16n8k16 bf16 MMAs with fp32
// accumulation (bf16 products are exact in fp32, so S is fp32-accurate); then
//     a_j = (1 / R2) * sum_r exp(s_rj - M_p,r) / L_p,r          (splitk.py:320-359)
// as column sums: per thread over its rows, across lanes by shuffles, across warps in
// a fixed order (deterministic). With a centre requested the CTA also accumulates
// sum_j a_j v_j and sum_j a_j over its slots from the V tiles it streams, and the last
// CTA of the head reduces those partials in slot order into
//     c = sum_j a_j v_j / max(sum_j a_j, 1e-12)                  (session.py:27-40, 870-899)
// which the value-apply kernel turns into a_j * ||v_j - c||.
#include "ma_kernels.cuh"
#include "ma_mma.cuh"

namespace ma {

namespace {

constexpr int kWarps = 8;
constexpr int kThreads = kWarps * 32;
constexpr int kRows = 256;          // selection rows (R2 = G * T2 <= 256)
constexpr int kBN = 64;             // slots per tile
constexpr int kQBytes = kRows * kTileD * 2;
constexpr int kKBytes = kBN * kTileD * 2;
constexpr int kSmemBytes = kQBytes + 4 * kKBytes + (2 * kRows + kWarps * kBN + 2 * kBN) * 4 + 2 * kBN;

struct MassArgs {
  ma_rows q;
  ma_kv kv;
  const int32_t* q_rows;
  const float* m_p;
  const float* l_p;
  float* mass;
  int64_t sm0, sm1;
  float* part;          // [BH][ctas][D+1] centre partials (CENTRE only)
  unsigned* counters;   // [BH]
  float* centre;        // [BH][D]
  float scale;
  int H, T2, slots_per_cta;
};

// stage slots [j0, j0+kBN) of (b, h): keys swizzled (MMA operand), values plain (row-major)
template <bool PACKED, bool CENTRE>
__device__ __forceinline__ void load_slots(const MassArgs& A, int b, int h, int j0, int end, uint8_t* sK,
                                           uint8_t* sV, uint8_t* sOk) {
  const __nv_bfloat16* kf = reinterpret_cast<const __nv_bfloat16*>(A.kv.kf);
  const __nv_bfloat16* vf = reinterpret_cast<const __nv_bfloat16*>(A.kv.vf);
  for (int c = threadIdx.x; c < kBN * kRowChunks; c += kThreads) {
    const int jj = c / kRowChunks, ch = c % kRowChunks;
    const int j = j0 + jj;
    const bool ok = j < end && kv_live(A.kv, A.H, b, h, j);
    uint8_t* dk = sK + swz(jj, ch);
    uint8_t* dv = sV + jj * (kTileD * 2) + ch * 16;
    if (!ok) {
      *reinterpret_cast<uint4*>(dk) = make_uint4(0, 0, 0, 0);
      if (CENTRE) *reinterpret_cast<uint4*>(dv) = make_uint4(0, 0, 0, 0);
    } else if (!PACKED || j >= A.kv.nq) {
      const int row = j - A.kv.nq;
      cp_async16(smem_u32(dk), kf + (int64_t)b * A.kv.skf[0] + (int64_t)h * A.kv.skf[1] + (int64_t)row * A.kv.skf[2] + ch * 8, true);
      if (CENTRE)
        cp_async16(smem_u32(dv), vf + (int64_t)b * A.kv.svf[0] + (int64_t)h * A.kv.svf[1] + (int64_t)row * A.kv.svf[2] + ch * 8, true);
    } else {
      float f[8];
      kv_read8<true>(A.kv, b, h, j, ch, f);
      *reinterpret_cast<uint4*>(dk) = float8_to_bf16x8(f);
      if (CENTRE) {
        kv_read8<false>(A.kv, b, h, j, ch, f);
        *reinterpret_cast<uint4*>(dv) = float8_to_bf16x8(f);
      }
    }
    if (ch == 0) sOk[jj] = ok ? 1 : 0;
  }
  cp_async_commit();
}

template <bool PACKED, bool CENTRE>
__global__ void __launch_bounds__(kThreads, 1) prefix_mass_mma(const MassArgs A) {
  extern __shared__ __align__(128) uint8_t smem[];
  uint8_t* sQ = smem;
  uint8_t* sKb[2] = {smem + kQBytes, smem + kQBytes + kKBytes};
  uint8_t* sVb[2] = {smem + kQBytes + 2 * kKBytes, smem + kQBytes + 3 * kKBytes};
  float* sM = reinterpret_cast<float*>(smem + kQBytes + 4 * kKBytes);
  float* sL = sM + kRows;
  float* sCol = sL + kRows;               // [kWarps][kBN]
  float* sMass = sCol + kWarps * kBN;     // [kBN]
  float* sRed = sMass + kBN;              // [kBN] scratch for the centre reduction
  uint8_t* sOkb[2] = {reinterpret_cast<uint8_t*>(sRed + kBN), reinterpret_cast<uint8_t*>(sRed + kBN) + kBN};

  const int n = A.kv.nq + A.kv.nf;
  const int bh = blockIdx.y;
  const int H = A.H;
  const int b = bh / H, h = bh - (bh / H) * H;
  const int G = A.q.Hq / H;
  const int T = A.q.T;
  const int R2 = G * A.T2;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int begin = blockIdx.x * A.slots_per_cta;
  const int end = min(n, begin + A.slots_per_cta);
  const float inv_rows = 1.f / (float)R2;

  float cacc = 0.f, asum = 0.f;           // centre partial of channel (tid % 128)
  const int cd = threadIdx.x & (kTileD - 1), chalf = threadIdx.x >> 7;
  const int rp = 0;                       // R2 <= kRows: one pass over the rows
  {
    // selection rows: r2 = g*T2 + i -> query row (h*G + g, q_rows[i])
    {
      const __nv_bfloat16* qp = reinterpret_cast<const __nv_bfloat16*>(A.q.q);
      for (int c = threadIdx.x; c < kRows * kRowChunks; c += kThreads) {
        const int rr = c / kRowChunks, ch = c % kRowChunks;
        const int r2 = rp + rr;
        const int g = r2 / A.T2;
        const int t = r2 < R2 ? A.q_rows[r2 - g * A.T2] : -1;
        const bool ok = t >= 0 && t < T;
        const __nv_bfloat16* src = ok ? qp + (int64_t)b * A.q.sq[0] + (int64_t)(h * G + g) * A.q.sq[1] +
                                            (int64_t)t * A.q.sq[2] + ch * 8
                                      : qp;
        cp_async16(smem_u32(sQ + swz(rr, ch)), src, ok);
        if (ch == 0) {
          const int64_t ri = (int64_t)bh * G * T + (int64_t)g * T + t;
          const float L = ok ? A.l_p[ri] : 0.f;
          sM[rr] = ok ? A.m_p[ri] : 0.f;
          sL[rr] = L > 0.f ? L : 0.f;   // the divisor; 0 marks a row that contributes nothing
        }
      }
    }
    if (begin < end) load_slots<PACKED, CENTRE>(A, b, h, begin, end, sKb[0], sVb[0], sOkb[0]);
    else cp_async_commit();

    const int wrow = warp * 32;
    int stage = 0;
    for (int j0 = begin; j0 < end; j0 += kBN) {
      cp_async_wait_all();
      __syncthreads();
      if (j0 + kBN < end) load_slots<PACKED, CENTRE>(A, b, h, j0 + kBN, end, sKb[stage ^ 1], sVb[stage ^ 1], sOkb[stage ^ 1]);
      const uint8_t* sK = sKb[stage];
      const uint8_t* sOk = sOkb[stage];
      float col[8][2];
#pragma unroll
      for (int nt = 0; nt < 8; ++nt) col[nt][0] = col[nt][1] = 0.f;
      if (rp + wrow < R2) {
        float s[2][8][4];
#pragma unroll
        for (int mt = 0; mt < 2; ++mt)
#pragma unroll
          for (int nt = 0; nt < 8; ++nt)
#pragma unroll
            for (int e = 0; e < 4; ++e) s[mt][nt][e] = 0.f;
#pragma unroll
        for (int kk = 0; kk < kTileD / 16; ++kk) {
          uint32_t a[2][4];
#pragma unroll
          for (int mt = 0; mt < 2; ++mt)
            ldsm_x4(smem_u32(sQ + swz(wrow + mt * 16 + (lane & 15), kk * 2 + (lane >> 4))), a[mt][0], a[mt][1],
                    a[mt][2], a[mt][3]);
#pragma unroll
          for (int np = 0; np < 4; ++np) {
            uint32_t b0, b1, b2, b3;
            const int key = np * 16 + (lane & 7) + ((lane >> 4) << 3);
            ldsm_x4(smem_u32(sK + swz(key, kk * 2 + ((lane >> 3) & 1))), b0, b1, b2, b3);
#pragma unroll
            for (int mt = 0; mt < 2; ++mt) {
              mma_bf16(s[mt][2 * np], a[mt], b0, b1);
              mma_bf16(s[mt][2 * np + 1], a[mt], b2, b3);
            }
          }
        }
#pragma unroll
        for (int mt = 0; mt < 2; ++mt)
#pragma unroll
          for (int hf = 0; hf < 2; ++hf) {
            const int rr = wrow + mt * 16 + hf * 8 + (lane >> 2);
            const float L = sL[rr];
            if (L > 0.f) {
              const float M = sM[rr];
#pragma unroll
              for (int nt = 0; nt < 8; ++nt)
#pragma unroll
                for (int e = 0; e < 2; ++e) col[nt][e] += expf(s[mt][nt][hf * 2 + e] * A.scale - M) / L;
            }
          }
      }
      // lanes sharing (lane & 3) hold the same columns
#pragma unroll
      for (int nt = 0; nt < 8; ++nt)
#pragma unroll
        for (int e = 0; e < 2; ++e) {
          float v = col[nt][e];
          v += __shfl_xor_sync(0xffffffffu, v, 4);
          v += __shfl_xor_sync(0xffffffffu, v, 8);
          v += __shfl_xor_sync(0xffffffffu, v, 16);
          col[nt][e] = v;
        }
      if (lane < 4) {
#pragma unroll
        for (int nt = 0; nt < 8; ++nt) {
          sCol[warp * kBN + nt * 8 + lane * 2] = col[nt][0];
          sCol[warp * kBN + nt * 8 + lane * 2 + 1] = col[nt][1];
        }
      }
      __syncthreads();
      if (threadIdx.x < kBN) {
        const int jj = threadIdx.x;
        float a = 0.f;
#pragma unroll
        for (int w = 0; w < kWarps; ++w) a += sCol[w * kBN + jj];
        const int j = j0 + jj;
        const float out = sOk[jj] ? a * inv_rows : 0.f;
        if (j < end) A.mass[(int64_t)b * A.sm0 + (int64_t)h * A.sm1 + j] = out;
        sMass[jj] = j < end ? out : 0.f;
      }
      if (CENTRE) {
        __syncthreads();
        const __nv_bfloat16* sV = reinterpret_cast<const __nv_bfloat16*>(sVb[stage]);
        const int j_lo = chalf * (kBN / 2);
        for (int jj = j_lo; jj < j_lo + kBN / 2; ++jj) {
          const float a = sMass[jj];
          cacc = fmaf(a, __bfloat162float(sV[jj * kTileD + cd]), cacc);
          asum += a;
        }
      }
      stage ^= 1;
    }
    __syncthreads();
  }

  if (!CENTRE) return;
  // per-CTA partial: [D] weighted sums and the weight total, two halves added in order
  float* mine = A.part + ((int64_t)bh * gridDim.x + blockIdx.x) * (kTileD + 1);
  __shared__ float sHalf[kThreads];
  __shared__ float sHalfA[2];
  __shared__ bool sLast;
  sHalf[threadIdx.x] = cacc;
  if (cd == 0) sHalfA[chalf] = asum;
  __syncthreads();
  if (threadIdx.x < kTileD) mine[threadIdx.x] = sHalf[threadIdx.x] + sHalf[threadIdx.x + kTileD];
  if (threadIdx.x == 0) mine[kTileD] = sHalfA[0] + sHalfA[1];
  __threadfence();
  __syncthreads();
  if (threadIdx.x == 0) sLast = atomicAdd(&A.counters[bh], 1u) == gridDim.x - 1;
  __syncthreads();
  if (!sLast) return;
  __threadfence();
  const float* base = A.part + (int64_t)bh * gridDim.x * (kTileD + 1);
  if (threadIdx.x <= kTileD) {
    float tot = 0.f;
    for (unsigned t = 0; t < gridDim.x; ++t) tot += __ldcg(base + (int64_t)t * (kTileD + 1) + threadIdx.x);
    sHalf[threadIdx.x] = tot;
  }
  __syncthreads();
  if (threadIdx.x < kTileD)
    A.centre[(int64_t)bh * kTileD + threadIdx.x] = sHalf[threadIdx.x] / fmaxf(sHalf[kTileD], 1e-12f);
  if (threadIdx.x == 0) A.counters[bh] = 0u;
}

}  // namespace

int mass_mma_slots_per_cta(int n, int BH) {
  const int sms = device_sm_count();
  int per_head = sms / (BH > 0 ? BH : 1);
  if (per_head < 1) per_head = 1;
  int spc = (n + per_head - 1) / per_head;
  spc = ((spc + kBN - 1) / kBN) * kBN;
  return spc < kBN ? kBN : spc;
}

int launch_prefix_mass_mma(const ma_rows& q, const ma_kv& kv, int H, const int32_t* q_rows, int T2,
                           const float* m_p, const float* l_p, float scale, float* mass, int64_t sm0,
                           int64_t sm1, float* part, unsigned* counters, float* centre, cudaStream_t st) {
  const int n = kv.nq + kv.nf;
  MassArgs A;
  A.q = q;
  A.kv = kv;
  A.q_rows = q_rows;
  A.m_p = m_p;
  A.l_p = l_p;
  A.mass = mass;
  A.sm0 = sm0;
  A.sm1 = sm1;
  A.part = part;
  A.counters = counters;
  A.centre = centre;
  A.scale = scale;
  A.H = H;
  A.T2 = T2;
  A.slots_per_cta = mass_mma_slots_per_cta(n, q.B * H);
  dim3 grid((n + A.slots_per_cta - 1) / A.slots_per_cta, q.B * H);
  const bool packed = kv.layout != MA_KV_DENSE;
  const bool cen = centre != nullptr;
  auto go = [&](auto kernel) -> int {
    if (cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmemBytes) != cudaSuccess)
      return MA_ERR_CUDA;
    kernel<<<grid, kThreads, kSmemBytes, st>>>(A);
    return cudaGetLastError() == cudaSuccess ? MA_OK : MA_ERR_CUDA;
  };
  if (packed) return cen ? go(prefix_mass_mma<true, true>) : go(prefix_mass_mma<true, false>);
  return cen ? go(prefix_mass_mma<false, true>) : go(prefix_mass_mma<false, false>);
}

}  // namespace ma
