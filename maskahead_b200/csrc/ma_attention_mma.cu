// Split-K attention over [prefix | current block] (or [read set | current block]) on
// the tensor cores, for bf16 queries and a bf16 (or dequantized-to-bf16) cache.
//
// One CTA = 8 warps = up to 256 query rows of one KV head (the R = G*T rows of the GQA
// group share every K/V tile, so a tile crosses HBM once per KV head); each warp owns
// 32 rows. Keys stream through shared memory in tiles of 32 (double-buffered
// cp.async for bf16 rows, dequantized stores for packed rows), S = Q K^T and O += P V
// run as m16n8k16 bf16 MMAs with fp32 accumulation, softmax is online per row.
// Output: the split's (m, l, acc) per row in the shared partial format (ma_common.cuh).
// Semantics follow src/maskahead/kernels/splitk.py:115-190 (_sk_fwd).
#include "ma_kernels.cuh"
#include "ma_mma.cuh"

namespace ma {

namespace {

constexpr int kWarps = 8;
constexpr int kThreads = kWarps * 32;
constexpr int kRowsPerWarp = 32;
constexpr int kRowTile = kWarps * kRowsPerWarp;  // 256
constexpr int kBN = 32;                          // keys per tile
constexpr int kD = 128;
constexpr int kChunks = kD / 8;                  // 16-byte chunks per row
constexpr float kLog2e = 1.4426950408889634f;

// shared memory layout (bytes)
constexpr int kQBytes = kRowTile * kD * 2;         // 64 KB
constexpr int kTileBytes = kBN * kD * 2;           // 8 KB per K or V tile
constexpr int kSmemBytes = kQBytes + 4 * kTileBytes + 2 * kBN;

struct Args {
  ma_rows q;
  ma_kv kv;
  ma_block cur;
  const int64_t* idx;
  int64_t si0, si1;
  float scale;
  int H, causal_block, q_pos0, c_pos0, n_keys, split_len, nsplit;
  Partials P;
};

// Stage keys [j0, j0+kBN) of this split into buffer `st`.
template <bool PACKED>
__device__ __forceinline__ void load_tile(const Args& A, int b, int h, bool is_cur, int j0, int end,
                                          uint8_t* sK, uint8_t* sV, uint8_t* sOk) {
  const __nv_bfloat16* ck = reinterpret_cast<const __nv_bfloat16*>(A.cur.k);
  const __nv_bfloat16* cv = reinterpret_cast<const __nv_bfloat16*>(A.cur.v);
  const __nv_bfloat16* kf = reinterpret_cast<const __nv_bfloat16*>(A.kv.kf);
  const __nv_bfloat16* vf = reinterpret_cast<const __nv_bfloat16*>(A.kv.vf);
  for (int c = threadIdx.x; c < kBN * kChunks; c += kThreads) {
    const int jj = c / kChunks, ch = c % kChunks;
    const int j = j0 + jj;
    bool ok = j < end;
    const uint32_t dk = smem_u32(sK + swz(jj, ch)), dv = smem_u32(sV + swz(jj, ch));
    if (is_cur) {
      const __nv_bfloat16* src_k = ok ? ck + (int64_t)b * A.cur.sk[0] + (int64_t)h * A.cur.sk[1] +
                                            (int64_t)j * A.cur.sk[2] + ch * 8
                                      : ck;
      const __nv_bfloat16* src_v = ok ? cv + (int64_t)b * A.cur.sv[0] + (int64_t)h * A.cur.sv[1] +
                                            (int64_t)j * A.cur.sv[2] + ch * 8
                                      : cv;
      cp_async16(dk, src_k, ok);
      cp_async16(dv, src_v, ok);
    } else {
      int slot = j;
      if (ok && A.idx) slot = (int)A.idx[(int64_t)b * A.si0 + (int64_t)h * A.si1 + j];
      ok = ok && kv_live(A.kv, A.H, b, h, slot);
      if (!ok) {
        *reinterpret_cast<uint4*>(sK + swz(jj, ch)) = make_uint4(0, 0, 0, 0);
        *reinterpret_cast<uint4*>(sV + swz(jj, ch)) = make_uint4(0, 0, 0, 0);
      } else if (!PACKED || slot >= A.kv.nq) {
        const int row = slot - A.kv.nq;
        cp_async16(dk, kf + (int64_t)b * A.kv.skf[0] + (int64_t)h * A.kv.skf[1] + (int64_t)row * A.kv.skf[2] + ch * 8, true);
        cp_async16(dv, vf + (int64_t)b * A.kv.svf[0] + (int64_t)h * A.kv.svf[1] + (int64_t)row * A.kv.svf[2] + ch * 8, true);
      } else {
        float fk[8], fv[8];
        kv_read8<true>(A.kv, b, h, slot, ch, fk);
        kv_read8<false>(A.kv, b, h, slot, ch, fv);
        *reinterpret_cast<uint4*>(sK + swz(jj, ch)) = float8_to_bf16x8(fk);
        *reinterpret_cast<uint4*>(sV + swz(jj, ch)) = float8_to_bf16x8(fv);
      }
    }
    if (ch == 0) sOk[jj] = ok ? 1 : 0;
  }
  cp_async_commit();
}

template <bool PACKED>
__global__ void __launch_bounds__(kThreads, 1) attn_partial_mma(const Args A) {
  extern __shared__ __align__(128) uint8_t smem[];
  uint8_t* sQ = smem;
  uint8_t* sKb[2] = {smem + kQBytes, smem + kQBytes + kTileBytes};
  uint8_t* sVb[2] = {smem + kQBytes + 2 * kTileBytes, smem + kQBytes + 3 * kTileBytes};
  uint8_t* sOkb[2] = {smem + kQBytes + 4 * kTileBytes, smem + kQBytes + 4 * kTileBytes + kBN};

  const int split = blockIdx.x;
  const int bh = blockIdx.y;
  const int H = A.H;
  const int b = bh / H, h = bh - (bh / H) * H;
  const int T = A.q.T;
  const int G = A.q.Hq / H;
  const int R = G * T;
  const int r0 = blockIdx.z * kRowTile;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

  const bool is_cur = split == A.nsplit;
  int begin, end;
  if (is_cur) {
    begin = 0;
    end = A.cur.Tc;
  } else {
    begin = split * A.split_len;
    end = min(A.n_keys, begin + A.split_len);
  }

  // Q rows (bf16), swizzled; rows beyond R are zero
  {
    const __nv_bfloat16* qp = reinterpret_cast<const __nv_bfloat16*>(A.q.q);
    for (int c = threadIdx.x; c < kRowTile * kChunks; c += kThreads) {
      const int rr = c / kChunks, ch = c % kChunks;
      const int r = r0 + rr;
      const bool ok = r < R;
      const int g = ok ? r / T : 0, t = ok ? r - (r / T) * T : 0;
      const __nv_bfloat16* src =
          qp + (int64_t)b * A.q.sq[0] + (int64_t)(h * G + g) * A.q.sq[1] + (int64_t)t * A.q.sq[2] + ch * 8;
      cp_async16(smem_u32(sQ + swz(rr, ch)), ok ? src : qp, ok);
    }
  }
  if (begin < end) load_tile<PACKED>(A, b, h, is_cur, begin, end, sKb[0], sVb[0], sOkb[0]);
  else cp_async_commit();

  const int wrow = warp * kRowsPerWarp;          // first row of this warp within the tile
  const bool warp_active = r0 + wrow < R;
  // row block positions t of this thread's 4 rows (for the block-causal mask)
  int trow[2][2];
#pragma unroll
  for (int mt = 0; mt < 2; ++mt)
#pragma unroll
    for (int hf = 0; hf < 2; ++hf) {
      const int r = r0 + wrow + mt * 16 + hf * 8 + (lane >> 2);
      trow[mt][hf] = (r < R) ? r % T : 0;
    }

  float o[2][16][4];
#pragma unroll
  for (int mt = 0; mt < 2; ++mt)
#pragma unroll
    for (int nt = 0; nt < 16; ++nt)
#pragma unroll
      for (int e = 0; e < 4; ++e) o[mt][nt][e] = 0.f;
  float m[2][2], l[2][2];
#pragma unroll
  for (int mt = 0; mt < 2; ++mt)
#pragma unroll
    for (int hf = 0; hf < 2; ++hf) {
      m[mt][hf] = -INFINITY;
      l[mt][hf] = 0.f;
    }

  int stage = 0;
  for (int j0 = begin; j0 < end; j0 += kBN) {
    cp_async_wait_all();
    __syncthreads();  // tile `stage` (and Q) visible; the other buffer is free
    if (j0 + kBN < end) load_tile<PACKED>(A, b, h, is_cur, j0 + kBN, end, sKb[stage ^ 1], sVb[stage ^ 1], sOkb[stage ^ 1]);
    const uint8_t* sK = sKb[stage];
    const uint8_t* sV = sVb[stage];
    const uint8_t* sOk = sOkb[stage];
    if (warp_active) {
      float s[2][4][4];
#pragma unroll
      for (int mt = 0; mt < 2; ++mt)
#pragma unroll
        for (int nt = 0; nt < 4; ++nt)
#pragma unroll
          for (int e = 0; e < 4; ++e) s[mt][nt][e] = 0.f;
      // S = Q K^T
#pragma unroll
      for (int kk = 0; kk < kD / 16; ++kk) {
        uint32_t a[2][4];
#pragma unroll
        for (int mt = 0; mt < 2; ++mt) {
          const int row = wrow + mt * 16 + (lane & 15);
          ldsm_x4(smem_u32(sQ + swz(row, kk * 2 + (lane >> 4))), a[mt][0], a[mt][1], a[mt][2], a[mt][3]);
        }
#pragma unroll
        for (int np = 0; np < 2; ++np) {
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
      // mask, online softmax (log2 domain inside the tile)
#pragma unroll
      for (int mt = 0; mt < 2; ++mt) {
#pragma unroll
        for (int hf = 0; hf < 2; ++hf) {
          float mx = -INFINITY;
#pragma unroll
          for (int nt = 0; nt < 4; ++nt)
#pragma unroll
            for (int e = 0; e < 2; ++e) {
              const int jj = nt * 8 + (lane & 3) * 2 + e;
              bool vis = sOk[jj] != 0;
              if (is_cur && A.causal_block > 0)
                vis = vis && ((A.c_pos0 + j0 + jj) / A.causal_block <= (A.q_pos0 + trow[mt][hf]) / A.causal_block);
              const float v = vis ? s[mt][nt][hf * 2 + e] * A.scale : -INFINITY;
              s[mt][nt][hf * 2 + e] = v;
              mx = fmaxf(mx, v);
            }
          mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 1));
          mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 2));
          const float m_new = fmaxf(m[mt][hf], mx);
          const float m_safe = (m_new == -INFINITY) ? 0.f : m_new;
          const float alpha = exp2f((m[mt][hf] - m_safe) * kLog2e);
          float rs = 0.f;
#pragma unroll
          for (int nt = 0; nt < 4; ++nt)
#pragma unroll
            for (int e = 0; e < 2; ++e) {
              const float p = exp2f((s[mt][nt][hf * 2 + e] - m_safe) * kLog2e);
              s[mt][nt][hf * 2 + e] = p;
              rs += p;
            }
          rs += __shfl_xor_sync(0xffffffffu, rs, 1);
          rs += __shfl_xor_sync(0xffffffffu, rs, 2);
          l[mt][hf] = l[mt][hf] * alpha + rs;
          m[mt][hf] = m_new;
#pragma unroll
          for (int nt = 0; nt < 16; ++nt) {
            o[mt][nt][hf * 2] *= alpha;
            o[mt][nt][hf * 2 + 1] *= alpha;
          }
        }
      }
      // O += P V
#pragma unroll
      for (int kk = 0; kk < kBN / 16; ++kk) {
        uint32_t a[2][4];
#pragma unroll
        for (int mt = 0; mt < 2; ++mt) {
          a[mt][0] = pack_bf16(s[mt][2 * kk][0], s[mt][2 * kk][1]);
          a[mt][1] = pack_bf16(s[mt][2 * kk][2], s[mt][2 * kk][3]);
          a[mt][2] = pack_bf16(s[mt][2 * kk + 1][0], s[mt][2 * kk + 1][1]);
          a[mt][3] = pack_bf16(s[mt][2 * kk + 1][2], s[mt][2 * kk + 1][3]);
        }
#pragma unroll
        for (int dp = 0; dp < kD / 16; ++dp) {
          uint32_t b0, b1, b2, b3;
          const int key = kk * 16 + (lane & 7) + (((lane >> 3) & 1) << 3);
          ldsm_x4_t(smem_u32(sV + swz(key, dp * 2 + (lane >> 4))), b0, b1, b2, b3);
#pragma unroll
          for (int mt = 0; mt < 2; ++mt) {
            mma_bf16(o[mt][2 * dp], a[mt], b0, b1);
            mma_bf16(o[mt][2 * dp + 1], a[mt], b2, b3);
          }
        }
      }
    }
    stage ^= 1;
  }

  // partials
  if (!warp_active) return;
  const int D = kD;
#pragma unroll
  for (int mt = 0; mt < 2; ++mt)
#pragma unroll
    for (int hf = 0; hf < 2; ++hf) {
      const int r = r0 + wrow + mt * 16 + hf * 8 + (lane >> 2);
      if (r >= R) continue;
      const int64_t prow = ((int64_t)bh * A.P.S + split) * A.P.Rp + r;
      if ((lane & 3) == 0) A.P.ml[prow] = make_float2(m[mt][hf], l[mt][hf]);
      float* dst = A.P.acc + prow * D + (lane & 3) * 2;
#pragma unroll
      for (int nt = 0; nt < 16; ++nt)
        *reinterpret_cast<float2*>(dst + nt * 8) = make_float2(o[mt][nt][hf * 2], o[mt][nt][hf * 2 + 1]);
    }
}

}  // namespace

int mma_row_tile() { return kRowTile; }
int mma_key_tile() { return kBN; }

int launch_attn_partial_mma(const ma_rows& q, const ma_kv& kv, int H, const ma_block& cur,
                            float scale, int causal_block, int q_pos0, int c_pos0,
                            const int64_t* idx, int64_t si0, int64_t si1, int n_keys,
                            int split_len, int nsplit, const Partials& P, cudaStream_t st) {
  if (q.D != kD) return MA_ERR_UNSUPPORTED;
  Args A;
  A.q = q;
  A.kv = kv;
  A.cur = cur;
  A.idx = idx;
  A.si0 = si0;
  A.si1 = si1;
  A.scale = scale;
  A.H = H;
  A.causal_block = causal_block;
  A.q_pos0 = q_pos0;
  A.c_pos0 = c_pos0;
  A.n_keys = n_keys;
  A.split_len = split_len;
  A.nsplit = nsplit;
  A.P = P;
  const int G = q.Hq / H;
  const int R = G * q.T;
  dim3 grid(P.S, q.B * H, (R + kRowTile - 1) / kRowTile);
  const bool packed = kv.layout != MA_KV_DENSE;
  cudaError_t e;
  if (packed) {
    e = cudaFuncSetAttribute(attn_partial_mma<true>, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmemBytes);
    if (e != cudaSuccess) return MA_ERR_CUDA;
    attn_partial_mma<true><<<grid, kThreads, kSmemBytes, st>>>(A);
  } else {
    e = cudaFuncSetAttribute(attn_partial_mma<false>, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmemBytes);
    if (e != cudaSuccess) return MA_ERR_CUDA;
    attn_partial_mma<false><<<grid, kThreads, kSmemBytes, st>>>(A);
  }
  return cudaGetLastError() == cudaSuccess ? MA_OK : MA_ERR_CUDA;
}

}  // namespace ma
