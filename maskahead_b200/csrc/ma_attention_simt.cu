// Split-K attention over [prefix | current block] (or [read set | current block]) on
// CUDA cores in fp32. This is the kernel family for fp32 caches (the CPU-runnable
// configuration keeps K/V in fp32 and its selections need fp32-exact logits); bf16
// caches use the tcgen05 kernel in ma_attention_tc.cu; both write the split partials
// of ma_common.cuh and share the combine kernel.
//
// Semantics follow the reference's split-K kernels (src/maskahead/kernels/splitk.py:
// 115-190 _sk_fwd, 271-318 _sk_combine): every split keeps an online-softmax
// (max m, sum l, unnormalized acc) per row; dead prefix slots and block-causally hidden
// current keys get s = -inf; a row with no visible key keeps m = -inf, l = 0. The
// partial output is written normalized (acc / l, fp32).
#include "ma_kernels.cuh"

namespace ma {

namespace {

constexpr int kRB = 32;        // rows per CTA
constexpr int kBN = 16;        // keys per tile (static shared memory stays under 48 KB)
constexpr int kThreads = 256;  // 8 threads per row

template <typename QT>
__global__ void __launch_bounds__(kThreads)
attn_partial_simt(ma_rows q, ma_kv kv, int H, ma_block cur, float scale, int causal_block,
                  int q_pos0, int c_pos0, const int64_t* __restrict__ idx, int64_t si0,
                  int64_t si1, int n_keys, int split_len, int nsplit, Partials P) {
  const int D = q.D;
  const int split = blockIdx.x;
  const int bh = blockIdx.y;
  const int b = bh / H, h = bh - (bh / H) * H;
  const int G = q.Hq / H;
  const int R = G * q.T;
  const int r0 = blockIdx.z * kRB;
  const int tid = threadIdx.x;

  __shared__ float sQ[kRB][kMaxD];
  __shared__ float sK[kBN][kMaxD + 1];
  __shared__ float sV[kBN][kMaxD];
  __shared__ float sP[kRB][kBN + 1];
  __shared__ unsigned char sOk[kBN];

  // query rows of this CTA (fp32, unscaled)
  const QT* qp = reinterpret_cast<const QT*>(q.q);
  const int chunks = D / 8;
  for (int c = tid; c < kRB * chunks; c += kThreads) {
    const int rr = c / chunks, c8 = c - (c / chunks) * chunks;
    const int r = r0 + rr;
    float f[8];
    if (r < R) {
      const int g = r / q.T, t = r - (r / q.T) * q.T;
      load8(qp + (int64_t)b * q.sq[0] + (int64_t)(h * G + g) * q.sq[1] + (int64_t)t * q.sq[2] + 8 * c8, f);
    } else {
#pragma unroll
      for (int i = 0; i < 8; ++i) f[i] = 0.f;
    }
#pragma unroll
    for (int i = 0; i < 8; ++i) sQ[rr][8 * c8 + i] = f[i];
  }

  const int row = tid >> 3;     // 0..31
  const int lane8 = tid & 7;
  const int r = r0 + row;
  const int t_row = (r < R) ? (r % q.T) : 0;
  float m = -INFINITY, l = 0.f;
  float o[kMaxD / 8];
#pragma unroll
  for (int i = 0; i < kMaxD / 8; ++i) o[i] = 0.f;

  const bool is_cur = split == nsplit;
  int begin, end;
  if (is_cur) {
    begin = 0;
    end = cur.Tc;
  } else {
    begin = split * split_len;
    end = min(n_keys, begin + split_len);
  }
  const QT* ck = reinterpret_cast<const QT*>(cur.k);
  const QT* cv = reinterpret_cast<const QT*>(cur.v);

  for (int j0 = begin; j0 < end; j0 += kBN) {
    __syncthreads();  // previous tile fully consumed (and sQ written on the first pass)
    for (int c = tid; c < kBN * chunks; c += kThreads) {
      const int jj = c / chunks, c8 = c - (c / chunks) * chunks;
      const int j = j0 + jj;
      float fk[8], fv[8];
      bool ok = j < end;
      if (ok) {
        if (is_cur) {
          load8(ck + (int64_t)b * cur.sk[0] + (int64_t)h * cur.sk[1] + (int64_t)j * cur.sk[2] + 8 * c8, fk);
          load8(cv + (int64_t)b * cur.sv[0] + (int64_t)h * cur.sv[1] + (int64_t)j * cur.sv[2] + 8 * c8, fv);
        } else {
          const int slot = idx ? (int)idx[(int64_t)b * si0 + (int64_t)h * si1 + j] : j;
          ok = kv_live(kv, H, b, h, slot);
          if (ok) {
            kv_read8<true>(kv, b, h, slot, c8, fk);
            kv_read8<false>(kv, b, h, slot, c8, fv);
          }
        }
      }
      if (!ok) {
#pragma unroll
        for (int i = 0; i < 8; ++i) fk[i] = fv[i] = 0.f;
      }
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        sK[jj][8 * c8 + i] = fk[i];
        sV[jj][8 * c8 + i] = fv[i];
      }
      if (c8 == 0) sOk[jj] = ok ? 1 : 0;
    }
    __syncthreads();

    // logits of this thread's kBN/8 keys
    float s[kBN / 8];
    float tmax = -INFINITY;
#pragma unroll
    for (int i = 0; i < kBN / 8; ++i) {
      const int jj = lane8 + 8 * i;
      float acc = 0.f;
      for (int d = 0; d < D; ++d) acc = fmaf(sQ[row][d], sK[jj][d], acc);
      bool vis = sOk[jj] != 0;
      if (is_cur && causal_block > 0)
        vis = vis && ((c_pos0 + j0 + jj) / causal_block <= (q_pos0 + t_row) / causal_block);
      s[i] = vis ? acc * scale : -INFINITY;
      tmax = fmaxf(tmax, s[i]);
    }
#pragma unroll
    for (int o8 = 1; o8 < 8; o8 <<= 1) tmax = fmaxf(tmax, __shfl_xor_sync(0xffffffffu, tmax, o8));
    const float m_new = fmaxf(m, tmax);
    const float m_safe = (m_new == -INFINITY) ? 0.f : m_new;
    const float alpha = expf(m - m_safe);
    float psum = 0.f;
#pragma unroll
    for (int i = 0; i < kBN / 8; ++i) {
      const float p = expf(s[i] - m_safe);
      sP[row][lane8 + 8 * i] = p;
      psum += p;
    }
#pragma unroll
    for (int o8 = 1; o8 < 8; o8 <<= 1) psum += __shfl_xor_sync(0xffffffffu, psum, o8);
    l = l * alpha + psum;
    m = m_new;
    __syncwarp();
    // o[d] for d = lane8 + 8*i
#pragma unroll
    for (int i = 0; i < kMaxD / 8; ++i) o[i] *= alpha;
    for (int jj = 0; jj < kBN; ++jj) {
      const float p = sP[row][jj];
#pragma unroll
      for (int i = 0; i < kMaxD / 8; ++i) {
        const int d = lane8 + 8 * i;
        if (d < D) o[i] = fmaf(p, sV[jj][d], o[i]);
      }
    }
  }

  if (r < R) {
    const int64_t prow = ((int64_t)bh * P.S + split) * P.Rp + r;
    if (lane8 == 0) P.ml[prow] = make_float2(m, l);
    float* a = reinterpret_cast<float*>(P.o) + prow * D;
    const float inv = l > 0.f ? 1.f / l : 0.f;   // normalized output; 0 without a visible key
#pragma unroll
    for (int i = 0; i < kMaxD / 8; ++i) {
      const int d = lane8 + 8 * i;
      if (d < D) a[d] = o[i] * inv;
    }
  }
}

}  // namespace

int launch_attn_partial_simt(const ma_rows& q, const ma_kv& kv, int H, const ma_block& cur,
                             float scale, int causal_block, int q_pos0, int c_pos0,
                             const int64_t* idx, int64_t si0, int64_t si1, int n_keys,
                             int split_len, int nsplit, const Partials& P, cudaStream_t st) {
  const int G = q.Hq / H;
  const int R = G * q.T;
  dim3 grid(P.S, q.B * H, (R + kRB - 1) / kRB);
  if (q.dtype == MA_F32) {
    attn_partial_simt<float><<<grid, kThreads, 0, st>>>(q, kv, H, cur, scale, causal_block, q_pos0,
                                                        c_pos0, idx, si0, si1, n_keys, split_len,
                                                        nsplit, P);
  } else {
    attn_partial_simt<__nv_bfloat16><<<grid, kThreads, 0, st>>>(q, kv, H, cur, scale, causal_block,
                                                                q_pos0, c_pos0, idx, si0, si1,
                                                                n_keys, split_len, nsplit, P);
  }
  return cudaGetLastError() == cudaSuccess ? MA_OK : MA_ERR_CUDA;
}

int simt_row_block() { return kRB; }
int simt_key_tile() { return kBN; }

}  // namespace ma
