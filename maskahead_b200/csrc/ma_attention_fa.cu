// Split-K attention over [prefix | current block] for contiguous bf16 keys/values read by
// TMA, with the softmax of each M tile in its own warpgroup and P kept in tensor memory.
//
// CTA = 2 softmax warpgroups (warps 0-3: rows 0-127, warps 4-7: rows 128-255 of one KV
// head's R = G*T query rows) + 1 MMA/TMA warp. Keys come in tiles of 128: K through 3
// slots (a slot is refilled once its S was read), V through 2 (refilled when its P.V
// completes), 32 KB each. Tensor memory (512 columns): S_m = Q_m K^T in columns
// [128m, 128m+128) and O_m in [256+128m, 256+128m+128). Per tile t and M tile m:
//   MMA warp   S_m(t) = Q_m K(t)^T (8 MMAs 128x128x16, A = Q in shared memory)
//   warpgroup  row max over the 128 logits (lazy, base 2), P = 2^(u - m) rounded to bf16
//              and written back over the first 64 columns of S_m as bf16 pairs
//   MMA warp   O_m += P_m V(t) (8 MMAs, A = P_m from tensor memory, B = V MN-major)
// The two warpgroups run out of phase, so the tensor core works on one M tile while the
// other's softmax runs. S_m(t+1) is issued only once O_m += P_m(t) V(t) has completed
// (its P shares the columns), which also keeps the lazy rescale of O_m race-free. With
// one M tile (R - r0 <= 128) the warpgroups split the keys instead (even / odd tiles, the
// same rows, separate S, P and O) and merge their (m, l, O) at the end.
// Per split: (m, l) and o = acc / l as bf16 (ma_common.cuh), stored by TMA, the merge
// as in ma_attention_tc.cu (fused into a cooperative launch when it is one pass).
// Every wait is bounded. Semantics follow src/maskahead/kernels/splitk.py:115-190.
#include <string.h>

#include <algorithm>

#include "ma_combine.cuh"
#include "ma_kernels.cuh"
#include "ma_tcgen05.cuh"
#include "ma_tma.cuh"

namespace ma {

namespace {

using namespace tc;

constexpr int kSoftWarps = 8;
constexpr int kSoftThreads = kSoftWarps * 32;
constexpr int kWarps = kSoftWarps + 1;
constexpr int kThreads = kWarps * 32;
constexpr int kMTile = 128;
constexpr int kRowTile = 2 * kMTile;
constexpr int kBN = 128;                           // keys per tile
constexpr int kD = 128;
constexpr int kKSlots = 3;                        // K tiles in flight (freed once S was read)
constexpr int kVSlots = 2;                        // V tiles in flight (freed when P.V completes)
constexpr float kLog2e = 1.4426950408889634f;
constexpr float kLazyLog2 = 8.0f * kLog2e;

constexpr int kQBlock = kRowTile * 128;            // 32 KB: one 64-channel block of 256 rows
constexpr int kQBytes = 2 * kQBlock;
constexpr int kKVBlock = kBN * 128;                // 16 KB: [128 rows][128 B]
constexpr int kKVBytes = 2 * kKVBlock;             // a K or V tile: 32 KB
constexpr int kSmemBytes = 1024 + kQBytes + (kKSlots + kVSlots) * kKVBytes;   // 225 KB
constexpr uint32_t kTmemCols = 512;
constexpr uint32_t kColS = 0, kColO = 256;
constexpr int kOutBox = 32 * 128;
constexpr uint64_t kMergeWaitNs = 200000000ull;
constexpr uint64_t kStallNs = 500000000ull;        // MMA issuer: longest time without progress

struct __align__(64) Args {
  CUtensorMap kmap, vmap;       // prefix K/V [B][H][n][D]
  CUtensorMap ckmap, cvmap;     // current block K/V [B][H][Tc][D]
  CUtensorMap qmap;             // queries [B][Hq][T][D]
  CUtensorMap omap;             // partial outputs [BH * S * Rp][D] bf16 (stores)
  ma_rows q;
  ma_kv kv;
  ma_block cur;
  float scale;
  int H, causal_block, q_pos0, c_pos0, n_keys, split_len, nsplit;
  int tma_out;
  Partials P;
  int* err;
  int fuse;
  FusedMerge fm;
};

__device__ __forceinline__ void mbar_arrive(uint64_t* mbar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];\n" ::"r"(smem_addr(mbar)) : "memory");
}
// non-blocking test of a phase parity
__device__ __forceinline__ bool mbar_test(uint64_t* mbar, uint32_t phase) {
  uint32_t ok;
  asm volatile(
      "{\n.reg .pred p;\nmbarrier.test_wait.parity.shared::cta.b64 p, [%1], %2;\nselp.u32 %0, 1, 0, p;\n}\n"
      : "=r"(ok)
      : "r"(smem_addr(mbar)), "r"(phase)
      : "memory");
  return ok != 0;
}
__device__ __forceinline__ void prefetch_map(const CUtensorMap* m) {
  asm volatile("prefetch.tensormap [%0];\n" ::"l"(reinterpret_cast<uint64_t>(m)) : "memory");
}
// tensor-memory store of 16 consecutive 32-bit columns of this warp's 32 lanes
__device__ __forceinline__ void tmem_st16(uint32_t taddr, const uint32_t* r) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16};\n" ::"r"(
          taddr),
      "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]), "r"(r[8]), "r"(r[9]),
      "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15]));
}
// D[tmem] (+)= A[tmem] * B[smem]: the A operand (M x 16, bf16 pairs per column) in TMEM
__device__ __forceinline__ void mma_bf16_ta(uint32_t d_tmem, uint32_t a_tmem, uint64_t b_desc, uint32_t idesc,
                                            bool accumulate) {
  asm volatile(
      "{\n.reg .pred p;\nsetp.ne.b32 p, %4, 0;\n"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n}\n" ::"r"(d_tmem),
      "r"(a_tmem), "l"(b_desc), "r"(idesc), "r"(accumulate ? 1 : 0));
}
// packed fp32 pairs (sm_100): one instruction for two lanes of work
__device__ __forceinline__ uint64_t f2_bits(float2 a) {
  uint64_t u;
  asm("mov.b64 %0, {%1, %2};" : "=l"(u) : "f"(a.x), "f"(a.y));
  return u;
}
__device__ __forceinline__ float2 bits_f2(uint64_t u) {
  float2 a;
  asm("mov.b64 {%0, %1}, %2;" : "=f"(a.x), "=f"(a.y) : "l"(u));
  return a;
}
__device__ __forceinline__ float2 ffma2(float2 a, float2 b, float2 c) {
  uint64_t d;
  asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(d) : "l"(f2_bits(a)), "l"(f2_bits(b)), "l"(f2_bits(c)));
  return bits_f2(d);
}
__device__ __forceinline__ float2 fadd2(float2 a, float2 b) {
  uint64_t d;
  asm("add.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(f2_bits(a)), "l"(f2_bits(b)));
  return bits_f2(d);
}
// three-input maximum (sm_100)
__device__ __forceinline__ float max3f(float a, float b, float c) {
  float d;
  asm("max.f32 %0, %1, %2, %3;" : "=f"(d) : "f"(a), "f"(b), "f"(c));
  return d;
}
__device__ __forceinline__ uint32_t pack_bf16x2(float lo, float hi) {
  __nv_bfloat162 v = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<uint32_t*>(&v);
}
// barrier of one softmax warpgroup (ids 1 and 2; 0 is __syncthreads)
__device__ __forceinline__ void wg_sync(int m) {
  asm volatile("bar.sync %0, 128;\n" ::"r"(1 + m) : "memory");
}

// one 128-key tile of K or V (two 64-channel boxes) into dst, completing on `bar`
__device__ __forceinline__ void tma_tile(const CUtensorMap* map, int b, int h, int j0, uint8_t* dst, uint64_t* bar) {
  tma::expect_tx(bar, kKVBytes);
  tma::load_4d(dst, map, 0, j0, h, b, bar);
  tma::load_4d(dst + kKVBlock, map, 64, j0, h, b, bar);
}

__global__ void __launch_bounds__(kThreads, 1) attn_partial_fa(const __grid_constant__ Args A) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sQ = smem;                                   // [2 d blocks][256 rows][128 B]
  uint8_t* ring = sQ + kQBytes;                         // K slots, then V slots
  uint8_t* sKs = ring;
  uint8_t* sVs = ring + kKSlots * kKVBytes;
  __shared__ uint32_t s_taddr;
  __shared__ __align__(8) uint64_t kfull[kKSlots], vfull[kVSlots], s_full[2], p_full[2], o_done[2], q_full, mbar_fin;
  __shared__ int s_abort, s_merge_ok;

  const int split = blockIdx.x;
  const int bh = blockIdx.y;
  const int H = A.H;
  const int b = bh / H, h = bh - (bh / H) * H;
  const int T = A.q.T;
  const int G = A.q.Hq / H;
  const int R = G * T;
  const int r0 = blockIdx.z * kRowTile;
  const int mtiles = min(2, (R - r0 + kMTile - 1) / kMTile);
  // one M tile: the two warpgroups split the keys (even / odd tiles) over the same rows,
  // each with its own S, P and O, and merge at the end
  const bool dual = mtiles == 1;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const bool softmax_warp = warp < kSoftWarps;
  const int mt = (warp >> 2) & 1, quarter = warp & 3;
  const int mrow = dual ? 0 : mt;                        // the M tile whose rows this warp holds
  const int r = r0 + mrow * kMTile + quarter * 32 + lane;
  const int wrow0 = r0 + mrow * kMTile + quarter * 32;
  const bool wg_on = softmax_warp && mt < (dual ? 2 : mtiles);
  const bool warp_rows = wg_on && wrow0 < R;             // warp-uniform
  const bool row_ok = wg_on && r < R;
  const int t_row = row_ok ? r % T : 0;

  const bool is_cur = split == A.nsplit;
  int begin, end;
  if (is_cur) {
    begin = 0;
    end = A.cur.Tc;
  } else {
    begin = split * A.split_len;
    end = min(A.n_keys, begin + A.split_len);
  }
  int vis_end = end;
  if (is_cur && A.causal_block > 0)
    vis_end = min(end, ((A.q_pos0 + t_row) / A.causal_block + 1) * A.causal_block - A.c_pos0);
  if (!row_ok) vis_end = begin;
  const int ntiles = end > begin ? (end - begin + kBN - 1) / kBN : 0;
  // chain m (S_m, P_m, O_m): every tile for M tile m, or tiles m, m+2, ... in dual mode
  const int nt0 = dual ? (ntiles + 1) / 2 : ntiles;
  const int nt1 = dual ? ntiles / 2 : (mtiles > 1 ? ntiles : 0);
  const float c2 = A.scale * kLog2e;
  const int group = bh * gridDim.z + blockIdx.z;

  unsigned gen0 = 0;   // the merge generation, read before this CTA arrives (thread 0)
  if (A.fuse && threadIdx.x == 0) gen0 = *reinterpret_cast<volatile const unsigned*>(&A.fm.sync[group].y);
  if (threadIdx.x == kSoftThreads) {
    prefetch_map(&A.qmap);
    prefetch_map(is_cur ? &A.ckmap : &A.kmap);
    prefetch_map(is_cur ? &A.cvmap : &A.vmap);
    for (int i = 0; i < kKSlots; ++i) mbar_init(&kfull[i], 1);
    for (int i = 0; i < kVSlots; ++i) mbar_init(&vfull[i], 1);
    for (int m = 0; m < 2; ++m) {
      mbar_init(&s_full[m], 1);
      mbar_init(&p_full[m], 4);   // the warpgroup's warps
      mbar_init(&o_done[m], 1);
    }
    mbar_init(&q_full, 1);
    mbar_init(&mbar_fin, 1);
    s_abort = 0;
    asm volatile("fence.mbarrier_init.release.cluster;\n" ::: "memory");
  }
  if (warp == 0) tmem_alloc(&s_taddr, kTmemCols);
  fence_before_sync();
  __syncthreads();
  fence_after_sync();
  const uint32_t taddr = s_taddr;
  const uint32_t lane_base = (uint32_t)(quarter * 32) << 16;
  const uint32_t tS = taddr + lane_base + kColS + mt * 128;   // this warpgroup's S (and P)
  const uint32_t tO = taddr + lane_base + kColO + mt * 128;   // this warpgroup's O
  float m_run = -INFINITY, l_run = 0.f, m_true = -INFINITY;

  if (!softmax_warp) {
    // ------------------------------------------------------------ MMA / TMA warp
    if (lane == 0) {
      // Event loop over the chains S_m(0) PV_m(0) S_m(1) PV_m(1) ..., issuing whatever
      // became ready: S_m(u) needs its K tile and PV_m(u-1) completed (P_m lives in S_m's
      // columns), PV_m(u) needs its V tile and the warpgroup's P_m(u). A K slot takes the
      // next K tile once every S that read it was consumed (its P.V issued), a V slot once
      // every P.V that read it completed. Each barrier has at most one completed but
      // unobserved phase, so the parity tests are unambiguous.
      pdl_wait();   // with a programmatic launch, the inputs may come from the kernel before
      bool ok = true;
      int kIss = 0, kObs = 0, vIss = 0, vObs = 0;   // tiles issued / seen loaded
      int sN[2] = {0, 0}, pN[2] = {0, 0}, oD[2] = {0, 0};
      const int nt[2] = {nt0, nt1};
      const CUtensorMap* km = is_cur ? &A.ckmap : &A.kmap;
      const CUtensorMap* vm = is_cur ? &A.cvmap : &A.vmap;
      const int hq0 = h * G + r0 / T;
      tma::expect_tx(&q_full, (uint32_t)(kRowTile * 256));
      tma::load_4d(sQ, &A.qmap, 0, 0, hq0, b, &q_full);
      tma::load_4d(sQ + kQBlock, &A.qmap, 64, 0, hq0, b, &q_full);
      for (; kIss < kKSlots && kIss < ntiles; ++kIss)
        tma_tile(km, b, h, begin + kIss * kBN, sKs + kIss * kKVBytes, &kfull[kIss]);
      for (; vIss < kVSlots && vIss < ntiles; ++vIss)
        tma_tile(vm, b, h, begin + vIss * kBN, sVs + vIss * kKVBytes, &vfull[vIss]);
      const bool q_ok = mbar_wait(&q_full, 0);
      ok = q_ok;
      const uint32_t idS = idesc_bf16(kMTile, kBN, false, false);
      const uint32_t idO = idesc_bf16(kMTile, kD, false, true);
      // base descriptors; a K step or a slot only moves the start address (field bits
      // [0,14) = address >> 4, no carry below 256 KB), so each MMA adds a constant
      const uint64_t qdesc = smem_desc(smem_addr(sQ), 16, 1024);
      const uint64_t kdesc = smem_desc(smem_addr(sKs), 16, 1024);
      const uint64_t vdesc = smem_desc(smem_addr(sVs), kKVBlock, 1024);
      uint64_t t_idle = 0;
      bool armed = false;
      int spins = 0;
      while (ok && (pN[0] < nt[0] || pN[1] < nt[1])) {
        bool progress = false;
        if (kObs < kIss && mbar_test(&kfull[kObs % kKSlots], (uint32_t)(kObs / kKSlots) & 1u)) {
          ++kObs;
          progress = true;
        }
        if (vObs < vIss && mbar_test(&vfull[vObs % kVSlots], (uint32_t)(vObs / kVSlots) & 1u)) {
          ++vObs;
          progress = true;
        }
#pragma unroll
        for (int m = 0; m < 2; ++m) {
          if (oD[m] < pN[m] && mbar_test(&o_done[m], (uint32_t)oD[m] & 1u)) {
            ++oD[m];
            progress = true;
          }
          if (sN[m] == pN[m] && sN[m] < nt[m]) {
            const int u = sN[m];
            const int t = dual ? 2 * u + m : u;
            if (kObs > t && oD[m] >= u) {
              fence_after_sync();
              const uint64_t ad0 = qdesc + (uint64_t)((dual ? 0 : m) * (kMTile * 128 / 16));
              const uint64_t bd0 = kdesc + (uint64_t)((t % kKSlots) * (kKVBytes / 16));
              const uint32_t dS = taddr + kColS + m * 128;
#pragma unroll
              for (int kk = 0; kk < kD / 16; ++kk)
                mma_bf16(dS, ad0 + (uint64_t)(((kk >> 2) * kQBlock + (kk & 3) * 32) >> 4),
                         bd0 + (uint64_t)(((kk >> 2) * kKVBlock + (kk & 3) * 32) >> 4), idS, kk > 0);
              mma_commit(&s_full[m]);
              sN[m] = u + 1;
              progress = true;
            }
          } else if (pN[m] < sN[m]) {
            const int u = pN[m];
            const int t = dual ? 2 * u + m : u;
            if (vObs > t && mbar_test(&p_full[m], (uint32_t)u & 1u)) {
              fence_after_sync();
              const uint64_t bd0 = vdesc + (uint64_t)((t % kVSlots) * (kKVBytes / 16));
              const uint32_t dO = taddr + kColO + m * kD, aP = taddr + kColS + m * 128;
#pragma unroll
              for (int kk = 0; kk < kBN / 16; ++kk)
                mma_bf16_ta(dO, aP + kk * 8, bd0 + (uint64_t)(kk * (2048 / 16)), idO, u > 0 || kk > 0);
              mma_commit(&o_done[m]);
              pN[m] = u + 1;
              progress = true;
            }
          }
        }
        // K slot of tile kIss - kKSlots: free once that tile's P.V was issued by every chain
        // that reads it (the warpgroup had read its S)
        if (kIss < ntiles) {
          const int prev = kIss - kKSlots;
          const bool free_slot = dual ? pN[prev & 1] > (prev >> 1)
                                      : (pN[0] > prev && pN[1] > prev);
          if (free_slot) {
            tma_tile(km, b, h, begin + kIss * kBN, sKs + (kIss % kKSlots) * kKVBytes, &kfull[kIss % kKSlots]);
            ++kIss;
            progress = true;
          }
        }
        // V slot of tile vIss - kVSlots: free once its P.V completed in every chain
        if (vIss < ntiles) {
          const int prev = vIss - kVSlots;
          const bool free_slot = dual ? oD[prev & 1] > (prev >> 1)
                                      : (oD[0] > prev && oD[1] > prev);
          if (free_slot) {
            tma_tile(vm, b, h, begin + vIss * kBN, sVs + (vIss % kVSlots) * kKVBytes, &vfull[vIss % kVSlots]);
            ++vIss;
            progress = true;
          }
        }
        if (progress) {
          spins = 0;
          armed = false;
        } else if (++spins == 256) {   // idle: bound the time without progress
          spins = 0;
          const uint64_t now = global_ns();
          if (!armed) {
            t_idle = now;
            armed = true;
          } else if (now - t_idle > kStallNs) {
            ok = false;
          }
          if (s_abort) ok = false;
        }
      }
      if (!ok) s_abort = 1;
      // drain (bounded): every MMA issued, every TMA load still in flight
      mma_commit(&mbar_fin);
      mbar_wait(&mbar_fin, 0, 20000000ull);
      if (!q_ok) mbar_wait(&q_full, 0, 20000000ull);
      for (int tt = kObs; tt < kIss; ++tt)
        mbar_wait(&kfull[tt % kKSlots], (uint32_t)(tt / kKSlots) & 1u, 20000000ull);
      for (int tt = vObs; tt < vIss; ++tt)
        mbar_wait(&vfull[tt % kVSlots], (uint32_t)(tt / kVSlots) & 1u, 20000000ull);
    }
    __syncwarp();
  } else if (wg_on) {
    // ------------------------------------------------------------ softmax warpgroup mt
    pdl_wait();   // the partials and outputs may still be in use by the kernel before
    bool ok = true;
    const int nt_me = mt == 0 ? nt0 : nt1;
    const float2 c2x2 = make_float2(c2, c2);
    for (int u = 0; u < nt_me; ++u) {
      const int t = dual ? 2 * u + mt : u;
      const int j0 = begin + t * kBN;
      ok = mbar_wait(&s_full[mt], (uint32_t)u & 1u);
      fence_after_sync();
      if (!ok) s_abort = 1;
      if (s_abort) break;
      const int lim = vis_end - j0;   // keys i >= lim are hidden from this row
      if (warp_rows) {
        // pass 1: the tile max over the raw logits (scale > 0 keeps the order); the four
        // loads share one wait, hidden keys read as -inf
        const bool part = !__all_sync(0xffffffffu, lim >= kBN);
        float tmax;
        {
          float mx[4] = {-INFINITY, -INFINITY, -INFINITY, -INFINITY};
#pragma unroll 1
          for (int hh = 0; hh < 2; ++hh) {
            float s[64];
            tmem_ld32(tS + hh * 64, s);
            tmem_ld32(tS + hh * 64 + 32, s + 32);
            tmem_ld_wait();
            if (part) {
#pragma unroll
              for (int i = 0; i < 64; ++i) s[i] = hh * 64 + i < lim ? s[i] : -INFINITY;
            }
#pragma unroll
            for (int i = 0; i < 64; i += 8) {
#pragma unroll
              for (int j = 0; j < 4; ++j) mx[j] = max3f(mx[j], s[i + j], s[i + 4 + j]);
            }
          }
          tmax = fmaxf(max3f(mx[0], mx[1], mx[2]), mx[3]);
        }
        // lazy rescale of O_m (its last P.V completed before S_m(u) was issued)
        m_true = fmaxf(m_true, tmax);
        const float m_new = fmaxf(m_run, tmax * c2);
        const bool grow = u > 0 && m_new > m_run + kLazyLog2;
        if (__any_sync(0xffffffffu, grow)) {
          const float alpha = grow ? ex2(m_run - m_new) : 1.f;
#pragma unroll 1
          for (int c = 0; c < kD / 32; ++c) {
            float o[32];
            tmem_ld32(tO + c * 32, o);
            tmem_ld_wait();
#pragma unroll
            for (int i = 0; i < 32; ++i) o[i] *= alpha;
            tmem_st32(tO + c * 32, o);
          }
          tmem_st_wait();
          if (grow) {
            l_run *= alpha;
            m_run = m_new;
          }
        }
        if (u == 0) m_run = m_new;
        const float msl = (m_run == -INFINITY) ? 0.f : m_run;
        // pass 2: P = 2^(s c2 - m) (packed FMA, one ex2 per key) as bf16 pairs over the
        // first 64 columns of S_m (half hh's P lands on columns already read), the row sum
        // from the fp32 values
        const float2 nm2 = make_float2(-msl, -msl);
        float2 acc0 = make_float2(0.f, 0.f), acc1 = make_float2(0.f, 0.f);
#pragma unroll 1
        for (int hh = 0; hh < 2; ++hh) {
          float sc[64];
          tmem_ld32(tS + hh * 64, sc);
          tmem_ld32(tS + hh * 64 + 32, sc + 32);
          tmem_ld_wait();
          if (part) {
#pragma unroll
            for (int i = 0; i < 64; ++i) sc[i] = hh * 64 + i < lim ? sc[i] : -INFINITY;
          }
#pragma unroll
          for (int c = 0; c < 2; ++c) {
            uint32_t w[16];
#pragma unroll
            for (int i = 0; i < 16; ++i) {
              float2 x = ffma2(make_float2(sc[32 * c + 2 * i], sc[32 * c + 2 * i + 1]), c2x2, nm2);
              x.x = ex2(x.x);
              x.y = ex2(x.y);
              if (i & 1) acc1 = fadd2(acc1, x); else acc0 = fadd2(acc0, x);
              w[i] = pack_bf16x2(x.x, x.y);
            }
            tmem_st16(tS + hh * 32 + c * 16, w);
          }
        }
        tmem_st_wait();
        l_run += (acc0.x + acc0.y) + (acc1.x + acc1.y);
      }
      fence_before_sync();
      __syncwarp();
      if (lane == 0) mbar_arrive(&p_full[mt]);
    }
    if (ok && nt_me > 0) {
      ok = mbar_wait(&o_done[mt], (uint32_t)(nt_me - 1) & 1u);
      fence_after_sync();
    }
    if (!ok) s_abort = 1;
  }
  // join: every MMA done (the MMA warp drained), every warpgroup out of its loop
  fence_before_sync();
  __syncthreads();
  fence_after_sync();

  // dual mode: each chain's (m_run, l_run, m_true) per row, in the (drained) V slots
  float (*sMrg)[3][kMTile] = reinterpret_cast<float (*)[3][kMTile]>(sVs);
  if (dual && softmax_warp) {
    const int rl = quarter * 32 + lane;
    sMrg[mt][0][rl] = m_run;
    sMrg[mt][1][rl] = l_run;
    sMrg[mt][2][rl] = m_true;
    asm volatile("bar.sync 1, %0;\n" ::"r"(kSoftThreads) : "memory");
  }
  if (softmax_warp && wg_on) {
    const int64_t prow = ((int64_t)bh * A.P.S + split) * A.P.Rp + r;
    const int prow0 = (int)(((int64_t)bh * A.P.S + split) * A.P.Rp + wrow0);
    if (s_abort != 0) {
      if (threadIdx.x == 0) atomicExch(A.err, 1);
      if (row_ok && (!dual || mt == 0)) A.P.ml[prow] = make_float2(NAN, NAN);
    } else if (!dual) {
      // the exact max: l under m_run times 2^(m_run - m_true) <= 1; o = acc / l is the same
      // under either reference
      if (row_ok) {
        const float fix = (m_true == -INFINITY) ? 1.f : ex2(m_run - m_true * c2);
        A.P.ml[prow] = make_float2(m_true * A.scale, l_run * fix);
      }
      const float inv = l_run > 0.f ? 1.f / l_run : 0.f;
      if (warp_rows) {
        if (ntiles > 0 && A.tma_out) {
          // the warp's 32 rows -> two 32-row x 64-channel boxes in the (drained) ring,
          // 128-byte swizzled, then two TMA box stores by lane 0
          uint8_t* box = ring + warp * (2 * kOutBox);
#pragma unroll 1
          for (int c = 0; c < kD / 32; ++c) {
            float o[32];
            tmem_ld32(tO + c * 32, o);
            tmem_ld_wait();
            uint8_t* line = box + (c >> 1) * kOutBox + lane * 128;
#pragma unroll
            for (int qq = 0; qq < 4; ++qq) {
              float f8[8];
#pragma unroll
              for (int i = 0; i < 8; ++i) f8[i] = o[8 * qq + i] * inv;
              const int chunk = (c & 1) * 4 + qq;
              *reinterpret_cast<uint4*>(line + ((chunk ^ (lane & 7)) << 4)) = float8_to_bf16x8(f8);
            }
          }
          fence_proxy_async();
          __syncwarp();
          if (lane == 0) {
            tma::store_2d(&A.omap, 0, prow0, box);
            tma::store_2d(&A.omap, 64, prow0, box + kOutBox);
            tma::store_commit();
            if (A.fuse) {   // other CTAs read these rows: complete, then order for generic loads
              tma::store_wait_all();
              asm volatile("fence.proxy.async.global;\n" ::: "memory");
            } else {
              tma::store_wait_read();
            }
          }
          __syncwarp();
        } else {
          __nv_bfloat16* obase = reinterpret_cast<__nv_bfloat16*>(A.P.o);
#pragma unroll 1
          for (int c = 0; c < kD / 32; ++c) {
            float o[32];
            if (ntiles > 0) {
              tmem_ld32(tO + c * 32, o);
              tmem_ld_wait();
            }
#pragma unroll
            for (int i = 0; i < 32; ++i) o[i] = ntiles > 0 ? o[i] * inv : 0.f;
            if (row_ok) {
              uint4* dst = reinterpret_cast<uint4*>(obase + prow * kD + c * 32);
#pragma unroll
              for (int qq = 0; qq < 4; ++qq) dst[qq] = float8_to_bf16x8(o + 8 * qq);
            }
          }
        }
      }
    } else {
      // dual: merge the two chains' (m, l, O) per row; warpgroup m writes channels
      // [64m, 64m+64) of the warp's 32 rows
      const int rl = quarter * 32 + lane;
      const float m0 = sMrg[0][0][rl], m1 = sMrg[1][0][rl];
      const float M = fmaxf(m0, m1);
      const float f0 = (M == -INFINITY || nt0 == 0) ? 0.f : ex2(m0 - M);
      const float f1 = (M == -INFINITY || nt1 == 0) ? 0.f : ex2(m1 - M);
      const float l = sMrg[0][1][rl] * f0 + sMrg[1][1][rl] * f1;
      const float mtr = fmaxf(sMrg[0][2][rl], sMrg[1][2][rl]);
      if (row_ok && mt == 0) {
        const float fix = (mtr == -INFINITY) ? 1.f : ex2(M - mtr * c2);
        A.P.ml[prow] = make_float2(mtr * A.scale, l * fix);
      }
      const float inv = l > 0.f ? 1.f / l : 0.f;
      const float g0 = f0 * inv, g1 = f1 * inv;
      const uint32_t tO0 = taddr + lane_base + kColO + 64 * mt;   // chain 0's O, this half
      const uint32_t tO1 = tO0 + 128;                              // chain 1's O
      if (warp_rows) {
        float o[64];
        if (ntiles > 0) {
          tmem_ld32(tO0, o);
          tmem_ld32(tO0 + 32, o + 32);
          tmem_ld_wait();
#pragma unroll
          for (int i = 0; i < 64; ++i) o[i] *= g0;
          if (nt1 > 0) {
#pragma unroll
            for (int c = 0; c < 2; ++c) {
              float o1[32];
              tmem_ld32(tO1 + 32 * c, o1);
              tmem_ld_wait();
#pragma unroll
              for (int i = 0; i < 32; ++i) o[32 * c + i] = fmaf(o1[i], g1, o[32 * c + i]);
            }
          }
        } else {
#pragma unroll
          for (int i = 0; i < 64; ++i) o[i] = 0.f;
        }
        if (ntiles > 0 && A.tma_out) {
          uint8_t* box = ring + warp * kOutBox;
          uint8_t* line = box + lane * 128;
#pragma unroll
          for (int qq = 0; qq < 8; ++qq)
            *reinterpret_cast<uint4*>(line + ((qq ^ (lane & 7)) << 4)) = float8_to_bf16x8(o + 8 * qq);
          fence_proxy_async();
          __syncwarp();
          if (lane == 0) {
            tma::store_2d(&A.omap, 64 * mt, prow0, box);
            tma::store_commit();
            if (A.fuse) {
              tma::store_wait_all();
              asm volatile("fence.proxy.async.global;\n" ::: "memory");
            } else {
              tma::store_wait_read();
            }
          }
          __syncwarp();
        } else if (row_ok) {
          uint4* dst = reinterpret_cast<uint4*>(reinterpret_cast<__nv_bfloat16*>(A.P.o) + prow * kD + 64 * mt);
#pragma unroll
          for (int qq = 0; qq < 8; ++qq) dst[qq] = float8_to_bf16x8(o + 8 * qq);
        }
      }
    }
  }
  fence_before_sync();
  __syncthreads();
  fence_after_sync();
  if (warp == 0) tmem_dealloc(taddr, kTmemCols);
  if (!A.fuse) return;

  // ---- fused merge: every CTA of the (head, row block) group is resident (cooperative
  // launch); the last to arrive advances the group's generation, the others wait for it
  __threadfence();
  __syncthreads();
  if (threadIdx.x == 0) {
    bool ok = true;
    const unsigned prev = atomicAdd(&A.fm.sync[group].x, 1u);
    if (prev == gridDim.x - 1) {
      A.fm.sync[group].x = 0u;   // ready for the next call
      __threadfence();
      atomicAdd(&A.fm.sync[group].y, 1u);
    } else {
      const uint64_t t0 = global_ns();
      while (ld_acquire_u32(&A.fm.sync[group].y) == gen0) {
        if (global_ns() - t0 > kMergeWaitNs) {
          ok = false;
          atomicExch(A.err, 1);
          break;
        }
        __nanosleep(128);
      }
    }
    s_merge_ok = ok ? 1 : 0;
  }
  __syncthreads();
  // this split's share of the group's rows, one warp per row (weights scratch in the ring)
  const int R_blk = min(kRowTile, R - r0);
  const int per = (R_blk + (int)gridDim.x - 1) / (int)gridDim.x;
  const int lo = split * per, hi = min(R_blk, lo + per);
  float* sW = reinterpret_cast<float*>(ring) + warp * kCombineMaxSplits;
  __nv_bfloat16* out = reinterpret_cast<__nv_bfloat16*>(A.fm.out);
  for (int rr = lo + warp; rr < hi; rr += kWarps) {
    if (s_merge_ok) {
      combine_row<__nv_bfloat16, __nv_bfloat16>(A.q, H, A.P, A.nsplit, A.cur.Tc > 0, out, A.fm.so[0], A.fm.so[1],
                                                A.fm.so[2], A.fm.m_p, A.fm.l_p, A.fm.o_p, bh, r0 + rr, sW);
    } else if (lane == 0) {   // a split never arrived: the row is reported as NaN
      const int rw = r0 + rr;
      const int g = rw / T, t = rw - (rw / T) * T;
      __nv_bfloat16* dst = out + (int64_t)b * A.fm.so[0] + (int64_t)(h * G + g) * A.fm.so[1] + (int64_t)t * A.fm.so[2];
      for (int d = 0; d < kD; ++d) dst[d] = __float2bfloat16_rn(NAN);
    }
  }
}

bool tma_map_rows(CUtensorMap* map, const void* base, int B, int H, int n, const int64_t s[3]) {
  // bf16 [B][H][n][128] with element strides s (b, h, row); box: 64 channels x 128 rows
  const uint64_t dims[4] = {128, (uint64_t)n, (uint64_t)H, (uint64_t)B};
  const uint64_t strides[3] = {(uint64_t)s[2] * 2, (uint64_t)s[1] * 2, (uint64_t)s[0] * 2};
  const uint32_t box[4] = {64, (uint32_t)kBN, 1, 1};
  return make_tma_map_bf16_4d(map, base, dims, strides, box);
}

}  // namespace

int fa_key_tile() { return kBN; }

bool fa_eligible(const ma_rows& q, const ma_kv& kv, const int64_t* idx, const ma_block& cur, int n_keys) {
  const bool prefix_ok = n_keys == 0 || (kv.layout == MA_KV_DENSE && kv.dtype == MA_BF16 && !idx && !kv.mask &&
                                         !kv.pages && !kv.lens);
  return q.dtype == MA_BF16 && q.D == kD && q.T <= kRowTile && kRowTile % q.T == 0 && prefix_ok &&
         (n_keys > 0 || cur.Tc > 0);
}

int launch_attn_partial_fa(const ma_rows& q, const ma_kv& kv, int H, const ma_block& cur, float scale,
                           int causal_block, int q_pos0, int c_pos0, int n_keys, int split_len, int nsplit,
                           const Partials& P, int* err, const FusedMerge* fm, bool* fused, cudaStream_t st) {
  *fused = false;
  if (!fa_eligible(q, kv, nullptr, cur, n_keys) || !(scale > 0.f) || !P.o_bf16 || split_len % kBN != 0)
    return MA_ERR_UNSUPPORTED;
  Args A;
  memset(&A, 0, sizeof(A));
  A.q = q;
  A.kv = kv;
  A.cur = cur;
  A.scale = scale;
  A.H = H;
  A.causal_block = causal_block;
  A.q_pos0 = q_pos0;
  A.c_pos0 = c_pos0;
  A.n_keys = n_keys;
  A.split_len = split_len;
  A.nsplit = nsplit;
  A.P = P;
  A.err = err;
  if (n_keys > 0 && !(tma_map_rows(&A.kmap, kv.kf, q.B, H, kv.nf, kv.skf) &&
                      tma_map_rows(&A.vmap, kv.vf, q.B, H, kv.nf, kv.svf)))
    return MA_ERR_UNSUPPORTED;
  if (cur.Tc > 0 && !(tma_map_rows(&A.ckmap, cur.k, q.B, H, cur.Tc, cur.sk) &&
                      tma_map_rows(&A.cvmap, cur.v, q.B, H, cur.Tc, cur.sv)))
    return MA_ERR_UNSUPPORTED;
  {
    const uint64_t dims[4] = {128, (uint64_t)q.T, (uint64_t)q.Hq, (uint64_t)q.B};
    const uint64_t strides[3] = {(uint64_t)q.sq[2] * 2, (uint64_t)q.sq[1] * 2, (uint64_t)q.sq[0] * 2};
    const uint32_t box[4] = {64, (uint32_t)q.T, (uint32_t)(kRowTile / q.T), 1};
    if (!make_tma_map_bf16_4d(&A.qmap, q.q, dims, strides, box)) return MA_ERR_UNSUPPORTED;
  }
  const int G = q.Hq / H;
  const int R = G * q.T;
  // partial rows [BH * S * Rp][D] bf16, stored by 32-row x 64-channel boxes
  const uint64_t prow_total = (uint64_t)q.B * H * P.S * P.Rp;
  A.tma_out = (P.Rp % 32 == 0 && prow_total < (1ull << 31) &&
               make_tma_map_2d(&A.omap, true, P.o, kD, prow_total, kD * 2, 64, 32)) ? 1 : 0;
  dim3 grid(P.S, q.B * H, (R + kRowTile - 1) / kRowTile);
  auto kernel = attn_partial_fa;
  if (cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmemBytes) != cudaSuccess)
    return MA_ERR_CUDA;
  // fused merge: one wave of resident CTAs (cooperative launch), when each split's share of
  // the rows is one pass of its warps
  const int rows_per_split = (std::min(kRowTile, R) + (int)grid.x - 1) / (int)grid.x;
  if (fm != nullptr && (int)(grid.y * grid.z) <= fm->sync_slots && (int)grid.x <= kCombineMaxSplits &&
      rows_per_split <= kWarps) {
    int dev = 0, coop = 0, per_sm = 0;
    if (cudaGetDevice(&dev) == cudaSuccess &&
        cudaDeviceGetAttribute(&coop, cudaDevAttrCooperativeLaunch, dev) == cudaSuccess && coop &&
        cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kernel, kThreads, kSmemBytes) == cudaSuccess &&
        (long long)grid.x * grid.y * grid.z <= (long long)per_sm * device_sm_count()) {
      Args Af = A;
      Af.fuse = 1;
      Af.fm = *fm;
      cudaLaunchConfig_t cfg = {};
      cfg.gridDim = grid;
      cfg.blockDim = dim3(kThreads);
      cfg.dynamicSmemBytes = kSmemBytes;
      cfg.stream = st;
      cudaLaunchAttribute attr[1];
      attr[0].id = cudaLaunchAttributeCooperative;
      attr[0].val.cooperative = 1;
      cfg.attrs = attr;
      cfg.numAttrs = 1;
      if (cudaLaunchKernelEx(&cfg, kernel, Af) == cudaSuccess) {
        *fused = true;
        return MA_OK;
      }
      (void)cudaGetLastError();
    }
  }
  return launch_pdl(kernel, grid, dim3(kThreads), kSmemBytes, st, A) == cudaSuccess ? MA_OK : MA_ERR_CUDA;
}

}  // namespace ma
