// Split-K attention over [prefix | current block] (or [read set | current block]) with
// Blackwell tcgen05 MMAs, for bf16 queries over a bf16 (or dequantized packed) cache.
//
// CTA = 16 warps = up to 256 query rows of one KV head (two M = 128 tiles; the R = G*T
// rows of the GQA group share every K/V tile, so a tile crosses HBM once per KV head).
// Two threads own each row -- warps w and w + 4 of an M tile read the same TMEM lane
// quarter, one the first and one the second 32 logits of every tile -- and exchange
// their row maxima through shared memory.
// Keys stream through a ring of kStages shared-memory tiles of 64 keys (the whole
// per-CTA slice is in flight from the start):
//   * contiguous bf16 rows (dense prefix without a live mask, the current block) and the
//     query rows arrive by TMA -- one thread issues a box load per 64 channels, the
//     hardware applies the 128-byte swizzle the MMA descriptors expect;
//   * gathered rows (a read set), masked prefixes and packed (k4v4) rows go through
//     per-thread cp.async / dequantizing stores into the same layout.
// Per tile: thread 0 issues S_m = Q_m K^T (tcgen05.mma, M 128, N 64, accumulator in TMEM)
// and commits to an mbarrier; each thread loads its 32 logits of its row (tcgen05.ld),
// masks them, updates the running max lazily (O in TMEM is rescaled
// only when a row max grows by more than kLazy, so exp(s - m) <= e^kLazy) and writes
// P = exp(s - m) as bf16 into shared memory; thread 0 issues O_m += P_m V. The exact row
// max is tracked beside the lazy one and folded into (l, acc) at the end. The split's
// (m, l, acc) per row goes to the partial format (ma_common.cuh) through shared memory
// as coalesced row stores. Every wait on the tensor core or TMA is bounded; a timeout
// sets the CTA's abort flag, the CTA stops and reports through the error word.
// Semantics follow src/maskahead/kernels/splitk.py:115-190 (_sk_fwd).
#include <string.h>

#include "ma_kernels.cuh"
#include "ma_mma.cuh"
#include "ma_tcgen05.cuh"
#include "ma_tma.cuh"

namespace ma {

namespace {

using namespace tc;

constexpr int kWarps = 16;
constexpr int kThreads = kWarps * 32;
constexpr int kHalf = 32;                   // logits of a tile per thread (two threads per row)
constexpr int kMTile = 128;
constexpr int kRowTile = 2 * kMTile;        // 256 rows per CTA
constexpr int kBN = 64;                     // keys per tile
constexpr int kD = 128;
constexpr int kChunks = kD / 8;
constexpr int kStages = 3;                  // key tiles in flight
constexpr float kLazy = 8.0f;               // rescale O when a row max grows by more than this
constexpr float kLog2e = 1.4426950408889634f;

constexpr int kQBlock = kRowTile * 128;               // one 64-channel block of all rows: 32 KB
constexpr int kQBytes = 2 * kQBlock;                  // 64 KB: [d block][256 rows][128 B]
constexpr int kKVBlock = kBN * 128;                   // 8 KB: [64 rows][128 B]
constexpr int kKVBytes = 2 * kKVBlock;                // 16 KB per K or V tile
constexpr int kPBytes = kRowTile * kBN * 2;           // 32 KB: [M tile][128 rows][128 B]
constexpr int kSmemBytes = 1024 + kQBytes + 2 * kStages * kKVBytes + kPBytes;
constexpr uint32_t kTmemCols = 512;
constexpr uint32_t kColS = 0, kColO = 256;
constexpr uint32_t kTileTx = 2 * kKVBytes;            // bytes a K+V tile brings by TMA

struct __align__(64) Args {
  CUtensorMap kmap, vmap;       // prefix K/V [B][H][n][D] (dense, unmasked prefix)
  CUtensorMap ckmap, cvmap;     // current block K/V [B][H][Tc][D]
  CUtensorMap qmap;             // queries [B][Hq][T][D]
  CUtensorMap accmap;           // partial acc rows [BH * S * Rp][D] fp32 (stores)
  ma_rows q;
  ma_kv kv;
  ma_block cur;
  const int64_t* idx;
  int64_t si0, si1;
  float scale;
  int H, causal_block, q_pos0, c_pos0, n_keys, split_len, nsplit;
  int tma_kv, tma_cur, tma_q;   // which operands arrive by TMA
  int tma_acc;                  // partial rows leave by TMA
  Partials P;
  int* err;
};

// Per-thread staging of keys [j0, j0+kBN): gathered, masked or packed rows.
template <bool PACKED>
__device__ __forceinline__ void stage_rows(const Args& A, int b, int h, bool is_cur, int j0, int end, uint8_t* sK,
                                           uint8_t* sV, uint8_t* sOk) {
  const __nv_bfloat16* ck = reinterpret_cast<const __nv_bfloat16*>(A.cur.k);
  const __nv_bfloat16* cv = reinterpret_cast<const __nv_bfloat16*>(A.cur.v);
  const __nv_bfloat16* kf = reinterpret_cast<const __nv_bfloat16*>(A.kv.kf);
  const __nv_bfloat16* vf = reinterpret_cast<const __nv_bfloat16*>(A.kv.vf);
  const int ch = threadIdx.x % kChunks;                 // fixed channel chunk per thread
  for (int jj = threadIdx.x / kChunks; jj < kBN; jj += kThreads / kChunks) {
    const int j = j0 + jj;
    bool ok = j < end;
    const uint32_t off = kmajor_off(jj, ch, kBN);
    uint8_t* dk = sK + off;
    uint8_t* dv = sV + off;
    if (is_cur) {
      if (ok) {
        cp_async16(smem_addr(dk), ck + (int64_t)b * A.cur.sk[0] + (int64_t)h * A.cur.sk[1] + (int64_t)j * A.cur.sk[2] + ch * 8, true);
        cp_async16(smem_addr(dv), cv + (int64_t)b * A.cur.sv[0] + (int64_t)h * A.cur.sv[1] + (int64_t)j * A.cur.sv[2] + ch * 8, true);
      }
    } else {
      int slot = j;
      if (ok && A.idx) slot = (int)A.idx[(int64_t)b * A.si0 + (int64_t)h * A.si1 + j];
      ok = ok && kv_live(A.kv, A.H, b, h, slot);
      if (ok && (!PACKED || slot >= A.kv.nq)) {
        const int row = slot - A.kv.nq;
        cp_async16(smem_addr(dk), kf + (int64_t)b * A.kv.skf[0] + (int64_t)h * A.kv.skf[1] + (int64_t)row * A.kv.skf[2] + ch * 8, true);
        cp_async16(smem_addr(dv), vf + (int64_t)b * A.kv.svf[0] + (int64_t)h * A.kv.svf[1] + (int64_t)row * A.kv.svf[2] + ch * 8, true);
      } else if (ok) {
        float fk[8], fv[8];
        kv_read8<true>(A.kv, b, h, slot, ch, fk);
        kv_read8<false>(A.kv, b, h, slot, ch, fv);
        *reinterpret_cast<uint4*>(dk) = float8_to_bf16x8(fk);
        *reinterpret_cast<uint4*>(dv) = float8_to_bf16x8(fv);
      }
    }
    if (!ok) {  // zero rows: dead or missing slots contribute exact zeros to P.V
      *reinterpret_cast<uint4*>(dk) = make_uint4(0, 0, 0, 0);
      *reinterpret_cast<uint4*>(dv) = make_uint4(0, 0, 0, 0);
    }
    if (ch == 0) sOk[jj] = ok ? 1 : 0;
  }
}

// Issue the loads of key tile [j0, j0+kBN) into a stage (TMA or per-thread cp.async).
template <bool PACKED>
__device__ __forceinline__ void issue_tile(const Args& A, bool use_tma, int b, int h, bool is_cur, int j0, int end,
                                           uint8_t* sK, uint8_t* sV, uint8_t* sOk, uint64_t* full) {
  if (use_tma) {
    if (threadIdx.x == 0) {
      const CUtensorMap* km = is_cur ? &A.ckmap : &A.kmap;
      const CUtensorMap* vm = is_cur ? &A.cvmap : &A.vmap;
      tma::expect_tx(full, kTileTx);
      tma::load_4d(sK, km, 0, j0, h, b, full);
      tma::load_4d(sK + kKVBlock, km, 64, j0, h, b, full);
      tma::load_4d(sV, vm, 0, j0, h, b, full);
      tma::load_4d(sV + kKVBlock, vm, 64, j0, h, b, full);
    }
    if (threadIdx.x < kBN) sOk[threadIdx.x] = (j0 + (int)threadIdx.x < end) ? 1 : 0;
  } else {
    stage_rows<PACKED>(A, b, h, is_cur, j0, end, sK, sV, sOk);
  }
  cp_async_commit();  // one group per tile (empty on the TMA path)
}

template <bool PACKED>
__global__ void __launch_bounds__(kThreads, 1) attn_partial_tc(const __grid_constant__ Args A) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sQ = smem;                                   // [2 d blocks][256 rows][128 B]
  uint8_t* sKV = sQ + kQBytes;                          // [stage][K tile | V tile]
  uint8_t* sP = sKV + 2 * kStages * kKVBytes;           // [2 M tiles][128 rows][128 B]
  __shared__ __align__(16) uint8_t sOkb[kStages][kBN];
  __shared__ float sMax[2][kRowTile];                   // per row: the two halves' tile maxima
  __shared__ float sSum[kRowTile];
  __shared__ uint32_t s_taddr;
  __shared__ __align__(8) uint64_t mbar_s, mbar_o, mbar_q, full[kStages];
  __shared__ int s_abort;

  const int split = blockIdx.x;
  const int bh = blockIdx.y;
  const int H = A.H;
  const int b = bh / H, h = bh - (bh / H) * H;
  const int T = A.q.T;
  const int G = A.q.Hq / H;
  const int R = G * T;
  const int r0 = blockIdx.z * kRowTile;
  const int mtiles = min(2, (R - r0 + kMTile - 1) / kMTile);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int mt = warp >> 3, quarter = warp & 3, chalf = (warp >> 2) & 1;
  const int row_in_tile = quarter * 32 + lane;               // = the thread's TMEM lane
  const int r = r0 + mt * kMTile + row_in_tile;              // the thread's query row
  const bool row_ok = r < R && mt < mtiles;
  const int t_row = row_ok ? r % T : 0;

  const bool is_cur = split == A.nsplit;
  const bool tma_kv = is_cur ? A.tma_cur != 0 : A.tma_kv != 0;
  int begin, end;
  if (is_cur) {
    begin = 0;
    end = A.cur.Tc;
  } else {
    begin = split * A.split_len;
    end = min(A.n_keys, begin + A.split_len);
  }
  // Keys visible to this row: block-causal over the current block -- key j is visible iff
  // (c_pos0 + j) / cb <= (q_pos0 + t) / cb, i.e. j < vis_end (one division per thread).
  int vis_end = end;
  if (is_cur && A.causal_block > 0)
    vis_end = min(end, ((A.q_pos0 + t_row) / A.causal_block + 1) * A.causal_block - A.c_pos0);
  if (!row_ok) vis_end = begin;

  if (threadIdx.x == 0) {
    mbar_init(&mbar_s, 1);
    mbar_init(&mbar_o, 1);
    mbar_init(&mbar_q, 1);
    for (int st = 0; st < kStages; ++st) mbar_init(&full[st], 1);
    s_abort = 0;
    asm volatile("fence.mbarrier_init.release.cluster;\n" ::: "memory");
  }
  __syncthreads();

  // queries: TMA boxes of whole query heads when T divides the row tile, else cp.async
  if (A.tma_q) {
    if (threadIdx.x == 0) {
      const int hq0 = h * G + r0 / T;
      tma::expect_tx(&mbar_q, (uint32_t)(kRowTile * 256));
      tma::load_4d(sQ, &A.qmap, 0, 0, hq0, b, &mbar_q);
      tma::load_4d(sQ + kQBlock, &A.qmap, 64, 0, hq0, b, &mbar_q);
    }
  } else {
    const __nv_bfloat16* qp = reinterpret_cast<const __nv_bfloat16*>(A.q.q);
    const int ch = threadIdx.x % kChunks;
    for (int rr = threadIdx.x / kChunks; rr < kRowTile; rr += kThreads / kChunks) {
      const int rq = r0 + rr;
      uint8_t* dst = sQ + (ch >> 3) * kQBlock + rr * 128 + (((ch & 7) ^ (rr & 7)) << 4);
      if (rq < R) {
        const int g = rq / T, t = rq - (rq / T) * T;
        cp_async16(smem_addr(dst), qp + (int64_t)b * A.q.sq[0] + (int64_t)(h * G + g) * A.q.sq[1] + (int64_t)t * A.q.sq[2] + ch * 8, true);
      } else {
        *reinterpret_cast<uint4*>(dst) = make_uint4(0, 0, 0, 0);
      }
    }
  }
  // prologue: the first kStages tiles
  for (int st = 0; st < kStages; ++st) {
    const int j0 = begin + st * kBN;
    uint8_t* sK = sKV + 2 * st * kKVBytes;
    if (j0 < end) issue_tile<PACKED>(A, tma_kv, b, h, is_cur, j0, end, sK, sK + kKVBytes, sOkb[st], &full[st]);
    else cp_async_commit();
  }
  if (warp == 0) tmem_alloc(&s_taddr, kTmemCols);
  fence_before_sync();
  __syncthreads();
  fence_after_sync();
  const uint32_t taddr = s_taddr;
  const uint32_t lane_base = (uint32_t)(quarter * 32) << 16;
  const uint32_t tS = taddr + lane_base + kColS + mt * kBN + chalf * kHalf;   // this thread's S half-row
  const uint32_t tO = taddr + lane_base + kColO + mt * kD + chalf * (kD / 2);  // this thread's O half-row
  const int rloc = mt * kMTile + row_in_tile;                                   // row within the CTA

  const uint32_t idS = idesc_bf16(kMTile, kBN, false, false);
  const uint32_t idO = idesc_bf16(kMTile, kD, false, true);
  float m_run = -INFINITY, l_run = 0.f;   // exponent reference (lazy) and the sum under it
  float m_true = -INFINITY;                // exact running max
  uint32_t phase_s = 0, phase_o = 0;
  int stage = 0, tile = 0;
  bool first = true;
  bool aborted = false;
  bool q_ready = !A.tma_q;

  for (int j0 = begin; j0 < end; j0 += kBN, ++tile) {
    uint8_t* sKs = sKV + 2 * stage * kKVBytes;
    uint8_t* sVs = sKs + kKVBytes;
    cp_async_wait<kStages - 1>();   // the per-thread part of this tile (one group per tile)
    bool ok_w = true;
    if (!q_ready) {
      ok_w = mbar_wait(&mbar_q, 0);
      q_ready = true;
    }
    if (tma_kv) ok_w = mbar_wait(&full[stage], (uint32_t)(tile / kStages) & 1u) && ok_w;
    if (!ok_w) s_abort = 1;
    fence_proxy_async();
    fence_before_sync();
    __syncthreads();
    fence_after_sync();
    if (s_abort) {
      aborted = true;
      break;
    }
    if (threadIdx.x == 0) {
      for (int m = 0; m < mtiles; ++m) {
        const uint32_t qa = smem_addr(sQ + m * (kMTile * 128));
        const uint32_t ka = smem_addr(sKs);
#pragma unroll
        for (int kk = 0; kk < kD / 16; ++kk) {
          const uint64_t ad = smem_desc(qa + (kk >> 2) * kQBlock + (kk & 3) * 32, 16, 1024);
          const uint64_t bd = smem_desc(ka + (kk >> 2) * kKVBlock + (kk & 3) * 32, 16, 1024);
          mma_bf16(taddr + kColS + m * kBN, ad, bd, idS, kk > 0);
        }
      }
      mma_commit(&mbar_s);
    }
    const bool ok_s = mbar_wait(&mbar_s, phase_s);
    phase_s ^= 1;
    fence_after_sync();
    if (!ok_s) s_abort = 1;
    float s[kHalf];
    float tmax = -INFINITY;
    const int lim = vis_end - j0 - chalf * kHalf;    // keys i >= lim of this half are hidden
    if (mt < mtiles) {
      tmem_ld32(tS, s);
      tmem_ld_wait();
      // validity bytes of this half tile, 16 at a time
      uint32_t okw[kHalf / 4];
      {
        const uint4* okv = reinterpret_cast<const uint4*>(sOkb[stage] + chalf * kHalf);
#pragma unroll
        for (int q4 = 0; q4 < kHalf / 16; ++q4) {
          const uint4 w = okv[q4];
          okw[4 * q4] = w.x;
          okw[4 * q4 + 1] = w.y;
          okw[4 * q4 + 2] = w.z;
          okw[4 * q4 + 3] = w.w;
        }
      }
      bool full_tile = lim >= kHalf;
#pragma unroll
      for (int w = 0; w < kHalf / 4; ++w) full_tile = full_tile && okw[w] == 0x01010101u;
      if (full_tile) {  // every key of the half tile visible (the common case)
#pragma unroll
        for (int i = 0; i < kHalf; ++i) {
          s[i] *= A.scale;
          tmax = fmaxf(tmax, s[i]);
        }
      } else {
#pragma unroll
        for (int i = 0; i < kHalf; ++i) {
          const bool vis = ((okw[i >> 2] >> (8 * (i & 3))) & 0xFFu) != 0 && i < lim;
          s[i] = vis ? s[i] * A.scale : -INFINITY;
          tmax = fmaxf(tmax, s[i]);
        }
      }
      sMax[chalf][rloc] = tmax;
    }
    __syncthreads();
    if (mt < mtiles) {
      tmax = fmaxf(sMax[0][rloc], sMax[1][rloc]);     // the row's tile max (both halves agree)
      m_true = fmaxf(m_true, tmax);
      const float m_new = fmaxf(m_run, tmax);
      const bool grow = !first && m_new > m_run + kLazy;
      if (__any_sync(0xffffffffu, grow)) {
        // rescale this thread's half of O (and of l) for rows whose max grew a lot;
        // warp-collective TMEM access
        const float alpha = grow ? ex2((m_run - m_new) * kLog2e) : 1.f;
#pragma unroll 1
        for (int c = 0; c < kD / 64; ++c) {
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
      if (first) m_run = m_new;
      const float msl = (m_run == -INFINITY) ? 0.f : m_run * kLog2e;
      float psum = 0.f;
      uint8_t* prow = sP + mt * (kMTile * kBN * 2);
#pragma unroll
      for (int c = 0; c < kHalf / 8; ++c) {
        float p8[8];
#pragma unroll
        for (int i = 0; i < 8; ++i) {
          p8[i] = ex2(fmaf(s[c * 8 + i], kLog2e, -msl));   // exp2(-inf) = 0 for hidden keys
          psum += p8[i];
        }
        *reinterpret_cast<uint4*>(prow + kmajor_off(row_in_tile, chalf * (kHalf / 8) + c, kMTile)) =
            float8_to_bf16x8(p8);
      }
      l_run += psum;
    }
    fence_proxy_async();
    fence_before_sync();
    __syncthreads();
    fence_after_sync();
    if (s_abort) {
      aborted = true;
      break;
    }
    if (threadIdx.x == 0) {
      for (int m = 0; m < mtiles; ++m) {
        const uint32_t pa = smem_addr(sP + m * (kMTile * kBN * 2));
        const uint32_t va = smem_addr(sVs);
#pragma unroll
        for (int kk = 0; kk < kBN / 16; ++kk) {
          const uint64_t ad = smem_desc(pa + kk * 32, 16, 1024);
          const uint64_t bd = smem_desc(va + kk * 2048, kKVBlock, 1024);
          mma_bf16(taddr + kColO + m * kD, ad, bd, idO, !(first && kk == 0));
        }
      }
      mma_commit(&mbar_o);
    }
    const bool ok_o = mbar_wait(&mbar_o, phase_o);
    phase_o ^= 1;
    fence_after_sync();
    if (!ok_o) s_abort = 1;
    // refill this stage with the tile kStages ahead (the MMAs reading it have completed)
    const int jn = j0 + kStages * kBN;
    if (jn < end) issue_tile<PACKED>(A, tma_kv, b, h, is_cur, jn, end, sKs, sVs, sOkb[stage], &full[stage]);
    else cp_async_commit();
    first = false;
    stage = (stage + 1) % kStages;
  }

  // report the exact max: (l, acc) under m_run times exp(m_run - m_true) <= 1; the two
  // threads of a row hold halves of l
  const float fix = (m_true == -INFINITY) ? 1.f : ex2((m_run - m_true) * kLog2e);
  if (chalf == 1) sSum[rloc] = l_run;
  __syncthreads();
  if (!aborted && row_ok && chalf == 0) {
    const int64_t prow = ((int64_t)bh * A.P.S + split) * A.P.Rp + r;
    A.P.ml[prow] = make_float2(m_true, first ? 0.f : (l_run + sSum[rloc]) * fix);
    if (first) {  // no key in this split
      float* dst = A.P.acc + prow * kD;
#pragma unroll 1
      for (int c = 0; c < kD; c += 4) *reinterpret_cast<float4*>(dst + c) = make_float4(0.f, 0.f, 0.f, 0.f);
    }
  }
  // O rows -> shared memory in the 128-byte-swizzled layout of four 32-column boxes
  // ([box][256 rows][128 B], chunk q of row r at q ^ (r & 7): conflict-free writes), then
  // one thread stores the CTA's rows with four TMA box stores. The K/V ring is free now.
  // (Plain per-warp stores are the fallback when the tensor map is unavailable.)
  if (!aborted && !first) {
    cp_async_wait<0>();
    __syncthreads();
    uint8_t* sO = sKV;
    if (mt < mtiles) {
#pragma unroll 1
      for (int c = 0; c < kD / 64; ++c) {
        float o[32];
        tmem_ld32(tO + c * 32, o);
        tmem_ld_wait();
        uint8_t* box = sO + (chalf * 2 + c) * (kRowTile * 128) + rloc * 128;
#pragma unroll
        for (int q = 0; q < 8; ++q)
          *reinterpret_cast<float4*>(box + ((q ^ (rloc & 7)) << 4)) =
              make_float4(o[4 * q] * fix, o[4 * q + 1] * fix, o[4 * q + 2] * fix, o[4 * q + 3] * fix);
      }
    }
    fence_proxy_async();
    __syncthreads();
    const int64_t prow0 = ((int64_t)bh * A.P.S + split) * A.P.Rp + r0;
    if (A.tma_acc) {
      if (threadIdx.x == 0) {
#pragma unroll
        for (int c = 0; c < kD / 32; ++c) tma::store_2d(&A.accmap, c * 32, (int)prow0, sO + c * (kRowTile * 128));
        tma::store_commit();
        tma::store_wait_read();
      }
    } else {
      for (int rr = warp; rr < mtiles * kMTile; rr += kWarps) {
        if (r0 + rr >= R) continue;
        float* dst = A.P.acc + (prow0 + rr) * kD;
#pragma unroll
        for (int c = 0; c < kD / 32; ++c) {
          const uint8_t* box = sO + c * (kRowTile * 128) + rr * 128;
          dst[c * 32 + lane] = reinterpret_cast<const float*>(box + (((lane >> 2) ^ (rr & 7)) << 4))[lane & 3];
        }
      }
    }
  }
  if (aborted) {
    if (threadIdx.x == 0) atomicExch(A.err, 1);
    // let in-flight tensor-core work drain (bounded) before the TMEM is released
    mbar_wait(&mbar_s, phase_s);
    mbar_wait(&mbar_o, phase_o);
    if (row_ok && chalf == 0) {
      const int64_t prow = ((int64_t)bh * A.P.S + split) * A.P.Rp + r;
      A.P.ml[prow] = make_float2(NAN, NAN);
    }
  }
  fence_before_sync();
  __syncthreads();
  fence_after_sync();
  if (warp == 0) tmem_dealloc(taddr, kTmemCols);
}

bool tma_map_rows(CUtensorMap* map, const void* base, int B, int H, int n, const int64_t s[3]) {
  // bf16 [B][H][n][128] with element strides s (b, h, row); box: 64 channels x 64 rows
  const uint64_t dims[4] = {128, (uint64_t)n, (uint64_t)H, (uint64_t)B};
  const uint64_t strides[3] = {(uint64_t)s[2] * 2, (uint64_t)s[1] * 2, (uint64_t)s[0] * 2};
  const uint32_t box[4] = {64, (uint32_t)kBN, 1, 1};
  return make_tma_map_bf16_4d(map, base, dims, strides, box);
}

}  // namespace

int tc_row_tile() { return kRowTile; }
int tc_key_tile() { return kBN; }

int launch_attn_partial_tc(const ma_rows& q, const ma_kv& kv, int H, const ma_block& cur, float scale,
                           int causal_block, int q_pos0, int c_pos0, const int64_t* idx, int64_t si0, int64_t si1,
                           int n_keys, int split_len, int nsplit, const Partials& P, int* err, cudaStream_t st) {
  if (q.D != kD) return MA_ERR_UNSUPPORTED;
  Args A;
  memset(&A, 0, sizeof(A));
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
  A.err = err;
  const int G = q.Hq / H;
  const int R = G * q.T;
  // TMA for contiguous bf16 rows: the dense prefix without a mask, the current block, and
  // the queries when a row tile is made of whole query heads
  A.tma_kv = (kv.layout == MA_KV_DENSE && kv.dtype == MA_BF16 && !idx && !kv.mask && n_keys > 0 &&
              tma_map_rows(&A.kmap, kv.kf, q.B, H, kv.nf, kv.skf) &&
              tma_map_rows(&A.vmap, kv.vf, q.B, H, kv.nf, kv.svf)) ? 1 : 0;
  A.tma_cur = (cur.Tc > 0 && tma_map_rows(&A.ckmap, cur.k, q.B, H, cur.Tc, cur.sk) &&
               tma_map_rows(&A.cvmap, cur.v, q.B, H, cur.Tc, cur.sv)) ? 1 : 0;
  if (q.T <= kRowTile && kRowTile % q.T == 0) {
    const uint64_t dims[4] = {128, (uint64_t)q.T, (uint64_t)q.Hq, (uint64_t)q.B};
    const uint64_t strides[3] = {(uint64_t)q.sq[2] * 2, (uint64_t)q.sq[1] * 2, (uint64_t)q.sq[0] * 2};
    const uint32_t box[4] = {64, (uint32_t)q.T, (uint32_t)(kRowTile / q.T), 1};
    A.tma_q = make_tma_map_bf16_4d(&A.qmap, q.q, dims, strides, box) ? 1 : 0;
  }
  // partial rows: [BH * S * Rp][D] fp32, stored by 32-column x 256-row boxes (the row tile
  // never reaches past its (b, h, split) block: Rp is a multiple of the row tile)
  A.tma_acc = make_tma_map_f32_2d(&A.accmap, P.acc, kD, (uint64_t)q.B * H * P.S * P.Rp, kD * 4, 32, kRowTile) ? 1 : 0;
  dim3 grid(P.S, q.B * H, (R + kRowTile - 1) / kRowTile);
  auto go = [&](auto kernel) -> int {
    if (cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmemBytes) != cudaSuccess)
      return MA_ERR_CUDA;
    kernel<<<grid, kThreads, kSmemBytes, st>>>(A);
    return cudaGetLastError() == cudaSuccess ? MA_OK : MA_ERR_CUDA;
  };
  return kv.layout != MA_KV_DENSE ? go(attn_partial_tc<true>) : go(attn_partial_tc<false>);
}

}  // namespace ma
