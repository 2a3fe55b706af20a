// Split-K attention over [prefix | current block] (or [read set | current block]) with
// Blackwell tcgen05 MMAs, for bf16 queries over a bf16 (or dequantized packed) cache.
//
// CTA = 8 softmax warps + 1 MMA warp over up to 256 query rows of one KV head (two
// M = 128 tiles; the R = G*T rows of the GQA group share every K/V tile, so a tile
// crosses HBM once per KV head). One thread per row: softmax warp w reads TMEM lane
// quarter w % 4 of M tile w / 4.
// Keys stream through a ring of kStages shared-memory stages of 64 keys (K and V):
//   * contiguous bf16 rows (dense prefix without a live mask, the current block) and the
//     query rows arrive by TMA, issued by the MMA warp -- a box load per 64 channels, the
//     hardware applies the 128-byte swizzle the MMA descriptors expect;
//   * gathered rows (a read set), masked prefixes and packed (k4v4) rows are staged by
//     the softmax warps with cp.async / dequantizing stores into the same layout.
// Warp specialization (tcgen05 MMA issue blocks the issuing thread while the tensor core
// is busy, so no softmax row waits on it): lane 0 of the MMA warp issues every TMA load
// and MMA, the two roles meet on mbarriers only --
//   full[stage] -> S(t) = Q K(t)^T into S buffer t&1 -> s_full -> softmax warps read S(t)
//   -> s_free (the buffer may take S(t+2)) ... P(t) in shared memory -> p_full ->
//   O += P(t) V(t) -> o_done (P buffer and O free again) and empty[stage] (refill).
// S(t+1) is issued before P(t) is waited for, so the tensor core computes the next
// logits under the current softmax.
// The running max is lazy in base-2 units: O in TMEM is rescaled only when a row max
// grows by more than kLazy (natural units), so every p = 2^(u - m) stays <= e^kLazy; the
// exact max is tracked beside it and folded into l at the end. Each split writes per
// row (m, l) and its normalized output o = acc / l as bf16 (ma_common.cuh), staged in
// shared memory and stored by TMA, one 32-row box pair per warp. Every wait on the tensor
// core or TMA is bounded; a timeout sets the CTA's abort flag, the CTA drains its
// in-flight work (bounded), reports through the error word and marks its rows NaN.
// Semantics follow src/maskahead/kernels/splitk.py:115-190 (_sk_fwd).
#include <string.h>

#include <algorithm>

#include "ma_combine.cuh"
#include "ma_kernels.cuh"
#include "ma_cp_async.cuh"
#include "ma_stage.cuh"
#include "ma_tcgen05.cuh"
#include "ma_tma.cuh"

namespace ma {

namespace {

using namespace tc;

constexpr int kSoftWarps = 8;              // one query row per thread
constexpr int kSoftThreads = kSoftWarps * 32;
constexpr int kWarps = kSoftWarps + 1;      // + the MMA / TMA warp
constexpr int kThreads = kWarps * 32;
constexpr int kMTile = 128;
constexpr int kRowTile = 2 * kMTile;        // 256 rows per CTA
constexpr int kBN = 64;                     // keys per tile
constexpr int kD = 128;
constexpr int kChunks = kD / 8;
constexpr int kStages = 4;                  // key tiles in the ring
constexpr float kLog2e = 1.4426950408889634f;
constexpr float kLazyLog2 = 8.0f * kLog2e;  // rescale O when a row max grows by more than e^8

constexpr int kQBlock = kRowTile * 128;               // one 64-channel block of all rows: 32 KB
constexpr int kQBytes = 2 * kQBlock;                  // 64 KB: [d block][256 rows][128 B]
constexpr int kKVBlock = kBN * 128;                   // 8 KB: [64 rows][128 B]
constexpr int kKVBytes = 2 * kKVBlock;                // 16 KB per K or V tile
constexpr int kStageBytes = 2 * kKVBytes;             // K tile | V tile
constexpr int kPBytes = kRowTile * kBN * 2;           // 32 KB: [M tile][128 rows][128 B]
constexpr int kSmemBytes = 1024 + kQBytes + kStages * kStageBytes + kPBytes;   // 225 KB
constexpr uint32_t kTmemCols = 512;
constexpr uint32_t kColS = 0;                         // S buffers at 0 and 128, M tile m at +64m
constexpr uint32_t kColO = 256;                       // O: M tile m at 256 + 128m
constexpr uint32_t kTileTx = kStageBytes;             // bytes a K+V tile brings by TMA
constexpr int kOutBox = 32 * 128;                     // output box: 32 rows x 64 bf16 channels

struct __align__(64) Args {
  CUtensorMap kmap, vmap;       // prefix K/V [B][H][n][D] (dense, unmasked prefix)
  CUtensorMap ckmap, cvmap;     // current block K/V [B][H][Tc][D]
  CUtensorMap qmap;             // queries [B][Hq][T][D]
  CUtensorMap omap;             // partial outputs [BH * S * Rp][D] bf16 (stores)
  ma_rows q;
  ma_kv kv;
  ma_block cur;
  const int64_t* idx;
  int64_t si0, si1;
  float scale;
  int H, causal_block, q_pos0, c_pos0, n_keys, split_len, nsplit;
  int tma_kv, tma_cur, tma_q;   // which operands arrive by TMA
  int tma_out;                  // partial rows leave by TMA
  Partials P;
  int* err;
  int fuse;                     // merge the splits in this (cooperative) launch
  FusedMerge fm;
};

// Per-thread staging of keys [j0, j0+kBN): gathered, masked or packed rows.
template <bool PACKED>
__device__ __forceinline__ void stage_rows(const Args& A, int b, int h, bool is_cur, int j0, int end, uint8_t* sK,
                                           uint8_t* sV, uint8_t* sOk, const float* sKch) {
  if (PACKED && !is_cur) {   // packed prefix rows: wide loads, dequantized into the tile
    stage::packed_tile<kBN, true, true>(A.kv, A.H, b, h, j0, end, A.idx, A.si0, A.si1, sK, sV, sOk, sKch,
                                        threadIdx.x, kSoftThreads);
    return;
  }
  const __nv_bfloat16* ck = reinterpret_cast<const __nv_bfloat16*>(A.cur.k);
  const __nv_bfloat16* cv = reinterpret_cast<const __nv_bfloat16*>(A.cur.v);
  const __nv_bfloat16* kf = reinterpret_cast<const __nv_bfloat16*>(A.kv.kf);
  const __nv_bfloat16* vf = reinterpret_cast<const __nv_bfloat16*>(A.kv.vf);
  const int ch = threadIdx.x % kChunks;                 // fixed channel chunk per thread
  for (int jj = threadIdx.x / kChunks; jj < kBN; jj += kSoftThreads / kChunks) {
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
        int sb = b, row = slot - A.kv.nq;
        if (!PACKED && A.kv.pages) kv_page(A.kv, b, row, sb, row);   // a paged dense cache
        cp_async16(smem_addr(dk), kf + (int64_t)sb * A.kv.skf[0] + (int64_t)h * A.kv.skf[1] + (int64_t)row * A.kv.skf[2] + ch * 8, true);
        cp_async16(smem_addr(dv), vf + (int64_t)sb * A.kv.svf[0] + (int64_t)h * A.kv.svf[1] + (int64_t)row * A.kv.svf[2] + ch * 8, true);
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

// TMA loads of key tile [j0, j0+kBN) into a stage (MMA warp, lane 0).
__device__ __forceinline__ void tma_tile(const Args& A, bool is_cur, int b, int h, int j0, uint8_t* sK, uint8_t* sV,
                                         uint64_t* full) {
  const CUtensorMap* km = is_cur ? &A.ckmap : &A.kmap;
  const CUtensorMap* vm = is_cur ? &A.cvmap : &A.vmap;
  tma::expect_tx(full, kTileTx);
  tma::load_4d(sK, km, 0, j0, h, b, full);
  tma::load_4d(sK + kKVBlock, km, 64, j0, h, b, full);
  tma::load_4d(sV, vm, 0, j0, h, b, full);
  tma::load_4d(sV + kKVBlock, vm, 64, j0, h, b, full);
}

// S(t) = Q K(t)^T for every M tile into S buffer `buf` (MMA warp, lane 0). The M tiles
// alternate per K step, so consecutive MMAs never accumulate into the same TMEM columns.
__device__ __forceinline__ void issue_s(uint32_t taddr, const uint8_t* sQ, const uint8_t* sK, int mtiles, int buf,
                                        uint64_t* mbar) {
  const uint32_t idS = idesc_bf16(kMTile, kBN, false, false);
  const uint32_t qa = smem_addr(sQ);
  const uint32_t ka = smem_addr(sK);
#pragma unroll
  for (int kk = 0; kk < kD / 16; ++kk) {
    const uint64_t bd = smem_desc(ka + (kk >> 2) * kKVBlock + (kk & 3) * 32, 16, 1024);
    for (int m = 0; m < mtiles; ++m) {
      const uint64_t ad = smem_desc(qa + m * (kMTile * 128) + (kk >> 2) * kQBlock + (kk & 3) * 32, 16, 1024);
      mma_bf16(taddr + kColS + buf * 128 + m * kBN, ad, bd, idS, kk > 0);
    }
  }
  mma_commit(mbar);
}

// O += P(t) V(t) for every M tile (MMA warp, lane 0), M tiles alternating per K step.
__device__ __forceinline__ void issue_pv(uint32_t taddr, const uint8_t* sP, const uint8_t* sV, int mtiles,
                                         bool first) {
  const uint32_t idO = idesc_bf16(kMTile, kD, false, true);
  const uint32_t pa = smem_addr(sP);
  const uint32_t va = smem_addr(sV);
#pragma unroll
  for (int kk = 0; kk < kBN / 16; ++kk) {
    const uint64_t bd = smem_desc(va + kk * 2048, kKVBlock, 1024);
    for (int m = 0; m < mtiles; ++m) {
      const uint64_t ad = smem_desc(pa + m * (kMTile * kBN * 2) + kk * 32, 16, 1024);
      mma_bf16(taddr + kColO + m * kD, ad, bd, idO, !(first && kk == 0));
    }
  }
}

__device__ __forceinline__ void mbar_arrive(uint64_t* mbar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];\n" ::"r"(smem_addr(mbar)) : "memory");
}
// barrier among the softmax warps only (the MMA warp runs on)
__device__ __forceinline__ void softmax_sync() { asm volatile("bar.sync 1, %0;\n" ::"n"(kSoftThreads) : "memory"); }
__device__ __forceinline__ void prefetch_map(const CUtensorMap* m) {
  asm volatile("prefetch.tensormap [%0];\n" ::"l"(reinterpret_cast<uint64_t>(m)) : "memory");
}

template <bool PACKED>
__global__ void __launch_bounds__(kThreads, 1) attn_partial_tc(const __grid_constant__ Args A) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sQ = smem;                                   // [2 d blocks][256 rows][128 B]
  uint8_t* ring = sQ + kQBytes;                         // [stage][K tile | V tile]
  uint8_t* sP = ring + kStages * kStageBytes;           // [2 M tiles][128 rows][128 B]
  __shared__ __align__(16) uint8_t sOkb[kStages][kBN];
  __shared__ float sKch[kD];                            // token-mode key divisor of (b, h)
  __shared__ uint32_t s_taddr;
  // full: a stage's tile landed; s_full/s_free: an S buffer computed / read out;
  // p_full: P(t) written; o_done: O += P(t) V(t) completed; empty: a stage's last reader
  // (the P.V MMA) completed
  __shared__ __align__(8) uint64_t full[kStages], empty[kStages], s_full[2], s_free[2], p_full, o_done, q_full,
      mbar_fin;
  __shared__ int s_abort, s_merge_ok;
  __shared__ unsigned s_gen;

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
  const int mt = (warp >> 2) & 1, quarter = warp & 3;
  const int row_in_tile = quarter * 32 + lane;               // = the thread's TMEM lane
  const int r = r0 + mt * kMTile + row_in_tile;              // the thread's query row
  const int wrow0 = r0 + mt * kMTile + quarter * 32;         // the warp's first row
  const bool softmax_warp = warp < kSoftWarps;
  const bool warp_rows = softmax_warp && mt < mtiles && wrow0 < R;   // warp-uniform
  const bool row_ok = softmax_warp && r < R && mt < mtiles;
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
  const int ntiles = end > begin ? (end - begin + kBN - 1) / kBN : 0;
  const float c2 = A.scale * kLog2e;                         // logit -> base-2 exponent units

  const int group = bh * gridDim.z + blockIdx.z;            // fused merge: (head, row block)
  if (A.fuse && threadIdx.x == 0) s_gen = *reinterpret_cast<volatile const unsigned*>(&A.fm.sync[group].y);
  if (threadIdx.x == kSoftThreads) {   // MMA warp, lane 0
    if (A.tma_q) prefetch_map(&A.qmap);
    if (tma_kv) {
      prefetch_map(is_cur ? &A.ckmap : &A.kmap);
      prefetch_map(is_cur ? &A.cvmap : &A.vmap);
    }
    for (int st = 0; st < kStages; ++st) {
      mbar_init(&full[st], tma_kv ? 1 : kSoftWarps);
      mbar_init(&empty[st], 1);
    }
    mbar_init(&s_full[0], 1);
    mbar_init(&s_full[1], 1);
    mbar_init(&s_free[0], kSoftWarps);
    mbar_init(&s_free[1], kSoftWarps);
    mbar_init(&p_full, kSoftWarps);
    mbar_init(&o_done, 1);
    mbar_init(&q_full, A.tma_q ? 1 : kSoftWarps);
    mbar_init(&mbar_fin, 1);
    s_abort = 0;
    asm volatile("fence.mbarrier_init.release.cluster;\n" ::: "memory");
  }
  if (warp == 0) tmem_alloc(&s_taddr, kTmemCols);
  fence_before_sync();
  __syncthreads();
  fence_after_sync();
  const uint32_t taddr = s_taddr;

  // softmax-warp state (used after the join by the epilogue)
  const uint32_t lane_base = (uint32_t)(quarter * 32) << 16;
  const uint32_t tS = taddr + lane_base + kColS + mt * kBN;   // this warp's S rows (buffer 0)
  const uint32_t tO = taddr + lane_base + kColO + mt * kD;    // this warp's O rows
  float m_run = -INFINITY, l_run = 0.f;   // base-2 exponent reference (lazy) and the sum under it
  float m_true = -INFINITY;                // exact running max of the raw logits q.k
  if (!softmax_warp) {
    // ------------------------------------------------------------ MMA / TMA warp
    if (lane == 0) {
      pdl_wait();   // with a programmatic launch, the inputs may come from the kernel before
      bool ok = true;
      bool q_ok = !A.tma_q;
      int issued = 0, waited = 0;   // TMA tiles issued / seen complete
      if (A.tma_q) {  // queries: TMA boxes of whole query heads (T divides the row tile)
        const int hq0 = h * G + r0 / T;
        tma::expect_tx(&q_full, (uint32_t)(kRowTile * 256));
        tma::load_4d(sQ, &A.qmap, 0, 0, hq0, b, &q_full);
        tma::load_4d(sQ + kQBlock, &A.qmap, 64, 0, hq0, b, &q_full);
      }
      if (tma_kv) {
        for (int st = 0; st < kStages && st < ntiles; ++st) {
          uint8_t* sK = ring + st * kStageBytes;
          tma_tile(A, is_cur, b, h, begin + st * kBN, sK, sK + kKVBytes, &full[st]);
          issued = st + 1;
        }
      }
      if (ntiles > 0) {
        ok = mbar_wait(&q_full, 0);
        q_ok = q_ok || ok;
      }
      for (int t = 0; t < ntiles && ok; ++t) {
        const int stage = t % kStages;
        // tile t landed, S buffer t&1 read out (S(t-2))
        ok = mbar_wait(&full[stage], (uint32_t)(t / kStages) & 1u);
        if (ok && tma_kv) waited = t + 1;
        if (ok && t >= 2) ok = mbar_wait(&s_free[t & 1], (uint32_t)((t - 2) >> 1) & 1u);
        if (!ok || s_abort) break;
        fence_after_sync();
        issue_s(taddr, sQ, ring + stage * kStageBytes, mtiles, t & 1, &s_full[t & 1]);
        if (t >= 1) {
          // O += P(t-1) V(t-1) once the softmax warps wrote P(t-1)
          ok = mbar_wait(&p_full, (uint32_t)(t - 1) & 1u);
          if (!ok) break;
          fence_after_sync();
          const int sp = (t - 1) % kStages;
          issue_pv(taddr, sP, ring + sp * kStageBytes + kKVBytes, mtiles, t == 1);
          mma_commit(&o_done);
          mma_commit(&empty[sp]);
          // refill the stage of tile t-2 (its P.V was issued one tile ago) with tile t-2+kStages
          const int tr = t - 2 + kStages;
          if (tma_kv && t >= 2 && tr < ntiles) {
            const int sr = (t - 2) % kStages;
            ok = mbar_wait(&empty[sr], (uint32_t)((t - 2) / kStages) & 1u);
            if (!ok) break;
            uint8_t* sK = ring + sr * kStageBytes;
            tma_tile(A, is_cur, b, h, begin + tr * kBN, sK, sK + kKVBytes, &full[sr]);
            issued = tr + 1;
          }
        }
      }
      if (ok && ntiles > 0) {
        ok = mbar_wait(&p_full, (uint32_t)(ntiles - 1) & 1u);
        if (ok) {
          fence_after_sync();
          const int sp = (ntiles - 1) % kStages;
          issue_pv(taddr, sP, ring + sp * kStageBytes + kKVBytes, mtiles, ntiles == 1);
          mma_commit(&o_done);
        }
      }
      if (!ok) s_abort = 1;
      // drain (bounded): every MMA issued, every TMA load still in flight
      mma_commit(&mbar_fin);
      mbar_wait(&mbar_fin, 0, 20000000ull);
      if (!q_ok) mbar_wait(&q_full, 0, 20000000ull);
      for (int tt = waited; tt < issued; ++tt)
        mbar_wait(&full[tt % kStages], (uint32_t)(tt / kStages) & 1u, 20000000ull);
    }
    __syncwarp();
  } else {
    // ------------------------------------------------------------ softmax warps
    // (with a programmatic launch: the read set, the partials workspace and the outputs
    // may still be in use by the kernel before)
    pdl_wait();
    bool ok = true;
    if (!A.tma_q && ntiles > 0) {  // queries by cp.async (waited at once: a rare layout)
      const __nv_bfloat16* qp = reinterpret_cast<const __nv_bfloat16*>(A.q.q);
      const int ch = threadIdx.x % kChunks;
      for (int rr = threadIdx.x / kChunks; rr < kRowTile; rr += kSoftThreads / kChunks) {
        const int rq = r0 + rr;
        uint8_t* dst = sQ + (ch >> 3) * kQBlock + rr * 128 + (((ch & 7) ^ (rr & 7)) << 4);
        if (rq < R) {
          const int g = rq / T, t = rq - (rq / T) * T;
          cp_async16(smem_addr(dst), qp + (int64_t)b * A.q.sq[0] + (int64_t)(h * G + g) * A.q.sq[1] + (int64_t)t * A.q.sq[2] + ch * 8, true);
        } else {
          *reinterpret_cast<uint4*>(dst) = make_uint4(0, 0, 0, 0);
        }
      }
      cp_async_commit();
      cp_async_wait<0>();
      fence_proxy_async();
      __syncwarp();
      if (lane == 0) mbar_arrive(&q_full);
    }
    if (PACKED && !is_cur && A.kv.layout == MA_KV_PACKED_TOKEN) {
      if (threadIdx.x < kD) sKch[threadIdx.x] = A.kv.kchan[(int64_t)b * A.kv.skc[0] + (int64_t)h * A.kv.skc[1] + threadIdx.x];
      softmax_sync();
    }
    // packed token-mode prefix: the register-pipelined staging (ma_stage.cuh), one
    // (row, channel group) item per thread; tiles 0 and 1 up front, then tile t+2 is
    // dequantized at iteration t from loads issued one iteration earlier
    const bool tokpipe = PACKED && !is_cur && A.kv.layout == MA_KV_PACKED_TOKEN;
    const int tj = threadIdx.x >> 2, tg = threadIdx.x & 3;
    stage::TokItem pR, pC;
    int sI = -1;
    if (tokpipe) {
      for (int u = 0; u < 2 && u < ntiles; ++u) {
        stage::TokItem it;
        stage::tok_locate(A.kv, A.H, b, h, stage::tok_slot(b, h, begin + u * kBN + tj, end, A.idx, A.si0, A.si1), it);
        stage::tok_fetch(A.kv, h, tg, it);
        uint8_t* sK = ring + u * kStageBytes;
        stage::tok_store<kBN>(A.kv, b, h, tj, tg, it, sK, sK + kKVBytes, sOkb[u], sKch);
      }
      fence_proxy_async();
      __syncwarp();
      if (lane == 0)
        for (int u = 0; u < 2 && u < ntiles; ++u) mbar_arrive(&full[u]);
      pR.ok = pC.ok = false;
      if (2 < ntiles) {
        stage::tok_locate(A.kv, A.H, b, h, stage::tok_slot(b, h, begin + 2 * kBN + tj, end, A.idx, A.si0, A.si1), pR);
        stage::tok_fetch(A.kv, h, tg, pR);
      }
      if (3 < ntiles)
        stage::tok_locate(A.kv, A.H, b, h, stage::tok_slot(b, h, begin + 3 * kBN + tj, end, A.idx, A.si0, A.si1), pC);
      if (4 < ntiles) sI = stage::tok_slot(b, h, begin + 4 * kBN + tj, end, A.idx, A.si0, A.si1);
    } else if (!tma_kv) {
      // prologue: tiles 0 .. kStages-2, one cp.async group each (tile i = group i)
      for (int st = 0; st < kStages - 1; ++st) {
        uint8_t* sK = ring + st * kStageBytes;
        if (st < ntiles) stage_rows<PACKED>(A, b, h, is_cur, begin + st * kBN, end, sK, sK + kKVBytes, sOkb[st], sKch);
        cp_async_commit();
      }
      if (ntiles > 0) {
        cp_async_wait<kStages - 2>();
        fence_proxy_async();
        __syncwarp();
        if (lane == 0) mbar_arrive(&full[0]);
      }
    }
    for (int t = 0; t < ntiles; ++t) {
      const int stage = t % kStages;
      const int j0 = begin + t * kBN;
      // (a) S(t): this thread's 64 logits; the S buffer is free again once read out
      ok = mbar_wait(&s_full[t & 1], (uint32_t)(t >> 1) & 1u);
      fence_after_sync();
      float s[kBN];
      if (warp_rows) {
        const uint32_t ts = tS + (uint32_t)(t & 1) * 128u;
        tmem_ld32(ts, s);
        tmem_ld32(ts + 32, s + 32);
        tmem_ld_wait();
      }
      fence_before_sync();
      __syncwarp();
      if (lane == 0) mbar_arrive(&s_free[t & 1]);
      // (b) token pipeline: tile t+2 into its stage (its previous tile's P.V completed one
      // iteration ago), loads advance one tile; cp.async path: tile t+1's copies landed
      if (tokpipe) {
        if (t + 2 < ntiles) {
          uint8_t* sK = ring + ((t + 2) % kStages) * kStageBytes;
          stage::tok_store<kBN>(A.kv, b, h, tj, tg, pR, sK, sK + kKVBytes, sOkb[(t + 2) % kStages], sKch);
          fence_proxy_async();
          __syncwarp();
          if (lane == 0) mbar_arrive(&full[(t + 2) % kStages]);
        }
        pR = pC;
        if (t + 3 < ntiles) stage::tok_fetch(A.kv, h, tg, pR);
        if (t + 4 < ntiles) stage::tok_locate(A.kv, A.H, b, h, sI, pC);
        sI = (t + 5 < ntiles) ? stage::tok_slot(b, h, begin + (t + 5) * kBN + tj, end, A.idx, A.si0, A.si1) : -1;
      } else if (!tma_kv) {
        cp_async_wait<kStages - 3>();
        fence_proxy_async();
        __syncwarp();
        if (lane == 0 && t + 1 < ntiles) mbar_arrive(&full[(t + 1) % kStages]);
      }
      if (!ok) s_abort = 1;
      softmax_sync();   // validity bytes of the staged tiles; a common view of the abort flag
      if (s_abort) {
        ok = false;
        break;
      }
      // (c) visibility mask and the row's tile max (raw logits; scale > 0 keeps the order)
      float tmax = -INFINITY;
      if (warp_rows) {
        const int lim = vis_end - j0;               // keys i >= lim are hidden from this row
        bool full_tile = lim >= kBN;
        uint32_t okw[kBN / 4];
        if (!tma_kv) {
          const uint4* okv = reinterpret_cast<const uint4*>(sOkb[stage]);
#pragma unroll
          for (int q4 = 0; q4 < kBN / 16; ++q4) {
            const uint4 w = okv[q4];
            okw[4 * q4] = w.x;
            okw[4 * q4 + 1] = w.y;
            okw[4 * q4 + 2] = w.z;
            okw[4 * q4 + 3] = w.w;
          }
#pragma unroll
          for (int w = 0; w < kBN / 4; ++w) full_tile = full_tile && okw[w] == 0x01010101u;
        } else {
#pragma unroll
          for (int w = 0; w < kBN / 4; ++w) okw[w] = 0x01010101u;   // TMA tiles: keys < end exist
        }
        if (!full_tile) {
#pragma unroll
          for (int i = 0; i < kBN; ++i) {
            const bool vis = ((okw[i >> 2] >> (8 * (i & 3))) & 0xFFu) != 0 && i < lim;
            s[i] = vis ? s[i] : -INFINITY;
          }
        }
        float m4[4] = {s[0], s[1], s[2], s[3]};
#pragma unroll
        for (int i = 4; i < kBN; ++i) m4[i & 3] = fmaxf(m4[i & 3], s[i]);
        tmax = fmaxf(fmaxf(m4[0], m4[1]), fmaxf(m4[2], m4[3]));
      }
      // (d) O += P(t-1) V(t-1) complete: O and the P buffer are free (and, on the cp.async
      // path, tile t-1's stage: refill it with tile t + kStages - 1)
      if (t > 0) {
        ok = mbar_wait(&o_done, (uint32_t)(t - 1) & 1u);
        fence_after_sync();
        if (!ok) s_abort = 1;
      }
      if (!tma_kv && !tokpipe) {
        const int tn = t + kStages - 1;
        const int sn = tn % kStages;
        if (tn < ntiles && ok) {
          uint8_t* sK = ring + sn * kStageBytes;
          stage_rows<PACKED>(A, b, h, is_cur, begin + tn * kBN, end, sK, sK + kKVBytes, sOkb[sn], sKch);
        }
        cp_async_commit();
      }
      // (e) lazy rescale of O, then P(t) = 2^(u - m) as bf16 into shared memory
      if (warp_rows) {
        m_true = fmaxf(m_true, tmax);
        const float m_new = fmaxf(m_run, tmax * c2);
        const bool grow = t > 0 && m_new > m_run + kLazyLog2;
        if (__any_sync(0xffffffffu, grow)) {   // warp-collective TMEM access
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
        if (t == 0) m_run = m_new;
        const float msl = (m_run == -INFINITY) ? 0.f : m_run;
        float ps[4] = {0.f, 0.f, 0.f, 0.f};
        uint8_t* prow = sP + mt * (kMTile * kBN * 2);
#pragma unroll
        for (int c = 0; c < kBN / 8; ++c) {
          float p8[8];
#pragma unroll
          for (int i = 0; i < 8; ++i) {
            p8[i] = ex2(fmaf(s[c * 8 + i], c2, -msl));   // exp2(-inf) = 0 for hidden keys
            ps[i & 3] += p8[i];
          }
          *reinterpret_cast<uint4*>(prow + kmajor_off(row_in_tile, c, kMTile)) = float8_to_bf16x8(p8);
        }
        l_run += (ps[0] + ps[1]) + (ps[2] + ps[3]);
      }
      // (f) P(t) visible to the tensor core -> the MMA warp issues O += P(t) V(t)
      fence_proxy_async();
      fence_before_sync();
      __syncwarp();
      if (lane == 0) mbar_arrive(&p_full);
    }
    if (ok && ntiles > 0) {
      ok = mbar_wait(&o_done, (uint32_t)(ntiles - 1) & 1u);
      fence_after_sync();
    }
    if (!ok) s_abort = 1;
    cp_async_wait<0>();
  }
  // join: both roles done (or aborted); the epilogue runs on the softmax warps
  fence_before_sync();
  __syncthreads();
  fence_after_sync();
  if (softmax_warp) {
    const int64_t prow = ((int64_t)bh * A.P.S + split) * A.P.Rp + r;
    if (s_abort != 0) {
      if (threadIdx.x == 0) atomicExch(A.err, 1);
      if (row_ok) A.P.ml[prow] = make_float2(NAN, NAN);
    } else {
      // report the exact max: l under m_run times 2^(m_run - m_true) <= 1; o = acc / l is
      // the same under either reference
      if (row_ok) {
        const float fix = (m_true == -INFINITY) ? 1.f : ex2(m_run - m_true * c2);
        A.P.ml[prow] = make_float2(m_true * A.scale, l_run * fix);
      }
      const float inv = l_run > 0.f ? 1.f / l_run : 0.f;
      if (warp_rows) {
        __nv_bfloat16* obase = reinterpret_cast<__nv_bfloat16*>(A.P.o);
        if (ntiles > 0 && A.tma_out) {
          // the warp's 32 rows -> two 32-row x 64-channel boxes in the ring (free now:
          // every load was consumed and every MMA has completed), 128-byte swizzled
          // (chunk q of line i at q ^ (i & 7)), then two TMA box stores by lane 0
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
            const int prow0 = (int)(((int64_t)bh * A.P.S + split) * A.P.Rp + wrow0);
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
          // plain row stores (no tensor map), or zeros for a split without keys
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
      while (ld_acquire_u32(&A.fm.sync[group].y) == s_gen) {
        if (global_ns() - t0 > A.fm.wait_ns) {
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
      const int r = r0 + rr;
      const int g = r / T, t = r - (r / T) * T;
      __nv_bfloat16* dst = out + (int64_t)b * A.fm.so[0] + (int64_t)(h * G + g) * A.fm.so[1] + (int64_t)t * A.fm.so[2];
      for (int d = 0; d < kD; ++d) dst[d] = __float2bfloat16_rn(NAN);
    }
  }
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
                           int n_keys, int split_len, int nsplit, const Partials& P, int* err, const FusedMerge* fm,
                           bool* fused, cudaStream_t st) {
  *fused = false;
  if (q.D != kD || !(scale > 0.f) || !P.o_bf16) return MA_ERR_UNSUPPORTED;
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
  A.tma_kv = (kv.layout == MA_KV_DENSE && kv.dtype == MA_BF16 && !idx && !kv.mask && !kv.pages && !kv.lens &&
              n_keys > 0 &&
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
  // partial rows [BH * S * Rp][D] bf16, stored by 32-row x 64-channel boxes: a warp's box
  // never leaves its (b, h, split) block when Rp is a multiple of 32
  const uint64_t prow_total = (uint64_t)q.B * H * P.S * P.Rp;
  A.tma_out = (P.Rp % 32 == 0 && prow_total < (1ull << 31) &&
               make_tma_map_2d(&A.omap, true, P.o, kD, prow_total, kD * 2, 64, 32)) ? 1 : 0;
  dim3 grid(P.S, q.B * H, (R + kRowTile - 1) / kRowTile);
  auto go = [&](auto kernel) -> int {
    if (cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmemBytes) != cudaSuccess)
      return MA_ERR_CUDA;
    // fused merge: one wave of resident CTAs (cooperative launch), merge scratch in place
    // (only when each split's share of the rows is one pass of its warps: the merge of a
    // row is two dependent global round trips, so more rows per CTA serialize)
    const int rows_per_split = (std::min(kRowTile, R) + (int)grid.x - 1) / (int)grid.x;
    if (fm != nullptr && (int)(grid.y * grid.z) <= fm->sync_slots && (int)grid.x <= kCombineMaxSplits &&
        q.dtype == MA_BF16 && rows_per_split <= kWarps) {
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
  };
  return kv.layout != MA_KV_DENSE ? go(attn_partial_tc<true>) : go(attn_partial_tc<false>);
}

}  // namespace ma
