// Split-K attention over [prefix | current block] for contiguous bf16 keys/values read by
// TMA: one 128-row M tile per CTA (or two, below), S double-buffered and P kept in tensor
// memory.
//
// CTA = 8 softmax warps, 1 MMA warp and 1 TMA warp over 128 query rows (r0..r0+127 of one
// KV head's R = G*T rows, ordered g*T + t) and one key range (a split of the prefix, or the
// current block). Keys come in tiles of 128: K and V each through 3 slots of 32 KB (a K
// slot is refilled once its S was read, a V slot once its P.V completed: the MMA warp
// releases the slot on kfree / vfree, the TMA warp issues the load -- a TMA issue can hold
// its thread for hundreds of cycles, time the MMA issuer cannot give). Tensor memory (512
// columns): S(t) = Q K(t)^T in buffer t&1 (columns [128(t&1), +128)), and two output
// accumulators, O0 for the even tiles in [256, 384) and O1 for the odd ones in [384, 512).
// Per tile t:
//   MMA warp   S(t) = Q K(t)^T (8 MMAs 128x128x16, A = Q, B = K, K-major in shared memory),
//              issued once K(t) is loaded and P.V(t-2) (whose P lives in the buffer) issued
//   softmax    the four warps of group t&1 (warps 4(t&1)..+3), warp w holding rows 32(w&3)..
//              and all 128 keys: the row max, lazy rescale of its O(t&1), P = 2^(u - m)
//              rounded to bf16 written as bf16 pairs over S's columns 0..31 and 64..95
//   MMA warp   O(t&1) += P V(t) (8 MMAs, A = P from tensor memory, B = V MN-major)
// so the two groups work on consecutive tiles at once (the two warps of a sub-partition
// alternate between exponentials and tensor-memory traffic) while the tensor core runs the
// next S. Each group keeps its own running max and row sum (a rescale of O first waits for
// the group's previous P.V: lazy, only when the max grows by more than e^8); the epilogue
// merges the two states.
// Per split: (m, l) and o = acc / l as bf16 (ma_common.cuh), stored by TMA, the merge as
// in ma_attention_tc.cu (fused into a cooperative launch when it is one pass). With at
// most 16 splits a row block's splits form one thread-block cluster and merge on chip:
// every split keeps its partial in shared memory and the others pull their share of the
// rows from it, or -- every split one key tile, as in the sub-steps over the compact
// cache -- every split copies each CTA's share into that CTA with the bulk-copy engine
// (one copy per destination, counted on the receiver's mbarrier).
// Every wait is bounded. Semantics follow src/maskahead/kernels/splitk.py:115-190.
//
// Row-tile pairs (PAIR): with more than 128 rows per KV head (R = 224 for 28 query heads
// over 4 KV heads and 32-row blocks) one CTA takes rows r0..r0+255 as two M tiles that
// share every K and V tile: warp group g owns M tile g (S(u) for u = 2t + g in buffer g,
// its own O accumulator in O_g, its own running max and sum), the MMA warp issues
// S0(t) = Q0 K(t)^T, S1(t) = Q1 K(t)^T, P0 V(t), P1 V(t), and a K slot is refilled once
// both S of its tile were consumed, a V slot once both P.V completed. Each K/V byte then
// crosses into shared memory (and, for a packed prefix, is dequantized) once per head
// instead of once per row tile; the slots shrink to three K and two V (Q takes 64 KB).
//
// Packed (token-mode k4v4) prefixes: the PACKED instantiation adds three producer warps
// that build the K and V tiles from the packed bytes (ma_packed.cuh) instead of TMA loads:
// in place of the TMA warp they take the slots the MMA warp releases on kfree / vfree and
// arrive on kfull / vfull (three arrivals) once the slot's rows are stored. The current
// block stays TMA-fed (its loads issued by the MMA warp).
#include <string.h>

#include <algorithm>

#include "ma_combine.cuh"
#include "ma_kernels.cuh"
#include "ma_packed.cuh"
#include "ma_tcgen05.cuh"
#include "ma_tma.cuh"

namespace ma {

namespace {

using namespace tc;

constexpr int kSoftWarps = 8;
constexpr int kSoftThreads = kSoftWarps * 32;
constexpr int kWarps = kSoftWarps + 1;
constexpr int kThreads = kWarps * 32;              // the softmax and MMA warps (they take the merge rows)
constexpr int kThreadsB = kThreads + 32;           // bf16 kernels: + the TMA warp
constexpr int kRowTile = 128;                      // query rows per CTA (one M tile)
constexpr int kBN = 128;                           // keys per tile
constexpr int kD = 128;
constexpr int kDqWarps = 3;                        // dequantizing producer warps (PACKED): 12 warps,
                                                   // three per SM sub-partition (168 registers each)
constexpr int kDqThreads = kDqWarps * 32;
constexpr int kThreadsP = kThreads + kDqWarps * 32;
constexpr int kStages = 3;                         // PACKED: staged raw tiles in flight (bulk copies)
constexpr int kPackedSlots = 2;                    // PACKED: K and V slots each (the staging takes the rest)
constexpr int kKSlots = 3;                         // K tiles in flight (freed once S was read)
constexpr int kVSlots = 3;                         // V tiles in flight (freed when P.V completes)
constexpr float kLog2e = 1.4426950408889634f;
constexpr float kLazyLog2 = 8.0f * kLog2e;

constexpr int kQBlock = kRowTile * 128;            // 16 KB: one 64-channel block of 128 rows
constexpr int kQBytes = 2 * kQBlock;
constexpr int kKVBlock = kBN * 128;                // 16 KB: [128 rows][128 B]
constexpr int kKVBytes = 2 * kKVBlock;             // a K or V tile: 32 KB
constexpr int kSmemBytes = 1024 + kQBytes + (kKSlots + kVSlots) * kKVBytes;   // 225 KB
constexpr int kSmemBytesP = 1024 + kQBytes + 2 * kPackedSlots * kKVBytes + kStages * packed::kStageBytes;   // 221 KB
constexpr int kPairKSlots = 3;                     // PAIR: K tiles in flight (bf16)
constexpr int kPairVSlots = 2;                     // PAIR: V tiles in flight (bf16)
constexpr int kPairKSlotsP = 2;                    // PAIR + PACKED: K tiles in flight
constexpr int kPairVSlotsP = 1;                    // PAIR + PACKED: V tiles in flight
constexpr int kPairStages = 3;                     // PAIR + PACKED: staged raw tiles
constexpr int kPgCache = 256;                      // PACKED: page-table entries kept in shared memory
constexpr int kSmemBytes2 = 1024 + 2 * kQBytes + (kPairKSlots + kPairVSlots) * kKVBytes;   // 225 KB
constexpr int kSmemBytesP2 =                                                               // 221 KB
    1024 + 2 * kQBytes + (kPairKSlotsP + kPairVSlotsP) * kKVBytes + kPairStages * packed::kStageBytes;
constexpr uint32_t kTmemCols = 512;
constexpr uint32_t kColS = 0, kColO = 256;
constexpr int kOutBox = 32 * 128;
constexpr uint64_t kStallNs = 500000000ull;        // MMA issuer: longest time without progress
constexpr unsigned kIdleNs = 64;                   // MMA issuer back-off when nothing was ready
constexpr uint64_t kWaitNs = 500000000ull;

struct __align__(64) Args {
  CUtensorMap kmap, vmap;       // prefix K/V [B][H][n][D]
  CUtensorMap ckmap, cvmap;     // current block K/V [B][H][Tc][D]
  CUtensorMap qmap;             // queries [B][Hq][T][D]: boxes of 128 rows
  CUtensorMap omap;             // partial outputs [BH * S * Rp][D] bf16 (stores)
  ma_rows q;
  ma_kv kv;
  ma_block cur;
  float scale;
  int H, causal_block, q_pos0, c_pos0, n_keys, split_len, nsplit;
  int q_mode;                   // the query tile's boxes: 0 = 128/T whole heads, 1 = 128 rows of
                                // one head (T % 128 == 0), 2 = four 32-row pieces (T % 32 == 0)
  int tma_out;
  Partials P;
  int* err;
  int fuse;
  int cmerge;                   // the group's splits form one cluster: partials in shared memory
  int fold;                     // the current block is the last prefix split's final key tile
                                // (no split of its own; no prefix-only statistics)
  int direct;                   // one split per row block: the epilogue writes the output rows
  FusedMerge fm;
};

__device__ __forceinline__ void prefetch_map(const CUtensorMap* m) {
  asm volatile("prefetch.tensormap [%0];\n" ::"l"(reinterpret_cast<uint64_t>(m)) : "memory");
}
// D[tmem] (+)= A[tmem] * B[smem]: the A operand (M x 16, bf16 pairs per column) in TMEM
__device__ __forceinline__ void mma_bf16_ta(uint32_t d_tmem, uint32_t a_tmem, uint64_t b_desc, uint32_t idesc,
                                            bool accumulate) {
  asm volatile(
      "{\n.reg .pred p;\nsetp.ne.b32 p, %4, 0;\n"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n}\n" ::"r"(d_tmem),
      "r"(a_tmem), "l"(b_desc), "r"(idesc), "r"(accumulate ? 1 : 0));
}
__device__ __forceinline__ uint32_t pack_bf16x2(float lo, float hi) {
  __nv_bfloat162 v = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<uint32_t*>(&v);
}
// The partial rows of a cluster's splits in their CTAs' shared memory: split s is cluster
// rank s; its rows at sO (256 bytes per row, 16-byte chunk c of row i at c ^ (i & 15)) and
// its (m, l) pairs at sML.
struct ClusterPartials {
  static constexpr bool kLaneMl = true;   // one distributed-shared-memory load per pair
  uint32_t o_base, ml_base;   // this CTA's sO / sML as shared::cta addresses
  int row, l16;
  __device__ __forceinline__ uint4 o(int s) const {
    uint32_t a;
    asm volatile("mapa.shared::cluster.u32 %0, %1, %2;\n"
                 : "=r"(a) : "r"(o_base + (uint32_t)(row * 256 + ((l16 ^ (row & 15)) << 4))), "r"(s));
    uint4 v;
    asm volatile("ld.shared::cluster.v4.u32 {%0, %1, %2, %3}, [%4];\n"
                 : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w) : "r"(a) : "memory");
    return v;
  }
  __device__ __forceinline__ float2 ml(int s) const {
    uint32_t a;
    asm volatile("mapa.shared::cluster.u32 %0, %1, %2;\n" : "=r"(a) : "r"(ml_base + (uint32_t)(row * 8)), "r"(s));
    uint32_t x, y;
    asm volatile("ld.shared::cluster.v2.u32 {%0, %1}, [%2];\n" : "=r"(x), "=r"(y) : "r"(a) : "memory");
    return make_float2(__uint_as_float(x), __uint_as_float(y));
  }
};

// The partial rows every split of the cluster copied to this CTA (the pushed merge): the
// CTA that merges rows [lo, lo + per) holds split s's row lo + i at slot s per + i (256
// bytes, 16-byte chunk c at c ^ ((lo + i) & 15), the sender's layout) and its (m, l) in
// the 16-byte entry ml_base[s per + i].
struct PushedPartials {
  static constexpr bool kLaneMl = false;
  const uint8_t* o_base;
  const float4* ml_base;
  int per, lo, i, l16;
  __device__ __forceinline__ uint4 o(int s) const {
    return *reinterpret_cast<const uint4*>(o_base + (s * per + i) * 256 + ((l16 ^ ((lo + i) & 15)) << 4));
  }
  __device__ __forceinline__ float2 ml(int s) const {
    const float4 e = ml_base[s * per + i];
    return make_float2(e.x, e.y);
  }
};
constexpr int kRxMlOffset = 40960;   // the pushed (m, l) entries after at most 143 x 256 bytes of rows
constexpr int kPushMlOffset = 4096;  // a split's own (m, l) entries in its V slot 0 (after the scratch)
static_assert(kKSlots >= 3 && 143 * 256 <= kRxMlOffset && kRxMlOffset + 143 * 16 <= 2 * kKVBytes,
              "the pushed rows fit K slots 1 and 2");

// the max of 64 values (four independent max3 chains)
__device__ __forceinline__ float max64(const float (&v)[64]) {
  float mx[4];
#pragma unroll
  for (int j = 0; j < 4; ++j) mx[j] = max3f(v[j], v[4 + j], v[8 + j]);
#pragma unroll
  for (int i = 12; i + 8 <= 60; i += 8) {
#pragma unroll
    for (int j = 0; j < 4; ++j) mx[j] = max3f(mx[j], v[i + j], v[i + 4 + j]);
  }
  return max3f(max3f(mx[0], mx[1], v[60]), max3f(mx[2], mx[3], v[61]), fmaxf(v[62], v[63]));
}
__device__ __forceinline__ void softmax_sync() { asm volatile("bar.sync 5, %0;\n" ::"r"(kSoftThreads) : "memory"); }

// one 128-key tile of K or V (two 64-channel boxes) into dst, completing on `bar`
__device__ __forceinline__ void tma_tile(const CUtensorMap* map, int b, int h, int j0, uint8_t* dst, uint64_t* bar) {
  tma::expect_tx(bar, kKVBytes);
  tma::load_4d(dst, map, 0, j0, h, b, bar);
  tma::load_4d(dst + kKVBlock, map, 64, j0, h, b, bar);
}

// Bounded wait of a producer warp for a slot (lane 0 polls, the warp follows); false when
// the CTA aborted or the wait gave up.
__device__ __forceinline__ bool dq_wait(uint64_t* bar, uint32_t parity, volatile int* abort) {
  bool ok = true;
  if ((threadIdx.x & 31) == 0 && !mbar_try_wait(bar, parity)) {   // try_wait blocks a while itself
    const uint64_t t0 = global_ns();
    while (!mbar_try_wait(bar, parity)) {
      if (*abort || global_ns() - t0 > kWaitNs) {
        ok = false;
        *abort = 1;
        break;
      }
    }
  }
  return __shfl_sync(0xffffffffu, ok ? 1 : 0, 0) != 0;
}

template <bool PACKED, bool PAIR>
__device__ __forceinline__ void attn_fa_body(const Args& A) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sQ = smem;                                   // per M tile: [2 d blocks][128 rows][128 B]
  // K and V tiles in flight: the loads run two tiles ahead of the tensor core (PAIR: three
  // K and two V slots beside 64 KB of Q; PAIR + PACKED: two and one, so that three raw
  // tiles fit the staging ring, a V slot's next dequantization overlapping the next S)
  constexpr int KS = PAIR ? (PACKED ? kPairKSlotsP : kPairKSlots) : PACKED ? kPackedSlots : kKSlots;
  constexpr int VS = PAIR ? (PACKED ? kPairVSlotsP : kPairVSlots) : PACKED ? kPackedSlots : kVSlots;
  constexpr int NST = PAIR ? kPairStages : kStages;     // PACKED: staged raw tiles
  constexpr int kQT = PAIR ? 2 : 1;                     // M tiles per CTA
  constexpr int kRows = kQT * kRowTile;                 // query rows per CTA
  uint8_t* sKs = sQ + kQT * kQBytes;                    // K slots
  uint8_t* sVs = sKs + KS * kKVBytes;                   // V slots
  uint8_t* sStg = sVs + VS * kKVBytes;                  // PACKED: the staging ring of raw tiles
  __shared__ uint32_t s_taddr;
  __shared__ __align__(8) uint64_t kfull[KS], vfull[VS], s_full[2], p_full[2], o_done[2], q_full, mbar_fin, rx_full;
  __shared__ __align__(8) uint64_t kfree[KS], vfree[VS];
  __shared__ __align__(8) uint64_t rfull[PACKED ? NST : 1], rfree[PACKED ? NST : 1];
  __shared__ __align__(16) float sKch[PACKED ? kD : 1];   // the packed keys' divisor of this (b, h)
  __shared__ int sPg[PACKED ? kPgCache : 1];              // the page-table entries of [begin, end)
  __shared__ int s_abort, s_merge_ok, s_gather_ok;
  __shared__ uint32_t s_epoch, s_cum;   // the fused head gather: call number, CTAs of the calls before

  // grid (row tiles, splits, heads): the row tiles of one split run side by side, so the
  // second and later ones read that split's K/V from L2
  const int split = blockIdx.y;
  const int bh = blockIdx.z;
  const int H = A.H;
  const int b = bh / H, h = bh - (bh / H) * H;
  const int T = A.q.T;
  const int G = A.q.Hq / H;
  const int R = G * T;
  const int r0 = blockIdx.x * kRows;                     // the CTA's first row
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const bool softmax_warp = warp < kSoftWarps;
  // rows 32*quarter.. of the M tile; single: the tiles t = grp mod 2, PAIR: M tile grp
  const int quarter = warp & 3, grp = (warp >> 2) & 1;
  const int rg0 = r0 + (PAIR ? kRowTile * grp : 0);      // this warp group's M tile
  const int rl = quarter * 32 + lane;
  const int r = rg0 + rl;
  const int wrow0 = rg0 + quarter * 32;
  const bool warp_rows = softmax_warp && wrow0 < R;      // the same for both warps of a pair
  const bool row_ok = softmax_warp && r < R;
  const int t_row = row_ok ? r % T : 0;

  const bool is_cur = split == A.nsplit;
  const bool dq = PACKED && !is_cur;   // prefix tiles built by the producer warps
  const bool merge_warp = warp < kWarps;   // the producer warps take no merge rows
  // pushed cluster merge (every CTA of the cluster has at most one key tile, so K slots 1
  // and 2 stay free): split j of the cluster merges rows [j mper, +mper) of the row block;
  // every split lays its partial out in its own K slot 0 and copies those rows into CTA
  // j's K slots 1 and 2 with the bulk-copy engine
  const bool push = !PAIR && !PACKED && A.cmerge == 2;
  const int R_blk = min(kRows, R - r0);
  const int mper = (R_blk + (int)gridDim.y - 1) / (int)gridDim.y;
  uint8_t* sRx = sKs + kKVBytes;
  float4* sRxML = reinterpret_cast<float4*>(sRx + kRxMlOffset);
  int begin, end;
  if (is_cur) {
    begin = 0;
    end = A.cur.Tc;
  } else {
    begin = split * A.split_len;
    end = min(A.n_keys, begin + A.split_len);
    if (A.kv.lens) {   // a ragged batch: slots past lens[b] do not exist (lens may come from
      pdl_wait();      // the kernel before, with a programmatic launch)
      end = max(begin, min(end, A.kv.lens[b]));
    }
  }
  int vis_end = end;
  if (is_cur && A.causal_block > 0)
    vis_end = min(end, ((A.q_pos0 + t_row) / A.causal_block + 1) * A.causal_block - A.c_pos0);
  if (!row_ok) vis_end = begin;
  const int ntp = end > begin ? (end - begin + kBN - 1) / kBN : 0;   // key tiles of [begin, end)
  // folded: the last prefix split also takes the current block, as one more key tile (keys
  // [0, Tc) of the block's maps), so the block needs no split of its own
  const bool fold_here = !PACKED && A.fold && !is_cur && split == A.nsplit - 1 && A.cur.Tc > 0;
  const int ntiles = ntp + (fold_here ? 1 : 0);
  const bool has_cur = A.cur.Tc > 0 && !A.fold;   // the merges: a block split after the prefix ones
  // key tile t's tensor map (K or V) and first key: the prefix's, or the block's for the
  // block split and for a folded split's last tile
  auto tile_map = [&](int t, bool v, int& x) -> const CUtensorMap* {
    const bool blk = is_cur || (fold_here && t >= ntp);
    x = blk ? (t - (is_cur ? 0 : ntp)) * kBN : begin + t * kBN;
    return blk ? (v ? &A.cvmap : &A.ckmap) : (v ? &A.vmap : &A.kmap);
  };
  const int nU = kQT * ntiles;   // S tiles: u = kQT t + M tile
  const float c2 = A.scale * kLog2e;
  const int group = bh * gridDim.x + blockIdx.x;

  // PACKED paged prefix: the entries of the pages [begin, end) crosses, read once (the MMA
  // warp's lanes) for the staging copies and the producers' row checks
  const int pps = A.kv.pages ? A.kv.page_size : 1;
  const int npg = (dq && A.kv.pages && end > begin) ? (end - 1) / pps - begin / pps + 1 : 0;
  const packed::PageCache pc{sPg, begin / pps, npg <= kPgCache ? npg : 0};
  if (dq && pc.n > 0 && warp == kSoftWarps) {
    pdl_wait();
    for (int i = lane; i < pc.n; i += 32) sPg[i] = A.kv.pages[(int64_t)b * A.kv.spg + pc.p0 + i];
    __syncwarp();
  }

  unsigned gen0 = 0;   // the merge generation, read after pdl_wait, before this CTA arrives (thread 0)
  if (threadIdx.x == kSoftThreads) {
    prefetch_map(&A.qmap);
    if (!dq) {
      prefetch_map(is_cur ? &A.ckmap : &A.kmap);
      prefetch_map(is_cur ? &A.cvmap : &A.vmap);
      if (fold_here) {
        prefetch_map(&A.ckmap);
        prefetch_map(&A.cvmap);
      }
    }
    for (int i = 0; i < KS; ++i) mbar_init(&kfull[i], dq ? kDqWarps : 1);
    for (int i = 0; i < VS; ++i) mbar_init(&vfull[i], dq ? kDqWarps : 1);
    for (int i = 0; i < KS; ++i) mbar_init(&kfree[i], 1);
    for (int i = 0; i < VS; ++i) mbar_init(&vfree[i], 1);
    if (PACKED) {
      for (int i = 0; i < NST; ++i) {
        mbar_init(&rfull[i], 1);
        mbar_init(&rfree[i], kDqWarps);
      }
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&s_full[i], 1);
      mbar_init(&p_full[i], kSoftWarps / 2);
      mbar_init(&o_done[i], 1);
    }
    mbar_init(&q_full, 1);
    mbar_init(&mbar_fin, 1);
    if (push) mbar_init(&rx_full, 1);
    s_abort = 0;
    asm volatile("fence.mbarrier_init.release.cluster;\n" ::: "memory");
    if (push) {   // every split's rows of this CTA's share: 256 bytes + a 16-byte (m, l) each
      const int own = max(0, min(R_blk, (split + 1) * mper) - split * mper);
      tma::expect_tx(&rx_full, (uint32_t)((int)gridDim.y * own * (kD * 2 + 16)));
    }
    // the queries and the first K and V tiles start loading now, before the TMEM
    // allocation and the setup barrier
    pdl_wait();   // with a programmatic launch, the inputs may come from the kernel before
    tma::expect_tx(&q_full, (uint32_t)(kQT * kQBytes));
    for (int qt = 0; qt < kQT; ++qt) {
      const int rq = r0 + qt * kRowTile;   // rows past R load neighbouring or zero rows: never used
      uint8_t* dQ = sQ + qt * kQBytes;
      if (A.q_mode == 1) {          // 128 consecutive positions of one query head
        tma::load_4d(dQ, &A.qmap, 0, rq % T, h * G + rq / T, b, &q_full);
        tma::load_4d(dQ + kQBlock, &A.qmap, 64, rq % T, h * G + rq / T, b, &q_full);
      } else if (A.q_mode == 0) {   // 128 / T whole query heads
        tma::load_4d(dQ, &A.qmap, 0, 0, h * G + rq / T, b, &q_full);
        tma::load_4d(dQ + kQBlock, &A.qmap, 64, 0, h * G + rq / T, b, &q_full);
      } else {                      // four 32-row pieces, each inside one query head
        for (int i = 0; i < kRowTile / 32; ++i) {
          const int rp = rq + 32 * i;
          tma::load_4d(dQ + i * 32 * 128, &A.qmap, 0, rp % T, h * G + rp / T, b, &q_full);
          tma::load_4d(dQ + kQBlock + i * 32 * 128, &A.qmap, 64, rp % T, h * G + rp / T, b, &q_full);
        }
      }
    }
    if (!dq) {
      for (int i = 0; i < KS && i < ntiles; ++i) {
        int x;
        const CUtensorMap* m = tile_map(i, false, x);
        tma_tile(m, b, h, x, sKs + i * kKVBytes, &kfull[i]);
      }
      for (int i = 0; i < VS && i < ntiles; ++i) {
        int x;
        const CUtensorMap* m = tile_map(i, true, x);
        tma_tile(m, b, h, x, sVs + i * kKVBytes, &vfull[i]);
      }
    } else {   // the first raw tiles into the staging ring
      for (int i = 0; i < NST && i < ntiles; ++i)
        packed::stage_tile(A.kv, b, h, begin + i * kBN, min(end, begin + (i + 1) * kBN), sStg + i * packed::kStageBytes,
                           &rfull[i], pc);
    }
  }
  if (warp == 0) tmem_alloc(&s_taddr, kTmemCols);
  fence_before_sync();
  __syncthreads();
  fence_after_sync();
  if (push) cluster_arrive_relaxed();   // rx_full is initialized (waited on before the first send)
  const uint32_t taddr = s_taddr;
  const uint32_t lane_base = (uint32_t)(quarter * 32) << 16;
  const uint32_t tS = taddr + lane_base + kColS + 128 * grp;   // this warp's S buffer (its rows)
  const uint32_t tO = taddr + lane_base + kColO + 128 * grp;   // this warp's O accumulator
  float m_run = -INFINITY, l_run = 0.f, m_true = -INFINITY;

  if (warp == kSoftWarps) {
    // ------------------------------------------------------------ MMA warp
    if (lane == 0) {
      // Event loop over the S tiles u (single: u = t; PAIR: u = 2t + M tile): S(u) needs
      // K(t) loaded and P.V(u-2) issued -- P(u-2) lives in S(u)'s buffer, and tcgen05.mma
      // operations of one thread execute in issue order, so S(u) overwrites P(u-2) only
      // after P.V(u-2) read it (a softmax that rescales O(u&1) waits for P.V(u-2) itself);
      // P.V(u) needs V(t) and the softmax's P(u). P.V completes in issue order, so oD
      // counts completions over both o_done barriers alternately. A K slot takes its next
      // tile once every S it fed was consumed (the tile's last P.V issued), a V slot once the
      // tile's last P.V completed. Each barrier has at most one completed but unobserved
      // phase, so the parity tests are unambiguous.
      bool ok = true;
      // the queries and the first min(3, ntiles) K and V tiles were issued at setup
      int kIss = min(KS, ntiles), kObs = 0, vIss = min(VS, ntiles), vObs = 0;
      int sN = 0, pN = 0, oD = 0;                   // S issued, P.V issued, P.V seen complete
      // PACKED: raw tiles staged, staged tiles seen consumed by the producer warps
      int rIss = dq ? min(NST, ntiles) : ntiles, rfObs = 0;
      const bool q_ok = mbar_wait(&q_full, 0);
      ok = q_ok;
      const uint32_t idS = idesc_bf16(kRowTile, kBN, false, false);
      const uint32_t idO = idesc_bf16(kRowTile, kD, false, true);
      // base descriptors; a K step or a slot only moves the start address (field bits
      // [0,14) = address >> 4, no carry below 256 KB), so each MMA adds a constant
      const uint64_t qdesc = smem_desc(smem_addr(sQ), 16, 1024);
      const uint64_t kdesc = smem_desc(smem_addr(sKs), 16, 1024);
      const uint64_t vdesc = smem_desc(smem_addr(sVs), kKVBlock, 1024);
      uint64_t t_idle = 0;
      bool armed = false;
      int spins = 0;
      while (ok && pN < nU) {
        bool progress = false;
        if (kObs < kIss && mbar_test(&kfull[kObs % KS], (uint32_t)(kObs / KS) & 1u)) {
          ++kObs;
          progress = true;
        }
        if (vObs < vIss && mbar_test(&vfull[vObs % VS], (uint32_t)(vObs / VS) & 1u)) {
          ++vObs;
          progress = true;
        }
        if (oD < pN && mbar_test(&o_done[oD & 1], (uint32_t)(oD >> 1) & 1u)) {
          ++oD;
          progress = true;
        }
        if (sN < nU && kObs > sN / kQT && pN >= sN - 1) {
          fence_after_sync();
          const uint64_t bd0 = kdesc + (uint64_t)(((sN / kQT) % KS) * (kKVBytes / 16));
          const uint64_t qd0 = qdesc + (uint64_t)((sN % kQT) * (kQBytes / 16));
          const uint32_t dS = taddr + kColS + (sN & 1) * 128;
#pragma unroll
          for (int kk = 0; kk < kD / 16; ++kk)
            mma_bf16(dS, qd0 + (uint64_t)(((kk >> 2) * kQBlock + (kk & 3) * 32) >> 4),
                     bd0 + (uint64_t)(((kk >> 2) * kKVBlock + (kk & 3) * 32) >> 4), idS, kk > 0);
          mma_commit(&s_full[sN & 1]);
          ++sN;
          progress = true;
        }
        if (pN < sN && vObs > pN / kQT && mbar_test(&p_full[pN & 1], (uint32_t)(pN >> 1) & 1u)) {
          fence_after_sync();
          const uint64_t bd0 = vdesc + (uint64_t)(((pN / kQT) % VS) * (kKVBytes / 16));
          const uint32_t aP = taddr + kColS + (pN & 1) * 128;
#pragma unroll
          for (int kk = 0; kk < kBN / 16; ++kk)   // keys 16kk..: P columns 64 (kk / 4) + 8 (kk % 4)
            mma_bf16_ta(taddr + kColO + (pN & 1) * 128, aP + (kk >> 2) * 64 + (kk & 3) * 8,
                        bd0 + (uint64_t)(kk * (2048 / 16)), idO, pN > 1 || kk > 0);
          mma_commit(&o_done[pN & 1]);
          ++pN;
          progress = true;
        }
        // PACKED: a stage takes the next raw tile once the producer warps consumed its last
        if (dq) {
          if (rfObs < rIss && mbar_test(&rfree[rfObs % NST], (uint32_t)(rfObs / NST) & 1u)) {
            ++rfObs;
            progress = true;
          }
          if (rIss < ntiles && rfObs > rIss - NST) {
            packed::stage_tile(A.kv, b, h, begin + rIss * kBN, min(end, begin + (rIss + 1) * kBN),
                               sStg + (rIss % NST) * packed::kStageBytes, &rfull[rIss % NST], pc);
            ++rIss;
            progress = true;
          }
        }
        // a K slot is free once the S it fed were consumed (the tile's last P.V issued); the
        // TMA warp (bf16) or the producer warps (packed) refill it -- a TMA issue can stall
        // its thread for hundreds of cycles, which this loop must not spend
        if (kIss < ntiles && pN >= kQT * (kIss - KS + 1)) {
          if (dq || !PACKED) {
            mbar_arrive(&kfree[kIss % KS]);
          } else {
            int x;
            const CUtensorMap* m = tile_map(kIss, false, x);
            tma_tile(m, b, h, x, sKs + (kIss % KS) * kKVBytes, &kfull[kIss % KS]);
          }
          ++kIss;
          progress = true;
        }
        // a V slot is free once the tile's last P.V completed
        if (vIss < ntiles && oD >= kQT * (vIss - VS + 1)) {
          if (dq || !PACKED) {
            mbar_arrive(&vfree[vIss % VS]);
          } else {
            int x;
            const CUtensorMap* m = tile_map(vIss, true, x);
            tma_tile(m, b, h, x, sVs + (vIss % VS) * kKVBytes, &vfull[vIss % VS]);
          }
          ++vIss;
          progress = true;
        }
        if (progress) {
          spins = 0;
          armed = false;
        } else if (__nanosleep(kIdleNs), ++spins == 256) {   // idle: back off (the issue slots
          // of this sub-partition belong to two compute warps), bound the time without progress
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
      if (PACKED && !dq) {   // TMA loads still in flight (bf16: the TMA warp drains its own)
        for (int tt = kObs; tt < kIss; ++tt)
          mbar_wait(&kfull[tt % KS], (uint32_t)(tt / KS) & 1u, 20000000ull);
        for (int tt = vObs; tt < vIss; ++tt)
          mbar_wait(&vfull[tt % VS], (uint32_t)(tt / VS) & 1u, 20000000ull);
      } else if (dq) {   // bulk copies into the staging ring still in flight
        for (int tt = rfObs; tt < rIss; ++tt)
          mbar_wait(&rfull[tt % NST], (uint32_t)(tt / NST) & 1u, 20000000ull);
      }
    }
    __syncwarp();
  } else if (!PACKED && warp == kSoftWarps + 1) {
    // ------------------------------------------------------------ TMA warp (bf16)
    // K tile t >= KS goes into slot t % KS once the MMA warp released it (kfree), V tile t
    // into slot t % VS likewise (vfree); the first KS and VS were issued at setup. At most
    // KS K and VS V loads are in flight at a time (a slot is released only after its tile
    // was consumed), so at the end the last ones issued are waited for.
    if (lane == 0) {
      pdl_wait();   // with a programmatic launch, the cache may come from the kernel before
      int kN = min(KS, ntiles), vN = min(VS, ntiles);
      uint64_t t_idle = 0;
      bool armed = false;
      int spins = 0;
      while (kN < ntiles || vN < ntiles) {
        bool progress = false;
        if (kN < ntiles && mbar_test(&kfree[kN % KS], (uint32_t)((kN / KS) - 1) & 1u)) {
          int x;
          const CUtensorMap* m = tile_map(kN, false, x);
          tma_tile(m, b, h, x, sKs + (kN % KS) * kKVBytes, &kfull[kN % KS]);
          ++kN;
          progress = true;
        }
        if (vN < ntiles && mbar_test(&vfree[vN % VS], (uint32_t)((vN / VS) - 1) & 1u)) {
          int x;
          const CUtensorMap* m = tile_map(vN, true, x);
          tma_tile(m, b, h, x, sVs + (vN % VS) * kKVBytes, &vfull[vN % VS]);
          ++vN;
          progress = true;
        }
        if (progress) {
          spins = 0;
          armed = false;
        } else if (__nanosleep(kIdleNs), ++spins == 256) {   // idle: bounded like the MMA warp
          spins = 0;
          const uint64_t now = global_ns();
          if (!armed) {
            t_idle = now;
            armed = true;
          } else if (now - t_idle > kStallNs) {
            s_abort = 1;
          }
          if (s_abort) break;
        }
      }
      for (int x = max(0, kN - KS); x < kN; ++x) mbar_wait(&kfull[x % KS], (uint32_t)(x / KS) & 1u, 20000000ull);
      for (int x = max(0, vN - VS); x < vN; ++x) mbar_wait(&vfull[x % VS], (uint32_t)(x / VS) & 1u, 20000000ull);
    }
    __syncwarp();
  } else if (PACKED && !softmax_warp) {
    // ------------------------------------------------------------ producer warps (PACKED)
    // Tile t's raw rows arrive in stage t % NST (rfull); its K items go into slot t % KS
    // once the MMA warp released it (kfree; the first KS are free), its V items into slot
    // t % VS likewise, then the stage is handed back (rfree). An item is (row, 32-channel
    // group), item it = dt + kDqThreads * i being group it & 3 of row it >> 2, so a warp
    // reads 512 consecutive staged bytes.
    if (dq) {
      const int dt = threadIdx.x - (kSoftThreads + 32);
      pdl_wait();   // with a programmatic launch, the cache may come from the kernel before
      for (int c = dt; c < kD; c += kDqThreads)
        sKch[c] = A.kv.kchan[(int64_t)b * A.kv.skc[0] + (int64_t)h * A.kv.skc[1] + c];
      asm volatile("bar.sync 6, %0;\n" ::"r"(kDqThreads) : "memory");
      constexpr int kItems = (kBN * 4 + kDqThreads - 1) / kDqThreads;
      for (int t = 0; t < ntiles; ++t) {
        const int j0 = begin + t * kBN;
        const uint8_t* stg = sStg + (t % NST) * packed::kStageBytes;
        // the tile's rows that exist (below end, on a page of the pool), one bit per row:
        // four page-table lookups a lane, in parallel, instead of one per item
        uint32_t okm[4];
#pragma unroll
        for (int i = 0; i < 4; ++i) okm[i] = __ballot_sync(0xffffffffu, packed::row_ok(A.kv, b, j0 + 32 * i + lane, end, pc));
        auto ok_row = [&](int row) {
          const uint32_t m = row < 64 ? (row < 32 ? okm[0] : okm[1]) : (row < 96 ? okm[2] : okm[3]);
          return ((m >> (row & 31)) & 1u) != 0;
        };
        if (!dq_wait(&rfull[t % NST], (uint32_t)(t / NST) & 1u, &s_abort)) break;
        if (t >= KS && !dq_wait(&kfree[t % KS], (uint32_t)((t / KS) - 1) & 1u, &s_abort)) break;
#pragma unroll
        for (int i = 0; i < kItems; ++i) {
          const int it = dt + kDqThreads * i;
          if (it < kBN * 4)
            packed::dequant_item<true>(stg, it >> 2, it & 3, ok_row(it >> 2), sKs + (t % KS) * kKVBytes, sKch);
        }
        fence_proxy_async();   // generic stores -> the tensor core's reads
        __syncwarp();
        if (lane == 0) mbar_arrive(&kfull[t % KS]);
        if (t >= VS && !dq_wait(&vfree[t % VS], (uint32_t)((t / VS) - 1) & 1u, &s_abort)) break;
#pragma unroll
        for (int i = 0; i < kItems; ++i) {
          const int it = dt + kDqThreads * i;
          if (it < kBN * 4)
            packed::dequant_item<false>(stg, it >> 2, it & 3, ok_row(it >> 2), sVs + (t % VS) * kKVBytes, nullptr);
        }
        fence_proxy_async();
        __syncwarp();
        if (lane == 0) {
          mbar_arrive(&vfull[t % VS]);
          mbar_arrive(&rfree[t % NST]);   // the stage's raw rows are read
        }
      }
    }
  } else {
    // ------------------------------------------------------------ softmax warps
    // warp (quarter, grp): rows 32 quarter.. of the tiles t = grp, grp + 2, ... (PAIR: of
    // M tile grp, every tile t), all 128 keys of each, with its own running max, row sum
    // and O accumulator; the two warps that share a sub-partition work on different S
    // tiles, so one's exponentials overlap the other's tensor-memory reads, maxima and
    // stores
    pdl_wait();   // the partials and outputs may still be in use by the kernel before
    if (A.fuse && threadIdx.x == 0) gen0 = *reinterpret_cast<volatile const unsigned*>(&A.fm.sync[group].y);
    const float2 c2x2 = make_float2(c2, c2);
    const int nk = PAIR ? ntiles : (ntiles > grp ? (ntiles - grp + 1) / 2 : 0);   // this warp's S tiles
    for (int k = 0; k < nk; ++k) {
      const int t = PAIR ? k : grp + 2 * k;   // its k-th S tile reads K/V tile t
      const bool ok = mbar_wait(&s_full[grp], (uint32_t)k & 1u);
      fence_after_sync();
      if (!ok) s_abort = 1;
      if (s_abort) break;
      if (warp_rows) {
        // keys i >= lim of the tile are hidden (a folded block tile: its first Tc keys exist)
        const int lim = (fold_here && t == ntp) ? (row_ok ? A.cur.Tc : 0) : vis_end - (begin + t * kBN);
        const bool full = __all_sync(0xffffffffu, lim >= kBN);
        float sv[64];
        // the row max: keys 64..127 (read, not kept), then keys 0..63 (kept)
        tmem_ld32(tS + 64, sv);
        tmem_ld32(tS + 96, sv + 32);
        tmem_ld_wait();
        if (!full) {
#pragma unroll
          for (int i = 0; i < 64; ++i) sv[i] = 64 + i < lim ? sv[i] : -INFINITY;
        }
        float pm = max64(sv);
        tmem_ld32(tS, sv);
        tmem_ld32(tS + 32, sv + 32);
        tmem_ld_wait();
        if (!full) {
#pragma unroll
          for (int i = 0; i < 64; ++i) sv[i] = i < lim ? sv[i] : -INFINITY;
        }
        pm = fmaxf(pm, max64(sv));
        // lazy rescale of this warp's O, after its previous P.V completed
        m_true = fmaxf(m_true, pm);
        const float m_new = fmaxf(m_run, pm * c2);
        const bool grow = k > 0 && m_new > m_run + kLazyLog2;
        if (__any_sync(0xffffffffu, grow)) {
          if (!mbar_wait(&o_done[grp], (uint32_t)(k - 1) & 1u, kWaitNs)) s_abort = 1;
          fence_after_sync();
          const float alpha = grow ? ex2(m_run - m_new) : 1.f;
#pragma unroll 1
          for (int c = 0; c < 4; ++c) {
            float o[32];
            tmem_ld32(tO + c * 32, o);
            tmem_ld_wait();
#pragma unroll
            for (int i = 0; i < 32; ++i) o[i] *= alpha;
            tmem_st32(tO + c * 32, o);
          }
          if (grow) {
            l_run *= alpha;
            m_run = m_new;
          }
        }
        if (k == 0) m_run = m_new;
        const float msl = (m_run == -INFINITY) ? 0.f : m_run;
        // P = 2^(s c2 - m) (packed FMA, one ex2 per key) as bf16 pairs: keys 0..63 into
        // columns 0..31, keys 64..127 (read again) into columns 64..95; the row sum from the
        // fp32 values
        const float2 nm2 = make_float2(-msl, -msl);
        float2 acc0 = make_float2(0.f, 0.f), acc1 = make_float2(0.f, 0.f);
#pragma unroll 1
        for (int half = 0; half < 2; ++half) {
          if (half == 1) {
            tmem_ld32(tS + 64, sv);
            tmem_ld32(tS + 96, sv + 32);
            tmem_ld_wait();
            if (!full) {
#pragma unroll
              for (int i = 0; i < 64; ++i) sv[i] = 64 + i < lim ? sv[i] : -INFINITY;
            }
          }
#pragma unroll
          for (int c = 0; c < 2; ++c) {
            uint32_t w[16];
#pragma unroll
            for (int i = 0; i < 16; ++i) {
              float2 x = ffma2(make_float2(sv[32 * c + 2 * i], sv[32 * c + 2 * i + 1]), c2x2, nm2);
              x.x = ex2(x.x);
              x.y = ex2(x.y);
              if (i & 1) acc1 = fadd2(acc1, x); else acc0 = fadd2(acc0, x);
              w[i] = pack_bf16x2(x.x, x.y);
            }
            tmem_st16(tS + 64 * half + c * 16, w);
          }
        }
        tmem_st_wait();
        l_run += (acc0.x + acc0.y) + (acc1.x + acc1.y);
      }
      fence_before_sync();
      __syncwarp();
      if (lane == 0) mbar_arrive(&p_full[grp]);
    }
    if (nk > 0 && !s_abort) {   // this warp's last P.V
      if (!mbar_wait(&o_done[grp], (uint32_t)((nk - 1) & 1), kWaitNs)) s_abort = 1;
      fence_after_sync();
    }
  }
  // join: every MMA done (the MMA warp drained), every softmax warp out of its loop
  fence_before_sync();
  __syncthreads();
  fence_after_sync();
  if (threadIdx.x == 0) pdl_launch_dependents();   // the next kernel's prologue may start
  if (push) cluster_wait();   // every CTA's rx_full is initialized: the sends may start

  // direct (one split per row block): the row of the output this thread's row goes to
  uint4* out_row = nullptr;
  if (A.direct && row_ok) {
    const int g = r / T, tt = r - (r / T) * T;
    out_row = reinterpret_cast<uint4*>(reinterpret_cast<__nv_bfloat16*>(A.fm.out) + (int64_t)b * A.fm.so[0] +
                                       (int64_t)(h * G + g) * A.fm.so[1] + (int64_t)tt * A.fm.so[2]);
  }
  const uint4 nan8 = make_uint4(0x7fc07fc0u, 0x7fc07fc0u, 0x7fc07fc0u, 0x7fc07fc0u);   // bf16 NaN x 8
  if (PAIR && softmax_warp) {
    // each M tile's rows are final in their own group: o = O_g / l under the group's running
    // max; warp (quarter, grp) writes all 128 channels of its 32 rows (the slots are
    // drained: two output boxes per warp in the K and V slots, or the cluster's rows)
    const int rc = r - r0;   // the row within the CTA
    const int64_t prow = ((int64_t)bh * A.P.S + split) * A.P.Rp + r;
    const int prow0 = (int)(((int64_t)bh * A.P.S + split) * A.P.Rp + wrow0);
    float2* sML = reinterpret_cast<float2*>(sVs + 4096);   // cluster merge: this split's (m, l)
    uint8_t* sO = sKs;                                     // cluster merge: its rows (64 KB)
    if (s_abort != 0) {
      if (threadIdx.x == 0) atomicExch(A.err, 1);
      if (row_ok) {
        if (A.direct) {
          for (int i = 0; i < kD / 8; ++i) out_row[i] = nan8;
        } else if (A.cmerge) {
          sML[rc] = make_float2(NAN, NAN);
        } else {
          A.P.ml[prow] = make_float2(NAN, NAN);
        }
      }
    } else {
      if (row_ok) {
        const float fix = (m_true == -INFINITY) ? 1.f : ex2(m_run - m_true * c2);
        if (A.cmerge) sML[rc] = make_float2(m_true * A.scale, l_run * fix);
        else A.P.ml[prow] = make_float2(m_true * A.scale, l_run * fix);
      }
      const float inv = l_run > 0.f ? 1.f / l_run : 0.f;
      if (warp_rows) {
        const bool via_tma = ntiles > 0 && A.tma_out && !A.cmerge && !A.direct;
        uint8_t* box = sKs + warp * 2 * kOutBox;   // two 32-row boxes: channels 0..63, 64..127
        uint4* dst = A.direct ? out_row : reinterpret_cast<uint4*>(reinterpret_cast<__nv_bfloat16*>(A.P.o) + prow * kD);
        const uint32_t tOg = taddr + lane_base + kColO + 128 * grp;
#pragma unroll 1
        for (int c = 0; c < 4; ++c) {
          float o[32];
          if (ntiles > 0) {
            tmem_ld32(tOg + 32 * c, o);
            tmem_ld_wait();
#pragma unroll
            for (int i = 0; i < 32; ++i) o[i] *= inv;
          } else {
#pragma unroll
            for (int i = 0; i < 32; ++i) o[i] = 0.f;
          }
          if (A.cmerge) {   // the row into shared memory, chunk cc of row rc at cc ^ (rc & 15)
#pragma unroll
            for (int qq = 0; qq < 4; ++qq) {
              const int cc = 4 * c + qq;
              *reinterpret_cast<uint4*>(sO + rc * 256 + ((cc ^ (rc & 15)) << 4)) = float8_to_bf16x8(o + 8 * qq);
            }
          } else if (via_tma) {
            uint8_t* line = box + (c >> 1) * kOutBox + lane * 128;
#pragma unroll
            for (int qq = 0; qq < 4; ++qq)
              *reinterpret_cast<uint4*>(line + (((4 * (c & 1) + qq) ^ (lane & 7)) << 4)) = float8_to_bf16x8(o + 8 * qq);
          } else if (row_ok) {
#pragma unroll
            for (int qq = 0; qq < 4; ++qq) dst[4 * c + qq] = float8_to_bf16x8(o + 8 * qq);
          }
        }
        if (via_tma) {
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
        }
      }
    }
  } else if (softmax_warp) {
    // the two tile groups' row states meet (the slots are drained: scratch in the V slots):
    // both are rescaled to the larger running max M, l = l0 f0 + l1 f1, o = (O0 f0 + O1 f1) / l;
    // warp (quarter, grp) writes channels 64 grp.. of its rows
    float* sX = reinterpret_cast<float*>(sVs);   // [group][m_run, l_run, m_true][row]
    sX[(grp * 3 + 0) * kRowTile + rl] = m_run;
    sX[(grp * 3 + 1) * kRowTile + rl] = l_run;
    sX[(grp * 3 + 2) * kRowTile + rl] = m_true;
    softmax_sync();
    const int og = grp ^ 1;
    const float m_oth = sX[(og * 3 + 0) * kRowTile + rl], l_oth = sX[(og * 3 + 1) * kRowTile + rl];
    const float M = fmaxf(m_run, m_oth);
    const float f_me = m_run == -INFINITY ? 0.f : ex2(m_run - M);
    const float f_oth = m_oth == -INFINITY ? 0.f : ex2(m_oth - M);
    const float l = l_run * f_me + l_oth * f_oth;
    const float mt = fmaxf(m_true, sX[(og * 3 + 2) * kRowTile + rl]);
    const float f0 = grp == 0 ? f_me : f_oth, f1 = grp == 0 ? f_oth : f_me;
    const int64_t prow = ((int64_t)bh * A.P.S + split) * A.P.Rp + r;
    const int prow0 = (int)(((int64_t)bh * A.P.S + split) * A.P.Rp + wrow0);
    float2* sML = reinterpret_cast<float2*>(sVs + 4096);   // cluster merge: this split's (m, l)
    uint8_t* sO = sKs;                                     // cluster merge: its rows (32 KB)
    float4* sMLq = reinterpret_cast<float4*>(sVs + kPushMlOffset);   // pushed merge: 16-byte (m, l)
    if (s_abort != 0) {
      if (threadIdx.x == 0) atomicExch(A.err, 1);
      if (row_ok && grp == 0) {
        if (A.direct) {
          for (int i = 0; i < kD / 8; ++i) out_row[i] = nan8;
        } else if (push) {
          sMLq[rl] = make_float4(NAN, NAN, 0.f, 0.f);
        } else if (A.cmerge) {
          sML[rl] = make_float2(NAN, NAN);
        } else {
          A.P.ml[prow] = make_float2(NAN, NAN);
        }
      }
    } else {
      // the exact max: l under M times 2^(M - m_true) <= 1; o = acc / l is the same under
      // either reference
      if (row_ok && grp == 0) {
        const float fix = (mt == -INFINITY) ? 1.f : ex2(M - mt * c2);
        if (push) sMLq[rl] = make_float4(mt * A.scale, l * fix, 0.f, 0.f);
        else if (A.cmerge) sML[rl] = make_float2(mt * A.scale, l * fix);
        else A.P.ml[prow] = make_float2(mt * A.scale, l * fix);
      }
      const float inv = l > 0.f ? 1.f / l : 0.f;
      if (warp_rows) {
        const bool via_tma = ntiles > 0 && A.tma_out && !A.cmerge && !A.direct;
        // the warp's 32 rows x 64 channels -> one box in the K slots, 128-byte swizzled
        // (chunk q of line i at q ^ (i & 7)), stored by lane 0; else straight to global
        uint8_t* box = sKs + warp * kOutBox;
        uint8_t* line = box + lane * 128;
        uint4* dst = A.direct ? out_row + 8 * grp
                              : reinterpret_cast<uint4*>(reinterpret_cast<__nv_bfloat16*>(A.P.o) + prow * kD + 64 * grp);
        const uint32_t tO0 = taddr + lane_base + kColO + 64 * grp, tO1 = tO0 + 128;
#pragma unroll 1
        for (int c = 0; c < 2; ++c) {
          float o[32];
          if (ntiles > 0) {
            tmem_ld32(tO0 + 32 * c, o);   // O0 holds tiles 0, 2, ..., O1 tiles 1, 3, ...
            if (ntiles > 1) {
              float x[32];
              tmem_ld32(tO1 + 32 * c, x);
              tmem_ld_wait();
#pragma unroll
              for (int i = 0; i < 32; ++i) o[i] = (o[i] * f0 + x[i] * f1) * inv;
            } else {
              tmem_ld_wait();
#pragma unroll
              for (int i = 0; i < 32; ++i) o[i] = o[i] * f0 * inv;
            }
          } else {
#pragma unroll
            for (int i = 0; i < 32; ++i) o[i] = 0.f;
          }
          if (A.cmerge) {   // the row into shared memory, chunk cc of row rl at cc ^ (rl & 15)
#pragma unroll
            for (int qq = 0; qq < 4; ++qq) {
              const int cc = 8 * grp + 4 * c + qq;
              *reinterpret_cast<uint4*>(sO + rl * 256 + ((cc ^ (rl & 15)) << 4)) = float8_to_bf16x8(o + 8 * qq);
            }
          } else if (via_tma) {
#pragma unroll
            for (int qq = 0; qq < 4; ++qq)
              *reinterpret_cast<uint4*>(line + (((4 * c + qq) ^ (lane & 7)) << 4)) = float8_to_bf16x8(o + 8 * qq);
          } else if (row_ok) {
#pragma unroll
            for (int qq = 0; qq < 4; ++qq) dst[4 * c + qq] = float8_to_bf16x8(o + 8 * qq);
          }
        }
        if (via_tma) {
          fence_proxy_async();
          __syncwarp();
          if (lane == 0) {
            tma::store_2d(&A.omap, 64 * grp, prow0, box);
            tma::store_commit();
            if (A.fuse) {   // other CTAs read these rows: complete, then order for generic loads
              tma::store_wait_all();
              asm volatile("fence.proxy.async.global;\n" ::: "memory");
            } else {
              tma::store_wait_read();
            }
          }
          __syncwarp();
        }
      }
    }
  }
  if (push) fence_proxy_async();   // the partial's rows -> the copy engine's reads
  fence_before_sync();
  __syncthreads();
  fence_after_sync();
  if (warp == 0) tmem_dealloc(taddr, kTmemCols);
  if (push) {
    // ---- pushed merge: lane j of the MMA warp copies rows [j mper, +mper) of this split's
    // partial (K slot 0) and their (m, l) into CTA j; this CTA merges its rows [lo, hi) of
    // every split from its own shared memory once rx_full has counted every byte
    const int lo = split * mper, hi = min(R_blk, lo + mper);
    if (warp == kSoftWarps && lane < (int)gridDim.y) {
      const int jlo = lane * mper, own = max(0, min(R_blk, jlo + mper) - jlo);
      if (own > 0) {
        const uint32_t bar = peer_addr(&rx_full, (uint32_t)lane);
        bulk_copy_to_peer(peer_addr(sRx + split * mper * 256, (uint32_t)lane), smem_addr(sKs + jlo * 256),
                          (uint32_t)(own * 256), bar);
        bulk_copy_to_peer(peer_addr(sRxML + split * mper, (uint32_t)lane),
                          smem_addr(reinterpret_cast<float4*>(sVs + kPushMlOffset) + jlo), (uint32_t)(own * 16), bar);
      }
    }
    const bool rx_ok = mbar_wait(&rx_full, 0u, kWaitNs);
    if (!rx_ok && threadIdx.x == 0) atomicExch(A.err, 1);
    cluster_arrive_relaxed();   // every copy into this CTA is done (its own copies' sources
                                // are free once every CTA has arrived; no data rides on it)
    __nv_bfloat16* out = reinterpret_cast<__nv_bfloat16*>(A.fm.out);
    PushedPartials src;
    src.o_base = sRx;
    src.ml_base = sRxML;
    src.per = mper;
    src.lo = lo;
    src.l16 = lane & 15;
    for (int rr0 = lo + 2 * warp; merge_warp && rr0 < hi; rr0 += 2 * kWarps) {   // uniform per warp
      const int rr = rr0 + (lane >> 4);
      src.i = (rr < hi ? rr : rr0) - lo;
      combine_row16_from<__nv_bfloat16>(A.q, H, A.nsplit, has_cur, out, A.fm.so[0], A.fm.so[1], A.fm.so[2],
                                        A.fm.m_p, A.fm.l_p, A.fm.o_p, bh, r0 + rr, rr < hi, src);
    }
    cluster_wait();   // no CTA leaves while a copy out of its shared memory may be running
    if (!rx_ok) mbar_wait(&rx_full, 0u, kWaitNs);   // late copies land before this CTA exits
    return;
  }
  if (A.cmerge) {
    // ---- cluster merge: the group's splits are the cluster's CTAs (rank = split); each
    // merges its share of the rows from every rank's shared memory, by half warps
    cluster_sync();   // every split's rows and (m, l) are in its shared memory
    const int per = (R_blk + (int)gridDim.y - 1) / (int)gridDim.y;
    const int lo = split * per, hi = min(R_blk, lo + per);
    __nv_bfloat16* out = reinterpret_cast<__nv_bfloat16*>(A.fm.out);
    ClusterPartials src;
    src.o_base = static_cast<uint32_t>(__cvta_generic_to_shared(sKs));
    src.ml_base = static_cast<uint32_t>(__cvta_generic_to_shared(sVs + 4096));
    src.l16 = lane & 15;
    for (int rr0 = lo + 2 * warp; merge_warp && rr0 < hi; rr0 += 2 * kWarps) {   // uniform per warp
      const int rr = rr0 + (lane >> 4);
      src.row = rr < hi ? rr : rr0;
      combine_row16_from<__nv_bfloat16>(A.q, H, A.nsplit, has_cur, out, A.fm.so[0], A.fm.so[1], A.fm.so[2],
                                        A.fm.m_p, A.fm.l_p, A.fm.o_p, bh, r0 + rr, rr < hi, src);
    }
    cluster_sync();   // no CTA leaves while another may still read its shared memory
    return;
  }
  if (!A.fuse) return;

  // ---- fused merge: every CTA of the (head, row block) group is resident (cooperative
  // launch); the last to arrive advances the group's generation, the others wait for it
  __threadfence();
  __syncthreads();
  if (threadIdx.x == 0) {
    bool ok = true;
    const unsigned prev = atomicAdd(&A.fm.sync[group].x, 1u);
    if (prev == gridDim.y - 1) {
      A.fm.sync[group].x = 0u;   // ready for the next call
      __threadfence();
      atomicAdd(&A.fm.sync[group].y, 1u);
    } else {
      const uint64_t t0 = global_ns();
      while (ld_acquire_u32(&A.fm.sync[group].y) == gen0) {
        if (global_ns() - t0 > A.fm.wait_ns) {
          ok = false;
          atomicExch(A.err, 1);
          break;
        }
        __nanosleep(128);
      }
    }
    s_merge_ok = ok ? 1 : 0;
    // the fused head gather: this call's number and the CTAs of the calls before it (the
    // last CTA of the previous call wrote them; this launch reads them only after that
    // launch completed: pdl_wait above)
    if (A.fm.gather) {
      s_epoch = *reinterpret_cast<volatile const uint32_t*>(A.fm.po.ws + 2) + 1u;
      s_cum = *reinterpret_cast<volatile const uint32_t*>(A.fm.po.ws + 4);
    }
  }
  __syncthreads();
  const PeerOut* po = A.fm.gather ? &A.fm.po : nullptr;
  const uint32_t pslot = s_epoch & 1u;
  // this split's share of the group's rows: a half warp per row with at most 16 prefix
  // splits, else a warp per row (weights scratch in the slots)
  const int per = (R_blk + (int)gridDim.y - 1) / (int)gridDim.y;
  const int lo = split * per, hi = min(R_blk, lo + per);
  __nv_bfloat16* out = reinterpret_cast<__nv_bfloat16*>(A.fm.out);
  if (A.nsplit <= 16 && s_merge_ok) {
    for (int rr0 = lo + 2 * warp; merge_warp && rr0 < hi; rr0 += 2 * kWarps) {   // uniform per warp
      const int rr = rr0 + (lane >> 4);
      combine_row16<__nv_bfloat16>(A.q, H, A.P, A.nsplit, has_cur, out, A.fm.so[0], A.fm.so[1], A.fm.so[2],
                                   A.fm.m_p, A.fm.l_p, A.fm.o_p, bh, r0 + rr, rr < hi, po, pslot);
    }
  } else {
    float* sW = reinterpret_cast<float*>(sKs) + warp * kCombineMaxSplits;
    for (int rr = lo + warp; merge_warp && rr < hi; rr += kWarps) {
      if (s_merge_ok) {
        combine_row<__nv_bfloat16, __nv_bfloat16>(A.q, H, A.P, A.nsplit, has_cur, out, A.fm.so[0], A.fm.so[1],
                                                  A.fm.so[2], A.fm.m_p, A.fm.l_p, A.fm.o_p, bh, r0 + rr, sW, po,
                                                  pslot);
      } else if (lane == 0) {   // a split never arrived: the row is reported as NaN
        const int rw = r0 + rr;
        const int g = rw / T, tt = rw - (rw / T) * T;
        __nv_bfloat16* dst = out + (int64_t)b * A.fm.so[0] + (int64_t)(h * G + g) * A.fm.so[1] + (int64_t)tt * A.fm.so[2];
        for (int d = 0; d < kD; ++d) dst[d] = __float2bfloat16_rn(NAN);
      }
    }
  }
  if (po == nullptr) return;

  // ---- fused head gather (every CTA of the launch is resident: cooperative launch). Each
  // CTA, once its rows are stored, adds 1 to its rank's arrival counter in every rank's
  // region -- a release reduction at system scope: the CTA barrier makes every thread's
  // peer stores observed by thread 0 and the release is cumulative, so one per CTA orders
  // them all (a fence in every thread measured ~1.5 us slower per call) -- then waits
  // (bounded) until every rank's counter in this rank's region holds the CTAs of every
  // call so far (every rank runs the same calls with the same grids, so the running
  // totals agree), and copies its share of the slot -- every rank's rows -- into the
  // gathered output; the last CTA to finish records the call. A rank is at most one call
  // ahead of another (it cannot finish call e + 1 before every CTA of every rank arrived
  // for e + 1), so the two slots never mix calls.
  __syncthreads();
  const uint32_t nctas = gridDim.x * gridDim.y * gridDim.z;
  const uint32_t ep = s_epoch, want = s_cum + nctas;
  if (threadIdx.x == 0) {
    for (int p = 0; p < po->world; ++p) {
      uint32_t* cnt = reinterpret_cast<uint32_t*>(po->base[p] + 2 * po->slot_bytes) + po->rank;
      asm volatile("red.release.sys.global.add.u32 [%0], 1;\n" ::"l"(cnt) : "memory");
    }
    const uint32_t* mine = reinterpret_cast<const uint32_t*>(po->base[po->rank] + 2 * po->slot_bytes);
    const uint64_t t0 = global_ns();
    bool ok = true;
    for (int p = 0; p < po->world && ok; ++p) {
      for (;;) {
        uint32_t f;
        asm volatile("ld.acquire.sys.global.u32 %0, [%1];\n" : "=r"(f) : "l"(mine + p) : "memory");
        if ((int32_t)(f - want) >= 0) break;
        if (global_ns() - t0 > A.fm.wait_ns) {
          ok = false;
          break;
        }
      }
    }
    if (!ok) atomicExch(A.err, 1);
    s_gather_ok = ok ? 1 : 0;
  }
  __syncthreads();
  if (s_gather_ok) {
    asm volatile("fence.acq_rel.sys;\n" ::: "memory");
    const int Hq = po->Hl * po->world, Tg = po->Tg;
    const char* src = po->base[po->rank] + (int64_t)pslot * po->slot_bytes;
    __nv_bfloat16* gout = reinterpret_cast<__nv_bfloat16*>(po->out);
    const int64_t chunks = (int64_t)A.q.B * Hq * Tg * (kD / 8);
    const int64_t cta = ((int64_t)blockIdx.z * gridDim.y + blockIdx.y) * gridDim.x + blockIdx.x;
    for (int64_t i = cta * blockDim.x + threadIdx.x; i < chunks; i += (int64_t)nctas * blockDim.x) {
      const int c = (int)(i & 15);
      const int64_t row = i >> 4;
      const int t = (int)(row % Tg);
      const int64_t bq = row / Tg;
      const int hq = (int)(bq % Hq), bb = (int)(bq / Hq);
      const uint4 v = __ldcg(reinterpret_cast<const uint4*>(src + row * (kD * 2)) + c);
      reinterpret_cast<uint4*>(gout + (int64_t)bb * po->so[0] + (int64_t)hq * po->so[1] + (int64_t)t * po->so[2])[c] = v;
    }
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    uint32_t* gw = po->ws;
    if (atomicAdd(gw + 3, 1u) == nctas - 1) {
      gw[3] = 0u;
      gw[4] = want;
      gw[2] = ep;
    }
  }
}

// The bf16 kernels (320 threads: softmax, MMA and TMA warps) and the PACKED ones (384
// threads: 12 warps, three on each SM sub-partition, whose quarter of the register file
// leaves 168 registers a thread), for one M tile per CTA or a pair.
__global__ void __launch_bounds__(kThreadsB, 1) attn_partial_fa(const __grid_constant__ Args A) {
  attn_fa_body<false, false>(A);
}
__global__ void __launch_bounds__(kThreadsP, 1) attn_partial_fa_packed(const __grid_constant__ Args A) {
  attn_fa_body<true, false>(A);
}
__global__ void __launch_bounds__(kThreadsB, 1) attn_partial_fa_pair(const __grid_constant__ Args A) {
  attn_fa_body<false, true>(A);
}
__global__ void __launch_bounds__(kThreadsP, 1) attn_partial_fa_pair_packed(const __grid_constant__ Args A) {
  attn_fa_body<true, true>(A);
}

int g_pairs = 0;   // fa_set_pairs


bool tma_map_rows(CUtensorMap* map, const void* base, int B, int H, int n, const int64_t s[3]) {
  // bf16 [B][H][n][128] with element strides s (b, h, row); box: 64 channels x 128 rows
  const uint64_t dims[4] = {128, (uint64_t)n, (uint64_t)H, (uint64_t)B};
  const uint64_t strides[3] = {(uint64_t)s[2] * 2, (uint64_t)s[1] * 2, (uint64_t)s[0] * 2};
  const uint32_t box[4] = {64, (uint32_t)kBN, 1, 1};
  return make_tma_map_bf16_4d(map, base, dims, strides, box);
}

}  // namespace

int fa_key_tile() { return kBN; }
void fa_set_pairs(int mode) { g_pairs = mode; }
int fa_row_tile(int R, int BH) {
  // automatic: pairs when the (KV head, M tile) units alone fill the GPU (a serving batch),
  // so that sharing each K/V tile between two M tiles does not cost parallelism; below
  // that, one M tile per CTA and more splits (a single long sequence)
  const bool many = (long long)BH * ((R + kRowTile - 1) / kRowTile) > device_sm_count();
  const bool pair = g_pairs == 2 || (g_pairs == 0 && many);
  return pair && R > kRowTile ? 2 * kRowTile : kRowTile;
}

bool fa_eligible(const ma_rows& q, const ma_kv& kv, const int64_t* idx, const ma_block& cur, int n_keys) {
  const bool dense_ok = kv.layout == MA_KV_DENSE && kv.dtype == MA_BF16 && !kv.mask && !kv.pages;
  // a token-mode packed prefix: the PACKED instantiation's producer warps read it in place
  const bool packed_ok = kv.dtype == MA_BF16 && packed::eligible(kv) && n_keys == kv.nq;
  const bool prefix_ok = n_keys == 0 || (!idx && (dense_ok || packed_ok));
  // a row tile is 128 / T whole query heads, 128 positions of one head, or four 32-row
  // pieces (each within one head)
  const bool rows_ok = q.T > 0 && (kRowTile % q.T == 0 || q.T % 32 == 0);
  return q.dtype == MA_BF16 && q.D == kD && rows_ok && prefix_ok && (n_keys > 0 || cur.Tc > 0);
}

int launch_attn_partial_fa(const ma_rows& q, const ma_kv& kv, int H, const ma_block& cur, float scale,
                           int causal_block, int q_pos0, int c_pos0, int n_keys, int split_len, int nsplit,
                           const Partials& P, int* err, const FusedMerge* fm, bool fold, bool* fused,
                           bool* gathered, cudaStream_t st) {
  *fused = false;
  if (gathered) *gathered = false;
  if (!fa_eligible(q, kv, nullptr, cur, n_keys) || !(scale > 0.f) || !P.o_bf16 || split_len % kBN != 0)
    return MA_ERR_UNSUPPORTED;
  const bool packed = n_keys > 0 && kv.layout == MA_KV_PACKED_TOKEN;
  // a folded block: only into bf16 prefix splits, one key tile of the block, no causal mask
  if (fold && (packed || causal_block > 0 || cur.Tc <= 0 || cur.Tc > kBN || n_keys <= 0 || nsplit < 1 ||
               P.S != nsplit || fm == nullptr || fm->m_p || fm->l_p || fm->o_p))
    return MA_ERR_ARG;
  const int threads = packed ? kThreadsP : kThreadsB;
  const int G = q.Hq / H;
  const int R = G * q.T;
  const int rows = fa_row_tile(R, q.B * H);   // the plan's row blocks: one M tile per CTA or a pair
  const bool pair = rows > kRowTile;
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
  A.fold = fold ? 1 : 0;
  if (n_keys > 0 && !packed && !(tma_map_rows(&A.kmap, kv.kf, q.B, H, kv.nf, kv.skf) &&
                                  tma_map_rows(&A.vmap, kv.vf, q.B, H, kv.nf, kv.svf)))
    return MA_ERR_UNSUPPORTED;
  if (cur.Tc > 0 && !(tma_map_rows(&A.ckmap, cur.k, q.B, H, cur.Tc, cur.sk) &&
                      tma_map_rows(&A.cvmap, cur.v, q.B, H, cur.Tc, cur.sv)))
    return MA_ERR_UNSUPPORTED;
  {
    const uint64_t dims[4] = {128, (uint64_t)q.T, (uint64_t)q.Hq, (uint64_t)q.B};
    const uint64_t strides[3] = {(uint64_t)q.sq[2] * 2, (uint64_t)q.sq[1] * 2, (uint64_t)q.sq[0] * 2};
    A.q_mode = (q.T % kRowTile == 0) ? 1 : (kRowTile % q.T == 0) ? 0 : 2;
    const uint32_t box[4] = {64, (uint32_t)(A.q_mode == 1 ? kRowTile : A.q_mode == 0 ? q.T : 32),
                             (uint32_t)(A.q_mode == 0 ? kRowTile / q.T : 1), 1};
    if (!make_tma_map_bf16_4d(&A.qmap, q.q, dims, strides, box)) return MA_ERR_UNSUPPORTED;
  }
  // partial rows [BH * S * Rp][D] bf16, stored by 32-row x 64-channel boxes
  const uint64_t prow_total = (uint64_t)q.B * H * P.S * P.Rp;
  A.tma_out = (P.Rp % 32 == 0 && prow_total < (1ull << 31) &&
               make_tma_map_2d(&A.omap, true, P.o, kD, prow_total, kD * 2, 64, 32)) ? 1 : 0;
  dim3 grid((R + rows - 1) / rows, P.S, q.B * H);
  const int kid = (packed ? 1 : 0) + (pair ? 2 : 0);
  auto kernel = pair ? (packed ? attn_partial_fa_pair_packed : attn_partial_fa_pair)
                     : (packed ? attn_partial_fa_packed : attn_partial_fa);
  const int smem = pair ? (packed ? kSmemBytesP2 : kSmemBytes2) : (packed ? kSmemBytesP : kSmemBytes);
  if (cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, smem) != cudaSuccess)
    return MA_ERR_CUDA;
  const int rows_per_split = (std::min(rows, R) + (int)grid.y - 1) / (int)grid.y;
  // a head gather runs only inside the cooperative merge (its CTAs wait for one another);
  // without one the caller gathers in separate launches
  const bool gather = fm != nullptr && fm->gather;
  if (fold && grid.y == 1 && !gather) {
    // one split holds every key of its rows: they are final in the epilogue, no merge
    Args Ad = A;
    Ad.direct = 1;
    Ad.fm = *fm;
    if (launch_pdl(kernel, grid, dim3(threads), smem, st, Ad) != cudaSuccess) return MA_ERR_CUDA;
    *fused = true;
    return MA_OK;
  }
  // cluster merge: with at most 16 splits (prefix ones + the block) a group's CTAs form one
  // thread-block cluster and merge through distributed shared memory (no global round
  // trips); the hardware co-schedules a cluster's CTAs, so no cooperative launch is needed.
  // Only when every cluster is resident at once: a cluster of one-CTA-per-SM blocks needs
  // that many free SMs in one GPC, so fewer clusters than SMs / size fit (a second wave
  // of clusters cost more than the merge saves)
  if (fm != nullptr && !gather && nsplit <= 16 && (int)grid.y <= 16 && rows_per_split <= 2 * kWarps) {
    static int cluster_nc_of[4][17] = {{0}};   // per kernel and cluster size: resident clusters (-1: none)
    int* cluster_nc = cluster_nc_of[kid];
    const int cs = (int)grid.y;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = dim3(threads);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = st;
    cudaLaunchAttribute attr[2];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = 1;
    attr[0].val.clusterDim.y = cs;
    attr[0].val.clusterDim.z = 1;
    attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[1].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    if (cluster_nc[cs] == 0) {
      int nc = 0;
      const bool attr_ok = cs <= 8 ||
                           cudaFuncSetAttribute(kernel, cudaFuncAttributeNonPortableClusterSizeAllowed, 1) == cudaSuccess;
      cluster_nc[cs] = (attr_ok && cudaOccupancyMaxActiveClusters(&nc, kernel, &cfg) == cudaSuccess && nc >= 1) ? nc : -1;
      (void)cudaGetLastError();
    }
    if (cluster_nc[cs] > 0 && (long long)grid.x * grid.z <= cluster_nc[cs]) {
      Args Ac = A;
      // one key tile per CTA: the splits push their rows to the merging CTA (K slots 1
      // and 2 of every CTA stay free), else every CTA pulls them from the others
      Ac.cmerge = (!pair && !packed && !fold && split_len <= kBN && cur.Tc <= kBN) ? 2 : 1;
      Ac.fm = *fm;
      cfg.numAttrs = 2;
      if (cudaLaunchKernelEx(&cfg, kernel, Ac) == cudaSuccess) {
        *fused = true;
        return MA_OK;
      }
      (void)cudaGetLastError();
    }
  }
  // fused merge: one wave of resident CTAs (cooperative launch), when each split's share of
  // the rows is one pass of its warps
  const int rows_per_pass = nsplit <= 16 ? 2 * kWarps : kWarps;   // half warps or warps per row
  if (fm != nullptr && (int)(grid.x * grid.z) <= fm->sync_slots && (int)grid.y <= kCombineMaxSplits &&
      rows_per_split <= rows_per_pass) {
    int dev = 0, coop = 0, per_sm = 0;
    if (cudaGetDevice(&dev) == cudaSuccess &&
        cudaDeviceGetAttribute(&coop, cudaDevAttrCooperativeLaunch, dev) == cudaSuccess && coop &&
        cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kernel, threads, smem) == cudaSuccess &&
        (long long)grid.x * grid.y * grid.z <= (long long)per_sm * device_sm_count()) {
      Args Af = A;
      Af.fuse = 1;
      Af.fm = *fm;
      cudaLaunchConfig_t cfg = {};
      cfg.gridDim = grid;
      cfg.blockDim = dim3(threads);
      cfg.dynamicSmemBytes = smem;
      cfg.stream = st;
      cudaLaunchAttribute attr[2];
      attr[0].id = cudaLaunchAttributeCooperative;
      attr[0].val.cooperative = 1;
      attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;   // tried first
      attr[1].val.programmaticStreamSerializationAllowed = 1;
      cfg.attrs = attr;
      for (int na = 2; na >= 1; --na) {
        cfg.numAttrs = na;
        if (cudaLaunchKernelEx(&cfg, kernel, Af) == cudaSuccess) {
          *fused = true;
          if (gathered) *gathered = gather;
          return MA_OK;
        }
        (void)cudaGetLastError();
      }
    }
  }
  return launch_pdl(kernel, grid, dim3(threads), smem, st, A) == cudaSuccess ? MA_OK : MA_ERR_CUDA;
}

}  // namespace ma

