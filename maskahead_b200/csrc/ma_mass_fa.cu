// Prefix mass, value-score centre and value score for contiguous bf16 caches read by TMA,
// with a warp-specialized pipeline (the TMA-fed counterpart of ma_mass_tc.cu).
//
// Per slot j of the prefix, over the R2 = G*T2 selection rows r of its KV head:
//     a_j = (1/R2) sum_r 2^(s_rj * scale * log2e - B_r),  B_r = M_p,r log2e + log2 L_p,r
// (splitk.py:320-359; reference.py:318-366), the head's centre
//     c = sum_j a_j v_j / max(sum_j a_j, 1e-12)            (session.py:27-40, 870-899)
// and the value score a_j ||v_j - c||.
//
// CTA = 8 sum warps + 1 producer/MMA warp + 2 centre warps over one slot range of one head
// (one wave of CTAs). Phase 1, per tile of 128 slots: the producer streams K and V tiles by
// TMA (ring slots of 32 KB), issues S^T = K Q^T (tcgen05, M = 128 slots, N = the selection
// rows padded to 16, double-buffered in tensor memory); sum warp w owns slot lane 32(w&3)..
// and half of the rows (w>>2): it sums its exponentials from tensor memory, the halves meet
// in shared memory, a_j is written (and handed to the centre warps through a double
// buffer); centre warp c accumulates sum_j a_j v_j over slots 64c.. of the V tile while
// the sum warps go on to the next tile. The last CTA of the head reduces the per-CTA partials
// in CTA order into c and advances the head's generation word. Phase 2 (cooperative
// launch, every CTA resident): each CTA waits (bounded) for the generation, the producer
// streams its V tiles again (newest first: V was loaded with an L2 evict_last policy, so
// most come from L2) through all four slots, and the sum warps write a_j ||v_j - c||.
// Every wait is bounded.
//
// Packed (token-mode k4v4) prefixes: the PACKED instantiation adds four producer warps
// that build the K tiles (for S^T) and, with the centre, the V tiles of phase 1 from the
// packed bytes (ma_packed.cuh); the producer/MMA warp releases their slots on kfree / vfree
// where it would have issued TMA loads. Phase 2 reads V from its phase-1 slots when they
// still hold every tile, else the sum warps read the packed V rows themselves and dequantize
// them exactly as the tiles hold them.
#include <string.h>

#include "ma_kernels.cuh"
#include "ma_packed.cuh"
#include "ma_stage.cuh"
#include "ma_tcgen05.cuh"
#include "ma_tma.cuh"

namespace ma {

namespace {

using namespace tc;

constexpr int kSumWarps = 8;
constexpr int kSumThreads = kSumWarps * 32;
static_assert(kSumThreads == 256, "one selection row per sum thread");
constexpr int kCentreWarps = 2;              // sum_j a_j v_j: warp c takes slots 64c..64c+63 of each tile
constexpr int kThreads = kSumThreads + 32 + kCentreWarps * 32;
constexpr int kDqWarps = 4;                  // dequantizing producer warps (PACKED)
constexpr int kThreadsP = kThreads + kDqWarps * 32;
constexpr int kPrefetchTiles = 4;            // L2 prefetch distance of the packed rows (tiles)
constexpr int kTile = 128;                   // slots per tile (= M = TMEM lanes)
constexpr int kD = 128;
constexpr int kMaxRows = 256;                // selection rows (N of the MMA)
constexpr int kBlock = kTile * 128;          // one 64-channel box of a tile: 16 KB
constexpr int kTileBytes = 2 * kBlock;       // a K or V tile: 32 KB
constexpr int kMaxSlots = 6;                 // tile slots (phase 1: K ring, then V ring; phase 2: V in all)
constexpr int kSmemLimit = 227 * 1024;       // dynamic + static shared memory of one CTA
constexpr int kStaticSmem = 8 * 1024;        // bound on this kernel's static shared memory
constexpr uint32_t kTmemCols = 512;          // two S^T buffers of up to 256 columns
constexpr int kRaggedTiles = 16;             // tiles per CTA at most, for a ragged batch of few heads
constexpr float kLog2e = 1.4426950408889634f;
constexpr uint64_t kWaitNs = 200000000ull;
constexpr uint64_t kStallNs = 500000000ull;
constexpr unsigned kIdleNs = 64;                   // producer back-off when nothing was ready

struct __align__(64) Args {
  CUtensorMap kmap, vmap;   // K/V [B][H][n][D], boxes of 64 channels x 128 slots
  ma_rows q;
  ma_kv kv;
  const int32_t* q_rows;
  const float* m_p;
  const float* l_p;
  float* mass;
  int64_t sm0, sm1;
  float* score;             // phase 2 (cooperative launch), or null
  int64_t ss0, ss1;
  float* part;              // [BH][ctas][D+1] centre partials (centre only)
  uint2* sync;              // [BH]: arrival counter, centre generation
  float* centre;            // [BH][D]
  int* err;
  float scale;
  int H, T2, slots_per_cta, want_centre;
  int nK, nV;               // K ring and V ring slots (phase 2 streams V through nK + nV)
  int given;                // a_j given in `mass` (value score only: no K, no exponentials)
  int score_only;           // phase 2 alone: a_j in `mass` and the centre in `centre` are final
  uint64_t peer_wait_ns;    // bound on the wait for the head's centre (other CTAs)
};

__device__ __forceinline__ void sum_sync() { asm volatile("bar.sync 1, %0;\n" ::"r"(kSumThreads) : "memory"); }

__device__ __forceinline__ void tile_load(const CUtensorMap* map, int b, int h, int j0, uint8_t* dst, uint64_t* bar,
                                          uint64_t policy) {
  tma::expect_tx(bar, kTileBytes);
  tma::load_4d_hint(dst, map, 0, j0, h, b, bar, policy);
  tma::load_4d_hint(dst + kBlock, map, 64, j0, h, b, bar, policy);
}

// byte offset of channel chunk c (8 channels) of slot row j in a TMA tile (two 64-channel
// boxes of 128 lines, 128-byte swizzle)
__device__ __forceinline__ uint32_t chunk_off(int j, int c) {
  return (uint32_t)((c >> 3) * kBlock + j * 128 + (((c & 7) ^ (j & 7)) << 4));
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

template <bool PACKED>
__device__ __forceinline__ void mass_fa_body(const Args& A) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sQ = smem;                      // K-major [2 d blocks][Npad rows][128 B]
  __shared__ __align__(16) float sNB[kMaxRows];  // per selection row: -B_r (-inf: no contribution)
  __shared__ float sHalf[2][kTile];
  __shared__ __align__(16) float sA[2][kTile];   // a_j of tiles t&1 (sum warps -> centre warps)
  __shared__ float sTot[2][kD + 1];
  __shared__ uint32_t s_taddr;
  __shared__ __align__(8) uint64_t kfull[kMaxSlots], vfull[kMaxSlots], s_full[2], s_free[2], v_free[kMaxSlots],
      wfull[kMaxSlots], wfree[kMaxSlots], a_full[2], a_free[2], mbar_fin;
  __shared__ int s_abort, s_wait_ok, sLast;
  __shared__ __align__(8) uint64_t kfree[PACKED ? kMaxSlots : 1], vfree[PACKED ? kMaxSlots : 1];
  __shared__ __align__(16) float sKch[PACKED ? kD : 1];   // the packed keys' divisor of this (b, h)

  const int n = PACKED ? A.kv.nq : A.kv.nf;   // the packed layout has no dense slots
  const int bh = blockIdx.y;
  const int H = A.H;
  const int b = bh / H, h = bh - (bh / H) * H;
  const int G = A.q.Hq / H;
  const int T = A.q.T;
  const int R2 = G * A.T2;
  const int Npad = (R2 + 15) & ~15;
  uint8_t* sSlot = sQ + Npad * 256;        // nK + nV tile slots (Npad * 256 is a multiple of 4 KB)
  const int nK = A.nK, nV = A.nV, nS = A.nK + A.nV;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const bool sum_warp = warp < kSumWarps;
  const int quarter = warp & 3, chalf = (warp >> 2) & 1;
  const int slot_lane = quarter * 32 + lane;          // this thread's slot within a tile (TMEM lane)
  const int begin = blockIdx.x * A.slots_per_cta;
  const int end_all = min(n, begin + A.slots_per_cta);
  int end = end_all;
  if (A.kv.lens) {   // a ragged batch: no work past lens[b] (lens may come from the kernel
    pdl_wait();      // before, with a programmatic launch); those slots get 0 below
    end = max(begin, min(end_all, A.kv.lens[b]));
  }
  const bool score_only = A.score_only != 0;
  const int ntiles2 = end > begin ? (end - begin + kTile - 1) / kTile : 0;   // phase 2's tiles
  const int ntiles = score_only ? 0 : ntiles2;                               // phase 1's
  const float inv_rows = 1.f / (float)R2;
  const float c2 = A.scale * kLog2e;
  const bool centre = A.want_centre != 0;
  const bool given = A.given != 0;
  const int kTiles = given ? 0 : ntiles;     // tiles that need K and S^T

  // the head's centre generation before this CTA arrives (the last CTA advances it)
  unsigned gen0 = 0;   // read after pdl_wait (below), before this CTA arrives
  if (threadIdx.x == kSumThreads) {
    if (!PACKED) {   // the packed instantiation has no tensor maps
      asm volatile("prefetch.tensormap [%0];\n" ::"l"(reinterpret_cast<uint64_t>(&A.kmap)) : "memory");
      asm volatile("prefetch.tensormap [%0];\n" ::"l"(reinterpret_cast<uint64_t>(&A.vmap)) : "memory");
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&s_full[i], 1);
      mbar_init(&s_free[i], kSumWarps);
      mbar_init(&a_full[i], 1);
      mbar_init(&a_free[i], kCentreWarps);
    }
    for (int i = 0; i < kMaxSlots; ++i) {
      mbar_init(&kfull[i], PACKED ? kDqWarps : 1);
      mbar_init(&vfull[i], PACKED ? kDqWarps : 1);
      if (PACKED) {
        mbar_init(&kfree[i], 1);
        mbar_init(&vfree[i], 1);
      }
      mbar_init(&v_free[i], kCentreWarps);
      mbar_init(&wfull[i], 1);
      mbar_init(&wfree[i], kSumWarps);
    }
    mbar_init(&mbar_fin, 1);
    s_abort = 0;
    s_wait_ok = 1;
    asm volatile("fence.mbarrier_init.release.cluster;\n" ::: "memory");
    // the first K and V tiles start loading now, while the sum warps stage Q
    pdl_wait();   // with a programmatic launch, the cache may come from the kernel before
    const uint64_t pol_k = tma::policy_evict_first(), pol_v = tma::policy_evict_last();
    if (!PACKED) {
      for (int i = 0; i < nK && i < kTiles; ++i)
        tile_load(&A.kmap, b, h, begin + i * kTile, sSlot + i * kTileBytes, &kfull[i], pol_k);
      if (centre)
        for (int i = 0; i < nV && i < ntiles; ++i)
          tile_load(&A.vmap, b, h, begin + i * kTile, sSlot + (nK + i) * kTileBytes, &vfull[i], pol_v);
    }
  }
  if (sum_warp && given) {
    pdl_wait();   // a (and with a programmatic launch, the outputs) of the kernel before
    if (centre && threadIdx.x == 0) gen0 = *reinterpret_cast<volatile const unsigned*>(&A.sync[bh].y);
  } else if (sum_warp) {
    pdl_wait();   // m_p, l_p (and with a programmatic launch, the outputs) of the kernel before
    if (centre && threadIdx.x == 0) gen0 = *reinterpret_cast<volatile const unsigned*>(&A.sync[bh].y);
    // one selection row per thread (kSumThreads == kMaxRows): r2 = g*T2 + i -> query row
    // (h*G + g, q_rows[i]), -B_r, and the row's query into the K-major SW128 Q tile of Npad
    // rows (zeros for padding rows)
    {
      const int rr = threadIdx.x;
      const int g = rr / A.T2;
      const int t = rr < R2 ? A.q_rows[rr - g * A.T2] : -1;
      const bool ok = t >= 0 && t < T;
      if (rr < Npad) {
        const __nv_bfloat16* qrow = reinterpret_cast<const __nv_bfloat16*>(A.q.q) + (int64_t)b * A.q.sq[0] +
                                    (int64_t)(h * G + g) * A.q.sq[1] + (int64_t)(ok ? t : 0) * A.q.sq[2];
#pragma unroll
        for (int ch = 0; ch < kD / 8; ++ch) {
          uint8_t* dst = sQ + kmajor_off(rr, ch, Npad);
          if (ok) cp_async16(smem_addr(dst), qrow + ch * 8, true);
          else *reinterpret_cast<uint4*>(dst) = make_uint4(0, 0, 0, 0);
        }
      }
      float Bv = INFINITY;   // exp2(s - inf) = 0: no contribution
      if (ok) {
        const int64_t ri = (int64_t)bh * G * T + (int64_t)g * T + t;
        const float L = A.l_p[ri];
        if (L > 0.f) Bv = fmaf(A.m_p[ri], kLog2e, log2f(L));
      }
      sNB[rr] = -Bv;
    }
    cp_async_commit();
    cp_async_wait<0>();
    fence_proxy_async();
  }
  if (warp == 0) tmem_alloc(&s_taddr, kTmemCols);
  fence_before_sync();
  __syncthreads();
  fence_after_sync();
  const uint32_t taddr = s_taddr;
  // centre warps: warp c accumulates a_j v_j over slots 64c.. of each tile, lane l over
  // channels 4l..4l+3
  float2 cacc0 = make_float2(0.f, 0.f), cacc1 = cacc0;
  float asum = 0.f;
  const int cw = warp - kSumWarps - 1;   // 0.. for the centre warps
  const bool dq_warp = PACKED && cw >= kCentreWarps;   // the producer warps (PACKED)

  if (dq_warp) {
    // ------------------------------------------------------------ producer warps (PACKED)
    // thread dt builds row dt of every K tile (slot t % nK, once released on kfree; the
    // first nK are free) and, with the centre, of every V tile (slot nK + t % nV)
    const int dt = threadIdx.x - kThreads;
    const bool want_k = kTiles > 0, want_v = centre;
    pdl_wait();   // with a programmatic launch, the cache may come from the kernel before
    if (want_k) sKch[dt] = A.kv.kchan[(int64_t)b * A.kv.skc[0] + (int64_t)h * A.kv.skc[1] + dt];
    if (dt == 0)
      for (int t = 0; t < kPrefetchTiles && t < ntiles; ++t)
        packed::prefetch_rows(A.kv, b, h, begin + t * kTile, min(end, begin + (t + 1) * kTile));
    asm volatile("bar.sync 6, %0;\n" ::"r"(kDqWarps * 32) : "memory");
    if (want_k || want_v) {
      packed::RawRow cur, nxt;
      packed::load_row(A.kv, b, h, begin + dt, end, cur, want_k, want_v);
      for (int t = 0; t < ntiles; ++t) {
        const int tp = t + kPrefetchTiles;
        if (dt == 0 && tp < ntiles)
          packed::prefetch_rows(A.kv, b, h, begin + tp * kTile, min(end, begin + (tp + 1) * kTile));
        if (t + 1 < ntiles) packed::load_row(A.kv, b, h, begin + (t + 1) * kTile + dt, end, nxt, want_k, want_v);
        if (want_k) {
          if (t >= nK && !dq_wait(&kfree[t % nK], (uint32_t)((t / nK) - 1) & 1u, &s_abort)) break;
          packed::store_row<true>(cur.k, cur.ok, sSlot + (t % nK) * kTileBytes, dt, sKch);
          fence_proxy_async();   // generic stores -> the tensor core's reads
          __syncwarp();
          if (lane == 0) mbar_arrive(&kfull[t % nK]);
        }
        if (want_v) {
          if (t >= nV && !dq_wait(&vfree[t % nV], (uint32_t)((t / nV) - 1) & 1u, &s_abort)) break;
          packed::store_row<false>(cur.v, cur.ok, sSlot + (nK + t % nV) * kTileBytes, dt, nullptr);
          __syncwarp();
          if (lane == 0) mbar_arrive(&vfull[t % nV]);
        }
        cur = nxt;
      }
    }
  } else if (cw >= 0) {
    // ------------------------------------------------------------ centre warps
    if (centre) {
      const uint32_t lane_off = (uint32_t)((lane & 1) * 8);   // channels 4l..: half of chunk l/2
      for (int t = 0; t < ntiles; ++t) {
        bool ok = mbar_wait(&a_full[t & 1], (uint32_t)(t >> 1) & 1u, kWaitNs);
        ok = ok && mbar_wait(&vfull[t % nV], (uint32_t)(t / nV) & 1u, kWaitNs);
        if (!ok) s_abort = 1;
        if (!ok || s_abort) break;
        const uint8_t* sV = sSlot + (nK + t % nV) * kTileBytes;
        const float* a = sA[t & 1];
#pragma unroll 8
        for (int i = 0; i < 64; ++i) {
          const int j = 64 * cw + i;
          const float aj = a[j];
          const uint2 u = *reinterpret_cast<const uint2*>(sV + chunk_off(j, lane >> 1) + lane_off);
          const float2 v0 = make_float2(__uint_as_float(u.x << 16), __uint_as_float(u.x & 0xFFFF0000u));
          const float2 v1 = make_float2(__uint_as_float(u.y << 16), __uint_as_float(u.y & 0xFFFF0000u));
          cacc0 = ffma2(make_float2(aj, aj), v0, cacc0);
          cacc1 = ffma2(make_float2(aj, aj), v1, cacc1);
          asum += aj;
        }
        __syncwarp();
        if (lane == 0) {
          mbar_arrive(&v_free[t % nV]);
          mbar_arrive(&a_free[t & 1]);
        }
      }
    }
  } else if (!sum_warp) {
    // ------------------------------------------------------------ producer / MMA warp
    if (lane == 0) {
      bool ok = true;
      // the first min(nK, ntiles) K and min(nV, ntiles) V tiles were issued at setup
      int kIss = min(nK, kTiles), kObs = 0, vIss = centre ? min(nV, ntiles) : 0, vObs = 0;
      int sN = 0, sDone = 0, sfObs = 0, vfObs = 0;
      const uint64_t pol_k = tma::policy_evict_first(), pol_v = tma::policy_evict_last();
      const int vTiles = centre ? ntiles : 0;
      const uint32_t idesc = idesc_bf16(kTile, Npad, false, false);
      const uint64_t kdesc = smem_desc(smem_addr(sSlot), 16, 1024);
      const uint64_t qdesc = smem_desc(smem_addr(sQ), 16, 1024);
      const uint32_t qblk = (uint32_t)(Npad * 128);   // bytes of one 64-channel block of Q
      uint64_t t_idle = 0;
      bool armed = false;
      int spins = 0;
      while (ok && (sN < kTiles || kIss < kTiles || vIss < vTiles)) {
        bool progress = false;
        if (kObs < kIss && mbar_test(&kfull[kObs % nK], (uint32_t)(kObs / nK) & 1u)) {
          ++kObs;
          progress = true;
        }
        if (sDone < sN && mbar_test(&s_full[sDone & 1], (uint32_t)(sDone >> 1) & 1u)) {
          ++sDone;
          progress = true;
        }
        if (sfObs < sDone && mbar_test(&s_free[sfObs & 1], (uint32_t)(sfObs >> 1) & 1u)) {
          ++sfObs;
          progress = true;
        }
        if (vfObs < vObs && mbar_test(&v_free[vfObs % nV], (uint32_t)(vfObs / nV) & 1u)) {
          ++vfObs;
          progress = true;
        }
        if (vObs < vIss && mbar_test(&vfull[vObs % nV], (uint32_t)(vObs / nV) & 1u)) {
          ++vObs;
          progress = true;
        }
        // S^T(t) = K(t) Q^T into buffer t&1, once K(t) is in and the sum warps released
        // the buffer's previous tile
        if (sN < kTiles && kObs > sN && sfObs >= sN - 1 && sDone >= sN - 1) {
          fence_after_sync();
          const uint64_t ad0 = kdesc + (uint64_t)((sN % nK) * (kTileBytes >> 4));
          const uint32_t d = taddr + (sN & 1) * 256;
#pragma unroll
          for (int kk = 0; kk < kD / 16; ++kk)
            mma_bf16(d, ad0 + (uint64_t)(((kk >> 2) * kBlock + (kk & 3) * 32) >> 4),
                     qdesc + (uint64_t)(((kk >> 2) * qblk + (kk & 3) * 32) >> 4), idesc, kk > 0);
          mma_commit(&s_full[sN & 1]);
          ++sN;
          progress = true;
        }
        // K slot of tile kIss - nK is free once its S^T completed
        if (kIss < kTiles && sDone > kIss - nK) {
          if (PACKED) mbar_arrive(&kfree[kIss % nK]);   // the producer warps may refill it
          else tile_load(&A.kmap, b, h, begin + kIss * kTile, sSlot + (kIss % nK) * kTileBytes, &kfull[kIss % nK],
                         pol_k);
          ++kIss;
          progress = true;
        }
        // V slot of tile vIss - nV is free once the sum warps released it
        if (vIss < vTiles && vfObs > vIss - nV) {
          if (PACKED) mbar_arrive(&vfree[vIss % nV]);
          else tile_load(&A.vmap, b, h, begin + vIss * kTile, sSlot + (nK + vIss % nV) * kTileBytes,
                         &vfull[vIss % nV], pol_v);
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
      // drain (bounded): every MMA, every load still in flight
      mma_commit(&mbar_fin);
      mbar_wait(&mbar_fin, 0, 20000000ull);
      if (!PACKED) {   // TMA loads still in flight (the producer warps' stores end with them)
        for (int tt = kObs; tt < kIss; ++tt) mbar_wait(&kfull[tt % nK], (uint32_t)(tt / nK) & 1u, 20000000ull);
        for (int tt = vObs; tt < vIss; ++tt) mbar_wait(&vfull[tt % nV], (uint32_t)(tt / nV) & 1u, 20000000ull);
      }
    }
    __syncwarp();
  } else {
    // ------------------------------------------------------------ sum warps
    __shared__ int sDecide;
    const uint32_t tRow = taddr + ((uint32_t)(quarter * 32) << 16);
    const float2 c2x2 = make_float2(c2, c2);
    // the two warps of a slot quarter split the Npad row columns evenly: half 0 takes
    // [0, h0), half 1 [h0, Npad) (h0 = Npad / 2 rounded up to 16), in 32-column chunks and
    // a 16-column tail; rows past R2 read -inf from sNB
    const int h0 = ((Npad / 2 + 15) / 16) * 16;
    const int col_lo = chalf ? h0 : 0, col_hi = chalf ? Npad : h0;
    for (int t = 0; t < ntiles; ++t) {
      const int j0 = begin + t * kTile;
      if (!given) {
      if (!mbar_wait(&s_full[t & 1], (uint32_t)(t >> 1) & 1u, kWaitNs)) s_abort = 1;
      fence_after_sync();
      // this thread: slot slot_lane, row columns [col_lo, col_hi)
      float2 a0 = make_float2(0.f, 0.f), a1 = a0, a2 = a0, a3 = a0;
      const uint32_t tS = tRow + (t & 1) * 256;
      // 32-column chunks, the next one's tensor-memory load in flight during this one's
      // exponentials (a wait covers every load issued before it), then a 16-column tail
      auto chunk = [&](const float* v, int col, int width) {
        const float* nb = sNB + col;
#pragma unroll
        for (int i = 0; i < 32; i += 8) {
          if (i >= width) break;
          const float4 b0 = *reinterpret_cast<const float4*>(nb + i);
          const float4 b1 = *reinterpret_cast<const float4*>(nb + i + 4);
          float2 x0 = ffma2(make_float2(v[i], v[i + 1]), c2x2, make_float2(b0.x, b0.y));
          float2 x1 = ffma2(make_float2(v[i + 2], v[i + 3]), c2x2, make_float2(b0.z, b0.w));
          float2 x2 = ffma2(make_float2(v[i + 4], v[i + 5]), c2x2, make_float2(b1.x, b1.y));
          float2 x3 = ffma2(make_float2(v[i + 6], v[i + 7]), c2x2, make_float2(b1.z, b1.w));
          x0 = make_float2(ex2(x0.x), ex2(x0.y));
          x1 = make_float2(ex2(x1.x), ex2(x1.y));
          x2 = make_float2(ex2(x2.x), ex2(x2.y));
          x3 = make_float2(ex2(x3.x), ex2(x3.y));
          a0 = fadd2(a0, x0);
          a1 = fadd2(a1, x1);
          a2 = fadd2(a2, x2);
          a3 = fadd2(a3, x3);
        }
      };
      float sa[32], sb[32];
      const int n32 = (col_hi - col_lo) / 32;   // full chunks
      if (n32 > 0) tmem_ld32(tS + col_lo, sa);
      tmem_ld_wait();
#pragma unroll 1
      for (int i = 0; i < n32; i += 2) {
        const int col = col_lo + 32 * i;
        if (i + 1 < n32) tmem_ld32(tS + col + 32, sb);
        chunk(sa, col, 32);
        tmem_ld_wait();
        if (i + 1 < n32) {
          if (i + 2 < n32) tmem_ld32(tS + col + 64, sa);
          chunk(sb, col + 32, 32);
          tmem_ld_wait();
        }
      }
      if (col_lo + 32 * n32 < col_hi) {   // the 16-column tail
        tmem_ld16(tS + col_lo + 32 * n32, sa);
        tmem_ld_wait();
        chunk(sa, col_lo + 32 * n32, 16);
      }
      sHalf[chalf][slot_lane] = ((a0.x + a0.y) + (a1.x + a1.y)) + ((a2.x + a2.y) + (a3.x + a3.y));
      fence_before_sync();
      __syncwarp();
      if (lane == 0) mbar_arrive(&s_free[t & 1]);
      }
      sum_sync();
      if (threadIdx.x < kTile) {
        const int j = j0 + threadIdx.x;
        const bool live = j < end && kv_live(A.kv, H, b, h, j);
        float a;
        if (given) {   // the caller's a_j (dead slots 0)
          a = live ? A.mass[(int64_t)b * A.sm0 + (int64_t)h * A.sm1 + j] : 0.f;
        } else {
          a = live ? (sHalf[0][threadIdx.x] + sHalf[1][threadIdx.x]) * inv_rows : 0.f;
          if (j < end) A.mass[(int64_t)b * A.sm0 + (int64_t)h * A.sm1 + j] = a;
        }
        if (centre) {
          // sA[t&1] held tile t-2: both centre warps must be done with it
          if (t >= 2 && !mbar_wait(&a_free[t & 1], (uint32_t)((t >> 1) - 1) & 1u, kWaitNs)) s_abort = 1;
          sA[t & 1][threadIdx.x] = a;
        }
      }
      if (threadIdx.x == 0) sDecide = s_abort;
      sum_sync();
      if (sDecide) break;   // every sum warp leaves at the same tile
      if (centre && threadIdx.x == 0) mbar_arrive(&a_full[t & 1]);   // the tile's a_j are in
    }
  }
  // slots past lens[b]: mass (and score) 0
  if (sum_warp && end < end_all) {
    for (int j = end + threadIdx.x; j < end_all; j += kSumThreads) {
      if (!given) A.mass[(int64_t)b * A.sm0 + (int64_t)h * A.sm1 + j] = 0.f;
      if (A.score) A.score[(int64_t)b * A.ss0 + (int64_t)h * A.ss1 + j] = 0.f;
    }
  }
  // join: the producer drained, the sum warps are out of their loop
  fence_before_sync();
  __syncthreads();
  fence_after_sync();
  if (threadIdx.x == 0) pdl_launch_dependents();   // the next kernel's prologue may start
  if (warp == 0) tmem_dealloc(taddr, kTmemCols);
  const bool aborted = s_abort != 0;
  if (aborted && threadIdx.x == 0) atomicExch(A.err, 1);
  if (!centre && !score_only) return;
  if (!score_only) {

  // centre partials per centre warp, in K slot 0 (drained; V tiles may stay in their slots;
  // nK >= 1 in every mode)
  float* sRed = reinterpret_cast<float*>(sSlot);           // [kCentreWarps][kD]
  float* sAsum = sRed + kCentreWarps * kD;                 // [kCentreWarps]
  // per-CTA centre partial (the centre warps' halves summed in order); the last CTA of the head
  // reduces the partials in CTA order and publishes c by advancing the generation
  if (cw >= 0 && cw < kCentreWarps) {
    *reinterpret_cast<float4*>(sRed + cw * kD + 4 * lane) = make_float4(cacc0.x, cacc0.y, cacc1.x, cacc1.y);
    if (lane == 0) sAsum[cw] = asum;
  }
  __syncthreads();
  float* mine = A.part + ((int64_t)bh * gridDim.x + blockIdx.x) * (kD + 1);
  if (threadIdx.x < kD) {   // the centre warps' halves, in order
    float tot = 0.f;
#pragma unroll
    for (int g = 0; g < kCentreWarps; ++g) tot += sRed[g * kD + threadIdx.x];
    mine[threadIdx.x] = aborted ? NAN : tot;
  }
  if (threadIdx.x == 0) {
    float tot = 0.f;
#pragma unroll
    for (int g = 0; g < kCentreWarps; ++g) tot += sAsum[g];
    mine[kD] = tot;
  }
  __threadfence();
  __syncthreads();
  if (threadIdx.x == 0) sLast = atomicAdd(&A.sync[bh].x, 1u) == gridDim.x - 1 ? 1 : 0;
  __syncthreads();
  if (sLast) {
    __threadfence();
    // two threads per column, each over one half of the CTAs in CTA order, up to 32 loads
    // in flight; the halves are added in order
    if (threadIdx.x < 2 * (kD + 1)) {
      const int col = threadIdx.x % (kD + 1), hh = threadIdx.x / (kD + 1);
      const int P = (int)gridDim.x, mid = (P + 1) / 2;
      const int p0 = hh ? mid : 0, p1 = hh ? P : mid;
      const float* base = A.part + (int64_t)bh * P * (kD + 1) + col;
      float tot = 0.f;
      for (int t0 = p0; t0 < p1; t0 += 32) {
        float v[32];
#pragma unroll
        for (int i = 0; i < 32; ++i) v[i] = t0 + i < p1 ? __ldcg(base + (int64_t)(t0 + i) * (kD + 1)) : 0.f;
#pragma unroll
        for (int i = 0; i < 32; ++i) tot += v[i];   // CTA order
      }
      sTot[hh][col] = tot;
    }
    __syncthreads();
    if (threadIdx.x < kD)
      A.centre[(int64_t)bh * kD + threadIdx.x] =
          (sTot[0][threadIdx.x] + sTot[1][threadIdx.x]) / fmaxf(sTot[0][kD] + sTot[1][kD], 1e-12f);
    if (threadIdx.x == 0) A.sync[bh].x = 0u;
    __threadfence();
    __syncthreads();
    if (threadIdx.x == 0) {
      __threadfence();
      atomicAdd(&A.sync[bh].y, 1u);
    }
  }
  }   // !score_only
  if (A.score == nullptr) return;

  // ---- phase 2: a_j ||v_j - c|| for this CTA's slots (cooperative launch: every CTA of
  // the head is resident, so the generation advances)
  if (!score_only && !sLast && threadIdx.x == 0) {
    const uint64_t t0 = global_ns();
    while (ld_acquire_u32(&A.sync[bh].y) == gen0) {
      if (global_ns() - t0 > A.peer_wait_ns) {
        s_wait_ok = 0;
        atomicExch(A.err, 1);
        break;
      }
      __nanosleep(64);
    }
  }
  __syncthreads();
  const bool ok_c = s_wait_ok != 0 && !aborted;
  // every V tile of the CTA still in its phase-1 slot (the V ring never wrapped)
  const bool resident = !score_only && ntiles <= nV;
  if (!sum_warp) {
    if (!PACKED && warp == kSumWarps && lane == 0 && ok_c && !resident) {
      // the CTA's V tiles again, newest first, through every slot
      const uint64_t pol = tma::policy_evict_first();
      int u = 0;
      for (; u < ntiles2; ++u) {
        const int slot = u % nS;
        if (u >= nS && !mbar_wait(&wfree[slot], (uint32_t)((u / nS) - 1) & 1u, kWaitNs)) break;
        tile_load(&A.vmap, b, h, begin + (ntiles2 - 1 - u) * kTile, sSlot + slot * kTileBytes, &wfull[slot], pol);
      }
      // drain (bounded): the last load of every slot
      for (int uu = max(0, u - nS); uu < u; ++uu)
        mbar_wait(&wfull[uu % nS], (uint32_t)(uu / nS) & 1u, 20000000ull);
    }
    __syncwarp();
  } else {
    // thread = slot row rl of the tile (TMEM-lane order, as in phase 1) and channel half
    // chalf; the halves' sums meet in shared memory (the Q region, free now)
    float* sc = A.score + (int64_t)b * A.ss0 + (int64_t)h * A.ss1;
    float* sC = reinterpret_cast<float*>(sQ);      // [kD] the centre
    float* sPart = sC + kD;                        // [2 tile parities][kTile] upper-half sums
    if (!ok_c) {
      for (int j = begin + threadIdx.x; j < end; j += kSumThreads) sc[j] = NAN;
    } else {
      if (threadIdx.x < kD) sC[threadIdx.x] = __ldcg(A.centre + (int64_t)bh * kD + threadIdx.x);
      sum_sync();
      const float* ms = A.mass + (int64_t)b * A.sm0 + (int64_t)h * A.sm1;
      const float* cb = sC + 64 * chalf;
      for (int u = 0; u < ntiles2; ++u) {
        const int slot = resident ? nK + (ntiles2 - 1 - u) : u % nS;
        const int j0 = begin + (ntiles2 - 1 - u) * kTile;
        const int j = j0 + slot_lane;
        float aj = 0.f;   // issued before the tile's wait
        if (chalf == 0 && j < end) aj = __ldcg(ms + j);
        const bool direct = PACKED && !resident;   // packed rows read here, not from a slot
        bool ok_t = resident || direct || mbar_wait(&wfull[slot], (uint32_t)(u / nS) & 1u, kWaitNs);
        float2 s0 = make_float2(0.f, 0.f), s1 = s0;
        if (direct) {
          // this thread's half row, dequantized as the tiles hold it (bf16), then as below
          packed::RawRow rr;
          packed::load_row(A.kv, b, h, j, end, rr, false, true);
          if (rr.ok) {
            packed::Raw hv;   // this half's payload words and scale/zero pairs (constant indices below)
            hv.p[0] = chalf ? rr.v.p[2] : rr.v.p[0];
            hv.p[1] = chalf ? rr.v.p[3] : rr.v.p[1];
            hv.s = make_uint2(chalf ? rr.v.s.y : rr.v.s.x, 0u);
            hv.z = make_uint2(chalf ? rr.v.z.y : rr.v.z.x, 0u);
#pragma unroll
            for (int c = 0; c < 8; ++c) {
              float f[8];
              bf16x8_to_float(packed::chunk<false>(hv, c, nullptr), f);
              const float4 c0 = *reinterpret_cast<const float4*>(cb + 8 * c);
              const float4 c1 = *reinterpret_cast<const float4*>(cb + 8 * c + 4);
              const float2 x0 = make_float2(f[0] - c0.x, f[1] - c0.y), x1 = make_float2(f[2] - c0.z, f[3] - c0.w);
              const float2 x2 = make_float2(f[4] - c1.x, f[5] - c1.y), x3 = make_float2(f[6] - c1.z, f[7] - c1.w);
              s0 = ffma2(x0, x0, s0);
              s1 = ffma2(x1, x1, s1);
              s0 = ffma2(x2, x2, s0);
              s1 = ffma2(x3, x3, s1);
            }
          }
        } else if (ok_t) {
          const uint8_t* sV = sSlot + slot * kTileBytes;
#pragma unroll
          for (int c = 0; c < 8; ++c) {
            float f[8];
            bf16x8_to_float(*reinterpret_cast<const uint4*>(sV + chunk_off(slot_lane, 8 * chalf + c)), f);
            const float4 c0 = *reinterpret_cast<const float4*>(cb + 8 * c);
            const float4 c1 = *reinterpret_cast<const float4*>(cb + 8 * c + 4);
            const float2 x0 = make_float2(f[0] - c0.x, f[1] - c0.y), x1 = make_float2(f[2] - c0.z, f[3] - c0.w);
            const float2 x2 = make_float2(f[4] - c1.x, f[5] - c1.y), x3 = make_float2(f[6] - c1.z, f[7] - c1.w);
            s0 = ffma2(x0, x0, s0);
            s1 = ffma2(x1, x1, s1);
            s0 = ffma2(x2, x2, s0);
            s1 = ffma2(x3, x3, s1);
          }
        }
        const float s2 = (s0.x + s0.y) + (s1.x + s1.y);
        if (chalf == 1) sPart[(u & 1) * kTile + slot_lane] = s2;
        if (!ok_t) atomicExch(A.err, 1);
        sum_sync();   // the upper halves are in; this tile's slot is read
        if (chalf == 0 && j < end) {
          const float tot = s2 + sPart[(u & 1) * kTile + slot_lane];
          sc[j] = !ok_t ? NAN : (kv_live(A.kv, H, b, h, j) ? aj * sqrtf(tot) : 0.f);
        }
        if (lane == 0 && !resident && !PACKED) mbar_arrive(&wfree[slot]);
      }
    }
  }
}

// The bf16 kernel (352 threads) and the PACKED one (480 threads: 15 warps, four of them on
// three of the SM sub-partitions, whose quarter of the register file leaves 128 registers
// a thread).
__global__ void __launch_bounds__(kThreads, 1) prefix_mass_fa(const __grid_constant__ Args A) { mass_fa_body<false>(A); }
__global__ void __launch_bounds__(kThreadsP, 1) prefix_mass_fa_packed(const __grid_constant__ Args A) { mass_fa_body<true>(A); }


bool tma_map_rows(CUtensorMap* map, const void* base, int B, int H, int n, const int64_t s[3]) {
  // bf16 [B][H][n][128] with element strides s (b, h, row); box: 64 channels x 128 rows
  const uint64_t dims[4] = {128, (uint64_t)n, (uint64_t)H, (uint64_t)B};
  const uint64_t strides[3] = {(uint64_t)s[2] * 2, (uint64_t)s[1] * 2, (uint64_t)s[0] * 2};
  const uint32_t box[4] = {64, (uint32_t)kTile, 1, 1};
  return make_tma_map_bf16_4d(map, base, dims, strides, box);
}

}  // namespace

int g_mass_tiles = 0;   // fa_set_mass_tiles: 0 automatic, > 0 a fixed cap, -1 none

void fa_set_mass_tiles(int tiles) { g_mass_tiles = tiles < 0 ? -1 : tiles; }
int fa_mass_tiles() { return g_mass_tiles; }

int launch_prefix_mass_fa(const ma_rows& q, const ma_kv& kv, int H, const int32_t* q_rows, int T2, const float* m_p,
                          const float* l_p, float scale, float* mass, int64_t sm0, int64_t sm1, float* score,
                          int64_t ss0, int64_t ss1, const ValueWs& w, bool want_centre, bool* fused, cudaStream_t st) {
  *fused = false;
  // a dense bf16 cache read by TMA, or a token-mode packed one built by the producer warps
  const bool packed = kv.layout == MA_KV_PACKED_TOKEN;
  const int n = packed ? kv.nq : kv.nf;
  const int BH = q.B * H;
  const int G = q.Hq / H;
  const bool dense_ok = kv.layout == MA_KV_DENSE && kv.dtype == MA_BF16 && !kv.pages && kv.nq == 0;
  const bool packed_ok = packed && kv.dtype == MA_BF16 && packed::eligible(kv);
  if (!((dense_ok || packed_ok) && q.dtype == MA_BF16 && q.D == kD && G * T2 <= kMaxRows && n > 0))
    return MA_ERR_UNSUPPORTED;
  auto kernel = packed ? prefix_mass_fa_packed : prefix_mass_fa;
  const int threads = packed ? kThreadsP : kThreads;
  Args A;
  memset(&A, 0, sizeof(A));
  if (!packed &&
      (!tma_map_rows(&A.kmap, kv.kf, q.B, H, n, kv.skf) || !tma_map_rows(&A.vmap, kv.vf, q.B, H, n, kv.svf)))
    return MA_ERR_UNSUPPORTED;
  A.q = q;
  A.kv = kv;
  A.q_rows = q_rows;
  A.m_p = m_p;
  A.l_p = l_p;
  A.mass = mass;
  A.sm0 = sm0;
  A.sm1 = sm1;
  A.score = nullptr;
  A.ss0 = ss0;
  A.ss1 = ss1;
  A.part = want_centre ? w.part : nullptr;
  A.sync = w.sync;
  A.centre = want_centre ? w.centre : nullptr;
  A.err = w.err;
  A.peer_wait_ns = peer_wait_ns();
  A.scale = scale;
  A.H = H;
  A.T2 = T2;
  A.want_centre = want_centre ? 1 : 0;
  // Q takes Npad * 256 bytes; the rest holds up to six 32 KB tile slots. With the centre,
  // K gets the deeper ring (a K slot is needed again one tile after its S^T completes, a
  // V slot only after the next tiles' sums): 5 slots -> K 3 + V 2.
  const int Npad = (G * T2 + 15) & ~15;
  int nslots = (kSmemLimit - kStaticSmem - 1024 - Npad * 256) / kTileBytes;
  if (nslots > kMaxSlots) nslots = kMaxSlots;
  if (nslots < 4) return MA_ERR_UNSUPPORTED;
  if (want_centre) {
    A.nV = nslots >= 5 ? nslots - 3 : 2;
    A.nK = nslots - A.nV;
  } else {
    A.nK = nslots;
    A.nV = 0;
  }
  const int smem = 1024 + Npad * 256 + nslots * kTileBytes;
  // one wave of CTAs over the heads, whole tiles each
  const int sms = device_sm_count();
  int per_head = sms / (BH > 0 ? BH : 1);
  if (per_head < 1) per_head = 1;
  int spc = (n + per_head - 1) / per_head;
  spc = ((spc + kTile - 1) / kTile) * kTile;
  // a ragged batch (a serving batch of sequences of different lengths) with fewer heads
  // than two waves of CTAs: a CTA per head, or a fixed share of each head, would leave the
  // longest sequences' heads on the critical path; CTAs of at most kRaggedTiles tiles
  // balance it over several waves (the centre is reduced by each head's last CTA, the score
  // follows in a second launch). With more heads one CTA per head balances well enough and
  // keeps the score in the same launch (V partly from L2).
  const int cap = g_mass_tiles > 0 ? g_mass_tiles : (g_mass_tiles == 0 && BH < 2 * sms) ? kRaggedTiles : 0;
  if (kv.lens && cap > 0 && spc > cap * kTile) spc = cap * kTile;
  A.slots_per_cta = spc;
  dim3 grid((n + spc - 1) / spc, BH);
  if (cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, smem) != cudaSuccess)
    return MA_ERR_CUDA;
  if (score != nullptr && want_centre && grid.x == 1) {
    // one CTA per head: it reduces its own centre, so the score needs no other CTA
    Args As = A;
    As.score = score;
    *fused = true;
    return launch_pdl(kernel, grid, dim3(threads), smem, st, As) == cudaSuccess ? MA_OK : MA_ERR_CUDA;
  }
  if (score != nullptr && want_centre) {
    // the fused score needs every CTA resident at once: a cooperative launch that fits
    int dev = 0, coop = 0, per_sm = 0;
    if (cudaGetDevice(&dev) == cudaSuccess &&
        cudaDeviceGetAttribute(&coop, cudaDevAttrCooperativeLaunch, dev) == cudaSuccess && coop &&
        cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kernel, threads, smem) == cudaSuccess &&
        (long long)grid.x * grid.y <= (long long)per_sm * sms) {
      Args Ac = A;
      Ac.score = score;
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
        if (cudaLaunchKernelEx(&cfg, kernel, Ac) == cudaSuccess) {
          *fused = true;
          return MA_OK;
        }
        (void)cudaGetLastError();
      }
    }
  }
  if (launch_pdl(kernel, grid, dim3(threads), smem, st, A) != cudaSuccess) return MA_ERR_CUDA;
  if (score != nullptr && want_centre && !packed) {
    // the score in a second launch of the same grid: phase 2 alone, once every head's mass
    // and centre are final (no CTA waits for another)
    Args As = A;
    As.given = 1;
    As.score_only = 1;
    As.want_centre = 0;
    As.score = score;
    As.centre = w.centre;
    if (launch_pdl(kernel, grid, dim3(threads), smem, st, As) != cudaSuccess) return MA_ERR_CUDA;
    *fused = true;
  }
  return MA_OK;
}

int launch_value_score_fa(const ma_kv& kv, int B, int H, int D, const float* a, int64_t sa0, int64_t sa1,
                          float* score, int64_t ss0, int64_t ss1, void* ws, cudaStream_t st) {
  const bool packed = kv.layout == MA_KV_PACKED_TOKEN;
  const int n = packed ? kv.nq : kv.nf;
  const int BH = B * H;
  const bool dense_ok = kv.layout == MA_KV_DENSE && kv.dtype == MA_BF16 && !kv.pages && kv.nq == 0;
  const bool packed_ok = packed && kv.dtype == MA_BF16 && packed::eligible(kv);
  if (!((dense_ok || packed_ok) && D == kD && n > 0)) return MA_ERR_UNSUPPORTED;
  auto kernel = packed ? prefix_mass_fa_packed : prefix_mass_fa;
  const int threads = packed ? kThreadsP : kThreads;
  Args A;
  memset(&A, 0, sizeof(A));
  if (!packed && !tma_map_rows(&A.vmap, kv.vf, B, H, n, kv.svf)) return MA_ERR_UNSUPPORTED;
  const ValueWs w = carve_value_ws(ws, BH, D);
  A.kv = kv;
  A.q.B = B;
  A.q.Hq = H;   // one "query head" per KV head, one selection row: only the value pass runs
  A.q.T = 1;
  A.q.D = D;
  A.T2 = 1;
  A.mass = const_cast<float*>(a);   // read only in this mode
  A.sm0 = sa0;
  A.sm1 = sa1;
  A.score = nullptr;
  A.ss0 = ss0;
  A.ss1 = ss1;
  A.part = w.part;
  A.sync = w.sync;
  A.centre = w.centre;
  A.err = w.err;
  A.peer_wait_ns = peer_wait_ns();
  A.H = H;
  A.want_centre = 1;
  A.given = 1;
  // the K ring is unused: one K slot remains as the centre-partial scratch (slot 0, which
  // must not hold a V tile that phase 2 reads in place), the others hold V
  const int Npad = 16;
  int nslots = (kSmemLimit - kStaticSmem - 1024 - Npad * 256) / kTileBytes;
  if (nslots > kMaxSlots) nslots = kMaxSlots;
  A.nK = 1;
  A.nV = nslots - 1;
  const int smem = 1024 + Npad * 256 + nslots * kTileBytes;
  const int sms = device_sm_count();
  int per_head = sms / (BH > 0 ? BH : 1);
  if (per_head < 1) per_head = 1;
  int spc = (n + per_head - 1) / per_head;
  spc = ((spc + kTile - 1) / kTile) * kTile;
  A.slots_per_cta = spc;
  dim3 grid((n + spc - 1) / spc, BH);
  if (cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, smem) != cudaSuccess)
    return MA_ERR_CUDA;
  A.score = score;
  if (grid.x == 1)   // one CTA per head: it reduces its own centre
    return launch_pdl(kernel, grid, dim3(threads), smem, st, A) == cudaSuccess ? MA_OK : MA_ERR_CUDA;
  int dev = 0, coop = 0, per_sm = 0;
  if (cudaGetDevice(&dev) == cudaSuccess && cudaDeviceGetAttribute(&coop, cudaDevAttrCooperativeLaunch, dev) == cudaSuccess &&
      coop && cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kernel, threads, smem) == cudaSuccess &&
      (long long)grid.x * grid.y <= (long long)per_sm * sms) {
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
      if (cudaLaunchKernelEx(&cfg, kernel, A) == cudaSuccess) return MA_OK;
      (void)cudaGetLastError();
    }
  }
  return MA_ERR_UNSUPPORTED;
}

}  // namespace ma
