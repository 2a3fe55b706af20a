// Selection kernels: the per-head top-k read set and the lookahead retained set, plus
// the indexed gather of dequantized rows.
//
// Top-k is a block-wide MSB-first radix select on order-preserving uint32 keys (four
// 8-bit digits, shared-memory histograms; the keys of rows up to 16384 slots stay in
// registers), followed by an index-order compaction, so
// the read set comes out already sorted ascending (the reference sorts after
// torch.topk: src/maskahead/kernels/ops.py:377-380, 509-516). Ties at the k-th score
// go to the lower slot index.
#include "ma_kernels.cuh"
#include "ma_packed.cuh"

namespace ma {

namespace {

constexpr int kSelThreads = 1024;

// Exclusive block-wide prefix sum over one int per thread (blockDim.x == 1024).
__device__ __forceinline__ int block_exclusive_scan(int v, int* sWarp, int& total) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  int x = v;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const int y = __shfl_up_sync(0xffffffffu, x, o);
    if (lane >= o) x += y;
  }
  if (lane == 31) sWarp[warp] = x;
  __syncthreads();
  if (warp == 0) {
    int w = sWarp[lane];
    int wx = w;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int y = __shfl_up_sync(0xffffffffu, wx, o);
      if (lane >= o) wx += y;
    }
    sWarp[lane] = wx - w;       // exclusive prefix of warp totals
    if (lane == 31) sWarp[32] = wx;
  }
  __syncthreads();
  const int res = sWarp[warp] + x - v;
  total = sWarp[32];
  __syncthreads();
  return res;
}

struct KthResult {
  uint32_t key;   // the k-th largest key
  int need;       // how many keys equal to `key` belong to the top k
};

// k-th largest of n keys (1 <= k <= n); key(j) must be cheap and pure.
template <class KeyFn>
__device__ KthResult radix_kth(KeyFn key, int n, int k, unsigned* sHist, int* sSel) {
  uint32_t prefix = 0, mask = 0;
  int kk = k;
  for (int pass = 0; pass < 4; ++pass) {
    const int shift = 24 - 8 * pass;
    for (int i = threadIdx.x; i < 256; i += blockDim.x) sHist[i] = 0u;
    __syncthreads();
    for (int j0 = 0; j0 < n; j0 += blockDim.x) {
      // lanes that hit the same bin add once (scores of one head share their top bits,
      // so per-element atomics would serialize on a handful of bins)
      const int j = j0 + threadIdx.x;
      const uint32_t x = j < n ? key(j) : 0u;
      const bool take = j < n && (x & mask) == prefix;
      const uint32_t bin = take ? ((x >> shift) & 255u) : 256u;
      const unsigned peers = __match_any_sync(0xffffffffu, bin);
      if (take && (threadIdx.x & 31) == __ffs(peers) - 1) atomicAdd(&sHist[bin], (unsigned)__popc(peers));
    }
    __syncthreads();
    if (threadIdx.x < 32) {
      // lane l owns digits 255-8l .. 248-8l (descending order)
      const int lane = threadIdx.x;
      int c[8];
      int loc = 0;
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        c[i] = (int)sHist[255 - (lane * 8 + i)];
        loc += c[i];
      }
      int incl = loc;
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const int y = __shfl_up_sync(0xffffffffu, incl, o);
        if (lane >= o) incl += y;
      }
      int cum = incl - loc;  // keys with a larger digit than this lane's first digit
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        if (cum < kk && cum + c[i] >= kk) {
          sSel[0] = 255 - (lane * 8 + i);
          sSel[1] = cum;
        }
        cum += c[i];
      }
    }
    __syncthreads();
    prefix |= (uint32_t)sSel[0] << shift;
    mask |= 255u << shift;
    kk -= sSel[1];
    __syncthreads();
  }
  return KthResult{prefix, kk};
}

// Write, in increasing j, every j whose key is above the threshold plus the first
// `need` ties; calls emit(rank, j) with rank the output position.
template <class KeyFn, class EmitFn>
__device__ void emit_selected(KeyFn key, int n, KthResult th, int* sWarp, EmitFn emit) {
  const int per = (n + blockDim.x - 1) / blockDim.x;
  const int lo = min(n, (int)threadIdx.x * per), hi = min(n, lo + per);
  int gt = 0, eq = 0;
  for (int j = lo; j < hi; ++j) {
    const uint32_t x = key(j);
    gt += x > th.key;
    eq += x == th.key;
  }
  int tot;
  const int eq_before = block_exclusive_scan(eq, sWarp, tot);
  const int take = max(0, min(eq, th.need - eq_before));
  int off = block_exclusive_scan(gt + take, sWarp, tot);
  int taken = 0;
  for (int j = lo; j < hi; ++j) {
    const uint32_t x = key(j);
    if (x > th.key || (x == th.key && taken < take)) {
      if (x == th.key) ++taken;
      emit(off++, j);
    }
  }
}

// One CTA per (b, h). The order keys are staged in shared memory when they fit
// (n <= kSelSmemKeys), so the four histogram passes and the two compaction passes read
// them on-chip; larger rows re-read the scores (from L2).
constexpr int kSelSmemKeys = 48 * 1024;

__global__ void __launch_bounds__(kSelThreads)
select_topk_kernel(const float* __restrict__ score, int H, int n, int64_t ss0, int64_t ss1,
                   const uint8_t* __restrict__ mask, const int32_t* __restrict__ lens, int k,
                   int64_t* __restrict__ indices,
                   float* __restrict__ values, int64_t si0, int64_t si1, int staged) {
  extern __shared__ uint32_t sKeys[];
  __shared__ unsigned sHist[256];
  __shared__ int sSel[2];
  __shared__ int sWarp[33];
  const int bh = blockIdx.x;
  const int b = bh / H, h = bh - (bh / H) * H;
  const float* s = score + (int64_t)b * ss0 + (int64_t)h * ss1;
  const uint8_t* m = mask ? mask + (int64_t)bh * n : nullptr;
  const int len = lens ? lens[b] : n;
  auto gkey = [&](int j) -> uint32_t {
    if (j >= len || (m && m[j] == 0)) return 0u;
    return order_key(s[j]);
  };
  int64_t* oi = indices + (int64_t)b * si0 + (int64_t)h * si1;
  float* ov = values ? values + (int64_t)b * si0 + (int64_t)h * si1 : nullptr;
  auto emit = [&](int r, int j) {
    oi[r] = j;
    if (ov) ov[r] = s[j];
  };
  if (staged) {
    for (int j = threadIdx.x; j < n; j += blockDim.x) sKeys[j] = gkey(j);
    __syncthreads();
    auto skey = [&](int j) -> uint32_t { return sKeys[j]; };
    const KthResult th = radix_kth(skey, n, k, sHist, sSel);
    emit_selected(skey, n, th, sWarp, emit);
  } else {
    const KthResult th = radix_kth(gkey, n, k, sHist, sSel);
    emit_selected(gkey, n, th, sWarp, emit);
  }
}

// Register-resident variant for n <= 1024 * PER (PER keys per thread, thread t owning
// slots [t*PER, t*PER + PER)): the keys are read once from global memory and stay in
// registers through the four radix passes and the emission, so the passes touch shared
// memory only for the 256-bin histogram. Histogram updates are aggregated per warp on
// lane 0's bin (ballot), which absorbs the heavy collisions of the leading digits; the
// remaining lanes add individually. The emission needs one block scan of the packed
// counts (ties << 16 | larger): the ties taken before a thread are min(ties before, need).
template <int PER>
__global__ void __launch_bounds__(kSelThreads)
select_topk_reg(const float* __restrict__ score, int H, int n, int64_t ss0, int64_t ss1,
                const uint8_t* __restrict__ mask, const int32_t* __restrict__ lens, int k,
                int64_t* __restrict__ indices,
                float* __restrict__ values, int64_t si0, int64_t si1) {
  __shared__ unsigned sHist[256];
  __shared__ int sSel[2][2];
  __shared__ int sWarp[33];
  pdl_wait();   // the scores of the kernel before
  const int bh = blockIdx.x;
  const int b = bh / H, h = bh - (bh / H) * H;
  const float* s = score + (int64_t)b * ss0 + (int64_t)h * ss1;
  const uint8_t* m = mask ? mask + (int64_t)bh * n : nullptr;
  const int lane = threadIdx.x & 31;
  const int j0 = threadIdx.x * PER;
  uint32_t key[PER];
  const bool vec = ((reinterpret_cast<uintptr_t>(s) & 15) == 0) && j0 + PER <= n;
  if (vec) {
#pragma unroll
    for (int c = 0; c < PER / 4; ++c) {
      const float4 v = __ldcg(reinterpret_cast<const float4*>(s + j0) + c);
      key[4 * c] = order_key(v.x);
      key[4 * c + 1] = order_key(v.y);
      key[4 * c + 2] = order_key(v.z);
      key[4 * c + 3] = order_key(v.w);
    }
  } else {
#pragma unroll
    for (int i = 0; i < PER; ++i) key[i] = j0 + i < n ? order_key(__ldcg(s + j0 + i)) : 0u;
  }
  if (m) {
#pragma unroll
    for (int i = 0; i < PER; ++i)
      if (j0 + i < n && m[j0 + i] == 0) key[i] = 0u;   // dead slots rank below every live one
  }
  if (lens) {
    const int len = lens[b];
#pragma unroll
    for (int i = 0; i < PER; ++i)
      if (j0 + i >= len) key[i] = 0u;
  }
  const int nv = max(0, min(PER, n - j0));   // this thread's slots inside the row

  uint32_t prefix = 0, pmask = 0;
  int kk = k;
#pragma unroll 1
  for (int pass = 0; pass < 4; ++pass) {
    const int shift = 24 - 8 * pass;
    if (threadIdx.x < 256) sHist[threadIdx.x] = 0u;
    __syncthreads();
#pragma unroll
    for (int i = 0; i < PER; ++i) {
      const uint32_t x = key[i];
      const bool take = i < nv && (x & pmask) == prefix;
      const uint32_t bin = take ? ((x >> shift) & 255u) : 256u;
      const uint32_t b0 = __shfl_sync(0xffffffffu, bin, 0);
      const unsigned same = __ballot_sync(0xffffffffu, bin == b0);
      if (lane == 0 && b0 < 256u) atomicAdd(&sHist[b0], (unsigned)__popc(same));
      if (take && bin != b0) atomicAdd(&sHist[bin], 1u);
    }
    __syncthreads();
    if (threadIdx.x < 32) {
      // lane l owns digits 255-8l .. 248-8l (descending order)
      int c[8];
      int loc = 0;
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        c[i] = (int)sHist[255 - (lane * 8 + i)];
        loc += c[i];
      }
      int incl = loc;
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const int y = __shfl_up_sync(0xffffffffu, incl, o);
        if (lane >= o) incl += y;
      }
      int cum = incl - loc;  // keys with a larger digit than this lane's first digit
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        if (cum < kk && cum + c[i] >= kk) {
          sSel[pass & 1][0] = 255 - (lane * 8 + i);
          sSel[pass & 1][1] = cum;
        }
        cum += c[i];
      }
    }
    __syncthreads();
    prefix |= (uint32_t)sSel[pass & 1][0] << shift;
    pmask |= 255u << shift;
    kk -= sSel[pass & 1][1];
  }
  if (threadIdx.x == 0) pdl_launch_dependents();   // the next kernel's prologue may start
  // emission in slot order: keys above the k-th plus the first kk ties
  int gt = 0, eq = 0;
#pragma unroll
  for (int i = 0; i < PER; ++i) {
    gt += (i < nv && key[i] > prefix) ? 1 : 0;
    eq += (i < nv && key[i] == prefix) ? 1 : 0;
  }
  int tot;
  const int before = block_exclusive_scan((eq << 16) | gt, sWarp, tot);
  const int gt_before = before & 0xFFFF, eq_before = before >> 16;
  const int take = max(0, min(eq, kk - eq_before));
  int off = gt_before + min(eq_before, kk);
  int taken = 0;
  int64_t* oi = indices + (int64_t)b * si0 + (int64_t)h * si1;
  float* ov = values ? values + (int64_t)b * si0 + (int64_t)h * si1 : nullptr;
#pragma unroll
  for (int i = 0; i < PER; ++i) {
    const uint32_t x = key[i];
    const bool tie = x == prefix;
    if (i < nv && (x > prefix || (tie && taken < take))) {
      taken += tie ? 1 : 0;
      oi[off] = j0 + i;
      if (ov) ov[off] = s[j0 + i];
      ++off;
    }
  }
}

// Cluster variant for rows longer than one CTA's registers hold: a cluster of kSelCluster
// CTAs per (b, h), CTA rank r owning the contiguous chunk [r*chunk, r*chunk + chunk) with
// PER keys per thread in registers. Each radix pass builds the CTA's 256-bin histogram,
// adds it into rank 0's shared memory (distributed shared memory atomics; one buffer per
// pass, zeroed before the first cluster barrier), and after a cluster barrier every CTA
// reads the summed histogram and picks the same digit. The emission ranks the CTAs' (larger,
// ties) counts in rank order through rank 0 as well, so the read set stays ascending and
// ties go to the lower slots. Cluster barriers wait only on the cluster's own CTAs, which
// the hardware co-schedules; every CTA takes the same barriers in the same order.
constexpr int kSelCluster = 8;

// The radix select and the rank-ordered emission shared by the cluster kernels: thread t of
// cluster rank r holds the order keys of slots j0 .. j0 + nv - 1 (j0 increasing with r and t)
// in key[]; emit(off, j) is called for the k largest, off their output position in slot
// order, ties at the k-th key going to the lower slots. sGlob (4 x 256) and sCnt
// (kSelCluster) are rank 0's; they must be zero and the cluster synchronized before the call.
// Ends with a cluster barrier, after which no CTA reads another's shared memory.
template <int PER, class EmitFn>
__device__ __forceinline__ void cluster_select(const uint32_t (&key)[PER], int nv, int j0, int k, uint32_t rank,
                                               unsigned* sHist, unsigned (*sGlob)[256], unsigned* sCnt,
                                               int (*sSel)[2], int* sWarp, EmitFn emit) {
  const int lane = threadIdx.x & 31;
  uint32_t prefix = 0, pmask = 0;
  int kk = k;
#pragma unroll 1
  for (int pass = 0; pass < 4; ++pass) {
    const int shift = 24 - 8 * pass;
    if (threadIdx.x < 256) sHist[threadIdx.x] = 0u;
    __syncthreads();
#pragma unroll
    for (int i = 0; i < PER; ++i) {
      const uint32_t x = key[i];
      const bool take = i < nv && (x & pmask) == prefix;
      const uint32_t bin = take ? ((x >> shift) & 255u) : 256u;
      const uint32_t b0 = __shfl_sync(0xffffffffu, bin, 0);
      const unsigned same = __ballot_sync(0xffffffffu, bin == b0);
      if (lane == 0 && b0 < 256u) atomicAdd(&sHist[b0], (unsigned)__popc(same));
      if (take && bin != b0) atomicAdd(&sHist[bin], 1u);
    }
    __syncthreads();
    if (threadIdx.x < 256 && sHist[threadIdx.x] != 0u)
      peer_add(peer_addr(&sGlob[pass][threadIdx.x], 0), sHist[threadIdx.x]);
    cluster_sync();   // the cluster's histogram for this pass is complete in rank 0
    if (threadIdx.x < 32) {
      // lane l owns digits 255-8l .. 248-8l (descending order)
      int c[8];
      int loc = 0;
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        c[i] = (int)peer_ld(peer_addr(&sGlob[pass][255 - (lane * 8 + i)], 0));
        loc += c[i];
      }
      int incl = loc;
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const int y = __shfl_up_sync(0xffffffffu, incl, o);
        if (lane >= o) incl += y;
      }
      int cum = incl - loc;  // keys with a larger digit than this lane's first digit
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        if (cum < kk && cum + c[i] >= kk) {
          sSel[pass & 1][0] = 255 - (lane * 8 + i);
          sSel[pass & 1][1] = cum;
        }
        cum += c[i];
      }
    }
    __syncthreads();
    prefix |= (uint32_t)sSel[pass & 1][0] << shift;
    pmask |= 255u << shift;
    kk -= sSel[pass & 1][1];
  }
  // emission in slot order: keys above the k-th plus the first kk ties, ranks in order
  int gt = 0, eq = 0;
#pragma unroll
  for (int i = 0; i < PER; ++i) {
    gt += (i < nv && key[i] > prefix) ? 1 : 0;
    eq += (i < nv && key[i] == prefix) ? 1 : 0;
  }
  int tot;
  const int before = block_exclusive_scan((eq << 16) | gt, sWarp, tot);
  if (threadIdx.x == 0) peer_st(peer_addr(&sCnt[rank], 0), (uint32_t)tot);
  cluster_sync();   // every rank's counts are in rank 0
  int gt_r = 0, eq_r = 0;   // larger keys and ties in the lower ranks
  for (uint32_t rr = 0; rr < rank; ++rr) {
    const uint32_t c = peer_ld(peer_addr(&sCnt[rr], 0));
    gt_r += (int)(c & 0xFFFFu);
    eq_r += (int)(c >> 16);
  }
  const int kk_cta = max(0, min(tot >> 16, kk - eq_r));   // ties this CTA takes
  const int gt_before = before & 0xFFFF, eq_before = before >> 16;
  const int take = max(0, min(eq, kk_cta - eq_before));
  int off = gt_r + min(eq_r, kk) + gt_before + min(eq_before, kk_cta);
  int taken = 0;
#pragma unroll
  for (int i = 0; i < PER; ++i) {
    const uint32_t x = key[i];
    const bool tie = x == prefix;
    if (i < nv && (x > prefix || (tie && taken < take))) {
      taken += tie ? 1 : 0;
      emit(off, j0 + i);
      ++off;
    }
  }
  cluster_sync();   // no CTA leaves while another may still read rank 0's shared memory
}

template <int PER>
__global__ void __launch_bounds__(kSelThreads)
select_topk_cluster(const float* __restrict__ score, int H, int n, int64_t ss0, int64_t ss1,
                    const uint8_t* __restrict__ mask, const int32_t* __restrict__ lens, int k,
                    int64_t* __restrict__ indices, float* __restrict__ values, int64_t si0, int64_t si1) {
  __shared__ unsigned sHist[256];                  // this CTA's histogram
  __shared__ unsigned sGlob[4][256];               // rank 0: the cluster's, one per pass
  __shared__ unsigned sCnt[kSelCluster];           // rank 0: (ties << 16 | larger) per rank
  __shared__ int sSel[2][2];
  __shared__ int sWarp[33];
  const uint32_t rank = cluster_rank();
  for (int i = threadIdx.x; i < 4 * 256; i += blockDim.x) (&sGlob[0][0])[i] = 0u;
  cluster_sync();   // every CTA of the cluster started, rank 0's buffers are zero
  pdl_wait();
  const int bh = blockIdx.y;
  const int b = bh / H, h = bh - (bh / H) * H;
  const float* s = score + (int64_t)b * ss0 + (int64_t)h * ss1;
  const uint8_t* m = mask ? mask + (int64_t)bh * n : nullptr;
  const int chunk = kSelThreads * PER;
  const int j0 = (int)rank * chunk + threadIdx.x * PER;
  uint32_t key[PER];
  const bool vec = ((reinterpret_cast<uintptr_t>(s) & 15) == 0) && j0 + PER <= n;
  if (vec) {
#pragma unroll
    for (int c = 0; c < PER / 4; ++c) {
      const float4 v = __ldcg(reinterpret_cast<const float4*>(s + j0) + c);
      key[4 * c] = order_key(v.x);
      key[4 * c + 1] = order_key(v.y);
      key[4 * c + 2] = order_key(v.z);
      key[4 * c + 3] = order_key(v.w);
    }
  } else {
#pragma unroll
    for (int i = 0; i < PER; ++i) key[i] = j0 + i < n ? order_key(__ldcg(s + j0 + i)) : 0u;
  }
  if (m) {
#pragma unroll
    for (int i = 0; i < PER; ++i)
      if (j0 + i < n && m[j0 + i] == 0) key[i] = 0u;   // dead slots rank below every live one
  }
  if (lens) {
    const int len = lens[b];
#pragma unroll
    for (int i = 0; i < PER; ++i)
      if (j0 + i >= len) key[i] = 0u;
  }
  const int nv = max(0, min(PER, n - j0));   // this thread's slots inside the row

  int64_t* oi = indices + (int64_t)b * si0 + (int64_t)h * si1;
  float* ov = values ? values + (int64_t)b * si0 + (int64_t)h * si1 : nullptr;
  cluster_select<PER>(key, nv, j0, k, rank, sHist, sGlob, sCnt, sSel, sWarp, [&](int off, int j) {
    oi[off] = j;
    if (ov) ov[off] = s[j];
  });
}

// Lookahead survivors when the live axis is ordered by position, as the reference keeps it
// (eviction.py:404-409, "recent stays the tail"): the window is then the last W entries, the
// contest for the other C - W slots runs over entries 0 .. live - W - 1, and the union in
// slot order is already the position order -- one radix select over a cluster of CTAs
// (gridDim.x ranks, PER entries per thread), no sort. The cluster first checks that the
// lane's positions strictly increase; a lane where they do not gets keep[lane][0] = -1 and
// is left to retain_kernel, launched after this one.
template <int PER>
__global__ void __launch_bounds__(kSelThreads, 1)
retain_sorted(const float* __restrict__ score, const int32_t* __restrict__ phys, int n_phys,
              const int32_t* __restrict__ pos, int live, int capacity, int W, int sinks,
              int64_t* __restrict__ keep) {
  __shared__ unsigned sHist[256];
  __shared__ unsigned sGlob[4][256];     // rank 0: the cluster's histograms
  __shared__ unsigned sCnt[kSelCluster];  // rank 0: (ties << 16 | larger) per rank
  __shared__ unsigned sUnsorted;          // rank 0: CTAs that saw positions out of order
  __shared__ int sFlag;
  __shared__ int sSel[2][2];
  __shared__ int sWarp[33];
  const uint32_t rank = cluster_rank();
  for (int i = threadIdx.x; i < 4 * 256; i += blockDim.x) (&sGlob[0][0])[i] = 0u;
  if (threadIdx.x == 0) sUnsorted = 0u;
  cluster_sync();   // every CTA of the cluster started, rank 0's buffers are zero
  const int lane_id = blockIdx.y;
  const int32_t* p = pos + (int64_t)lane_id * live;
  const float* sc = score + (int64_t)lane_id * (phys ? n_phys : live);
  const int32_t* ph = phys ? phys + (int64_t)lane_id * live : nullptr;
  int64_t* out = keep + (int64_t)lane_id * capacity;
  const int j0 = (int)rank * (kSelThreads * PER) + threadIdx.x * PER;
  const int m = live - W;   // the contest's entries

  int pv[PER];
  if (((reinterpret_cast<uintptr_t>(p + j0) & 15) == 0) && j0 + PER <= live) {
#pragma unroll
    for (int c = 0; c < PER / 4; ++c) {
      const int4 v = __ldg(reinterpret_cast<const int4*>(p + j0) + c);
      pv[4 * c] = v.x;
      pv[4 * c + 1] = v.y;
      pv[4 * c + 2] = v.z;
      pv[4 * c + 3] = v.w;
    }
  } else {
#pragma unroll
    for (int i = 0; i < PER; ++i) pv[i] = j0 + i < live ? __ldg(p + j0 + i) : 0;
  }
  bool bad = false;
#pragma unroll
  for (int i = 0; i + 1 < PER; ++i) bad |= (j0 + i + 1 < live) && pv[i] >= pv[i + 1];
  if (j0 + PER < live) bad |= pv[PER - 1] >= __ldg(p + j0 + PER);   // into the next thread's slots
  if (__syncthreads_or(bad) && threadIdx.x == 0) peer_add(peer_addr(&sUnsorted, 0), 1u);
  cluster_sync();   // every CTA's verdict is in rank 0
  if (threadIdx.x == 0) sFlag = peer_ld(peer_addr(&sUnsorted, 0)) != 0u ? 1 : 0;
  __syncthreads();
  if (sFlag) {   // the same for every CTA of the cluster
    if (rank == 0 && threadIdx.x == 0) out[0] = -1;
    cluster_sync();   // rank 0 stays until every CTA has read its verdict
    return;
  }

  const uint32_t kInf = 0xFF800000u;   // order_key(+inf): sinks win their slots outright
  uint32_t key[PER];
  const bool vec = !ph && ((reinterpret_cast<uintptr_t>(sc + j0) & 15) == 0) && j0 + PER <= m;
  if (vec) {
#pragma unroll
    for (int c = 0; c < PER / 4; ++c) {
      const float4 v = __ldg(reinterpret_cast<const float4*>(sc + j0) + c);
      key[4 * c] = order_key(v.x);
      key[4 * c + 1] = order_key(v.y);
      key[4 * c + 2] = order_key(v.z);
      key[4 * c + 3] = order_key(v.w);
    }
  } else {
#pragma unroll
    for (int i = 0; i < PER; ++i) {
      const int j = j0 + i;
      uint32_t x = 0u;
      if (j < m) {
        if (ph) {
          const int slot = __ldg(ph + j);
          x = (slot >= 0 && slot < n_phys) ? order_key(__ldg(sc + slot)) : 0u;   // bad slot: never kept by score
        } else {
          x = order_key(__ldg(sc + j));
        }
      }
      key[i] = x;
    }
  }
  if (sinks > 0) {
#pragma unroll
    for (int i = 0; i < PER; ++i)
      if (pv[i] < sinks) key[i] = kInf;
  }
  const int nv = max(0, min(PER, m - j0));   // this thread's entries in the contest
  const int rest = capacity - W;
  // the window: entries m .. live - 1, after the contest's winners
  const int stride = (int)gridDim.x * kSelThreads;
  for (int t = (int)rank * kSelThreads + threadIdx.x; t < W; t += stride) out[rest + t] = m + t;
  if (rest > 0) {
    cluster_select<PER>(key, nv, j0, rest, rank, sHist, sGlob, sCnt, sSel, sWarp,
                        [&](int off, int j) { out[off] = j; });
  } else {
    cluster_sync();   // rank 0 stays until every CTA has read its verdict
  }
}

// Lookahead survivors of one lane (eviction.py:364-409): recent window by position,
// sinks at +inf, window excluded from the score contest, union ordered by position.
// gated: only the lanes retain_sorted handed over (keep[lane][0] == -1) are computed.
__global__ void __launch_bounds__(kSelThreads)
retain_kernel(const float* __restrict__ score, const int32_t* __restrict__ phys, int n_phys,
              const int32_t* __restrict__ pos, int live, int capacity, int W, int sinks,
              int64_t* __restrict__ keep, int sort_cap, int gated) {
  extern __shared__ unsigned char smem[];
  unsigned long long* sSort = reinterpret_cast<unsigned long long*>(smem);   // [sort_cap]
  unsigned char* sRecent = smem + (size_t)sort_cap * sizeof(unsigned long long);  // [live]
  __shared__ unsigned sHist[256];
  __shared__ int sSel[2];
  __shared__ int sWarp[33];
  const int lane_id = blockIdx.x;
  if (gated && keep[(int64_t)lane_id * capacity] != -1) return;   // done by retain_sorted
  const int32_t* p = pos + (int64_t)lane_id * live;
  const float* sc = phys ? score + (int64_t)lane_id * n_phys : score + (int64_t)lane_id * live;
  const int32_t* ph = phys ? phys + (int64_t)lane_id * live : nullptr;

  for (int i = threadIdx.x; i < live; i += blockDim.x) sRecent[i] = 0;
  __syncthreads();
  if (W > 0) {
    auto pkey = [&](int i) -> uint32_t { return (uint32_t)p[i] ^ 0x80000000u; };
    const KthResult th = radix_kth(pkey, live, W, sHist, sSel);
    emit_selected(pkey, live, th, sWarp, [&](int, int i) { sRecent[i] = 1; });
    __syncthreads();
  }
  const int rest = capacity - W;
  const uint32_t kInf = 0xFF800000u;  // order_key(+inf)
  auto rkey = [&](int i) -> uint32_t {
    if (sRecent[i]) return 0u;
    if (p[i] < sinks) return kInf;
    if (ph) {
      const int slot = ph[i];
      return (slot >= 0 && slot < n_phys) ? order_key(sc[slot]) : 0u;  // bad slot: never kept by score
    }
    return order_key(sc[i]);
  };
  // union, in live-index order, as (position, index) sort keys
  auto ukey = [&](int i) -> unsigned long long {
    return ((unsigned long long)((uint32_t)p[i] ^ 0x80000000u) << 32) | (unsigned)i;
  };
  if (rest > 0) {
    const KthResult th = radix_kth(rkey, live, rest, sHist, sSel);
    // mark extras in sRecent with value 2 (keeps window entries at 1)
    emit_selected(rkey, live, th, sWarp, [&](int, int i) { sRecent[i] = 2; });
    __syncthreads();
  }
  // compact the kept set in index order
  const int per = (live + blockDim.x - 1) / blockDim.x;
  const int lo = min(live, (int)threadIdx.x * per), hi = min(live, lo + per);
  int cnt = 0;
  for (int i = lo; i < hi; ++i) cnt += sRecent[i] != 0;
  int tot;
  int off = block_exclusive_scan(cnt, sWarp, tot);
  for (int i = lo; i < hi; ++i)
    if (sRecent[i]) sSort[off++] = ukey(i);
  for (int i = tot + threadIdx.x; i < sort_cap; i += blockDim.x) sSort[i] = ~0ull;
  __syncthreads();
  // bitonic sort by position (already sorted when the live axis is, as the reference keeps it)
  for (int size = 2; size <= sort_cap; size <<= 1) {
    for (int stride = size >> 1; stride > 0; stride >>= 1) {
      for (int i = threadIdx.x; i < sort_cap; i += blockDim.x) {
        const int j = i ^ stride;
        if (j > i) {
          const bool up = (i & size) == 0;
          const unsigned long long a = sSort[i], c = sSort[j];
          if ((a > c) == up) {
            sSort[i] = c;
            sSort[j] = a;
          }
        }
      }
      __syncthreads();
    }
  }
  int64_t* out = keep + (int64_t)lane_id * capacity;
  for (int i = threadIdx.x; i < capacity; i += blockDim.x) out[i] = (int64_t)(sSort[i] & 0xffffffffull);
}

constexpr int kGatherTok = 32;

template <typename OT>
__global__ void gather_kv_kernel(ma_kv kv, int H, int D, const int64_t* __restrict__ idx, int k,
                                 int64_t si0, int64_t si1, OT* __restrict__ ok_,
                                 OT* __restrict__ ov_, int64_t sok0, int64_t sok1, int64_t sok2,
                                 int64_t sov0, int64_t sov1, int64_t sov2) {
  pdl_wait();   // the read set of the kernel before
  if (threadIdx.x == 0) pdl_launch_dependents();
  const int bh = blockIdx.y;
  const int b = bh / H, h = bh - (bh / H) * H;
  const int chunks = D / 8;
  const int i0 = blockIdx.x * kGatherTok;
  for (int c = threadIdx.x; c < kGatherTok * chunks; c += blockDim.x) {
    const int ii = c / chunks, c8 = c - (c / chunks) * chunks;
    const int i = i0 + ii;
    if (i >= k) continue;
    const int64_t slot64 = idx ? idx[(int64_t)b * si0 + (int64_t)h * si1 + i] : (int64_t)i;   // no index: slot i
    const int slot = (int)slot64;
    float fk[8], fv[8];
    if (slot64 >= 0 && slot64 < (int64_t)kv.nq + kv.nf && kv_exists(kv, b, slot)) {
      kv_read8<true>(kv, b, h, slot, c8, fk);
      kv_read8<false>(kv, b, h, slot, c8, fv);
    } else {  // a slot outside the prefix (or its sequence, or its page table) gathers zeros
#pragma unroll
      for (int e = 0; e < 8; ++e) fk[e] = fv[e] = 0.f;
    }
    OT* dk = ok_ + (int64_t)b * sok0 + (int64_t)h * sok1 + (int64_t)i * sok2 + 8 * c8;
    OT* dv = ov_ + (int64_t)b * sov0 + (int64_t)h * sov1 + (int64_t)i * sov2 + 8 * c8;
    store4(dk, fk[0], fk[1], fk[2], fk[3]);
    store4(dk + 4, fk[4], fk[5], fk[6], fk[7]);
    store4(dv, fv[0], fv[1], fv[2], fv[3]);
    store4(dv + 4, fv[4], fv[5], fv[6], fv[7]);
  }
}


// The whole token-mode packed prefix of one (b, h) dequantized in slot order (no index):
// thread = (slot jj of 64, 32-channel group g); 16-byte payload loads, the group's fp16
// scale/zero, codes to fp32 exactly (2^23 + code, minus 2^23), code*scale + zero in fp32
// (times the per-channel divisor for keys), rounded once to bf16 -- kv_read8's values.
// Slots past lens[b], on a bad page or past nq (a dense tail) go through kv_read8 or zero.
constexpr int kUnpackTok = 64;

__device__ __forceinline__ void unpack32(const uint4& p, float s, float z, const float* mul, float* f) {
  const uint32_t w[4] = {p.x, p.y, p.z, p.w};
#pragma unroll
  for (int i = 0; i < 32; ++i) {
    const float code = __uint_as_float(0x4B000000u | ((w[i >> 3] >> (4 * (i & 7))) & 0xFu)) - 8388608.f;
    f[i] = fmaf(code, s, z);
    if (mul) f[i] *= mul[i];
  }
}

// live_only: slots at or past lens[b] are skipped (not written) instead of zero-filled
__global__ void __launch_bounds__(256) unpack_token_kernel(ma_kv kv, int H, int n, __nv_bfloat16* __restrict__ ok_,
                                                           __nv_bfloat16* __restrict__ ov_, int64_t sok0, int64_t sok1,
                                                           int64_t sok2, int64_t sov0, int64_t sov1, int64_t sov2,
                                                           int live_only) {
  const int bh = blockIdx.y;
  const int b = bh / H, h = bh - (bh / H) * H;
  const int jj = threadIdx.x >> 2, g = threadIdx.x & 3;
  const float* kch = kv.kchan + (int64_t)b * kv.skc[0] + (int64_t)h * kv.skc[1] + 32 * g;
  if (live_only && kv.lens) n = max(0, min(n, kv.lens[b]));
  for (int j = blockIdx.x * kUnpackTok + jj; j < n; j += gridDim.x * kUnpackTok) {
    __nv_bfloat16* dk = ok_ + (int64_t)b * sok0 + (int64_t)h * sok1 + (int64_t)j * sok2 + 32 * g;
    __nv_bfloat16* dv = ov_ + (int64_t)b * sov0 + (int64_t)h * sov1 + (int64_t)j * sov2 + 32 * g;
    const bool live = kv_exists(kv, b, j);
    float f[32];
    if (j < kv.nq && live) {
      int sb = b, sj = j;
      if (kv_paged(kv, j)) kv_page(kv, b, j, sb, sj);
      const uint4 pk = __ldg(reinterpret_cast<const uint4*>(kv.kq + (int64_t)sb * kv.skq[0] + (int64_t)h * kv.skq[1] + (int64_t)sj * kv.skq[2] + 16 * g));
      const uint4 pv = __ldg(reinterpret_cast<const uint4*>(kv.vq + (int64_t)sb * kv.svq[0] + (int64_t)h * kv.svq[1] + (int64_t)sj * kv.svq[2] + 16 * g));
      const int64_t kso = (int64_t)sb * kv.sks[0] + (int64_t)h * kv.sks[1] + (int64_t)sj * kv.sks[2] + g;
      const int64_t vso = (int64_t)sb * kv.svs[0] + (int64_t)h * kv.svs[1] + (int64_t)sj * kv.svs[2] + g;
      const float ks = half_bits_to_float(kv.ks[kso]), kz = half_bits_to_float(kv.kz[kso]);
      const float vs = half_bits_to_float(kv.vs[vso]), vz = half_bits_to_float(kv.vz[vso]);
      unpack32(pk, ks, kz, kch, f);
#pragma unroll
      for (int c = 0; c < 4; ++c) reinterpret_cast<uint4*>(dk)[c] = float8_to_bf16x8(f + 8 * c);
      unpack32(pv, vs, vz, nullptr, f);
#pragma unroll
      for (int c = 0; c < 4; ++c) reinterpret_cast<uint4*>(dv)[c] = float8_to_bf16x8(f + 8 * c);
    } else if (j >= kv.nq && live) {   // the dense tail
#pragma unroll
      for (int c = 0; c < 4; ++c) kv_read8<true>(kv, b, h, j, 4 * g + c, f + 8 * c);
#pragma unroll
      for (int c = 0; c < 4; ++c) reinterpret_cast<uint4*>(dk)[c] = float8_to_bf16x8(f + 8 * c);
#pragma unroll
      for (int c = 0; c < 4; ++c) kv_read8<false>(kv, b, h, j, 4 * g + c, f + 8 * c);
#pragma unroll
      for (int c = 0; c < 4; ++c) reinterpret_cast<uint4*>(dv)[c] = float8_to_bf16x8(f + 8 * c);
    } else {
#pragma unroll
      for (int c = 0; c < 4; ++c) {
        reinterpret_cast<uint4*>(dk)[c] = make_uint4(0, 0, 0, 0);
        reinterpret_cast<uint4*>(dv)[c] = make_uint4(0, 0, 0, 0);
      }
    }
  }
}

// The same unpack with thread = (slot, 16-channel half of a 32-channel group): 8 threads a
// slot, 32 slots a pass, 8-byte code loads and the thread's 16 key divisors in registers.
// Twice the CTAs of unpack_token_kernel for the same slots: faster on a short prefix (cfg3:
// 7.6 against 10.2 µs a layer), slower on a long batch, whose wider loads keep more bytes
// in flight (cfg5: 2.07 against 1.83 ms).
constexpr int kUnpack16Tok = 32;
__global__ void __launch_bounds__(256) unpack_token16_kernel(ma_kv kv, int H, int n, __nv_bfloat16* __restrict__ ok_,
                                                           __nv_bfloat16* __restrict__ ov_, int64_t sok0, int64_t sok1,
                                                           int64_t sok2, int64_t sov0, int64_t sov1, int64_t sov2,
                                                           int live_only) {
  const int bh = blockIdx.y;
  const int b = bh / H, h = bh - (bh / H) * H;
  const int jj = threadIdx.x >> 3, c = threadIdx.x & 7, g = c >> 1;   // channels 16c..16c+15
  float kc[16];
  {
    const float4* kp = reinterpret_cast<const float4*>(kv.kchan + (int64_t)b * kv.skc[0] + (int64_t)h * kv.skc[1] + 16 * c);
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const float4 x = __ldg(kp + i);
      kc[4 * i] = x.x;
      kc[4 * i + 1] = x.y;
      kc[4 * i + 2] = x.z;
      kc[4 * i + 3] = x.w;
    }
  }
  if (live_only && kv.lens) n = max(0, min(n, kv.lens[b]));
  for (int j = blockIdx.x * kUnpack16Tok + jj; j < n; j += gridDim.x * kUnpack16Tok) {
    uint4* dk = reinterpret_cast<uint4*>(ok_ + (int64_t)b * sok0 + (int64_t)h * sok1 + (int64_t)j * sok2 + 16 * c);
    uint4* dv = reinterpret_cast<uint4*>(ov_ + (int64_t)b * sov0 + (int64_t)h * sov1 + (int64_t)j * sov2 + 16 * c);
    const bool live = kv_exists(kv, b, j);
    float f[16];
    if (j < kv.nq && live) {
      int sb = b, sj = j;
      if (kv_paged(kv, j)) kv_page(kv, b, j, sb, sj);
      // half c & 1 of group c >> 1: payload bytes 8c..8c+7, element k in nibble k
      const uint2 pk = __ldg(reinterpret_cast<const uint2*>(
          kv.kq + (int64_t)sb * kv.skq[0] + (int64_t)h * kv.skq[1] + (int64_t)sj * kv.skq[2] + 8 * c));
      const uint2 pv = __ldg(reinterpret_cast<const uint2*>(
          kv.vq + (int64_t)sb * kv.svq[0] + (int64_t)h * kv.svq[1] + (int64_t)sj * kv.svq[2] + 8 * c));
      const int64_t kso = (int64_t)sb * kv.sks[0] + (int64_t)h * kv.sks[1] + (int64_t)sj * kv.sks[2] + g;
      const int64_t vso = (int64_t)sb * kv.svs[0] + (int64_t)h * kv.svs[1] + (int64_t)sj * kv.svs[2] + g;
      const float ks = half_bits_to_float(kv.ks[kso]), kz = half_bits_to_float(kv.kz[kso]);
      const float vs = half_bits_to_float(kv.vs[vso]), vz = half_bits_to_float(kv.vz[vso]);
#pragma unroll
      for (int i = 0; i < 16; ++i) {
        const uint32_t w = i < 8 ? pk.x : pk.y;
        const float code = __uint_as_float(0x4B000000u | ((w >> (4 * (i & 7))) & 0xFu)) - 8388608.f;
        f[i] = fmaf(code, ks, kz) * kc[i];
      }
      dk[0] = float8_to_bf16x8(f);
      dk[1] = float8_to_bf16x8(f + 8);
#pragma unroll
      for (int i = 0; i < 16; ++i) {
        const uint32_t w = i < 8 ? pv.x : pv.y;
        const float code = __uint_as_float(0x4B000000u | ((w >> (4 * (i & 7))) & 0xFu)) - 8388608.f;
        f[i] = fmaf(code, vs, vz);
      }
      dv[0] = float8_to_bf16x8(f);
      dv[1] = float8_to_bf16x8(f + 8);
    } else if (j >= kv.nq && live) {   // the dense tail
      kv_read8<true>(kv, b, h, j, 2 * c, f);
      kv_read8<true>(kv, b, h, j, 2 * c + 1, f + 8);
      dk[0] = float8_to_bf16x8(f);
      dk[1] = float8_to_bf16x8(f + 8);
      kv_read8<false>(kv, b, h, j, 2 * c, f);
      kv_read8<false>(kv, b, h, j, 2 * c + 1, f + 8);
      dv[0] = float8_to_bf16x8(f);
      dv[1] = float8_to_bf16x8(f + 8);
    } else {
      const uint4 z = make_uint4(0, 0, 0, 0);
      dk[0] = z;
      dk[1] = z;
      dv[0] = z;
      dv[1] = z;
    }
  }
}


// The unpack of a long batch with its input staged by bulk copies: a CTA takes consecutive
// 128-slot units of one (b, h); one thread copies each unit's raw rows (K and V payloads,
// scales, zeros: 20 KB, per page crossed) into a ring of kUnpackStages stages a few units
// ahead (cp.async.bulk, completion on an mbarrier), so each SM keeps far more bytes in
// flight than register loads can; all 8 warps convert a staged unit, thread = (slot,
// 8-channel chunk), 16-byte stores two slots a warp. The arithmetic is kv_read8's.
constexpr int kUnpackStages = 3;
constexpr int kUnpackUnits = 8;   // units a CTA takes
__global__ void __launch_bounds__(256) unpack_staged_kernel(ma_kv kv, int H, int n, __nv_bfloat16* __restrict__ ok_,
                                                            __nv_bfloat16* __restrict__ ov_, int64_t sok0, int64_t sok1,
                                                            int64_t sok2, int64_t sov0, int64_t sov1, int64_t sov2,
                                                            int live_only) {
  extern __shared__ __align__(128) uint8_t stg_raw[];
  __shared__ __align__(8) uint64_t sfull[kUnpackStages];
  const int bh = blockIdx.y;
  const int b = bh / H, h = bh - (bh / H) * H;
  const int c = threadIdx.x & 15, g = c >> 2;
  pdl_wait();   // with a programmatic launch, the cache may come from the kernel before
  const int nq = min(n, kv.nq);
  int end = nq;
  if (kv.lens) end = max(0, min(end, kv.lens[b]));
  const int u0 = blockIdx.x * kUnpackUnits;
  const int last = live_only ? end : nq;   // slots written: below lens[b], or every one (zeros past it)
  const int units = max(0, min(kUnpackUnits, (last - u0 * 128 + 127) / 128));
  const packed::PageCache pc{nullptr, 0, 0};
  if (threadIdx.x == 0) {
    for (int i = 0; i < kUnpackStages; ++i) tc::mbar_init(&sfull[i], 1);
    asm volatile("fence.mbarrier_init.release.cluster;\n" ::: "memory");
    for (int i = 0; i < kUnpackStages && i < units; ++i) {
      const int j0 = (u0 + i) * 128;
      packed::stage_tile(kv, b, h, j0, min(end, j0 + 128), stg_raw + i * packed::kStageBytes, &sfull[i], pc);
    }
  }
  float kc[8];
  {
    const float4* kp = reinterpret_cast<const float4*>(kv.kchan + (int64_t)b * kv.skc[0] + (int64_t)h * kv.skc[1] + 8 * c);
    const float4 a = __ldg(kp), d = __ldg(kp + 1);
    kc[0] = a.x; kc[1] = a.y; kc[2] = a.z; kc[3] = a.w;
    kc[4] = d.x; kc[5] = d.y; kc[6] = d.z; kc[7] = d.w;
  }
  __syncthreads();
  for (int u = 0; u < units; ++u) {
    const int j0 = (u0 + u) * 128;
    const uint8_t* stg = stg_raw + (u % kUnpackStages) * packed::kStageBytes;
    const bool ok = tc::mbar_wait(&sfull[u % kUnpackStages], (uint32_t)(u / kUnpackStages) & 1u, 200000000ull);
#pragma unroll 2
    for (int i = 0; i < 8; ++i) {
      const int r = (threadIdx.x >> 4) + 16 * i;
      const int j = j0 + r;
      if (j >= last) continue;
      uint4* dk = reinterpret_cast<uint4*>(ok_ + (int64_t)b * sok0 + (int64_t)h * sok1 + (int64_t)j * sok2 + 8 * c);
      uint4* dv = reinterpret_cast<uint4*>(ov_ + (int64_t)b * sov0 + (int64_t)h * sov1 + (int64_t)j * sov2 + 8 * c);
      int sb, sj;
      if (!ok || j >= end || !packed::locate(kv, b, j, sb, sj)) {
        *dk = make_uint4(0, 0, 0, 0);
        *dv = make_uint4(0, 0, 0, 0);
        continue;
      }
      float f[8];
      const uint32_t wk = *reinterpret_cast<const uint32_t*>(stg + packed::kStgKq + r * 64 + 4 * c);
      const uint32_t wv = *reinterpret_cast<const uint32_t*>(stg + packed::kStgVq + r * 64 + 4 * c);
      const float ks = half_bits_to_float(*reinterpret_cast<const uint16_t*>(stg + packed::kStgKs + r * 8 + 2 * g));
      const float kz = half_bits_to_float(*reinterpret_cast<const uint16_t*>(stg + packed::kStgKz + r * 8 + 2 * g));
      const float vs = half_bits_to_float(*reinterpret_cast<const uint16_t*>(stg + packed::kStgVs + r * 8 + 2 * g));
      const float vz = half_bits_to_float(*reinterpret_cast<const uint16_t*>(stg + packed::kStgVz + r * 8 + 2 * g));
#pragma unroll
      for (int k = 0; k < 8; ++k) {
        const float code = __uint_as_float(0x4B000000u | ((wk >> (4 * k)) & 0xFu)) - 8388608.f;
        f[k] = fmaf(code, ks, kz) * kc[k];
      }
      *dk = float8_to_bf16x8(f);
#pragma unroll
      for (int k = 0; k < 8; ++k) {
        const float code = __uint_as_float(0x4B000000u | ((wv >> (4 * k)) & 0xFu)) - 8388608.f;
        f[k] = fmaf(code, vs, vz);
      }
      *dv = float8_to_bf16x8(f);
    }
    __syncthreads();   // every thread is done with the stage
    if (threadIdx.x == 0 && u + kUnpackStages < units) {
      const int jn = (u0 + u + kUnpackStages) * 128;
      packed::stage_tile(kv, b, h, jn, min(end, jn + 128), stg_raw + (u % kUnpackStages) * packed::kStageBytes,
                         &sfull[u % kUnpackStages], pc);
    }
  }
}

// the unpack of n slots of BH (b, h) pairs: the 16-channel form up to 2^20 slot-heads (a
// single sequence), the 32-channel one above; each CTA takes about four passes
void launch_unpack(const ma_kv& kv, int BH, int H, int n, void* out_k, void* out_v, const int64_t sok[3],
                   const int64_t sov[3], int live_only, cudaStream_t st) {
  // a long batch of a purely packed prefix (no dense tail): the staged form
  if ((long long)BH * n > (1ll << 20) && kv.nf == 0 && packed::eligible(kv)) {
    static bool attr = false;
    const int smem = kUnpackStages * packed::kStageBytes;
    if (!attr && cudaFuncSetAttribute(unpack_staged_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, smem) ==
                     cudaSuccess)
      attr = true;
    const dim3 grid((n + 128 * kUnpackUnits - 1) / (128 * kUnpackUnits), BH);
    unpack_staged_kernel<<<grid, 256, smem, st>>>(kv, H, n, (__nv_bfloat16*)out_k, (__nv_bfloat16*)out_v, sok[0],
                                                  sok[1], sok[2], sov[0], sov[1], sov[2], live_only);
    return;
  }
  const bool narrow = (long long)BH * n <= (1ll << 20);
  const int tok = narrow ? kUnpack16Tok : kUnpackTok;
  int gx = (n + tok - 1) / tok;
  if (gx > 8) gx = (gx + 3) / 4;
  const dim3 ugrid(gx, BH);
  if (narrow)
    unpack_token16_kernel<<<ugrid, 256, 0, st>>>(kv, H, n, (__nv_bfloat16*)out_k, (__nv_bfloat16*)out_v, sok[0],
                                                 sok[1], sok[2], sov[0], sov[1], sov[2], live_only);
  else
    unpack_token_kernel<<<ugrid, 256, 0, st>>>(kv, H, n, (__nv_bfloat16*)out_k, (__nv_bfloat16*)out_v, sok[0],
                                               sok[1], sok[2], sov[0], sov[1], sov[2], live_only);
}

}  // namespace

int launch_select_topk(const float* score, int B, int H, int n, int64_t ss0, int64_t ss1,
                       const uint8_t* mask, const int32_t* lens, int k, int64_t* indices, float* values,
                       int64_t si0, int64_t si1, cudaStream_t st) {
  if (n <= 1024 * 16) {  // keys in registers
    auto go = [&](auto kernel) {
      launch_pdl(kernel, dim3(B * H), dim3(kSelThreads), 0, st, score, H, n, ss0, ss1, mask, lens, k, indices,
                 values, si0, si1);
    };
    if (n <= 1024 * 4) go(select_topk_reg<4>);
    else if (n <= 1024 * 8) go(select_topk_reg<8>);
    else go(select_topk_reg<16>);
    return cudaGetLastError() == cudaSuccess ? MA_OK : MA_ERR_CUDA;
  }
  if (n <= kSelCluster * 1024 * 16) {  // keys in the registers of a cluster of CTAs
    auto go = [&](auto kernel) -> int {
      cudaLaunchConfig_t cfg = {};
      cfg.gridDim = dim3(kSelCluster, B * H);
      cfg.blockDim = dim3(kSelThreads);
      cfg.dynamicSmemBytes = 0;
      cfg.stream = st;
      cudaLaunchAttribute attr[1];
      attr[0].id = cudaLaunchAttributeClusterDimension;
      attr[0].val.clusterDim.x = kSelCluster;
      attr[0].val.clusterDim.y = 1;
      attr[0].val.clusterDim.z = 1;
      cfg.attrs = attr;
      cfg.numAttrs = 1;
      return cudaLaunchKernelEx(&cfg, kernel, score, H, n, ss0, ss1, mask, lens, k, indices, values, si0, si1) ==
                     cudaSuccess ? MA_OK : MA_ERR_CUDA;
    };
    if (n <= kSelCluster * 1024 * 4) return go(select_topk_cluster<4>);
    if (n <= kSelCluster * 1024 * 8) return go(select_topk_cluster<8>);
    return go(select_topk_cluster<16>);
  }
  const int staged = n <= kSelSmemKeys ? 1 : 0;
  const size_t smem = staged ? (size_t)n * sizeof(uint32_t) : 0;
  if (staged && smem > 48 * 1024 &&
      cudaFuncSetAttribute(select_topk_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem) !=
          cudaSuccess)
    return MA_ERR_CUDA;
  select_topk_kernel<<<B * H, kSelThreads, smem, st>>>(score, H, n, ss0, ss1, mask, lens, k, indices, values,
                                                       si0, si1, staged);
  return cudaGetLastError() == cudaSuccess ? MA_OK : MA_ERR_CUDA;
}

int retain_sort_cap(int capacity) {
  int c = 1;
  while (c < capacity) c <<= 1;
  return c;
}

int launch_retain(const float* score, const int32_t* phys, int n_phys, const int32_t* pos,
                  int lanes, int live, int capacity, int recent_window, int sink_tokens,
                  int64_t* keep, cudaStream_t st) {
  const int cap = retain_sort_cap(capacity);
  const size_t smem = (size_t)cap * sizeof(unsigned long long) + (((size_t)live + 15) / 16) * 16;
  if (smem > 200 * 1024) return MA_ERR_UNSUPPORTED;
  if (cudaFuncSetAttribute(retain_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem) !=
      cudaSuccess)
    return MA_ERR_CUDA;
  const int W = recent_window < capacity ? recent_window : capacity;
  int gated = 0;
  if (live <= kSelCluster * kSelThreads * 8) {   // positions in order: the cluster select
    auto go = [&](auto kernel, int per) -> bool {
      cudaLaunchConfig_t cfg = {};
      const int ncl = (live + kSelThreads * per - 1) / (kSelThreads * per);
      cfg.gridDim = dim3(ncl, lanes);
      cfg.blockDim = dim3(kSelThreads);
      cfg.dynamicSmemBytes = 0;
      cfg.stream = st;
      cudaLaunchAttribute attr[1];
      attr[0].id = cudaLaunchAttributeClusterDimension;
      attr[0].val.clusterDim.x = ncl;
      attr[0].val.clusterDim.y = 1;
      attr[0].val.clusterDim.z = 1;
      cfg.attrs = attr;
      cfg.numAttrs = 1;
      return cudaLaunchKernelEx(&cfg, kernel, score, phys, n_phys, pos, live, capacity, W, sink_tokens, keep) ==
             cudaSuccess;
    };
    bool ok;
    if (live <= kSelThreads * 4) ok = go(retain_sorted<4>, 4);
    else ok = go(retain_sorted<8>, 8);
    if (!ok) return MA_ERR_CUDA;
    gated = 1;
  }
  retain_kernel<<<lanes, kSelThreads, smem, st>>>(score, phys, n_phys, pos, live, capacity, W,
                                                  sink_tokens, keep, cap, gated);
  return cudaGetLastError() == cudaSuccess ? MA_OK : MA_ERR_CUDA;
}

int launch_unpack_live(const ma_kv& kv, int B, int H, int D, void* out_k, void* out_v, const int64_t sok[3],
                       const int64_t sov[3], cudaStream_t st) {
  const int k = kv.nq + kv.nf;
  if (!(kv.layout == MA_KV_PACKED_TOKEN && kv.dtype == MA_BF16 && D == 128 && kv.kchan && kv.vgroup == 32 &&
        kv.kgroup == 32 && (kv.nf == 0 || kv.kf)))
    return MA_ERR_UNSUPPORTED;
  if (k == 0) return MA_OK;
  launch_unpack(kv, B * H, H, k, out_k, out_v, sok, sov, 1, st);
  return cudaGetLastError() == cudaSuccess ? MA_OK : MA_ERR_CUDA;
}

int launch_gather_kv(const ma_kv& kv, int B, int H, int D, const int64_t* idx, int k, int64_t si0,
                     int64_t si1, void* out_k, void* out_v, const int64_t sok[3],
                     const int64_t sov[3], int out_dtype, cudaStream_t st) {
  if (k == 0) return MA_OK;
  if (!idx && kv.layout == MA_KV_PACKED_TOKEN && kv.dtype == MA_BF16 && out_dtype == MA_BF16 && D == 128 &&
      kv.kchan && kv.vgroup == 32 && kv.kgroup == 32 && (kv.nf == 0 || kv.kf)) {
    // the whole token-mode prefix: the contiguous unpack
    launch_unpack(kv, B * H, H, k, out_k, out_v, sok, sov, 0, st);
    return cudaGetLastError() == cudaSuccess ? MA_OK : MA_ERR_CUDA;
  }
  dim3 grid((k + kGatherTok - 1) / kGatherTok, B * H);
  if (out_dtype == MA_F32) {
    launch_pdl(gather_kv_kernel<float>, grid, dim3(256), 0, st, kv, H, D, idx, k, si0, si1, (float*)out_k,
               (float*)out_v, sok[0], sok[1], sok[2], sov[0], sov[1], sov[2]);
  } else {
    launch_pdl(gather_kv_kernel<__nv_bfloat16>, grid, dim3(256), 0, st, kv, H, D, idx, k, si0, si1,
               (__nv_bfloat16*)out_k, (__nv_bfloat16*)out_v, sok[0], sok[1], sok[2], sov[0], sov[1], sov[2]);
  }
  return cudaGetLastError() == cudaSuccess ? MA_OK : MA_ERR_CUDA;
}

}  // namespace ma
