// Compaction of the retained slots after an eviction: dst slot j of lane (b, h) gets the
// stored bytes of src slot keep[b, h, j] in every array of the layout, moved bit-exactly.
//
// The reference rebuilds per-token layouts this way (cache.py:659-678 compact_tokens:
// codes and fp16 scales move as they are, nothing is re-quantized) and dense bf16/fp32
// caches by a gather (cache.py:342-365 compact, whose bf16 re-staging is exact). It is
// pure data movement, bound by HBM: per kept slot each array's row is read once from a
// random slot and written once, contiguously. One launch moves every array: grid.y picks
// the array, grid.x the (lane, chunk of slots: 256, or more for arrays of short rows); each thread copies whole
// vectors (16 bytes when the row, the bases and the strides allow it) and issues
// kUnroll loads before their stores, so every warp keeps several row reads in flight.
#include "ma_kernels.cuh"

namespace ma {
namespace {

constexpr int kCompactThreads = 256;
constexpr int kCompactChunk = 256;     // kept slots per block (at least)
constexpr int kUnroll = 4;

template <typename V>
__device__ __forceinline__ V zero_vec() {
  V v;
  memset(&v, 0, sizeof(V));
  return v;
}

template <typename V>
__device__ __forceinline__ void compact_rows(const CompactArray& a, const int64_t* keep_lane, int64_t b,
                                             int64_t h, int j0, int count, int64_t n) {
  const int units = a.row_bytes / (int)sizeof(V);
  const int items = count * units;
  const unsigned char* src = a.src + b * a.ss[0] + h * a.ss[1];
  unsigned char* dst = a.dst + b * a.ds[0] + h * a.ds[1];
  for (int base = threadIdx.x; base < items; base += kCompactThreads * kUnroll) {
    V v[kUnroll];
    int64_t drow[kUnroll];
#pragma unroll
    for (int u = 0; u < kUnroll; ++u) {
      const int it = base + u * kCompactThreads;
      drow[u] = -1;
      if (it < items) {
        const int s = it / units, w = it - s * units;
        const int64_t slot = __ldg(keep_lane + j0 + s);
        drow[u] = (int64_t)(j0 + s) * a.ds[2] + (int64_t)w * (int64_t)sizeof(V);
        v[u] = (slot >= 0 && slot < n)
                   ? __ldg(reinterpret_cast<const V*>(src + slot * a.ss[2] + (int64_t)w * (int64_t)sizeof(V)))
                   : zero_vec<V>();
      }
    }
#pragma unroll
    for (int u = 0; u < kUnroll; ++u)
      if (drow[u] >= 0) *reinterpret_cast<V*>(dst + drow[u]) = v[u];
  }
}

__global__ void __launch_bounds__(kCompactThreads, 6) compact_kernel(CompactParams p) {
  const CompactArray& a = p.arrays[blockIdx.y];
  const int lane = blockIdx.x / p.chunks;
  const int chunk = blockIdx.x - lane * p.chunks;
  if (chunk >= a.chunks) return;   // an array of short rows covers its slots in fewer blocks
  const int64_t b = lane / p.H, h = lane - b * p.H;
  const int j0 = chunk * a.slots_per_block;
  const int count = min(a.slots_per_block, p.C - j0);
  const int64_t* keep_lane = p.keep + b * p.sk0 + h * p.sk1;
  switch (a.vec_bytes) {
    case 16: compact_rows<uint4>(a, keep_lane, b, h, j0, count, p.n); break;
    case 8: compact_rows<uint2>(a, keep_lane, b, h, j0, count, p.n); break;
    case 4: compact_rows<uint32_t>(a, keep_lane, b, h, j0, count, p.n); break;
    case 2: compact_rows<uint16_t>(a, keep_lane, b, h, j0, count, p.n); break;
    default: compact_rows<uint8_t>(a, keep_lane, b, h, j0, count, p.n); break;
  }
}

// The remap of a group-preserving rebuild (cache.py:236-335): one CTA per lane sets every
// old slot to -1, then writes the new slot of every slot that a kept group, the encoded
// list or the staged list names (entries < 0 are padding and name nothing). The lists are
// written one after another (groups before, groups after, encoded, staged), as the
// reference scatters them, so a slot named by two lists takes the later list's slot.
__global__ void __launch_bounds__(256) rebuild_remap_kernel(RemapParams p) {
  const int64_t lane = blockIdx.x;
  int64_t* remap = p.remap + lane * p.old_len;
  for (int i = threadIdx.x; i < p.old_len; i += blockDim.x) remap[i] = -1;
  __syncthreads();
  const int gk = p.kgroup;
  for (int pass = 0; pass < 2; ++pass) {
    const int64_t* gid = pass == 0 ? p.gb + lane * p.g1 : p.ga + lane * p.g3;
    const int count = (pass == 0 ? p.g1 : p.g3) * gk;
    const int at = pass == 0 ? 0 : (p.g1 + p.g2) * gk;
    for (int i = threadIdx.x; i < count; i += blockDim.x) {
      const int64_t g = gid[i / gk];
      const int64_t old = g * gk + i % gk;
      if (g >= 0 && old < p.old_len) remap[old] = at + i;
    }
    __syncthreads();
  }
  for (int i = threadIdx.x; i < p.m; i += blockDim.x) {
    const int64_t old = p.enc[lane * p.m + i];
    if (old >= 0 && old < p.old_len) remap[old] = (int64_t)p.g1 * gk + i;
  }
  __syncthreads();
  for (int i = threadIdx.x; i < p.st; i += blockDim.x) {
    const int64_t old = p.stg[lane * p.st + i];
    if (old >= 0 && old < p.old_len) remap[old] = p.ql + i;
  }
}

}  // namespace

// The planning of a group-preserving rebuild after an eviction (session.py:303-356), one
// CTA per lane. Live entry i (slot phys[i], position pos[i]) lies in key group
// phys / kgroup when phys < ql; a group is kept whole when at least `need` live entries
// lie in it (need 0: none is) and it is not one of the last tail_groups; an entry is
// staged when it is not packed (phys >= ql) and among the recent_window newest positions
// (pos >= the window's smallest); every other entry not in a kept group is re-encoded. The
// kept groups ascend; the encoded and staged slots follow the live axis, which is position
// order (the eviction state keeps it sorted: checked here, a lane out of order is counted
// in maxes[3] and its lists are not meaningful). Lists are padded with -1 to their full
// width; counts[lane] gets the three lengths and maxes[0..2] their maxima over lanes.
constexpr int kPlanThreads = 1024;

// exclusive prefix of `flag` over the block (every thread calls it), plus the block total
__device__ __forceinline__ int block_scan(bool flag, int* warp_tot, int* total) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const unsigned m = __ballot_sync(0xffffffffu, flag);
  const int in_warp = __popc(m & ((1u << lane) - 1u));
  __syncthreads();                      // warp_tot free (a previous call's reads are done)
  if (lane == 0) warp_tot[warp] = __popc(m);
  __syncthreads();
  if (warp == 0) {
    const int v = lane < (int)(blockDim.x >> 5) ? warp_tot[lane] : 0;
    int incl = v;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int u = __shfl_up_sync(0xffffffffu, incl, o);
      if (lane >= o) incl += u;
    }
    warp_tot[lane] = incl - v;          // exclusive prefix of the warp totals
    if (lane == 31) warp_tot[32] = incl;
  }
  __syncthreads();
  *total = warp_tot[32];
  return warp_tot[warp] + in_warp;
}

__global__ void __launch_bounds__(kPlanThreads) evict_plan_kernel(EvictPlanParams p) {
  __shared__ int cnt[kEvictMaxGroups + 1];
  __shared__ unsigned char keepg[kEvictMaxGroups];
  __shared__ int warp_tot[33];
  __shared__ int s_bad;
  const int64_t lane = blockIdx.x;
  const int32_t* phys = p.phys + lane * p.sphys;
  const int64_t* pos = p.pos + lane * p.spos;
  const int gk = p.kgroup, ql = p.ql, live = p.live;
  const int ng = max(1, ql / gk);
  for (int g = threadIdx.x; g <= ng; g += blockDim.x) cnt[g] = 0;
  if (threadIdx.x == 0) s_bad = 0;
  __syncthreads();
  for (int i = threadIdx.x; i < live; i += blockDim.x) {
    const int s = phys[i];
    atomicAdd(&cnt[(s >= 0 && s < ql) ? s / gk : ng], 1);
    if (i + 1 < live && pos[i + 1] <= pos[i]) s_bad = 1;
  }
  __syncthreads();
  const int keep_to = ng - p.tail_groups;
  for (int g = threadIdx.x; g < ng; g += blockDim.x) keepg[g] = (p.need > 0 && cnt[g] >= p.need && g < keep_to) ? 1 : 0;
  __syncthreads();
  // kept groups, ascending
  int total, n_groups = 0;
  for (int g0 = 0; g0 < ng; g0 += blockDim.x) {
    const int g = g0 + threadIdx.x;
    const bool f = g < ng && keepg[g];
    const int at = block_scan(f, warp_tot, &total);
    if (f) p.groups_before[lane * ng + n_groups + at] = g;
    n_groups += total;
  }
  for (int k = n_groups + threadIdx.x; k < ng; k += blockDim.x) p.groups_before[lane * ng + k] = -1;
  // the recent window's smallest position
  const int w = min(p.recent_window, live);
  const int64_t thr = w > 0 ? pos[live - w] : INT64_MAX;
  int n_enc = 0, n_stg = 0;
  for (int i0 = 0; i0 < live; i0 += blockDim.x) {
    const int i = i0 + threadIdx.x;
    bool enc = false, stg = false;
    int s = -1;
    if (i < live) {
      s = phys[i];
      const bool in_q = s >= 0 && s < ql;
      const bool kept = in_q && keepg[s / gk];
      stg = !in_q && pos[i] >= thr;
      enc = !kept && !stg;
    }
    int tot_e, tot_s;
    const int at_e = block_scan(enc, warp_tot, &tot_e);
    if (enc) p.encode[lane * live + n_enc + at_e] = s;
    const int at_s = block_scan(stg, warp_tot, &tot_s);
    if (stg) p.stage[lane * live + n_stg + at_s] = s;
    n_enc += tot_e;
    n_stg += tot_s;
  }
  for (int k = n_enc + threadIdx.x; k < live; k += blockDim.x) p.encode[lane * live + k] = -1;
  for (int k = n_stg + threadIdx.x; k < live; k += blockDim.x) p.stage[lane * live + k] = -1;
  if (threadIdx.x == 0) {
    p.counts[lane * 3 + 0] = n_groups;
    p.counts[lane * 3 + 1] = n_enc;
    p.counts[lane * 3 + 2] = n_stg;
    atomicMax(&p.maxes[0], n_groups);
    atomicMax(&p.maxes[1], n_enc);
    atomicMax(&p.maxes[2], n_stg);
    if (s_bad) atomicAdd(&p.maxes[3], 1);
  }
}

int launch_evict_plan(const EvictPlanParams& p, int lanes, cudaStream_t st) {
  if (cudaMemsetAsync(p.maxes, 0, 4 * sizeof(int32_t), st) != cudaSuccess) return MA_ERR_CUDA;
  if (lanes == 0) return MA_OK;
  evict_plan_kernel<<<lanes, kPlanThreads, 0, st>>>(p);
  return cudaGetLastError() == cudaSuccess ? MA_OK : MA_ERR_CUDA;
}

int launch_rebuild_remap(const RemapParams& p, int lanes, cudaStream_t st) {
  if (lanes <= 0 || p.old_len <= 0) return MA_OK;
  rebuild_remap_kernel<<<lanes, 256, 0, st>>>(p);
  return cudaGetLastError() == cudaSuccess ? MA_OK : MA_ERR_CUDA;
}

int launch_compact(CompactParams& p, int B, cudaStream_t st) {
  if (p.C == 0 || p.narrays == 0) return MA_OK;
  // every thread keeps kUnroll vectors in flight: arrays of short rows take more slots
  // per block (an 8-byte scale row: 1024 slots), long rows kCompactChunk
  p.chunks = 0;
  for (int i = 0; i < p.narrays; ++i) {
    CompactArray& a = p.arrays[i];
    const int units = a.row_bytes / a.vec_bytes;
    const int spb = (kCompactThreads * kUnroll) / units;
    a.slots_per_block = spb > kCompactChunk ? spb : kCompactChunk;
    a.chunks = (p.C + a.slots_per_block - 1) / a.slots_per_block;
    if (a.chunks > p.chunks) p.chunks = a.chunks;
  }
  const int64_t blocks = (int64_t)B * p.H * p.chunks;
  if (blocks > 0x7fffffffLL) return MA_ERR_UNSUPPORTED;
  dim3 grid((unsigned)blocks, (unsigned)p.narrays);
  compact_kernel<<<grid, kCompactThreads, 0, st>>>(p);
  return cudaGetLastError() == cudaSuccess ? MA_OK : MA_ERR_CUDA;
}

}  // namespace ma
