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
