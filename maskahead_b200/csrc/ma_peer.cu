// KV-head sharding's exchange of head outputs by this library's own kernel, over NVLink.
//
// Each rank of a KV-head-sharded layer step holds the outputs of its query heads,
// [B, Hl, T, D] bf16 (Hl = Hq / world), and every rank needs all of them, [B, Hq, T, D]
// (rank r's heads at [r Hl, (r+1) Hl)). Instead of a collective library call, every rank
// owns a receive region in its own HBM, mapped into every peer's address space through a
// CUDA IPC handle:
//
//   [slot 0: B Hq T D bf16][slot 1: same][counters: world u32]
//
// and call e (e = 1, 2, ...; kept in the caller's workspace, so a CUDA graph replays it)
// runs head_gather_kernel: its CTAs store the rank's rows straight into slot e & 1 of every
// rank's region (plain peer stores over NVLink, 16 bytes a thread; no TMA and no multicast
// on peer memory), and each CTA then adds 1 to counter `rank` of every region (a release
// reduction at system scope); the last CTA of the rank waits -- bounded -- until every
// rank's counter in its own region holds the CTAs of every call so far (all ranks run the
// same calls with the same grids, so the running totals agree). head_gather_copy_kernel
// then copies the slot to the caller's [B, Hq, T, D] output. The attention launch can run
// the same exchange itself (ma_prefix_attention_gather: its merge stores the rows, its CTAs
// arrive on the same counters); the two forms share the counters and may alternate. Two
// slots suffice: a rank writes slot s of call e + 2 only after every CTA of every rank
// arrived for call e + 1, which a rank's CTAs do only after its copy of call e (stream
// order). A wait that gives up sets the workspace's error word (ma_workspace_status reads
// it) and the call returns without the peers' rows.
#include <string.h>

#include <algorithm>

#include "ma_kernels.cuh"
#include "ma_tcgen05.cuh"

namespace ma {

namespace {

using namespace tc;

constexpr int kMaxWorld = 8;
constexpr int kD = 128;
constexpr int kGatherThreads = 256;

struct PeerBases {
  char* base[kMaxWorld];   // every rank's region as mapped here (this rank's own is local)
};

__device__ __forceinline__ void red_release_sys_add(uint32_t* p) {
  asm volatile("red.release.sys.global.add.u32 [%0], 1;\n" ::"l"(p) : "memory");
}
__device__ __forceinline__ uint32_t ld_acquire_sys_u32(const uint32_t* p) {
  uint32_t v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];\n" : "=r"(v) : "l"(p) : "memory");
  return v;
}

// ws (this rank's, 256-byte aligned): [0] error word, [1] CTA arrival counter, [2] calls done,
// [3] (the fused form's copy arrivals), [4] every rank's CTAs of the calls so far, per rank
__global__ void __launch_bounds__(kGatherThreads) head_gather_kernel(
    const __nv_bfloat16* __restrict__ part, int64_t sp0, int64_t sp1, int64_t sp2, int B, int Hl, int T, int world,
    int rank, int64_t slot_bytes, PeerBases peers, uint32_t* ws, uint64_t wait_ns) {
  pdl_wait();   // with a programmatic launch, the rows may come from the kernel before
  const uint32_t epoch = *reinterpret_cast<volatile uint32_t*>(ws + 2) + 1u;
  const int64_t slot_off = (int64_t)(epoch & 1u) * slot_bytes;
  const int Hq = Hl * world;
  const int64_t chunks = (int64_t)B * Hl * T * (kD / 8);   // 16-byte chunks of the rank's rows
  for (int64_t i = (int64_t)blockIdx.x * kGatherThreads + threadIdx.x; i < chunks;
       i += (int64_t)gridDim.x * kGatherThreads) {
    const int c = (int)(i & 15);
    const int64_t row = i >> 4;
    const int t = (int)(row % T);
    const int64_t bh = row / T;
    const int hl = (int)(bh % Hl), b = (int)(bh / Hl);
    const uint4 v = *reinterpret_cast<const uint4*>(part + (int64_t)b * sp0 + (int64_t)hl * sp1 + (int64_t)t * sp2 + 8 * c);
    const int64_t off = slot_off + ((((int64_t)b * Hq + (int64_t)rank * Hl + hl) * T + t) * kD + 8 * c) * 2;
    for (int p = 0; p < world; ++p) *reinterpret_cast<uint4*>(peers.base[p] + off) = v;
  }
  __syncthreads();
  if (threadIdx.x != 0) return;
  // this CTA arrives on its rank's counter in every rank's region: a release reduction at
  // system scope (the CTA barrier makes every thread's peer stores observed by thread 0,
  // the release is cumulative)
  const int64_t flags_off = 2 * slot_bytes;
  for (int p = 0; p < world; ++p) red_release_sys_add(reinterpret_cast<uint32_t*>(peers.base[p] + flags_off) + rank);
  if (atomicAdd(ws + 1, 1u) != gridDim.x - 1) return;
  // the last CTA of this rank: every rank's rows in this rank's region once every rank's
  // counter here holds the CTAs of every call so far (the same grids on every rank)
  ws[1] = 0u;
  const uint32_t want = *reinterpret_cast<volatile uint32_t*>(ws + 4) + gridDim.x;
  const uint32_t* mine = reinterpret_cast<const uint32_t*>(peers.base[rank] + flags_off);
  const uint64_t t0 = global_ns();
  bool ok = true;
  for (int q = 0; q < world && ok; ++q) {
    while ((int32_t)(ld_acquire_sys_u32(mine + q) - want) < 0) {
      if (global_ns() - t0 > wait_ns) {
        ok = false;
        break;
      }
    }
  }
  if (!ok) atomicExch(reinterpret_cast<int*>(ws), 1);
  ws[4] = want;
  ws[2] = epoch;   // the copy kernel reads the slot from it
}

// out [B, Hq, T, D] (strides so0..so2) <- slot (calls done & 1) of this rank's region
__global__ void __launch_bounds__(kGatherThreads) head_gather_copy_kernel(
    const char* __restrict__ region, int64_t slot_bytes, int B, int Hq, int T, __nv_bfloat16* __restrict__ out,
    int64_t so0, int64_t so1, int64_t so2, const uint32_t* ws) {
  pdl_wait();
  const uint32_t epoch = *reinterpret_cast<const volatile uint32_t*>(ws + 2);
  const __nv_bfloat16* src = reinterpret_cast<const __nv_bfloat16*>(region + (int64_t)(epoch & 1u) * slot_bytes);
  const int64_t chunks = (int64_t)B * Hq * T * (kD / 8);
  for (int64_t i = (int64_t)blockIdx.x * kGatherThreads + threadIdx.x; i < chunks;
       i += (int64_t)gridDim.x * kGatherThreads) {
    const int c = (int)(i & 15);
    const int64_t row = i >> 4;
    const int t = (int)(row % T);
    const int64_t bh = row / T;
    const int hq = (int)(bh % Hq), b = (int)(bh / Hq);
    reinterpret_cast<uint4*>(out + (int64_t)b * so0 + (int64_t)hq * so1 + (int64_t)t * so2)[c] =
        reinterpret_cast<const uint4*>(src + row * kD)[c];
  }
}

}  // namespace

size_t head_gather_region_bytes(int B, int Hq, int T) {
  const size_t slot = (((size_t)B * Hq * T * kD * 2) + 255) & ~size_t(255);
  return 2 * slot + 256;
}

int launch_head_gather(const void* part, const int64_t sp[3], int B, int Hl, int T, int world, int rank,
                       void* const* regions, void* out, const int64_t so[3], void* ws, uint64_t wait_ns,
                       cudaStream_t st) {
  if (world < 1 || world > kMaxWorld || rank < 0 || rank >= world || B <= 0 || Hl <= 0 || T <= 0) return MA_ERR_ARG;
  PeerBases peers;
  memset(&peers, 0, sizeof(peers));
  for (int p = 0; p < world; ++p) {
    if (!regions[p] || (reinterpret_cast<uintptr_t>(regions[p]) & 255)) return MA_ERR_ARG;
    peers.base[p] = reinterpret_cast<char*>(regions[p]);
  }
  const int Hq = Hl * world;
  const int64_t slot_bytes = (int64_t)((head_gather_region_bytes(B, Hq, T) - 256) / 2);
  uint32_t* w = reinterpret_cast<uint32_t*>((reinterpret_cast<uintptr_t>(ws) + 255) & ~uintptr_t(255));
  const int64_t chunks = (int64_t)B * Hl * T * (kD / 8);
  int grid = (int)std::min<int64_t>((chunks + kGatherThreads - 1) / kGatherThreads, 4 * device_sm_count());
  if (launch_pdl(head_gather_kernel, dim3(grid), dim3(kGatherThreads), 0, st, (const __nv_bfloat16*)part, sp[0],
                 sp[1], sp[2], B, Hl, T, world, rank, slot_bytes, peers, w, wait_ns) != cudaSuccess)
    return MA_ERR_CUDA;
  const int64_t out_chunks = chunks * world;
  grid = (int)std::min<int64_t>((out_chunks + kGatherThreads - 1) / kGatherThreads, 4 * device_sm_count());
  if (launch_pdl(head_gather_copy_kernel, dim3(grid), dim3(kGatherThreads), 0, st, (const char*)regions[rank],
                 slot_bytes, B, Hq, T, (__nv_bfloat16*)out, so[0], so[1], so[2], (const uint32_t*)w) != cudaSuccess)
    return MA_ERR_CUDA;
  return MA_OK;
}

}  // namespace ma
