// Tensor Memory Accelerator (TMA) loads for the tcgen05 kernels.
//
// A tensor map describes a 4-D bf16 tensor in global memory (dims innermost first:
// channels, rows, heads, batch) and a box; one thread issues
//   cp.async.bulk.tensor.4d.shared::cluster.global.mbarrier::complete_tx::bytes
// and the hardware writes the box into shared memory with the 128-byte swizzle, which is
// exactly the K-major SW128 layout the MMA descriptors read (ma_tcgen05.cuh): a box of
// 64 channels x R rows lands as R lines of 128 bytes, 16-byte chunk q of line r at
// q ^ (r & 7). Completion is signalled on an mbarrier whose expected transaction bytes
// the issuing thread sets first; boxes reaching past the tensor are zero-filled and
// still count their full size. Loads only, never with cluster multicast.
#pragma once

#include <cuda.h>
#include <stdint.h>

#include "ma_tcgen05.cuh"

namespace ma {
namespace tma {

__device__ __forceinline__ void expect_tx(uint64_t* mbar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%1], %0;\n" ::"r"(bytes), "r"(tc::smem_addr(mbar))
               : "memory");
}

__device__ __forceinline__ void load_4d(void* smem_dst, const CUtensorMap* map, int c0, int c1, int c2, int c3,
                                        uint64_t* mbar) {
  asm volatile(
      "cp.async.bulk.tensor.4d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4, %5, %6}], "
      "[%2];\n" ::"r"(tc::smem_addr(smem_dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(tc::smem_addr(mbar)), "r"(c0), "r"(c1), "r"(c2), "r"(c3)
      : "memory");
}

// The same load with an L2 cache policy (createpolicy): evict_last keeps the box in L2
// for a second pass over it, evict_first lets a read-once stream leave early.
__device__ __forceinline__ uint64_t policy_evict_last() {
  uint64_t p;
  asm volatile("createpolicy.fractional.L2::evict_last.b64 %0, 1.0;\n" : "=l"(p));
  return p;
}
__device__ __forceinline__ uint64_t policy_evict_first() {
  uint64_t p;
  asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;\n" : "=l"(p));
  return p;
}
__device__ __forceinline__ void load_4d_hint(void* smem_dst, const CUtensorMap* map, int c0, int c1, int c2, int c3,
                                             uint64_t* mbar, uint64_t policy) {
  asm volatile(
      "cp.async.bulk.tensor.4d.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint [%0], "
      "[%1, {%3, %4, %5, %6}], [%2], %7;\n" ::"r"(tc::smem_addr(smem_dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(tc::smem_addr(mbar)), "r"(c0), "r"(c1), "r"(c2), "r"(c3), "l"(policy)
      : "memory");
}

// Shared -> global tensor store of one box (never at a negative coordinate); completion
// is tracked per thread with bulk groups.
__device__ __forceinline__ void store_2d(const CUtensorMap* map, int c0, int c1, const void* smem_src) {
  asm volatile("cp.async.bulk.tensor.2d.global.shared::cta.bulk_group [%0, {%2, %3}], [%1];\n" ::"l"(
                   reinterpret_cast<uint64_t>(map)),
               "r"(tc::smem_addr(smem_src)), "r"(c0), "r"(c1)
               : "memory");
}
__device__ __forceinline__ void store_commit() { asm volatile("cp.async.bulk.commit_group;\n" ::: "memory"); }
// wait until the issued stores have finished reading shared memory
__device__ __forceinline__ void store_wait_read() { asm volatile("cp.async.bulk.wait_group.read 0;\n" ::: "memory"); }
// wait until the issued stores are complete (their writes performed)
__device__ __forceinline__ void store_wait_all() { asm volatile("cp.async.bulk.wait_group 0;\n" ::: "memory"); }

}  // namespace tma

// Host: a 4-D bf16 tensor map with the 128-byte swizzle. dims/box innermost first,
// strides_bytes for dims 1..3. Returns false if the driver rejects it (the caller then
// uses its cp.async path).
bool make_tma_map_bf16_4d(CUtensorMap* map, const void* base, const uint64_t dims[4],
                          const uint64_t strides_bytes[3], const uint32_t box[4]);
// Host: a 2-D tensor map [rows][cols] (bf16 or fp32, row stride in bytes), 128-byte swizzle.
bool make_tma_map_2d(CUtensorMap* map, bool bf16, const void* base, uint64_t cols, uint64_t rows,
                     uint64_t row_stride_bytes, uint32_t box_cols, uint32_t box_rows);

}  // namespace ma
