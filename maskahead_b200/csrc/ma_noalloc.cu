// Value-aware score for callers that cannot allocate device memory.
//
// ma_value_score needs scratch (per-head counters, the centre, per-tile partial sums)
// and takes it from a caller-provided workspace. Some callers cannot provide one: a
// host binding (JNI, cgo, a plugin interface) that is handed only the input and output
// device buffers by its framework and has no device allocator of its own, or code that
// must not call cudaMalloc/cudaFree at all because the framework owns every device
// allocation. ma_value_score_noalloc serves them with scratch that lives in this file:
// a static device array of kScratchBytes, which every GPU that loads the library holds
// until the process exits. Nothing here calls cudaMalloc, cudaFree or an allocating
// library routine.
#include <mutex>

#include "ma_kernels.cuh"

namespace {

constexpr size_t kScratchBytes = MA_NOALLOC_SCRATCH_BYTES;  // 8 MiB per device

// Host code may not use this name as a device address: on the host it names a
// stand-in, not the device array. Its device address comes from cudaGetSymbolAddress.
static __device__ __align__(256) unsigned char g_value_scratch[kScratchBytes];

constexpr int kMaxDevices = 64;
void* g_scratch_ptr[kMaxDevices] = {nullptr};
std::mutex g_scratch_mu;

// Device address of the scratch array on the current device, looked up once per device.
int scratch_address(void** out) {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) return MA_ERR_CUDA;
  std::lock_guard<std::mutex> lock(g_scratch_mu);
  if (g_scratch_ptr[dev] == nullptr) {
    void* p = nullptr;
    if (cudaGetSymbolAddress(&p, g_value_scratch) != cudaSuccess || p == nullptr) return MA_ERR_CUDA;
    g_scratch_ptr[dev] = p;
  }
  *out = g_scratch_ptr[dev];
  return MA_OK;
}

// Bytes at the front of the array that a call of BH heads needs zeroed: the error word
// (offset 0) and the (counter, generation) pairs of heads 0..BH-1 (from offset 8), in
// 256-byte units.
size_t noalloc_clear_bytes(int BH) { return ((8 + (size_t)BH * sizeof(uint2) + 255) / 256) * 256; }

}  // namespace

extern "C" {

int ma_value_score_noalloc(const ma_kv* kv, int B, int H, int D, const float* a, const int64_t sa[2],
                           float* score, const int64_t sscore[2], void* stream) {
  if (B <= 0 || H <= 0) return MA_ERR_ARG;
  if (D != 64 && D != 128) return MA_ERR_UNSUPPORTED;
  if (!kv || !a || !sa || !score || !sscore) return MA_ERR_ARG;
  const int n = kv->nq + kv->nf;
  if (n < 0) return MA_ERR_ARG;
  if (ma::value_score_ws_bytes(B, H, n, D) > kScratchBytes) return MA_ERR_UNSUPPORTED;
  void* ws = nullptr;
  int rc = scratch_address(&ws);
  if (rc != MA_OK) return rc;
  // the error word and this call's per-head (counter, generation) pairs must start at
  // zero; the rest of the array keeps what earlier calls left and is overwritten before
  // it is read
  if (cudaMemsetAsync(ws, 0, noalloc_clear_bytes(B * H), (cudaStream_t)stream) != cudaSuccess) return MA_ERR_CUDA;
  return ma_value_score(kv, B, H, D, a, sa, score, sscore, ws, kScratchBytes, stream);
}

int ma_value_score_noalloc_status(void* stream) {
  void* ws = nullptr;
  const int rc = scratch_address(&ws);
  if (rc != MA_OK) return rc;
  return ma_workspace_status(ws, kScratchBytes, stream);
}

}  // extern "C"
