// Quantize-on-append: dense K/V rows -> the packed k4v4 layouts the attention reads.
//
// Semantics of the reference's quantizers (src/maskahead/reference.py:58-90 quantize_keys,
// 182-213 quantize_values; token-mode keys cache.py:484-497), asymmetric 4-bit:
//     scale = max((max - min) / 15, 1e-8)     zero = min
//     code  = clamp(round_half_even((x - min) / scale), 0, 15)
// computed in the INPUT's dtype the way torch evaluates it: every elementwise op in fp32
// and rounded back to the tensor dtype (bf16 inputs: round-to-nearest-even to bf16 after
// each op), so codes and parameters match the reference bit for bit. scale and zero are
// stored as fp16 (param_dtype); element 2i of a byte is its low nibble (reference.py:
// 35-45). Token-mode keys are first divided by the per-channel divisor in fp32 and
// rounded to the input dtype (cache.py:491-497); the divisor is sqrt(max(max_t |K|, 1e-4))
// in fp32 (cache.py:488-490).
#include "ma_kernels.cuh"

namespace ma {

namespace {

constexpr int kGroup = 32;   // tokens or channels per quantization group (the shipped configs)

template <bool BF16>
__device__ __forceinline__ float rnd(float x) {
  return BF16 ? __bfloat162float(__float2bfloat16_rn(x)) : x;
}

template <typename T>
__device__ __forceinline__ float ld(const T* p);
template <>
__device__ __forceinline__ float ld<float>(const float* p) { return *p; }
template <>
__device__ __forceinline__ float ld<__nv_bfloat16>(const __nv_bfloat16* p) { return __bfloat162float(*p); }

// One group of 32 values (exact in the input dtype) -> packed codes, scale and zero bits.
template <bool BF16>
__device__ __forceinline__ void quantize_group(const float* x, uint32_t packed[4], uint16_t& scale_bits,
                                               uint16_t& zero_bits) {
  float mn = x[0], mx = x[0];
#pragma unroll
  for (int i = 1; i < kGroup; ++i) {
    mn = fminf(mn, x[i]);
    mx = fmaxf(mx, x[i]);
  }
  float s = rnd<BF16>(rnd<BF16>(mx - mn) / 15.0f);
  s = rnd<BF16>(fmaxf(s, 1e-8f));
#pragma unroll
  for (int w = 0; w < 4; ++w) packed[w] = 0u;
#pragma unroll
  for (int i = 0; i < kGroup; ++i) {
    const float t = rnd<BF16>(rnd<BF16>(x[i] - mn) / s);
    const float c = fminf(fmaxf(rintf(t), 0.f), 15.f);
    packed[i >> 3] |= (uint32_t)c << (4 * (i & 7));
  }
  scale_bits = __half_as_ushort(__float2half_rn(s));
  zero_bits = __half_as_ushort(__float2half_rn(mn));
}

// Token groups: one thread per (b, h, slot, channel group). kchan != null: token-mode keys.
template <typename T>
__global__ void quantize_tokens_kernel(const T* __restrict__ x, int H, int n, int D, int64_t sx0, int64_t sx1,
                                       int64_t sx2, const float* __restrict__ kchan, int64_t skc0, int64_t skc1,
                                       uint8_t* __restrict__ payload, int64_t sp0, int64_t sp1, int64_t sp2,
                                       uint16_t* __restrict__ scale, uint16_t* __restrict__ zero, int64_t ss0,
                                       int64_t ss1, int64_t ss2, int64_t total) {
  constexpr bool BF16 = sizeof(T) == 2;
  const int groups = D / kGroup;
  for (int64_t id = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; id < total; id += (int64_t)gridDim.x * blockDim.x) {
    const int g = (int)(id % groups);
    const int64_t rest = id / groups;
    const int j = (int)(rest % n);
    const int64_t bh = rest / n;
    const int h = (int)(bh % H), b = (int)(bh / H);
    const T* row = x + (int64_t)b * sx0 + (int64_t)h * sx1 + (int64_t)j * sx2 + g * kGroup;
    float v[kGroup];
#pragma unroll
    for (int i = 0; i < kGroup; ++i) v[i] = ld(row + i);
    if (kchan) {
      const float* c = kchan + (int64_t)b * skc0 + (int64_t)h * skc1 + g * kGroup;
#pragma unroll
      for (int i = 0; i < kGroup; ++i) v[i] = rnd<BF16>(v[i] / c[i]);
    }
    uint32_t packed[4];
    uint16_t sb, zb;
    quantize_group<BF16>(v, packed, sb, zb);
    uint4* dst = reinterpret_cast<uint4*>(payload + (int64_t)b * sp0 + (int64_t)h * sp1 + (int64_t)j * sp2 + g * 16);
    *dst = make_uint4(packed[0], packed[1], packed[2], packed[3]);
    const int64_t so = (int64_t)b * ss0 + (int64_t)h * ss1 + (int64_t)j * ss2 + g;
    scale[so] = sb;
    zero[so] = zb;
  }
}

// KIVI channel groups: one thread per (b, h, token group, channel); consecutive threads
// take consecutive channels, so every token row is read coalesced.
template <typename T>
__global__ void quantize_channels_kernel(const T* __restrict__ x, int H, int ng, int D, int64_t sx0, int64_t sx1,
                                         int64_t sx2, uint8_t* __restrict__ payload, int64_t sp0, int64_t sp1,
                                         int64_t sp2, uint16_t* __restrict__ scale, uint16_t* __restrict__ zero,
                                         int64_t ss0, int64_t ss1, int64_t ss2, int64_t total) {
  constexpr bool BF16 = sizeof(T) == 2;
  for (int64_t id = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; id < total; id += (int64_t)gridDim.x * blockDim.x) {
    const int d = (int)(id % D);
    const int64_t rest = id / D;
    const int gi = (int)(rest % ng);
    const int64_t bh = rest / ng;
    const int h = (int)(bh % H), b = (int)(bh / H);
    const T* col = x + (int64_t)b * sx0 + (int64_t)h * sx1 + (int64_t)gi * kGroup * sx2 + d;
    float v[kGroup];
#pragma unroll
    for (int i = 0; i < kGroup; ++i) v[i] = ld(col + (int64_t)i * sx2);
    uint32_t packed[4];
    uint16_t sb, zb;
    quantize_group<BF16>(v, packed, sb, zb);
    uint4* dst = reinterpret_cast<uint4*>(payload + (int64_t)b * sp0 + (int64_t)h * sp1 + (int64_t)gi * sp2 + d * 16);
    *dst = make_uint4(packed[0], packed[1], packed[2], packed[3]);
    const int64_t so = (int64_t)b * ss0 + (int64_t)h * ss1 + (int64_t)gi * ss2 + d;
    scale[so] = sb;
    zero[so] = zb;
  }
}

// Token-mode key divisor: one CTA per (b, h), 4 token lanes x D channels, max |K| then
// sqrt(max(., 1e-4)).
template <typename T>
__global__ void __launch_bounds__(512) key_divisor_kernel(const T* __restrict__ k, int H, int n, int D, int64_t sk0,
                                                          int64_t sk1, int64_t sk2, float* __restrict__ kchan,
                                                          int64_t skc0, int64_t skc1) {
  __shared__ float sMax[4][kMaxD];
  const int bh = blockIdx.x;
  const int b = bh / H, h = bh - (bh / H) * H;
  const int d = threadIdx.x % kMaxD, lane4 = threadIdx.x / kMaxD;
  float m = 0.f;
  if (d < D) {
    const T* base = k + (int64_t)b * sk0 + (int64_t)h * sk1 + d;
#pragma unroll 8
    for (int j = lane4; j < n; j += 4) m = fmaxf(m, fabsf(ld(base + (int64_t)j * sk2)));
  }
  sMax[lane4][d] = m;
  __syncthreads();
  if (lane4 == 0 && d < D) {
    const float mx = fmaxf(fmaxf(sMax[0][d], sMax[1][d]), fmaxf(sMax[2][d], sMax[3][d]));
    kchan[(int64_t)b * skc0 + (int64_t)h * skc1 + d] = sqrtf(fmaxf(mx, 1e-4f));
  }
}

int grid_for(int64_t total, int threads) {
  const int64_t blocks = (total + threads - 1) / threads;
  const int64_t cap = (int64_t)device_sm_count() * 16;
  return (int)(blocks < cap ? (blocks > 0 ? blocks : 1) : cap);
}

}  // namespace

int launch_quantize_tokens(const void* x, int dtype, int B, int H, int n, int D, const int64_t sx[3], const float* kchan,
                           const int64_t skc[2], uint8_t* payload, const int64_t sp[3], uint16_t* scale, uint16_t* zero,
                           const int64_t ss[3], cudaStream_t st) {
  const int64_t total = (int64_t)B * H * n * (D / kGroup);
  if (total == 0) return MA_OK;
  const int threads = 128, grid = grid_for(total, threads);
  const int64_t k0 = kchan ? skc[0] : 0, k1 = kchan ? skc[1] : 0;
  if (dtype == MA_BF16)
    quantize_tokens_kernel<__nv_bfloat16><<<grid, threads, 0, st>>>(
        reinterpret_cast<const __nv_bfloat16*>(x), H, n, D, sx[0], sx[1], sx[2], kchan, k0, k1, payload, sp[0], sp[1],
        sp[2], scale, zero, ss[0], ss[1], ss[2], total);
  else
    quantize_tokens_kernel<float><<<grid, threads, 0, st>>>(reinterpret_cast<const float*>(x), H, n, D, sx[0], sx[1],
                                                            sx[2], kchan, k0, k1, payload, sp[0], sp[1], sp[2], scale,
                                                            zero, ss[0], ss[1], ss[2], total);
  return cudaGetLastError() == cudaSuccess ? MA_OK : MA_ERR_CUDA;
}

int launch_quantize_channels(const void* x, int dtype, int B, int H, int n, int D, const int64_t sx[3],
                             uint8_t* payload, const int64_t sp[3], uint16_t* scale, uint16_t* zero, const int64_t ss[3],
                             cudaStream_t st) {
  const int ng = n / kGroup;
  const int64_t total = (int64_t)B * H * ng * D;
  if (total == 0) return MA_OK;
  const int threads = 128, grid = grid_for(total, threads);
  if (dtype == MA_BF16)
    quantize_channels_kernel<__nv_bfloat16><<<grid, threads, 0, st>>>(
        reinterpret_cast<const __nv_bfloat16*>(x), H, ng, D, sx[0], sx[1], sx[2], payload, sp[0], sp[1], sp[2], scale,
        zero, ss[0], ss[1], ss[2], total);
  else
    quantize_channels_kernel<float><<<grid, threads, 0, st>>>(reinterpret_cast<const float*>(x), H, ng, D, sx[0],
                                                              sx[1], sx[2], payload, sp[0], sp[1], sp[2], scale, zero,
                                                              ss[0], ss[1], ss[2], total);
  return cudaGetLastError() == cudaSuccess ? MA_OK : MA_ERR_CUDA;
}

int launch_key_divisor(const void* k, int dtype, int B, int H, int n, int D, const int64_t sk[3], float* kchan,
                       const int64_t skc[2], cudaStream_t st) {
  if (B * H == 0) return MA_OK;
  if (dtype == MA_BF16)
    key_divisor_kernel<__nv_bfloat16><<<B * H, 512, 0, st>>>(reinterpret_cast<const __nv_bfloat16*>(k), H, n, D, sk[0],
                                                             sk[1], sk[2], kchan, skc[0], skc[1]);
  else
    key_divisor_kernel<float><<<B * H, 512, 0, st>>>(reinterpret_cast<const float*>(k), H, n, D, sk[0], sk[1], sk[2],
                                                     kchan, skc[0], skc[1]);
  return cudaGetLastError() == cudaSuccess ? MA_OK : MA_ERR_CUDA;
}

}  // namespace ma
