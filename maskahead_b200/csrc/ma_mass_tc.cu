// Prefix mass with tcgen05 MMAs, with the value-score centre -- and the value score
// itself -- fused in.
//
// Transposed product: for a tile of 128 prefix slots, S^T = K Q^T (tcgen05.mma, M = 128
// slots, N = the selection rows padded to 16, K = 128 channels; accumulator in TMEM), so
// TMEM lane j holds slot j's logits against every selection row. Each thread owns one
// slot (its lane) and half of the rows: it loads its logits with tcgen05.ld and sums
//     exp(s_rj * scale - M_p,r) / L_p,r = 2^(s_rj * scale * log2e - B_r),
//     B_r = M_p,r * log2e + log2(L_p,r)            (splitk.py:320-359; reference.py:318-366)
// in registers; the two halves meet in shared memory in a fixed order, then
// a_j = sum / R2 (0 on dead slots). bf16 products are exact in fp32 and accumulate in
// fp32, so a_j is fp32-accurate.
//
// With a centre requested the CTA also accumulates sum_j a_j v_j and sum_j a_j from the
// V tiles it streams, and the last CTA of the head (a counter in the workspace) reduces
// the per-CTA partials in CTA order into c = sum a v / max(sum a, 1e-12) (session.py:
// 27-40, 870-899), then advances the head's generation word. With the score requested
// as well the launch is cooperative (every CTA resident): each CTA waits (bounded) for
// its head's generation to advance, reads c and writes a_j * ||v_j - c|| for its own slots
// -- one launch for mass, centre and score.
//
// Slot tiles stream through a 2-stage cp.async ring (each CTA holds its whole range,
// up to 256 slots, in flight from the start). Every wait is bounded.
#include "ma_kernels.cuh"
#include "ma_cp_async.cuh"
#include "ma_stage.cuh"
#include "ma_tcgen05.cuh"

namespace ma {

namespace {

using namespace tc;

constexpr int kWarps = 8;
constexpr int kThreads = kWarps * 32;
constexpr int kTile = 128;                  // slots per tile (= M, = TMEM lanes)
constexpr int kD = 128;
constexpr int kChunks = kD / 8;
constexpr int kMaxRows = 256;               // selection rows (N of the MMA)
constexpr int kStages = 2;
constexpr float kLog2e = 1.4426950408889634f;
constexpr int kQBytes = kMaxRows * kD * 2;  // 64 KB
constexpr int kTileBytes = kTile * kD * 2;  // 32 KB (K or V)
constexpr int kSmemBytes = 1024 + kQBytes + 2 * kStages * kTileBytes;
constexpr uint32_t kTmemCols = 256;
constexpr int kMaxCtas = 1024;              // partial slots per head (the launcher never exceeds)

struct Args {
  ma_rows q;
  ma_kv kv;
  const int32_t* q_rows;
  const float* m_p;
  const float* l_p;
  float* mass;
  int64_t sm0, sm1;
  float* score;         // fused value score (cooperative launch), or null
  int64_t ss0, ss1;
  float* part;          // [BH][ctas][D+1] centre partials (centre only)
  uint2* sync;          // [BH]: arrival counter, centre generation
  float* centre;        // [BH][D]
  int* err;
  float scale;
  int H, T2, slots_per_cta;
  uint64_t peer_wait_ns;  // bound on the wait for the head's centre (other CTAs)
};

template <bool PACKED, bool CENTRE>
__device__ __forceinline__ void load_tile(const Args& A, int b, int h, int j0, int end, uint8_t* sK, uint8_t* sV,
                                          uint8_t* sOk, const float* sKch) {
  if (PACKED) {   // packed slots: wide loads, dequantized into the tiles (dense tail by cp.async)
    stage::packed_tile<kTile, false, CENTRE>(A.kv, A.H, b, h, j0, end, nullptr, 0, 0, sK, sV, sOk, sKch, threadIdx.x,
                                             kThreads);
    cp_async_commit();
    return;
  }
  const __nv_bfloat16* kf = reinterpret_cast<const __nv_bfloat16*>(A.kv.kf);
  const __nv_bfloat16* vf = reinterpret_cast<const __nv_bfloat16*>(A.kv.vf);
  for (int c = threadIdx.x; c < kTile * kChunks; c += kThreads) {
    const int jj = c / kChunks, ch = c % kChunks;
    const int j = j0 + jj;
    const bool ok = j < end && kv_live(A.kv, A.H, b, h, j);
    uint8_t* dk = sK + kmajor_off(jj, ch, kTile);
    uint8_t* dv = sV + jj * (kD * 2) + ch * 16;
    if (ok && (!PACKED || j >= A.kv.nq)) {
      int sb = b, row = j - A.kv.nq;
      if (!PACKED && A.kv.pages) kv_page(A.kv, b, row, sb, row);   // a paged dense cache
      cp_async16(tc::smem_addr(dk), kf + (int64_t)sb * A.kv.skf[0] + (int64_t)h * A.kv.skf[1] + (int64_t)row * A.kv.skf[2] + ch * 8, true);
      if (CENTRE)
        cp_async16(tc::smem_addr(dv), vf + (int64_t)sb * A.kv.svf[0] + (int64_t)h * A.kv.svf[1] + (int64_t)row * A.kv.svf[2] + ch * 8, true);
    } else if (ok) {
      float f[8];
      kv_read8<true>(A.kv, b, h, j, ch, f);
      *reinterpret_cast<uint4*>(dk) = float8_to_bf16x8(f);
      if (CENTRE) {
        kv_read8<false>(A.kv, b, h, j, ch, f);
        *reinterpret_cast<uint4*>(dv) = float8_to_bf16x8(f);
      }
    } else {
      *reinterpret_cast<uint4*>(dk) = make_uint4(0, 0, 0, 0);
      if (CENTRE) *reinterpret_cast<uint4*>(dv) = make_uint4(0, 0, 0, 0);
    }
    if (ch == 0) sOk[jj] = ok ? 1 : 0;
  }
  cp_async_commit();
}


template <bool PACKED, bool CENTRE>
__global__ void __launch_bounds__(kThreads, 1) prefix_mass_tc(const Args A) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sQ = smem;                         // K-major [2 d blocks][Npad rows][128 B]
  uint8_t* sRing = sQ + kQBytes;              // [stage][K tile (swizzled) | V tile (row-major)]
  __shared__ __align__(16) float sB[kMaxRows];   // per selection row: B_r (+inf: no contribution)
  __shared__ int sRowT[kMaxRows];                // block position of selection row r (-1: none)
  __shared__ float sHalf[2][kTile];
  __shared__ __align__(16) float sA[kTile];
  __shared__ float sAres[kStages][kTile];        // a_j of the tiles still in the ring
  __shared__ uint8_t sOk[kStages][kTile];
  __shared__ float sRed[4][kD];
  __shared__ float sKch[kD];                     // token-mode key divisor of (b, h)
  __shared__ float sTot[kD + 1];
  __shared__ float sAsum[4];
  __shared__ uint32_t s_taddr;
  __shared__ __align__(8) uint64_t mbar;
  __shared__ int s_abort, s_wait_ok, sLast;
  __shared__ unsigned sGen;

  const int n = A.kv.nq + A.kv.nf;
  const int bh = blockIdx.y;
  const int H = A.H;
  const int b = bh / H, h = bh - (bh / H) * H;
  const int G = A.q.Hq / H;
  const int T = A.q.T;
  const int R2 = G * A.T2;
  const int Npad = (R2 + 15) & ~15;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int quarter = warp & 3, chalf = warp >> 2;
  const int slot_lane = quarter * 32 + lane;          // this thread's slot within a tile (TMEM lane)
  const int begin = blockIdx.x * A.slots_per_cta;
  const int end = min(n, begin + A.slots_per_cta);
  const float inv_rows = 1.f / (float)R2;
  const float c2 = A.scale * kLog2e;

  // the head's centre generation before this CTA arrives (the last CTA advances it)
  if (CENTRE && threadIdx.x == 0) sGen = *reinterpret_cast<volatile const unsigned*>(&A.sync[bh].y);
  if (PACKED && A.kv.layout == MA_KV_PACKED_TOKEN && threadIdx.x < kD)
    sKch[threadIdx.x] = A.kv.kchan[(int64_t)b * A.kv.skc[0] + (int64_t)h * A.kv.skc[1] + threadIdx.x];
  // selection rows r2 = g*T2 + i -> query row (h*G + g, q_rows[i]) and B_r, one row per thread
  for (int rr = threadIdx.x; rr < Npad; rr += kThreads) {
    const int g = rr / A.T2;
    const int t = rr < R2 ? A.q_rows[rr - g * A.T2] : -1;
    const bool ok = t >= 0 && t < T;
    float Bv = INFINITY;   // exp2(s - inf) = 0: no contribution
    if (ok) {
      const int64_t ri = (int64_t)bh * G * T + (int64_t)g * T + t;
      const float L = A.l_p[ri];
      if (L > 0.f) Bv = fmaf(A.m_p[ri], kLog2e, log2f(L));
    }
    sRowT[rr] = ok ? t : -1;
    sB[rr] = Bv;
  }
  __syncthreads();
  {
    const __nv_bfloat16* qp = reinterpret_cast<const __nv_bfloat16*>(A.q.q);
    for (int c = threadIdx.x; c < Npad * kChunks; c += kThreads) {
      const int rr = c / kChunks, ch = c % kChunks;
      const int t = sRowT[rr];
      uint8_t* dst = sQ + kmajor_off(rr, ch, Npad);
      if (t >= 0) {
        const int g = rr / A.T2;
        cp_async16(tc::smem_addr(dst), qp + (int64_t)b * A.q.sq[0] + (int64_t)(h * G + g) * A.q.sq[1] + (int64_t)t * A.q.sq[2] + ch * 8, true);
      } else {
        *reinterpret_cast<uint4*>(dst) = make_uint4(0, 0, 0, 0);
      }
    }
  }
  for (int st = 0; st < kStages; ++st) {   // the queries join the group of the first tile
    const int j0 = begin + st * kTile;
    uint8_t* sK = sRing + 2 * st * kTileBytes;
    if (j0 < end) load_tile<PACKED, CENTRE>(A, b, h, j0, end, sK, sK + kTileBytes, sOk[st], sKch);
    else cp_async_commit();
  }
  if (threadIdx.x == 0) {
    mbar_init(&mbar, 1);
    s_abort = 0;
    s_wait_ok = 1;
  }
  if (warp == 0) tmem_alloc(&s_taddr, kTmemCols);
  fence_before_sync();
  __syncthreads();
  fence_after_sync();
  const uint32_t taddr = s_taddr;
  const uint32_t tRow = taddr + ((uint32_t)(quarter * 32) << 16);   // this thread's lane
  const uint32_t idesc = idesc_bf16(kTile, Npad, false, false);
  const int cols_half = Npad / 2;                                    // rows handled per half
  const int c_lo = chalf * cols_half;
  uint32_t phase = 0;
  int stage = 0;
  // centre: channel pair cp (channels 2cp, 2cp+1) over key quarter kq of every tile
  const int cp = threadIdx.x & 63, kq = threadIdx.x >> 6;
  float cacc0 = 0.f, cacc1 = 0.f, asum = 0.f;
  bool aborted = false;

  const int ntiles = end > begin ? (end - begin + kTile - 1) / kTile : 0;
  const bool resident = ntiles <= kStages;   // every V tile of the CTA stays in the ring
  int tt = 0;
  for (int j0 = begin; j0 < end; j0 += kTile, ++tt) {
    uint8_t* sK = sRing + 2 * stage * kTileBytes;
    uint8_t* sV = sK + kTileBytes;
    cp_async_wait<kStages - 1>();
    fence_proxy_async();
    fence_before_sync();
    __syncthreads();
    fence_after_sync();
    if (s_abort) {
      aborted = true;
      break;
    }
    if (threadIdx.x == 0) {
      const uint32_t ka = tc::smem_addr(sK), qa = tc::smem_addr(sQ);
#pragma unroll
      for (int kk = 0; kk < kD / 16; ++kk) {
        const uint64_t ad = smem_desc(ka + (kk >> 2) * (kTile * 128) + (kk & 3) * 32, 16, 1024);
        const uint64_t bd = smem_desc(qa + (kk >> 2) * (Npad * 128) + (kk & 3) * 32, 16, 1024);
        mma_bf16(taddr, ad, bd, idesc, kk > 0);
      }
      mma_commit(&mbar);
    }
    const bool ok = mbar_wait(&mbar, phase);
    phase ^= 1;
    fence_after_sync();
    if (!ok) s_abort = 1;
    // this thread: slot slot_lane, rows [c_lo, c_lo + cols_half), in row order
    float acc[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll 1
    for (int c0 = 0; c0 < cols_half; c0 += 64) {
      // two 32-column loads per wait (columns stay inside the 256-column allocation)
      float sv[64];
      tmem_ld32(tRow + c_lo + c0, sv);
      tmem_ld32(tRow + c_lo + c0 + 32, sv + 32);
      tmem_ld_wait();
      const int lim = cols_half - c0;
#pragma unroll
      for (int i = 0; i < 64; i += 4) {
        const float4 b4 = *reinterpret_cast<const float4*>(&sB[(c_lo + c0 + i) & (kMaxRows - 1)]);
        if (i < lim) {   // lim is a multiple of 8
          acc[0] += ex2(fmaf(sv[i], c2, -b4.x));
          acc[1] += ex2(fmaf(sv[i + 1], c2, -b4.y));
          acc[2] += ex2(fmaf(sv[i + 2], c2, -b4.z));
          acc[3] += ex2(fmaf(sv[i + 3], c2, -b4.w));
        }
      }
    }
    sHalf[chalf][slot_lane] = (acc[0] + acc[1]) + (acc[2] + acc[3]);
    __syncthreads();
    if (threadIdx.x < kTile) {
      const int j = j0 + threadIdx.x;
      const float a = sOk[stage][threadIdx.x] ? (sHalf[0][threadIdx.x] + sHalf[1][threadIdx.x]) * inv_rows : 0.f;
      if (j < end) A.mass[(int64_t)b * A.sm0 + (int64_t)h * A.sm1 + j] = a;
      sA[threadIdx.x] = j < end ? a : 0.f;
      if (tt < kStages) sAres[tt][threadIdx.x] = j < end ? a : 0.f;
    }
    if (CENTRE) {
      __syncthreads();
      const __nv_bfloat162* v2 = reinterpret_cast<const __nv_bfloat162*>(sV);   // [key][64 channel pairs]
#pragma unroll 2
      for (int j4 = 0; j4 < kTile / 4; j4 += 4) {
        const float4 a4 = *reinterpret_cast<const float4*>(&sA[kq * (kTile / 4) + j4]);
        const float av[4] = {a4.x, a4.y, a4.z, a4.w};
#pragma unroll
        for (int u = 0; u < 4; ++u) {
          const float2 v = __bfloat1622float2(v2[(kq * (kTile / 4) + j4 + u) * (kD / 2) + cp]);
          cacc0 = fmaf(av[u], v.x, cacc0);
          cacc1 = fmaf(av[u], v.y, cacc1);
          asum += av[u];
        }
      }
    }
    fence_before_sync();
    __syncthreads();   // this stage and sA are consumed
    const int jn = j0 + kStages * kTile;
    if (jn < end) load_tile<PACKED, CENTRE>(A, b, h, jn, end, sK, sV, sOk[stage], sKch);
    else cp_async_commit();
    stage = (stage + 1) % kStages;
  }

  if (aborted && threadIdx.x == 0) atomicExch(A.err, 1);
  if (aborted) mbar_wait(&mbar, phase);     // drain the in-flight MMA (bounded)
  cp_async_wait<0>();
  fence_before_sync();
  __syncthreads();
  fence_after_sync();
  if (warp == 0) tmem_dealloc(taddr, kTmemCols);
  if (!CENTRE) return;

  // per-CTA centre partial (key quarters summed in order); the last CTA of the head
  // reduces the partials in CTA order and publishes c by advancing the generation
  sRed[kq][2 * cp] = cacc0;
  sRed[kq][2 * cp + 1] = cacc1;
  if (cp == 0) sAsum[kq] = asum;
  __syncthreads();
  float* mine = A.part + ((int64_t)bh * gridDim.x + blockIdx.x) * (kD + 1);
  if (threadIdx.x < kD)
    mine[threadIdx.x] = aborted ? NAN : ((sRed[0][threadIdx.x] + sRed[1][threadIdx.x]) + sRed[2][threadIdx.x]) + sRed[3][threadIdx.x];
  if (threadIdx.x == 0) mine[kD] = ((sAsum[0] + sAsum[1]) + sAsum[2]) + sAsum[3];
  __threadfence();
  __syncthreads();
  if (threadIdx.x == 0) sLast = atomicAdd(&A.sync[bh].x, 1u) == gridDim.x - 1 ? 1 : 0;
  __syncthreads();
  if (sLast) {
    __threadfence();
    if (threadIdx.x <= kD) {
      const float* base = A.part + (int64_t)bh * gridDim.x * (kD + 1) + threadIdx.x;
      float tot = 0.f;
      for (unsigned t0 = 0; t0 < gridDim.x; t0 += 16) {
        float v[16];
#pragma unroll
        for (int i = 0; i < 16; ++i) v[i] = t0 + i < gridDim.x ? __ldcg(base + (int64_t)(t0 + i) * (kD + 1)) : 0.f;
#pragma unroll
        for (int i = 0; i < 16; ++i) tot += v[i];   // CTA order
      }
      sTot[threadIdx.x] = tot;
    }
    __syncthreads();
    if (threadIdx.x < kD) A.centre[(int64_t)bh * kD + threadIdx.x] = sTot[threadIdx.x] / fmaxf(sTot[kD], 1e-12f);
    if (threadIdx.x == 0) A.sync[bh].x = 0u;
    __threadfence();
    __syncthreads();
    if (threadIdx.x == 0) {
      __threadfence();
      atomicAdd(&A.sync[bh].y, 1u);
    }
  }
  if (A.score == nullptr) return;

  // fused value score (cooperative launch: every CTA of the head is resident)
  if (!sLast && threadIdx.x == 0) {
    const uint64_t t0 = global_ns();
    while (ld_acquire_u32(&A.sync[bh].y) == sGen) {
      if (global_ns() - t0 > A.peer_wait_ns) {
        s_wait_ok = 0;
        atomicExch(A.err, 1);
        break;
      }
      __nanosleep(256);
    }
  }
  __syncthreads();
  const bool ok_c = s_wait_ok != 0;
  const int grp = threadIdx.x >> 4, l16 = threadIdx.x & 15;
  float cc[8];
#pragma unroll
  for (int i = 0; i < 8; ++i) cc[i] = __ldcg(A.centre + (int64_t)bh * kD + 8 * l16 + i);
  if (resident) {
    // V tiles and a_j still on chip: tile t sits in ring stage t (row-major bf16 rows)
    for (int t = 0; t < ntiles; ++t) {
      const uint8_t* sVt = sRing + (2 * t + 1) * kTileBytes;
#pragma unroll 2
      for (int jj = grp; jj < kTile; jj += kThreads / 16) {
        const int j = begin + t * kTile + jj;
        float f[8];
        bf16x8_to_float(*reinterpret_cast<const uint4*>(sVt + jj * (kD * 2) + l16 * 16), f);
        float s2 = 0.f;
#pragma unroll
        for (int i = 0; i < 8; ++i) {
          const float x = f[i] - cc[i];
          s2 = fmaf(x, x, s2);
        }
#pragma unroll
        for (int o = 8; o > 0; o >>= 1) s2 += __shfl_xor_sync(0xffffffffu, s2, o);
        if (l16 == 0 && j < end) A.score[(int64_t)b * A.ss0 + (int64_t)h * A.ss1 + j] = ok_c ? sAres[t][jj] * sqrtf(s2) : NAN;
      }
    }
    return;
  }
  constexpr int kBatch = 4;
  for (int jb = begin; jb < end; jb += (kThreads / 16) * kBatch) {
    float f[kBatch][8];
    bool live[kBatch];
#pragma unroll
    for (int u = 0; u < kBatch; ++u) {
      const int j = jb + u * (kThreads / 16) + grp;
      live[u] = j < end && kv_live(A.kv, H, b, h, j);
      if (live[u]) {
        kv_read8<false>(A.kv, b, h, j, l16, f[u]);
      } else {
#pragma unroll
        for (int i = 0; i < 8; ++i) f[u][i] = cc[i];
      }
    }
#pragma unroll
    for (int u = 0; u < kBatch; ++u) {
      float s2 = 0.f;
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        const float x = f[u][i] - cc[i];
        s2 = fmaf(x, x, s2);
      }
#pragma unroll
      for (int o = 8; o > 0; o >>= 1) s2 += __shfl_xor_sync(0xffffffffu, s2, o);
      const int j = jb + u * (kThreads / 16) + grp;
      if (l16 == 0 && j < end) {
        const float aj = live[u] ? A.mass[(int64_t)b * A.sm0 + (int64_t)h * A.sm1 + j] : 0.f;
        A.score[(int64_t)b * A.ss0 + (int64_t)h * A.ss1 + j] = ok_c ? aj * sqrtf(s2) : NAN;
      }
    }
  }
}

}  // namespace

int launch_prefix_mass_tc(const ma_rows& q, const ma_kv& kv, int H, const int32_t* q_rows, int T2, const float* m_p,
                          const float* l_p, float scale, float* mass, int64_t sm0, int64_t sm1, float* score,
                          int64_t ss0, int64_t ss1, const ValueWs& w, bool want_centre, bool* fused, cudaStream_t st) {
  *fused = false;
  const int n = kv.nq + kv.nf;
  const int BH = q.B * H;
  Args A;
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
  // CTAs: one wave over the heads, at least one tile each
  const int sms = device_sm_count();
  int per_head = sms / (BH > 0 ? BH : 1);
  if (per_head < 1) per_head = 1;
  int spc = (n + per_head - 1) / per_head;
  spc = ((spc + kTile - 1) / kTile) * kTile;
  A.slots_per_cta = spc < kTile ? kTile : spc;
  dim3 grid((n + A.slots_per_cta - 1) / A.slots_per_cta, BH);
  if ((int)grid.x > kMaxCtas) return MA_ERR_UNSUPPORTED;
  const bool packed = kv.layout != MA_KV_DENSE;
  auto go = [&](auto kernel) -> int {
    if (cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmemBytes) != cudaSuccess)
      return MA_ERR_CUDA;
    if (score != nullptr && want_centre) {
      // the fused score needs every CTA resident at once: a cooperative launch that fits
      int dev = 0, coop = 0, per_sm = 0;
      if (cudaGetDevice(&dev) == cudaSuccess &&
          cudaDeviceGetAttribute(&coop, cudaDevAttrCooperativeLaunch, dev) == cudaSuccess && coop &&
          cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kernel, kThreads, kSmemBytes) == cudaSuccess &&
          (long long)grid.x * grid.y <= (long long)per_sm * sms) {
        Args Ac = A;
        Ac.score = score;
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
        if (cudaLaunchKernelEx(&cfg, kernel, Ac) == cudaSuccess) {
          *fused = true;
          return MA_OK;
        }
        (void)cudaGetLastError();
      }
    }
    kernel<<<grid, kThreads, kSmemBytes, st>>>(A);
    return cudaGetLastError() == cudaSuccess ? MA_OK : MA_ERR_CUDA;
  };
  if (packed) return want_centre ? go(prefix_mass_tc<true, true>) : go(prefix_mass_tc<true, false>);
  return want_centre ? go(prefix_mass_tc<false, true>) : go(prefix_mass_tc<false, false>);
}

}  // namespace ma
