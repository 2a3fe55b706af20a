// C ABI of the select + attend hot path: argument validation, split planning and the
// launch sequence of every entry point declared in include/maskahead_b200.h.
#include <string.h>

#include "ma_kernels.cuh"
#include "ma_packed.cuh"

namespace ma {

int device_sm_count() {
  static int cached[64] = {0};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return 148;
  if (cached[dev] == 0) {
    int sms = 0;
    if (cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || sms <= 0)
      sms = 148;
    cached[dev] = sms;
  }
  return cached[dev];
}

namespace {
constexpr uint64_t kDefaultPeerWaitNs = 200000000ull;   // 200 ms
uint64_t g_peer_wait_ns = kDefaultPeerWaitNs;
}  // namespace

uint64_t peer_wait_ns() { return g_peer_wait_ns; }

}  // namespace ma

using namespace ma;

namespace {

int g_attention_kernel = 0;   // ma_set_attention_kernel
bool fa_disabled() { return g_attention_kernel == 1; }

inline bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }
inline int esize(int dtype) { return dtype == MA_F32 ? 4 : 2; }
inline bool valid_dtype(int dtype) { return dtype == MA_F32 || dtype == MA_BF16; }

// strides (elements) whose byte size keeps every row start 16-byte aligned
inline bool strides16(const int64_t* s, int count, int elem) {
  for (int i = 0; i < count; ++i)
    if (s[i] < 0 || ((s[i] * elem) & 15) != 0) return false;
  return true;
}

int check_rows(const ma_rows* q) {
  if (!q || !q->q) return MA_ERR_ARG;
  if (!valid_dtype(q->dtype)) return MA_ERR_ARG;
  if (q->B <= 0 || q->Hq <= 0 || q->T <= 0) return MA_ERR_ARG;
  if (q->D != 64 && q->D != 128) return MA_ERR_UNSUPPORTED;
  if (!aligned16(q->q) || !strides16(q->sq, 3, esize(q->dtype))) return MA_ERR_ARG;
  return MA_OK;
}

int check_kv(const ma_kv* kv, int D) {
  if (!kv) return MA_ERR_ARG;
  if (kv->nq < 0 || kv->nf < 0) return MA_ERR_ARG;
  if (!valid_dtype(kv->dtype)) return MA_ERR_ARG;
  if (kv->nf > 0) {
    if (!kv->kf || !kv->vf || !aligned16(kv->kf) || !aligned16(kv->vf)) return MA_ERR_ARG;
    if (!strides16(kv->skf, 3, esize(kv->dtype)) || !strides16(kv->svf, 3, esize(kv->dtype))) return MA_ERR_ARG;
  }
  if (kv->pages) {
    if (kv->page_size <= 0 || kv->num_pages <= 0 || kv->spg < 0) return MA_ERR_ARG;
    if (kv->layout == MA_KV_PACKED_CHANNEL && (kv->kgroup <= 0 || kv->page_size % kv->kgroup != 0))
      return MA_ERR_ARG;
  }
  if (kv->layout == MA_KV_DENSE) {
    if (kv->nq != 0) return MA_ERR_ARG;
    return MA_OK;
  }
  if (kv->layout != MA_KV_PACKED_TOKEN && kv->layout != MA_KV_PACKED_CHANNEL) return MA_ERR_ARG;
  if (kv->nq == 0) return MA_OK;
  if (kv->vgroup <= 0 || (kv->vgroup % 8) != 0 || D % kv->vgroup) return MA_ERR_UNSUPPORTED;
  if (!kv->vq || !kv->vs || !kv->vz || !kv->kq || !kv->ks || !kv->kz) return MA_ERR_ARG;
  // payload rows are read with 16-byte loads: 16-byte aligned bases and strides
  if (!aligned16(kv->vq) || !aligned16(kv->kq)) return MA_ERR_ARG;
  for (int i = 0; i < 3; ++i)
    if ((kv->svq[i] & 15) || (kv->skq[i] & 15) || kv->svq[i] < 0 || kv->skq[i] < 0 || kv->sks[i] < 0 ||
        kv->svs[i] < 0)
      return MA_ERR_ARG;
  if (kv->vgroup != 32 || (kv->layout == MA_KV_PACKED_CHANNEL && kv->kgroup != 32)) return MA_ERR_UNSUPPORTED;
  if (kv->layout == MA_KV_PACKED_TOKEN) {
    if (!kv->kchan) return MA_ERR_ARG;
  } else {
    if (kv->kgroup <= 0 || (kv->kgroup % 2) != 0) return MA_ERR_UNSUPPORTED;
    if (!kv->pages && kv->nq % kv->kgroup) return MA_ERR_ARG;
  }
  return MA_OK;
}

int check_block(const ma_block* cur, const ma_rows* q, int H) {
  if (!cur) return MA_ERR_ARG;
  if (cur->Tc < 0) return MA_ERR_ARG;
  if (cur->Tc == 0) return MA_OK;
  if (!cur->k || !cur->v || !aligned16(cur->k) || !aligned16(cur->v)) return MA_ERR_ARG;
  if (!strides16(cur->sk, 3, esize(q->dtype)) || !strides16(cur->sv, 3, esize(q->dtype))) return MA_ERR_ARG;
  (void)H;
  return MA_OK;
}

bool use_mma(const ma_rows& q, const ma_kv& kv) {
  // bf16 queries over a bf16 (or bf16-dequantized packed) cache go to the tensor cores
  return q.dtype == MA_BF16 && kv.dtype == MA_BF16 && q.D == 128;
}
// the attention kernel also needs a positive scale (its row maxima are taken on the raw
// logits q.k)
bool use_mma_attention(const ma_rows& q, const ma_kv& kv, float scale) { return use_mma(q, kv) && scale > 0.f; }

struct Plan {
  int nsplit;     // splits over the keys
  int split_len;  // keys per split (a multiple of the key tile)
  int S;          // partial slots per (b, h): nsplit (+1 for the current block)
  int Rp;         // padded rows
  bool o_bf16;    // partial outputs in bf16 (tensor-core kernel)
};

int row_tile(bool mma) { return mma ? tc_row_tile() : simt_row_block(); }
int key_tile(bool mma) { return mma ? tc_key_tile() : simt_key_tile(); }

// Splits over the keys: enough CTAs for one wave (tensor-core CTAs hold an SM each) or
// two (CUDA-core CTAs, several per SM), the current block included, but no split shorter
// than a few key tiles -- each split pays for staging its rows and writing R x D partials.
Plan plan_splits(int BH, int R, int n, int Tc, bool mma, bool fa = false) {
  Plan p;
  const int rt = fa ? fa_row_tile(R, BH) : row_tile(mma), kt = fa ? fa_key_tile() : key_tile(mma);
  const int row_blocks = (R + rt - 1) / rt;
  // tensor-core partial rows are stored per 32-row warp box
  p.Rp = mma ? ((R + 31) / 32) * 32 : row_blocks * rt;
  if (n <= 0) {
    p.nsplit = 0;
    p.split_len = kt;
  } else {
    const int sms = device_sm_count();
    const int per_split = BH * row_blocks;
    const int waves = mma ? 1 : 2;
    int target = (waves * sms) / (per_split > 0 ? per_split : 1) - (Tc > 0 ? 1 : 0);
    if (target < 1) target = 1;
    const int min_len = (mma ? 1 : 2) * kt;
    const int max_splits = (n + min_len - 1) / min_len;
    int ns = target < max_splits ? target : max_splits;
    // the pipelined kernel: at most 32 key tiles per split, so long rows of a large batch
    // spread over many short CTAs (several waves balance ragged lengths)
    if (fa) {
      const int by_len = (n + 32 * kt - 1) / (32 * kt);
      if (ns < by_len) ns = by_len < max_splits ? by_len : max_splits;
    }
    if (ns > 255) ns = 255;
    int len = (n + ns - 1) / ns;
    len = ((len + kt - 1) / kt) * kt;
    p.split_len = len;
    p.nsplit = (n + len - 1) / len;
  }
  p.S = p.nsplit + (Tc > 0 ? 1 : 0);
  if (p.S == 0) p.S = 1;
  p.o_bf16 = mma;
  return p;
}

// The fused merge's (counter, generation) pairs: a fixed-size block at the front of the
// workspace, so its words never move with the call's sizes.
constexpr int kSyncSlots = 8192;
constexpr size_t kSyncBytes = (size_t)kSyncSlots * sizeof(uint2);

size_t attention_ws(int B, int H, int R, int n, int D, int Tc) {
  size_t best = 0;
  for (int m = 0; m < 3; ++m) {
    const Plan p = plan_splits(B * H, R, n, Tc, m >= 1, m == 2);
    const size_t bytes = partials_bytes(B * H, p.S, p.Rp, D, p.o_bf16) + 512 + kSyncBytes;
    if (bytes > best) best = bytes;
  }
  return best;
}

// workspace: [256-byte aligned] error word block (256 B), the merge sync block, then the
// split partials
Partials carve_partials(void* ws, int BH, const Plan& p, int D, int** err, uint2** sync) {
  Partials P;
  char* base = reinterpret_cast<char*>((reinterpret_cast<uintptr_t>(ws) + 255) & ~uintptr_t(255));
  *err = reinterpret_cast<int*>(base);
  base += 256;
  *sync = reinterpret_cast<uint2*>(base);
  base += kSyncBytes;
  P.ml = reinterpret_cast<float2*>(base);
  P.o = base + (size_t)BH * p.S * p.Rp * sizeof(float2);
  P.o_bf16 = p.o_bf16 ? 1 : 0;
  P.S = p.S;
  P.Rp = p.Rp;
  (void)D;
  return P;
}

// The head gather in its own launches (ma_head_gather's kernels), when the attention's merge
// could not run it: the call's rows t < Tg of `out` go to every rank, the gathered rows
// into po->out.
int separate_gather(const ma_rows& q, const PeerOut* po, void* const* regions, const void* out, const int64_t so[3],
                    cudaStream_t st) {
  return launch_head_gather(out, so, q.B, q.Hq, po->Tg, po->world, po->rank, regions, po->out, po->so, po->ws,
                            peer_wait_ns(), st);
}

// shared by the prefix and the read-set attention: partial pass + combine
int run_attention(const ma_rows& q, const ma_kv& kv, int H, const ma_block& cur, float scale,
                  int causal_block, int q_pos0, int c_pos0, const int64_t* idx, int64_t si0,
                  int64_t si1, int n_keys, void* out, const int64_t so[3], float* m_p, float* l_p,
                  float* o_p, void* ws, size_t ws_bytes, cudaStream_t st, const PeerOut* po = nullptr,
                  void* const* regions = nullptr) {
  const int G = q.Hq / H;
  const int R = G * q.T;
  const bool mma = use_mma_attention(q, kv, scale);
  // TMA-fed dense bf16 calls take the 128 x 128-tile kernel (its plan is sized into the
  // workspace too)
  const bool fa = mma && !fa_disabled() && fa_eligible(q, kv, idx, cur, n_keys);
  Plan p = plan_splits(q.B * H, R, n_keys, cur.Tc, mma, fa);
  // the current block as the last prefix split's final key tile, when no prefix-only
  // statistics are asked for and that split is long (or the only one): a block split of its
  // own would be a CTA of one short tile per row block, plus a merge of one more split
  const int kt = fa ? fa_key_tile() : 0;
  const bool fold = fa && !idx && n_keys > 0 && kv.layout != MA_KV_PACKED_TOKEN && !m_p && !l_p && !o_p &&
                    causal_block == 0 && cur.Tc > 0 && cur.Tc <= kt && p.nsplit >= 1 &&
                    (p.nsplit == 1 || p.split_len >= 4 * kt);
  if (fold) p.S = p.nsplit;
  bool folded = false;
  bool gathered = false;   // the head gather ran inside the attention launch
  if (!ws || ws_bytes < partials_bytes(q.B * H, p.S, p.Rp, q.D, p.o_bf16) + 512 + kSyncBytes)
    return MA_ERR_WORKSPACE;
  int* err = nullptr;
  uint2* sync = nullptr;
  Partials P = carve_partials(ws, q.B * H, p, q.D, &err, &sync);
  int rc;
  if (p.nsplit + (cur.Tc > 0 ? 1 : 0) > 0) {
    if (mma) {
      FusedMerge fm;
      fm.out = out;
      fm.so[0] = so[0];
      fm.so[1] = so[1];
      fm.so[2] = so[2];
      fm.m_p = m_p;
      fm.l_p = l_p;
      fm.o_p = o_p;
      fm.sync = sync;
      fm.sync_slots = kSyncSlots;
      fm.wait_ns = peer_wait_ns();
      fm.gather = po != nullptr ? 1 : 0;
      if (po != nullptr) fm.po = *po;
      bool fused = false;
      rc = MA_ERR_UNSUPPORTED;
      if (fa) {
        rc = launch_attn_partial_fa(q, kv, H, cur, scale, causal_block, q_pos0, c_pos0, n_keys, p.split_len,
                                    p.nsplit, P, err, &fm, fold, &fused, &gathered, st);
        if (rc == MA_ERR_UNSUPPORTED) {   // a tensor map the TMA cannot describe: 64-key kernel
          p = plan_splits(q.B * H, R, n_keys, cur.Tc, mma);
          P = carve_partials(ws, q.B * H, p, q.D, &err, &sync);
        } else {
          folded = fold;
        }
      }
      if (rc == MA_ERR_UNSUPPORTED) {
        fm.gather = 0;   // only the pipelined kernel's cooperative merge gathers
        rc = launch_attn_partial_tc(q, kv, H, cur, scale, causal_block, q_pos0, c_pos0, idx, si0, si1, n_keys,
                                    p.split_len, p.nsplit, P, err, &fm, &fused, st);
      }
      if (rc != MA_OK) return rc;
      if (fused) return (po != nullptr && !gathered) ? separate_gather(q, po, regions, out, so, st) : MA_OK;
    } else {
      rc = launch_attn_partial_simt(q, kv, H, cur, scale, causal_block, q_pos0, c_pos0, idx, si0, si1, n_keys,
                                    p.split_len, p.nsplit, P, st);
      if (rc != MA_OK) return rc;
    }
  }
  rc = launch_attn_combine(q, H, P, p.nsplit, cur.Tc > 0 && !folded, out, so, m_p, l_p, o_p, st);
  if (rc != MA_OK || po == nullptr) return rc;
  return separate_gather(q, po, regions, out, so, st);
}

}  // namespace

extern "C" {

int ma_version(void) { return (0 << 16) | 1; }

int64_t ma_set_peer_wait_ns(int64_t ns) {
  const int64_t prev = (int64_t)g_peer_wait_ns;
  g_peer_wait_ns = ns > 0 ? (uint64_t)ns : kDefaultPeerWaitNs;
  return prev;
}

int ma_workspace_status(void* workspace, size_t workspace_bytes, void* stream) {
  if (!workspace || workspace_bytes < 256 + sizeof(int)) return MA_ERR_ARG;
  // the error word sits at the first 256-byte boundary of every workspace layout
  char* base = reinterpret_cast<char*>((reinterpret_cast<uintptr_t>(workspace) + 255) & ~uintptr_t(255));
  if (base + sizeof(int) > reinterpret_cast<char*>(workspace) + workspace_bytes) return MA_ERR_ARG;
  cudaStream_t st = (cudaStream_t)stream;
  int word = 0;
  if (cudaMemcpyAsync(&word, base, sizeof(int), cudaMemcpyDeviceToHost, st) != cudaSuccess ||
      cudaStreamSynchronize(st) != cudaSuccess)
    return MA_ERR_CUDA;
  if (word == 0) return MA_OK;
  if (cudaMemsetAsync(base, 0, sizeof(int), st) != cudaSuccess) return MA_ERR_CUDA;
  return MA_ERR_TIMEOUT;
}

const char* ma_last_cuda_error(void) {
  const cudaError_t e = cudaGetLastError();
  return e == cudaSuccess ? "no CUDA error pending" : cudaGetErrorString(e);
}

int ma_kv_read_in_place(const ma_kv* kv, int D) {
  if (!kv || check_kv(kv, D) != MA_OK || D != 128) return 0;
  if (kv->layout == MA_KV_DENSE) return kv->dtype == MA_BF16 && !kv->mask && !kv->pages ? 1 : 0;
  return kv->dtype == MA_BF16 && packed::eligible(*kv) ? 1 : 0;
}

int ma_set_attention_kernel(int which) {
  const int prev = g_attention_kernel;
  g_attention_kernel = (which >= 1 && which <= 3) ? which : 0;
  fa_set_pairs(g_attention_kernel == 2 ? 1 : g_attention_kernel == 3 ? 2 : 0);
  return prev;
}

int ma_set_mass_tiles(int tiles) {
  const int prev = fa_mass_tiles();
  fa_set_mass_tiles(tiles);
  return prev;
}

const char* ma_status_string(int status) {
  switch (status) {
    case MA_OK: return "ok";
    case MA_ERR_ARG: return "invalid argument";
    case MA_ERR_UNSUPPORTED: return "unsupported configuration";
    case MA_ERR_WORKSPACE: return "workspace missing or too small";
    case MA_ERR_CUDA: return "CUDA error";
    case MA_ERR_TIMEOUT: return "device-side wait timed out";
    default: return "unknown status";
  }
}

size_t ma_prefix_attention_workspace(int B, int H, int R, int n, int D, int Tc) {
  if (B <= 0 || H <= 0 || R <= 0 || n < 0 || D <= 0 || Tc < 0) return 0;
  return attention_ws(B, H, R, n, D, Tc);
}

int ma_prefix_attention(const ma_rows* q, const ma_kv* kv, int H, const ma_block* cur, float scale,
                        int causal_block, int q_pos0, int c_pos0, void* out, const int64_t so[3],
                        float* m_p, float* l_p, float* o_p, void* workspace, size_t workspace_bytes,
                        void* stream) {
  int rc = check_rows(q);
  if (rc) return rc;
  if (H <= 0 || q->Hq % H) return MA_ERR_ARG;
  if ((rc = check_kv(kv, q->D))) return rc;
  if ((rc = check_block(cur, q, H))) return rc;
  if (!out || !so || !aligned16(out) || !strides16(so, 3, esize(q->dtype))) return MA_ERR_ARG;
  if ((m_p == nullptr) != (l_p == nullptr)) return MA_ERR_ARG;
  if (o_p && !aligned16(o_p)) return MA_ERR_ARG;
  if (causal_block < 0) return MA_ERR_ARG;
  if (kv->nq + kv->nf == 0 && cur->Tc == 0) return MA_ERR_ARG;
  return run_attention(*q, *kv, H, *cur, scale, causal_block, q_pos0, c_pos0, nullptr, 0, 0,
                       kv->nq + kv->nf, out, so, m_p, l_p, o_p, workspace, workspace_bytes,
                       (cudaStream_t)stream);
}

int ma_prefix_attention_gather(const ma_rows* q, const ma_kv* kv, int H, const ma_block* cur, float scale,
                               int causal_block, int q_pos0, int c_pos0, void* out, const int64_t so[3],
                               float* m_p, float* l_p, float* o_p, void* workspace, size_t workspace_bytes,
                               int world, int rank, void* const* regions, int Tg, void* gout,
                               const int64_t sgo[3], void* gather_ws, size_t gather_ws_bytes, void* stream) {
  int rc = check_rows(q);
  if (rc) return rc;
  if (H <= 0 || q->Hq % H) return MA_ERR_ARG;
  if ((rc = check_kv(kv, q->D))) return rc;
  if ((rc = check_block(cur, q, H))) return rc;
  if (!out || !so || !aligned16(out) || !strides16(so, 3, esize(q->dtype))) return MA_ERR_ARG;
  if ((m_p == nullptr) != (l_p == nullptr)) return MA_ERR_ARG;
  if (o_p && !aligned16(o_p)) return MA_ERR_ARG;
  if (causal_block < 0) return MA_ERR_ARG;
  if (kv->nq + kv->nf == 0 && cur->Tc == 0) return MA_ERR_ARG;
  if (q->dtype != MA_BF16 || q->D != 128) return MA_ERR_UNSUPPORTED;
  if (world < 1 || world > kPeerMaxWorld || rank < 0 || rank >= world || !regions) return MA_ERR_ARG;
  if (Tg < 1 || Tg > q->T || !gout || !sgo || !aligned16(gout) || !strides16(sgo, 3, 2)) return MA_ERR_ARG;
  if (!gather_ws || gather_ws_bytes < ma_head_gather_workspace()) return MA_ERR_WORKSPACE;
  PeerOut po;
  memset(&po, 0, sizeof(po));
  for (int p = 0; p < world; ++p) {
    if (!regions[p] || (reinterpret_cast<uintptr_t>(regions[p]) & 255)) return MA_ERR_ARG;
    po.base[p] = reinterpret_cast<char*>(regions[p]);
  }
  po.ws = reinterpret_cast<uint32_t*>((reinterpret_cast<uintptr_t>(gather_ws) + 255) & ~uintptr_t(255));
  po.slot_bytes = (int64_t)((head_gather_region_bytes(q->B, q->Hq * world, Tg) - 256) / 2);
  po.out = gout;
  for (int i = 0; i < 3; ++i) po.so[i] = sgo[i];
  po.world = world;
  po.rank = rank;
  po.Hl = q->Hq;
  po.Tg = Tg;
  return run_attention(*q, *kv, H, *cur, scale, causal_block, q_pos0, c_pos0, nullptr, 0, 0, kv->nq + kv->nf, out,
                       so, m_p, l_p, o_p, workspace, workspace_bytes, (cudaStream_t)stream, &po, regions);
}

int ma_prefix_scores(const ma_rows* q, const ma_kv* kv, int H, const int32_t* q_rows, int T2,
                     const float* m_p, const float* l_p, float scale, float* mass, const int64_t smass[2],
                     float* score, const int64_t sscore[2], void* workspace, size_t workspace_bytes,
                     void* stream) {
  int rc = check_rows(q);
  if (rc) return rc;
  if (H <= 0 || q->Hq % H) return MA_ERR_ARG;
  if ((rc = check_kv(kv, q->D))) return rc;
  if (!q_rows || T2 <= 0 || !m_p || !l_p || !mass || !smass) return MA_ERR_ARG;
  if (smass[0] < 0 || smass[1] < 0) return MA_ERR_ARG;
  if (score && (!sscore || sscore[0] < 0 || sscore[1] < 0)) return MA_ERR_ARG;
  const int n = kv->nq + kv->nf;
  if (n == 0) return MA_OK;
  const int BH = q->B * H;
  const int G = q->Hq / H;
  const bool tc = use_mma(*q, *kv) && G * T2 <= 256;
  ValueWs w = {nullptr, nullptr, nullptr, nullptr};
  if (score || tc) {  // the tensor-core kernel reports bounded-wait timeouts in the workspace
    if (BH > value_sync_slots()) return MA_ERR_UNSUPPORTED;
    if (!workspace || workspace_bytes < value_score_ws_bytes(q->B, H, n, q->D)) return MA_ERR_WORKSPACE;
    if ((reinterpret_cast<uintptr_t>(workspace) & 255) != 0) return MA_ERR_WORKSPACE;
    w = carve_value_ws(workspace, BH, q->D);
  }
  cudaStream_t st = (cudaStream_t)stream;
  if (tc) {
    bool fused = false;
    rc = MA_ERR_UNSUPPORTED;
    if (!fa_disabled())   // TMA-fed dense bf16 cache: the pipelined kernel
      rc = launch_prefix_mass_fa(*q, *kv, H, q_rows, T2, m_p, l_p, scale, mass, smass[0], smass[1], score,
                                 score ? sscore[0] : 0, score ? sscore[1] : 0, w, score != nullptr, &fused, st);
    if (rc == MA_ERR_UNSUPPORTED)
      rc = launch_prefix_mass_tc(*q, *kv, H, q_rows, T2, m_p, l_p, scale, mass, smass[0], smass[1], score,
                                 score ? sscore[0] : 0, score ? sscore[1] : 0, w, score != nullptr, &fused, st);
    if (rc || !score || fused) return rc;
    return launch_value_apply(*kv, q->B, H, q->D, mass, smass[0], smass[1], w.centre, score, sscore[0],
                              sscore[1], st);
  }
  rc = launch_prefix_mass(*q, *kv, H, q_rows, T2, m_p, l_p, scale, mass, smass[0], smass[1], st);
  if (rc || !score) return rc;
  return launch_value_score(*kv, q->B, H, q->D, mass, smass[0], smass[1], score, sscore[0], sscore[1], workspace,
                            st);
}

size_t ma_value_score_workspace(int B, int H, int n, int D) {
  if (B <= 0 || H <= 0 || n < 0 || D <= 0) return 0;
  return value_score_ws_bytes(B, H, n, D);
}

int ma_value_score(const ma_kv* kv, int B, int H, int D, const float* a, const int64_t sa[2],
                   float* score, const int64_t sscore[2], void* workspace, size_t workspace_bytes,
                   void* stream) {
  if (B <= 0 || H <= 0) return MA_ERR_ARG;
  if (D != 64 && D != 128) return MA_ERR_UNSUPPORTED;
  int rc = check_kv(kv, D);
  if (rc) return rc;
  if (!a || !sa || !score || !sscore) return MA_ERR_ARG;
  const int n = kv->nq + kv->nf;
  if ((int64_t)B * H > value_sync_slots()) return MA_ERR_UNSUPPORTED;
  if (!workspace || workspace_bytes < value_score_ws_bytes(B, H, n, D)) return MA_ERR_WORKSPACE;
  if ((reinterpret_cast<uintptr_t>(workspace) & 255) != 0) return MA_ERR_WORKSPACE;
  if (!fa_disabled()) {
    rc = launch_value_score_fa(*kv, B, H, D, a, sa[0], sa[1], score, sscore[0], sscore[1], workspace,
                               (cudaStream_t)stream);
    if (rc != MA_ERR_UNSUPPORTED) return rc;
  }
  return launch_value_score(*kv, B, H, D, a, sa[0], sa[1], score, sscore[0], sscore[1], workspace,
                            (cudaStream_t)stream);
}

int ma_select_topk(const float* score, int B, int H, int n, const int64_t sscore[2], const uint8_t* mask,
                   const int32_t* lens, int k, int64_t* indices, float* values, const int64_t sidx[2],
                   void* stream) {
  if (!score || !sscore || !indices || !sidx || B <= 0 || H <= 0 || n <= 0) return MA_ERR_ARG;
  if (k < 0 || k > n) return MA_ERR_ARG;
  if (k == 0) return MA_OK;
  return launch_select_topk(score, B, H, n, sscore[0], sscore[1], mask, lens, k, indices, values, sidx[0],
                            sidx[1], (cudaStream_t)stream);
}

int ma_quantize_tokens(const void* x, int32_t dtype, int B, int H, int n, int D, const int64_t sx[3],
                       const float* kchan, const int64_t skc[2], int group, uint8_t* payload, const int64_t sp[3],
                       uint16_t* scale, uint16_t* zero, const int64_t ss[3], void* stream) {
  if (!x || !payload || !scale || !zero || !sx || !sp || !ss || B < 0 || H < 0 || n < 0 || D <= 0) return MA_ERR_ARG;
  if (!valid_dtype(dtype)) return MA_ERR_ARG;
  if (group != 32 || D % 32 != 0) return MA_ERR_UNSUPPORTED;
  if (kchan && (!skc || skc[0] < 0 || skc[1] < 0)) return MA_ERR_ARG;
  if ((reinterpret_cast<uintptr_t>(payload) & 15) != 0 || !strides16(sp, 3, 1)) return MA_ERR_ARG;
  if ((reinterpret_cast<uintptr_t>(x) & (esize(dtype) - 1)) != 0) return MA_ERR_ARG;
  for (int i = 0; i < 3; ++i)
    if (sx[i] < 0 || ss[i] < 0) return MA_ERR_ARG;
  return launch_quantize_tokens(x, dtype, B, H, n, D, sx, kchan, skc, payload, sp, scale, zero, ss,
                                (cudaStream_t)stream);
}

int ma_quantize_keys_channel(const void* k, int32_t dtype, int B, int H, int n, int D, const int64_t sk[3], int group,
                             uint8_t* payload, const int64_t sp[3], uint16_t* scale, uint16_t* zero,
                             const int64_t ss[3], void* stream) {
  if (!k || !payload || !scale || !zero || !sk || !sp || !ss || B < 0 || H < 0 || n < 0 || D <= 0) return MA_ERR_ARG;
  if (!valid_dtype(dtype)) return MA_ERR_ARG;
  if (group != 32) return MA_ERR_UNSUPPORTED;
  if (n % 32 != 0) return MA_ERR_ARG;
  if ((reinterpret_cast<uintptr_t>(payload) & 15) != 0 || !strides16(sp, 3, 1)) return MA_ERR_ARG;
  if ((reinterpret_cast<uintptr_t>(k) & (esize(dtype) - 1)) != 0) return MA_ERR_ARG;
  for (int i = 0; i < 3; ++i)
    if (sk[i] < 0 || ss[i] < 0) return MA_ERR_ARG;
  return launch_quantize_channels(k, dtype, B, H, n, D, sk, payload, sp, scale, zero, ss, (cudaStream_t)stream);
}

int ma_key_divisor(const void* k, int32_t dtype, int B, int H, int n, int D, const int64_t sk[3], float* kchan,
                   const int64_t skc[2], void* stream) {
  if (!k || !kchan || !sk || !skc || B < 0 || H < 0 || n < 0 || D <= 0) return MA_ERR_ARG;
  if (!valid_dtype(dtype)) return MA_ERR_ARG;
  if (D > kMaxD) return MA_ERR_UNSUPPORTED;
  for (int i = 0; i < 3; ++i)
    if (sk[i] < 0) return MA_ERR_ARG;
  if (skc[0] < 0 || skc[1] < 0) return MA_ERR_ARG;
  return launch_key_divisor(k, dtype, B, H, n, D, sk, kchan, skc, (cudaStream_t)stream);
}

int ma_retain(const float* score, const int32_t* phys, int n_phys, const int32_t* pos, int lanes, int live,
              int capacity, int recent_window, int sink_tokens, int64_t* keep, void* stream) {
  if (!score || !pos || !keep || lanes <= 0 || live <= 0) return MA_ERR_ARG;
  if (capacity <= 0 || capacity > live || recent_window < 0 || sink_tokens < 0) return MA_ERR_ARG;
  if (phys && n_phys <= 0) return MA_ERR_ARG;
  if (capacity > 16384 || live > 65536) return MA_ERR_UNSUPPORTED;
  return launch_retain(score, phys, n_phys, pos, lanes, live, capacity, recent_window, sink_tokens, keep,
                       (cudaStream_t)stream);
}

size_t ma_sparse_attention_workspace(int B, int H, int R, int k, int D, int Tc) {
  if (B <= 0 || H <= 0 || R <= 0 || k < 0 || D <= 0 || Tc < 0) return 0;
  return attention_ws(B, H, R, k, D, Tc);
}

int ma_sparse_attention(const ma_rows* q, const ma_kv* kv, int H, const int64_t* idx, int k,
                        const int64_t sidx[2], const ma_block* cur, float scale, void* out,
                        const int64_t so[3], void* workspace, size_t workspace_bytes, void* stream) {
  int rc = check_rows(q);
  if (rc) return rc;
  if (H <= 0 || q->Hq % H) return MA_ERR_ARG;
  if ((rc = check_kv(kv, q->D))) return rc;
  if ((rc = check_block(cur, q, H))) return rc;
  if (k < 0 || (k > 0 && (!idx || !sidx))) return MA_ERR_ARG;
  if (k == 0 && cur->Tc == 0) return MA_ERR_ARG;
  if (!out || !so || !aligned16(out) || !strides16(so, 3, esize(q->dtype))) return MA_ERR_ARG;
  return run_attention(*q, *kv, H, *cur, scale, 0, 0, 0, idx, k ? sidx[0] : 0, k ? sidx[1] : 0, k, out,
                       so, nullptr, nullptr, nullptr, workspace, workspace_bytes, (cudaStream_t)stream);
}

int ma_gather_kv(const ma_kv* kv, int B, int H, int D, const int64_t* idx, int k, const int64_t sidx[2],
                 void* out_k, void* out_v, const int64_t sok[3], const int64_t sov[3], int32_t out_dtype,
                 void* stream) {
  if (B <= 0 || H <= 0 || k < 0) return MA_ERR_ARG;
  if (D != 64 && D != 128) return MA_ERR_UNSUPPORTED;
  int rc = check_kv(kv, D);
  if (rc) return rc;
  if (!valid_dtype(out_dtype)) return MA_ERR_ARG;
  if (k > 0 && ((idx && !sidx) || !out_k || !out_v || !sok || !sov)) return MA_ERR_ARG;
  if (k > 0 && (!aligned16(out_k) || !aligned16(out_v) || !strides16(sok, 3, esize(out_dtype)) ||
                !strides16(sov, 3, esize(out_dtype))))
    return MA_ERR_ARG;
  return launch_gather_kv(*kv, B, H, D, idx, k, (k && idx) ? sidx[0] : 0, (k && idx) ? sidx[1] : 0, out_k, out_v, sok, sov,
                          out_dtype, (cudaStream_t)stream);
}

int ma_unpack_prefix(const ma_kv* kv, int B, int H, int D, void* out_k, void* out_v, const int64_t sok[3],
                     const int64_t sov[3], void* stream) {
  if (B <= 0 || H <= 0) return MA_ERR_ARG;
  if (D != 128) return MA_ERR_UNSUPPORTED;
  int rc = check_kv(kv, D);
  if (rc) return rc;
  if (!out_k || !out_v || !sok || !sov) return MA_ERR_ARG;
  if (!aligned16(out_k) || !aligned16(out_v) || !strides16(sok, 3, 2) || !strides16(sov, 3, 2)) return MA_ERR_ARG;
  return launch_unpack_live(*kv, B, H, D, out_k, out_v, sok, sov, (cudaStream_t)stream);
}

namespace {

// largest power-of-two vector (<= 16 bytes) that divides the row, both bases and every stride
int compact_vec(const void* src, const void* dst, int row_bytes, const int64_t ss[3], const int64_t ds[3]) {
  uint64_t bits = (uint64_t)row_bytes | reinterpret_cast<uintptr_t>(src) | reinterpret_cast<uintptr_t>(dst);
  for (int i = 0; i < 3; ++i) bits |= (uint64_t)ss[i] | (uint64_t)ds[i];
  int v = 16;
  while (v > 1 && (bits & (uint64_t)(v - 1))) v >>= 1;
  return v;
}

// appends one array (element strides es/ed of an element of `elem` bytes) to the plan
int compact_add(CompactParams& p, const void* src, const void* dst, const int64_t es[3], const int64_t ed[3],
                int elem, int row_bytes) {
  if (!src || !dst) return MA_ERR_ARG;
  if (src == dst) return MA_ERR_ARG;   // out of place only
  CompactArray& a = p.arrays[p.narrays++];
  a.src = static_cast<const unsigned char*>(src);
  a.dst = static_cast<unsigned char*>(const_cast<void*>(dst));
  for (int i = 0; i < 3; ++i) {
    if (es[i] < 0 || ed[i] < 0) return MA_ERR_ARG;
    a.ss[i] = es[i] * elem;
    a.ds[i] = ed[i] * elem;
  }
  if (a.ds[2] < row_bytes) return MA_ERR_ARG;   // destination rows must not overlap
  a.row_bytes = row_bytes;
  a.vec_bytes = compact_vec(src, dst, row_bytes, a.ss, a.ds);
  return MA_OK;
}

}  // namespace

int ma_compact_tokens(const ma_kv* src, const ma_kv* dst, int B, int H, int D, const int64_t* keep, int C,
                      const int64_t skeep[2], void* stream) {
  if (B <= 0 || H <= 0 || C < 0 || !src || !dst) return MA_ERR_ARG;
  if (D != 64 && D != 128) return MA_ERR_UNSUPPORTED;
  int rc = check_kv(src, D);
  if (rc) return rc;
  if (src->pages || dst->pages) return MA_ERR_UNSUPPORTED;
  if (dst->layout != src->layout || dst->dtype != src->dtype) return MA_ERR_ARG;
  CompactParams p{};
  p.H = H;
  p.C = C;
  if (src->layout == MA_KV_DENSE) {
    p.n = src->nf;
    if (C > src->nf || C > dst->nf) return MA_ERR_ARG;
    if (C == 0) return MA_OK;
    const int row = D * esize(src->dtype);
    if ((rc = compact_add(p, src->kf, dst->kf, src->skf, dst->skf, esize(src->dtype), row))) return rc;
    if ((rc = compact_add(p, src->vf, dst->vf, src->svf, dst->svf, esize(src->dtype), row))) return rc;
  } else if (src->layout == MA_KV_PACKED_CHANNEL) {
    // whole key groups: keep indexes groups of kgroup tokens; a group's key payload and
    // scale/zero rows move with its kgroup value slots, which must be packed back to back
    // so that they form one row (the group copy of cache.py:236-335 rebuild). The dense
    // tail is not touched.
    if (dst->vgroup != src->vgroup || dst->kgroup != src->kgroup) return MA_ERR_ARG;
    const int kg = src->kgroup, groups = D / src->vgroup;
    if (src->svq[2] != D / 2 || dst->svq[2] != D / 2 || src->svs[2] != groups || dst->svs[2] != groups)
      return MA_ERR_UNSUPPORTED;
    p.n = src->nq / kg;
    if ((int64_t)C * kg > src->nq || (int64_t)C * kg > dst->nq) return MA_ERR_ARG;
    if (C == 0) return MA_OK;
    const int64_t svq_s[3] = {src->svq[0], src->svq[1], src->svq[2] * kg};
    const int64_t svq_d[3] = {dst->svq[0], dst->svq[1], dst->svq[2] * kg};
    const int64_t svs_s[3] = {src->svs[0], src->svs[1], src->svs[2] * kg};
    const int64_t svs_d[3] = {dst->svs[0], dst->svs[1], dst->svs[2] * kg};
    if ((rc = compact_add(p, src->kq, dst->kq, src->skq, dst->skq, 1, D * kg / 2))) return rc;
    if ((rc = compact_add(p, src->ks, dst->ks, src->sks, dst->sks, 2, D * 2))) return rc;
    if ((rc = compact_add(p, src->kz, dst->kz, src->sks, dst->sks, 2, D * 2))) return rc;
    if ((rc = compact_add(p, src->vq, dst->vq, svq_s, svq_d, 1, kg * D / 2))) return rc;
    if ((rc = compact_add(p, src->vs, dst->vs, svs_s, svs_d, 2, kg * groups * 2))) return rc;
    if ((rc = compact_add(p, src->vz, dst->vz, svs_s, svs_d, 2, kg * groups * 2))) return rc;
  } else {
    // per-token codes only: a dense tail must have been quantized first (cache.py:662-663)
    if (src->nf != 0) return MA_ERR_UNSUPPORTED;
    if (dst->vgroup != src->vgroup) return MA_ERR_ARG;
    p.n = src->nq;
    if (C > src->nq || C > dst->nq) return MA_ERR_ARG;
    if (C == 0) return MA_OK;
    const int groups = D / src->vgroup;
    if ((rc = compact_add(p, src->kq, dst->kq, src->skq, dst->skq, 1, D / 2))) return rc;
    if ((rc = compact_add(p, src->ks, dst->ks, src->sks, dst->sks, 2, groups * 2))) return rc;
    if ((rc = compact_add(p, src->kz, dst->kz, src->sks, dst->sks, 2, groups * 2))) return rc;
    if ((rc = compact_add(p, src->vq, dst->vq, src->svq, dst->svq, 1, D / 2))) return rc;
    if ((rc = compact_add(p, src->vs, dst->vs, src->svs, dst->svs, 2, groups * 2))) return rc;
    if ((rc = compact_add(p, src->vz, dst->vz, src->svs, dst->svs, 2, groups * 2))) return rc;
  }
  if (!keep || !skeep || skeep[0] < 0 || skeep[1] < 0) return MA_ERR_ARG;
  p.keep = keep;
  p.sk0 = skeep[0];
  p.sk1 = skeep[1];
  return launch_compact(p, B, (cudaStream_t)stream);
}

int ma_evict_plan(const int32_t* phys, const int64_t* pos, int lanes, int live, const int64_t sphys_spos[2],
                  int quantized_length, int kgroup, int need, int tail_groups, int recent_window,
                  int64_t* groups_before, int64_t* encode, int64_t* stage, int32_t* counts, int32_t* maxes,
                  void* stream) {
  if (lanes < 0 || live < 0 || quantized_length < 0 || kgroup <= 0 || need < 0 || tail_groups < 0 ||
      recent_window < 0 || !sphys_spos || !maxes)
    return MA_ERR_ARG;
  const int ng = quantized_length / kgroup > 1 ? quantized_length / kgroup : 1;
  if (ng > kEvictMaxGroups || tail_groups > ng) return MA_ERR_UNSUPPORTED;
  if (lanes > 0 && live > 0 && (!phys || !pos || !groups_before || !encode || !stage || !counts)) return MA_ERR_ARG;
  if (lanes > 0 && (!groups_before || !counts)) return MA_ERR_ARG;
  if (sphys_spos[0] < live || sphys_spos[1] < live) return MA_ERR_ARG;
  EvictPlanParams p{phys, pos, sphys_spos[0], sphys_spos[1], live, quantized_length, kgroup, need, tail_groups,
                    recent_window, groups_before, encode, stage, counts, maxes};
  return launch_evict_plan(p, lanes, (cudaStream_t)stream);
}

int ma_rebuild_remap(int B, int H, int old_len, int kgroup, const int64_t* groups_before, int g1,
                     const int64_t* encode, int m, const int64_t* groups_after, int g3, const int64_t* stage, int st,
                     int64_t* remap, void* stream) {
  if (B <= 0 || H <= 0 || old_len < 0 || kgroup <= 0 || g1 < 0 || m < 0 || g3 < 0 || st < 0) return MA_ERR_ARG;
  if ((g1 && !groups_before) || (m && !encode) || (g3 && !groups_after) || (st && !stage)) return MA_ERR_ARG;
  if (old_len > 0 && !remap) return MA_ERR_ARG;
  const int64_t g2 = ((int64_t)m + kgroup - 1) / kgroup;
  const int64_t ql = ((int64_t)g1 + g2 + g3) * kgroup;
  if (ql + st > 0x7fffffffLL) return MA_ERR_ARG;
  const int64_t lanes = (int64_t)B * H;   // one CTA per lane: the grid's x extent
  if (lanes > 0x7fffffffLL) return MA_ERR_UNSUPPORTED;
  RemapParams p{groups_before, encode, groups_after, stage, remap, g1, (int)g2, g3, m, st, kgroup, old_len, (int)ql};
  return launch_rebuild_remap(p, (int)lanes, (cudaStream_t)stream);
}

// ------------------------------------------------------------------ KV-head sharding
size_t ma_head_gather_region_bytes(int B, int Hq, int T) {
  if (B <= 0 || Hq <= 0 || T <= 0) return 0;
  return ma::head_gather_region_bytes(B, Hq, T);
}

size_t ma_head_gather_workspace(void) { return 512; }

int ma_peer_alloc(size_t bytes, void** ptr) {
  if (!ptr || bytes == 0) return MA_ERR_ARG;
  *ptr = nullptr;
  void* p = nullptr;
  if (cudaMalloc(&p, bytes) != cudaSuccess) return MA_ERR_CUDA;
  if (cudaMemset(p, 0, bytes) != cudaSuccess) {
    cudaFree(p);
    return MA_ERR_CUDA;
  }
  *ptr = p;
  return MA_OK;
}

int ma_peer_free(void* ptr) { return cudaFree(ptr) == cudaSuccess ? MA_OK : MA_ERR_CUDA; }

size_t ma_ipc_handle_bytes(void) { return sizeof(cudaIpcMemHandle_t); }

int ma_ipc_get_handle(void* ptr, void* handle) {
  if (!ptr || !handle) return MA_ERR_ARG;
  cudaIpcMemHandle_t h;
  if (cudaIpcGetMemHandle(&h, ptr) != cudaSuccess) return MA_ERR_CUDA;
  memcpy(handle, &h, sizeof(h));
  return MA_OK;
}

int ma_ipc_open_handle(const void* handle, void** ptr) {
  if (!handle || !ptr) return MA_ERR_ARG;
  cudaIpcMemHandle_t h;
  memcpy(&h, handle, sizeof(h));
  *ptr = nullptr;
  return cudaIpcOpenMemHandle(ptr, h, cudaIpcMemLazyEnablePeerAccess) == cudaSuccess ? MA_OK : MA_ERR_CUDA;
}

int ma_ipc_close_handle(void* ptr) { return cudaIpcCloseMemHandle(ptr) == cudaSuccess ? MA_OK : MA_ERR_CUDA; }

int ma_head_gather(const void* part, const int64_t sp[3], int B, int Hl, int T, int D, int world, int rank,
                   void* const* regions, void* out, const int64_t so[3], void* workspace, size_t workspace_bytes,
                   void* stream) {
  if (!part || !sp || !regions || !out || !so) return MA_ERR_ARG;
  if (D != 128) return MA_ERR_UNSUPPORTED;
  if (!workspace || workspace_bytes < ma_head_gather_workspace()) return MA_ERR_WORKSPACE;
  if (!aligned16(part) || !aligned16(out) || !strides16(sp, 3, 2) || !strides16(so, 3, 2)) return MA_ERR_ARG;
  return ma::launch_head_gather(part, sp, B, Hl, T, world, rank, regions, out, so, workspace, peer_wait_ns(),
                                (cudaStream_t)stream);
}

}  // extern "C"
