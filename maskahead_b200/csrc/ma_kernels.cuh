// Internal launcher declarations shared by the kernel translation units and the C ABI.
#pragma once

#include "ma_common.cuh"

namespace ma {

// ma_attention_simt.cu
int launch_attn_partial_simt(const ma_rows& q, const ma_kv& kv, int H, const ma_block& cur,
                             float scale, int causal_block, int q_pos0, int c_pos0,
                             const int64_t* idx, int64_t si0, int64_t si1, int n_keys,
                             int split_len, int nsplit, const Partials& P, cudaStream_t st);
int simt_row_block();
int simt_key_tile();

// ma_attention_tc.cu (bf16 queries and caches, tcgen05 / TMEM)
// The merge of the splits fused into the same (cooperative) launch: every split CTA of a
// (head, row block) arrives on sync[group].x, the last advances sync[group].y, and each
// CTA then merges its share of the group's rows into out / m_p / l_p / o_p.
struct FusedMerge {
  void* out;
  int64_t so[3];
  float* m_p;
  float* l_p;
  float* o_p;
  uint2* sync;      // [B*H*row blocks], zero counters between calls
  int sync_slots;   // capacity of sync
  uint64_t wait_ns; // bound on a CTA's wait for the other splits of its group
  int gather;       // the merge also runs the head gather `po` (cooperative launch only)
  PeerOut po;
};
// The bound on every wait of one CTA for other CTAs of the same launch (the split merge's
// and the value-score centre's generation words); ma_set_peer_wait_ns. The waits on a
// CTA's own asynchronous copies and MMAs keep their fixed bounds.
uint64_t peer_wait_ns();
// Returns MA_OK with *fused = true when the merge ran inside the launch (the caller
// then skips launch_attn_combine).
int launch_attn_partial_tc(const ma_rows& q, const ma_kv& kv, int H, const ma_block& cur, float scale,
                           int causal_block, int q_pos0, int c_pos0, const int64_t* idx, int64_t si0, int64_t si1,
                           int n_keys, int split_len, int nsplit, const Partials& P, int* err, const FusedMerge* fm,
                           bool* fused, cudaStream_t st);
int tc_row_tile();
int tc_key_tile();

// ma_attention_fa.cu (TMA-fed bf16: the dense prefix without a read set, mask or paging,
// and the current block; 128-row x 128-key tiles, S double-buffered and P in tensor
// memory). split_len must be a multiple of fa_key_tile() and the plan's row blocks are
// fa_row_tile(R, B*H) rows (128, or 256 when a CTA takes a pair of M tiles);
// MA_ERR_UNSUPPORTED when the call is not TMA-eligible (the caller then uses
// launch_attn_partial_tc). fa_set_pairs: 0 = automatic, 1 = one M tile per CTA, 2 = pairs
// whenever R > 128.
bool fa_eligible(const ma_rows& q, const ma_kv& kv, const int64_t* idx, const ma_block& cur, int n_keys);
int fa_key_tile();
int fa_row_tile(int R, int BH);
void fa_set_pairs(int mode);
// the mass kernel's CTAs over a ragged batch: at most `tiles` 128-slot tiles each (0: the
// automatic policy, < 0: no cap)
void fa_set_mass_tiles(int tiles);
int fa_mass_tiles();
int launch_attn_partial_fa(const ma_rows& q, const ma_kv& kv, int H, const ma_block& cur, float scale,
                           int causal_block, int q_pos0, int c_pos0, int n_keys, int split_len, int nsplit,
                           const Partials& P, int* err, const FusedMerge* fm, bool fold, bool* fused,
                           bool* gathered, cudaStream_t st);

// ma_combine.cu
int launch_attn_combine(const ma_rows& q, int H, const Partials& P, int nsplit, bool has_cur,
                        void* out, const int64_t so[3], float* m_p, float* l_p, float* o_p,
                        cudaStream_t st);

// ma_score.cu
int launch_prefix_mass(const ma_rows& q, const ma_kv& kv, int H, const int32_t* q_rows, int T2,
                       const float* m_p, const float* l_p, float scale, float* mass,
                       int64_t sm0, int64_t sm1, cudaStream_t st);
size_t value_score_ws_bytes(int B, int H, int n, int D);
// The sync block's layout does not depend on B*H, so a workspace shared by calls of
// different sizes never reads one call's words as another's counters.
struct ValueWs {
  int* err;            // device-side error word (a bounded wait gave up)
  uint2* sync;         // [BH]: x = arrival counter (zero between calls), y = centre generation
  float* centre;       // [BH][D]
  float* part;         // [BH][tiles][D+1]
};
size_t value_sync_bytes(int BH);
int value_sync_slots();   // the most heads (B * H) one call may have
ValueWs carve_value_ws(void* ws, int BH, int D);
int launch_value_apply(const ma_kv& kv, int B, int H, int D, const float* a, int64_t sa0, int64_t sa1,
                       const float* centre, float* score, int64_t ss0, int64_t ss1, cudaStream_t st);
int launch_value_score(const ma_kv& kv, int B, int H, int D, const float* a, int64_t sa0,
                       int64_t sa1, float* score, int64_t ss0, int64_t ss1, void* ws,
                       cudaStream_t st);

// ma_mass_tc.cu (bf16, R2 = G*T2 <= 256): mass, optionally the value-score centre
// With score != NULL the value score a_j ||v_j - c|| is computed in the same (cooperative)
// launch; *fused reports whether it was (else the caller runs launch_value_apply).
int launch_prefix_mass_tc(const ma_rows& q, const ma_kv& kv, int H, const int32_t* q_rows, int T2, const float* m_p,
                          const float* l_p, float scale, float* mass, int64_t sm0, int64_t sm1, float* score,
                          int64_t ss0, int64_t ss1, const ValueWs& w, bool want_centre, bool* fused, cudaStream_t st);

// ma_mass_fa.cu (TMA-fed dense bf16 cache without paging or a packed part): the same
// contract as launch_prefix_mass_tc; MA_ERR_UNSUPPORTED when the cache is not eligible.
int launch_prefix_mass_fa(const ma_rows& q, const ma_kv& kv, int H, const int32_t* q_rows, int T2, const float* m_p,
                          const float* l_p, float scale, float* mass, int64_t sm0, int64_t sm1, float* score,
                          int64_t ss0, int64_t ss1, const ValueWs& w, bool want_centre, bool* fused, cudaStream_t st);

// a_j ||v_j - c|| from given a_j over a TMA-fed dense bf16 V (the value pass of
// prefix_mass_fa); MA_ERR_UNSUPPORTED when V or the launch does not qualify.
int launch_value_score_fa(const ma_kv& kv, int B, int H, int D, const float* a, int64_t sa0, int64_t sa1,
                          float* score, int64_t ss0, int64_t ss1, void* ws, cudaStream_t st);

// ma_select.cu
int launch_select_topk(const float* score, int B, int H, int n, int64_t ss0, int64_t ss1,
                       const uint8_t* mask, const int32_t* lens, int k, int64_t* indices, float* values,
                       int64_t si0, int64_t si1, cudaStream_t st);

// ma_quant.cu
int launch_quantize_tokens(const void* x, int dtype, int B, int H, int n, int D, const int64_t sx[3], const float* kchan,
                           const int64_t skc[2], uint8_t* payload, const int64_t sp[3], uint16_t* scale, uint16_t* zero,
                           const int64_t ss[3], cudaStream_t st);
int launch_quantize_channels(const void* x, int dtype, int B, int H, int n, int D, const int64_t sx[3],
                             uint8_t* payload, const int64_t sp[3], uint16_t* scale, uint16_t* zero, const int64_t ss[3],
                             cudaStream_t st);
int launch_key_divisor(const void* k, int dtype, int B, int H, int n, int D, const int64_t sk[3], float* kchan,
                       const int64_t skc[2], cudaStream_t st);
int launch_retain(const float* score, const int32_t* phys, int n_phys, const int32_t* pos,
                  int lanes, int live, int capacity, int recent_window, int sink_tokens,
                  int64_t* keep, cudaStream_t st);
// every slot below lens[b] (all nq + nf without lens) of a token-mode packed prefix into
// contiguous bf16 rows; slots at or past lens[b] are not written
int launch_unpack_live(const ma_kv& kv, int B, int H, int D, void* out_k, void* out_v, const int64_t sok[3],
                       const int64_t sov[3], cudaStream_t st);
int launch_gather_kv(const ma_kv& kv, int B, int H, int D, const int64_t* idx, int k, int64_t si0,
                     int64_t si1, void* out_k, void* out_v, const int64_t sok[3],
                     const int64_t sov[3], int out_dtype, cudaStream_t st);

// ma_compact.cu: one array of a cache layout moved by the compaction, byte strides over
// (b, h, slot); vec_bytes divides row_bytes, both bases and every stride
struct CompactArray {
  const unsigned char* src;
  unsigned char* dst;
  int64_t ss[3];
  int64_t ds[3];
  int row_bytes;
  int vec_bytes;
  int slots_per_block;   // set by launch_compact
  int chunks;            // set by launch_compact
};
constexpr int kCompactMaxArrays = 6;
struct CompactParams {
  CompactArray arrays[kCompactMaxArrays];
  int narrays;
  const int64_t* keep;   // [B, H, C], strides sk0, sk1 over (b, h), slot axis contiguous
  int64_t sk0, sk1;
  int H, C;
  int64_t n;             // source slots: a keep index outside [0, n) writes a zero row
  int chunks;            // set by launch_compact: the most blocks any array needs per lane
};
int launch_compact(CompactParams& p, int B, cudaStream_t st);
// the remap of a group-preserving rebuild; index lists contiguous [lanes][count]
struct RemapParams {
  const int64_t* gb;
  const int64_t* enc;
  const int64_t* ga;
  const int64_t* stg;
  int64_t* remap;        // [lanes][old_len]
  int g1, g2, g3, m, st, kgroup, old_len, ql;
};
int launch_rebuild_remap(const RemapParams& p, int lanes, cudaStream_t st);
// The index lists of a group-preserving rebuild after an eviction (ma_evict_plan).
struct EvictPlanParams {
  const int32_t* phys;   // [lanes][live] physical slot of each live entry
  const int64_t* pos;    // [lanes][live] its position (increasing along the live axis)
  int64_t sphys, spos;   // lane strides
  int live, ql, kgroup, need, tail_groups, recent_window;
  int64_t* groups_before;   // [lanes][ng]
  int64_t* encode;          // [lanes][live]
  int64_t* stage;           // [lanes][live]
  int32_t* counts;          // [lanes][3]
  int32_t* maxes;           // [4]: the three maxima over lanes, lanes out of position order
};
constexpr int kEvictMaxGroups = 8192;
int launch_evict_plan(const EvictPlanParams& p, int lanes, cudaStream_t st);

// ma_peer.cu: KV-head sharding's exchange of head outputs by peer stores
size_t head_gather_region_bytes(int B, int Hq, int T);
int launch_head_gather(const void* part, const int64_t sp[3], int B, int Hl, int T, int world, int rank,
                       void* const* regions, void* out, const int64_t so[3], void* ws, uint64_t wait_ns,
                       cudaStream_t st);

// device properties, cached per device
int device_sm_count();

}  // namespace ma
