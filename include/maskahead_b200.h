/*
 * maskahead_b200 -- C ABI of the B200 (sm_100a) select + attend hot path.
 *
 * Every entry point takes plain device pointers, element strides and sizes, enqueues
 * its kernels on the given CUDA stream (cudaStream_t passed as void*, NULL = legacy
 * default stream), never synchronizes (the status queries ma_workspace_status and
 * ma_value_score_noalloc_status excepted), never allocates device memory, and returns an
 * int status: MA_OK (0) or a negative MA_ERR_* code. Arguments are validated on the
 * host before anything is launched; a rejected call launches nothing. Scratch memory
 * is caller-provided ("workspace") and sized by the matching *_workspace() function;
 * a workspace must be zero-filled once when it is allocated (kernels leave it ready
 * for the next call) and must not be shared by calls that can overlap on the GPU.
 *
 * Device-side failures: every wait of a kernel is bounded. A wait that gives up records
 * it in the error word of the call's workspace and the rows it could not finish are
 * written as NaN; the status of the call itself (MA_OK) only covers the host-side checks
 * and the launch. ma_workspace_status reads (and clears) that error word and returns
 * MA_ERR_TIMEOUT when it is set.
 *
 * Conventions
 *   query rows:  Q [B, Hq, T, D], Hq = G * H (GQA); the R = G*T rows of KV head h are
 *                r = g*T + t for query head h*G + g and block position t.
 *   prefix:      described by ma_kv (layout, strides, optional live-slot mask).
 *   strides:     in ELEMENTS of the tensor's own type; the innermost dimension is
 *                contiguous unless stated otherwise.
 *   D:           head_dim, 64 or 128.
 *
 * The entry points replace the reference package's operator bodies (file:line within
 * brain-lab-research/MaskAhead, src/maskahead/):
 *   ma_prefix_attention  kernels/splitk.py:493-579 (splitk_attention) and
 *                        kernels/ops.py:130-264, 766-787 (dense_packed_attention)
 *   ma_prefix_scores     kernels/splitk.py:582-614 (prefix_scores) and
 *                        kernels/ops.py:333-521 (selector_topk importance)
 *   ma_value_score       runtime/session.py:27-40 (value_score) and 870-954
 *                        (_rescore_by_value, value_center="attn")
 *   ma_select_topk       kernels/ops.py:377-380, 509-516; runtime/session.py:1434-1438
 *   ma_retain            eviction.py:325-409 (EvictionState.survivors, lookahead)
 *   ma_sparse_attention  runtime/session.py:1286-1336 + reference.py:403-426
 *                        (_compact_attention -> sdpa_compact over the read set)
 *   ma_gather_kv         kernels/ops.py:570-662, 835-855 (gather_packed_kv)
 *   ma_quantize_tokens, ma_quantize_keys_channel, ma_key_divisor
 *                        reference.py:58-90, 182-213 and cache.py:484-497 (the packing
 *                        of the append path)
 *   ma_compact_tokens    cache.py:659-678 (compact_tokens) and 342-365 (compact): the
 *                        cache compaction after an eviction (runtime/session.py:270-302)
 *   ma_rebuild_remap     cache.py:236-335 (the remap of rebuild)
 *   ma_evict_plan        runtime/session.py:303-356 (_evict_to: the rebuild's index lists)
 */
#ifndef MASKAHEAD_B200_H
#define MASKAHEAD_B200_H

#include <stddef.h>
#include <stdint.h>

#if defined(__GNUC__)
#define MA_API __attribute__((visibility("default")))
#else
#define MA_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

/* ---- status codes ---------------------------------------------------------------- */
#define MA_OK 0
#define MA_ERR_ARG (-1)          /* invalid shape, stride, pointer or parameter        */
#define MA_ERR_UNSUPPORTED (-2)  /* valid request outside what the kernels implement   */
#define MA_ERR_WORKSPACE (-3)    /* workspace missing or smaller than *_workspace()     */
#define MA_ERR_CUDA (-4)         /* a CUDA runtime call or launch failed                */
#define MA_ERR_TIMEOUT (-5)      /* a bounded device-side wait gave up                  */

/* ---- element types ----------------------------------------------------------------- */
#define MA_F32 0
#define MA_BF16 1
#define MA_F16 2

/* ---- KV layouts -------------------------------------------------------------------- */
/* Dense: K/V [B,H,n,D] in `dtype` (fp32 or bf16) -- LayerCacheView k_fp/v_fp
 * (cache.py:142-143). */
#define MA_KV_DENSE 0
/* Packed, token-mode keys: the first nq slots hold 4-bit codes of every token over
 * channel groups of vgroup (payload [.., D/vgroup, vgroup/2] u8, fp16 scale/zero
 * [.., D/vgroup]) for both K and V; keys are multiplied by the per-channel divisor
 * kchan [B,H,D] fp32 after dequantization; slots nq..nq+nf-1 are a `dtype` tail
 * (cache.py:146-152, 172-189; splitk.py:389-395). */
#define MA_KV_PACKED_TOKEN 1
/* Packed, KIVI channel-mode keys: key payload [B,H,ng,D,kgroup/2] u8 and fp16
 * scale/zero [B,H,ng,D] per group of kgroup tokens; values as in the token layout
 * (cache.py:154-169). */
#define MA_KV_PACKED_CHANNEL 2

typedef struct ma_kv {
  int32_t layout;        /* MA_KV_*                                                   */
  int32_t dtype;         /* element type of dense K/V and of the tail: MA_F32/MA_BF16  */
  int32_t nq;            /* packed slots (0 for MA_KV_DENSE)                           */
  int32_t nf;            /* dense / tail slots after them (all n for MA_KV_DENSE)      */
  int32_t kgroup;        /* channel-mode key token group (32)                          */
  int32_t vgroup;        /* value (and token-mode key) channel group (32)              */
  /* dense K/V or the tail: strides over (b, h, slot), D contiguous                    */
  const void* kf;
  const void* vf;
  int64_t skf[3];
  int64_t svf[3];
  /* packed keys: token mode strides over (b, h, slot) of a slot's contiguous
   * D/2-byte payload; channel mode strides over (b, h, group) of a group's contiguous
   * [D][kgroup/2] payload. Scale/zero (fp16 bit patterns) strides follow the same axes
   * with the channel (group) index contiguous.                                          */
  const uint8_t* kq;
  const uint16_t* ks;
  const uint16_t* kz;
  int64_t skq[3];
  int64_t sks[3];
  /* packed values: strides over (b, h, slot)                                          */
  const uint8_t* vq;
  const uint16_t* vs;
  const uint16_t* vz;
  int64_t svq[3];
  int64_t svs[3];
  /* token-mode key divisor [B,H,D] fp32: strides over (b, h)                          */
  const float* kchan;
  int64_t skc[2];
  /* optional live-slot mask, uint8 [B,H,nq+nf] contiguous; 0 = dead slot, never read  */
  const uint8_t* mask;
  /* Paged storage (optional; the reference has none -- the serving batch uses it): with
   * pages != NULL, slot j of sequence b in the paged part -- slots [0, nq) of a packed
   * layout, every slot of MA_KV_DENSE -- lives in page pages[b*spg + j/page_size] at
   * position j % page_size, and that part's strides run over (page, h, position)
   * instead of (b, h, slot); for channel-mode keys over (page, h, token group within
   * the page), page_size a multiple of kgroup. A page index outside [0, num_pages)
   * reads as a dead slot. The dense tail of a packed layout stays per sequence.       */
  const int32_t* pages;
  int64_t spg;
  int32_t page_size;
  int32_t num_pages;
  /* optional live length per sequence, int32 [B]: slots >= lens[b] are dead            */
  const int32_t* lens;
} ma_kv;

/* The query block: Q [B,Hq,T,D], strides over (b, hq, t). */
typedef struct ma_rows {
  const void* q;
  int32_t dtype;         /* MA_F32 or MA_BF16; the output has the same type             */
  int32_t B, Hq, T, D;
  int64_t sq[3];
} ma_rows;

/* The current block's keys/values [B,H,Tc,D] (query dtype), strides over (b, h, t). */
typedef struct ma_block {
  const void* k;
  const void* v;
  int32_t Tc;
  int64_t sk[3];
  int64_t sv[3];
} ma_block;

/* ---- library ----------------------------------------------------------------------- */
MA_API int ma_version(void);                       /* (major << 16) | minor                   */
MA_API const char* ma_status_string(int status);
/* Kernel choice for TMA-eligible dense bf16 calls (process-wide; for tests and A/B
 * timing): 0 = automatic (the TMA-pipelined attention and mass kernels), 1 = always the
 * general kernels (64-key attention tiles, cp.async-staged mass), 2 = the pipelined
 * attention with one 128-row M tile per CTA, 3 = with a pair of M tiles per CTA whenever
 * a KV head has more than 128 query rows. Returns the previous setting. A workspace size
 * queried under one setting may be too small under another. Not part of the reference's
 * interface.                                                                          */
MA_API int ma_set_attention_kernel(int which);
/* Work per CTA of the mass / value-score kernel over a ragged batch (ma_kv.lens set; process-
 * wide; for tests and A/B timing): at most `tiles` 128-slot tiles per CTA, so that heads of
 * long sequences spread over several CTAs (the score then follows in a second launch);
 * 0 = automatic (16 tiles when the batch has fewer heads than twice the SM count, else
 * no cap), < 0 = no cap (one CTA per head when the heads fill the GPU, the score in the
 * same launch). Returns the previous setting. Not part of the reference's interface.  */
MA_API int ma_set_mass_tiles(int tiles);
/* 1 when the TMA-pipelined attention and scoring kernels read this prefix as it is stored
 * (dense bf16 without mask or paging; token-mode k4v4 without a dense tail or mask, its
 * tiles dequantized by producer warps of those kernels), 0 when a caller is better served
 * by unpacking it to bf16 first (the other kernels still read it in place, slower). Not
 * part of the reference's interface.                                                  */
MA_API int ma_kv_read_in_place(const ma_kv* kv, int D);
/* The CUDA runtime's message for the error behind the last MA_ERR_CUDA of this thread
 * (the library links its own runtime, so a caller's cudaGetLastError cannot see it);
 * reading it clears it.                                                              */
MA_API const char* ma_last_cuda_error(void);

/* ---- device-side status --------------------------------------------------------------
 * ma_workspace_status: waits for the work queued on `stream` (a stream synchronization),
 * reads the error word of `workspace` (the first 256-byte boundary inside it, for every
 * workspace layout of this library), clears it and returns MA_ERR_TIMEOUT if a bounded
 * device wait of a call that used the workspace gave up since the last query, MA_OK if
 * none did. Not part of the reference's interface (its Triton launches have no device
 * waits).
 * ma_set_peer_wait_ns: the bound on a CTA's wait for other CTAs of the same launch (the
 * split merge of the attention calls and the value-score centre), process-wide; ns <= 0
 * restores the default (200 ms). Returns the previous bound. A CTA whose wait ends early
 * writes its rows as NaN and records the timeout; the launch stays consistent for the next
 * call. The waits on a CTA's own copies and MMAs keep their fixed bounds.            */
MA_API int ma_workspace_status(void* workspace, size_t workspace_bytes, void* stream);
MA_API int64_t ma_set_peer_wait_ns(int64_t ns);

/* ---- attention over [prefix | current block] ----------------------------------------
 * out[b, h*G+g, t, :] = softmax over the live prefix slots and the visible current keys.
 * causal_block > 0: query t sees current key j iff (c_pos0+j)/cb <= (q_pos0+t)/cb.
 * m_p, l_p ([B,H,R] fp32) and o_p ([B,H,R,D] fp32), all optional (NULL): prefix-only
 * softmax max, sum of exp(s - m_p) and normalized output per row.                    */
MA_API size_t ma_prefix_attention_workspace(int B, int H, int R, int n, int D, int Tc);
MA_API int ma_prefix_attention(const ma_rows* q, const ma_kv* kv, int H, const ma_block* cur,
                        float scale, int causal_block, int q_pos0, int c_pos0,
                        void* out, const int64_t so[3],
                        float* m_p, float* l_p, float* o_p,
                        void* workspace, size_t workspace_bytes, void* stream);

/* ---- prefix scores (mass and value-aware score) -------------------------------------
 * mass[b,h,j] = mean over rows (g, t in q_rows[0..T2)) of exp(s - m_p[r]) / l_p[r],
 * s = scale * q_r . k_j; 0 on dead slots. With score != NULL also
 * score[b,h,j] = mass_j * ||v_j - c||, c = sum_j mass_j v_j / max(sum_j mass_j, 1e-12)
 * over live slots (fp32), as ma_value_score. mass/score strides over (b, h). Rows whose
 * q_rows entry lies outside [0, T) are skipped. The workspace is sized by
 * ma_value_score_workspace(B, H, n, D); calls with any B*H may share one workspace (its
 * per-head counters sit in a block of fixed size at the front). B*H above 65536 returns
 * MA_ERR_UNSUPPORTED.                                                                  */
MA_API int ma_prefix_scores(const ma_rows* q, const ma_kv* kv, int H, const int32_t* q_rows, int T2,
                     const float* m_p, const float* l_p, float scale,
                     float* mass, const int64_t smass[2], float* score, const int64_t sscore[2],
                     void* workspace, size_t workspace_bytes, void* stream);

/* ---- value-aware score --------------------------------------------------------------
 * c = sum_j a_j v_j / max(sum_j a_j, 1e-12) over live slots, score_j = a_j*||v_j - c||
 * (fp32; dead slots: 0). a and score strides over (b, h). One workspace serves calls of
 * every size, and ma_prefix_scores's; B*H above 65536 returns MA_ERR_UNSUPPORTED.       */
MA_API size_t ma_value_score_workspace(int B, int H, int n, int D);
MA_API int ma_value_score(const ma_kv* kv, int B, int H, int D, const float* a, const int64_t sa[2],
                   float* score, const int64_t sscore[2],
                   void* workspace, size_t workspace_bytes, void* stream);

/* ---- value-aware score without a workspace -------------------------------------------
 * No counterpart in the reference. The same result as ma_value_score for callers that
 * cannot allocate device memory -- a host binding (JNI, cgo, a plugin interface) that
 * is handed only its input and output buffers and has no device allocator, or code whose
 * framework owns every device allocation. Its scratch is a static device array of
 * MA_NOALLOC_SCRATCH_BYTES (8 MiB) inside the library, held by every GPU that loads the
 * library until the process exits. Sizes whose scratch (ma_value_score_workspace(B, H,
 * n, D)) exceeds it return MA_ERR_UNSUPPORTED. The first call on a device looks up the
 * array's device address; make that first call before any stream capture. Every call
 * shares the array: calls that can overlap on the GPU (two streams, two threads) race.
 * Allocates nothing (no cudaMalloc, cudaFree or allocating library routine).
 * ma_value_score_noalloc_status: ma_workspace_status on that array (the current device's)
 * -- MA_ERR_TIMEOUT if a bounded device wait of the last call gave up (its scores then
 * hold NaN rows). Query it before the next call, which clears the word.               */
#define MA_NOALLOC_SCRATCH_BYTES ((size_t)8 << 20)
MA_API int ma_value_score_noalloc(const ma_kv* kv, int B, int H, int D, const float* a,
                                  const int64_t sa[2], float* score, const int64_t sscore[2],
                                  void* stream);
MA_API int ma_value_score_noalloc_status(void* stream);

/* ---- top-k read set -----------------------------------------------------------------
 * Per (b, h): the k largest scores among live slots (ties: lower slot first), written
 * as ascending slot indices (int64) with their scores (values optional). Live: mask
 * (optional, uint8 [B,H,n]) nonzero and slot < lens[b] (optional, int32 [B]); dead
 * slots rank below every live one.                                                    */
MA_API int ma_select_topk(const float* score, int B, int H, int n, const int64_t sscore[2],
                   const uint8_t* mask, const int32_t* lens, int k, int64_t* indices, float* values,
                   const int64_t sidx[2], void* stream);

/* ---- lookahead retention ------------------------------------------------------------
 * Per lane (the flattened [L,B,H] axis): keep the W = min(recent_window, capacity)
 * largest positions, the sinks (pos < sink_tokens) and the best remaining slots by
 * score, capacity in total, as live-axis indices ordered by position. score and pos
 * are [lanes, live] contiguous; when phys is not NULL the score of live entry i is
 * score_phys[lane, phys[lane, i]] with score row length n_phys.                       */
MA_API int ma_retain(const float* score, const int32_t* phys, int n_phys, const int32_t* pos,
              int lanes, int live, int capacity, int recent_window, int sink_tokens,
              int64_t* keep, void* stream);

/* ---- attention over the read set and the current block ------------------------------
 * Keys/values of prefix slots idx[b,h,0..k) (read directly from the cache layout,
 * dequantized in the staging), then the current block, for every row.               */
MA_API size_t ma_sparse_attention_workspace(int B, int H, int R, int k, int D, int Tc);
MA_API int ma_sparse_attention(const ma_rows* q, const ma_kv* kv, int H,
                        const int64_t* idx, int k, const int64_t sidx[2],
                        const ma_block* cur, float scale,
                        void* out, const int64_t so[3],
                        void* workspace, size_t workspace_bytes, void* stream);

/* ---- gather + dequantize ------------------------------------------------------------
 * out_k/out_v [B,H,k,D] (out_dtype) = the prefix slots idx[b,h,:]; idx = NULL (sidx
 * ignored): slots 0..k-1, i.e. the whole prefix dequantized when k = nq + nf. Slots past
 * lens[b] or on a bad page read as zeros.                                             */
MA_API int ma_gather_kv(const ma_kv* kv, int B, int H, int D, const int64_t* idx, int k,
                 const int64_t sidx[2], void* out_k, void* out_v, const int64_t sok[3],
                 const int64_t sov[3], int32_t out_dtype, void* stream);

/* ---- unpack of the live slots --------------------------------------------------------
 * The step-0 unpack of a token-mode packed prefix (splitk.py:465-480 dequantizes the
 * prefix before attending): out_k/out_v [B,H,nq+nf,128] bf16 get every slot below
 * lens[b] (every slot without lens) dequantized as ma_gather_kv(idx = NULL) does; slots
 * at or past lens[b] are NOT written (ma_gather_kv zero-fills them), which spares a
 * ragged batch the writes for its padding. Consumers that honour lens never read them.
 * Other layouts: MA_ERR_UNSUPPORTED.                                                  */
MA_API int ma_unpack_prefix(const ma_kv* kv, int B, int H, int D, void* out_k, void* out_v,
                            const int64_t sok[3], const int64_t sov[3], void* stream);

/* ---- compaction of the retained slots ------------------------------------------------
 * After an eviction decision keep [B,H,C] (int64 physical slot indices, slot axis
 * contiguous, strides skeep over (b, h)), slot j < C of dst gets the stored bytes of
 * slot keep[b,h,j] of src, every array of the layout moved bit-exactly: the payloads and
 * fp16 scale/zero of a token-mode packed cache (cache.py:659-678 compact_tokens, which
 * re-quantizes nothing), K/V of a dense bf16/fp32 cache (cache.py:342-365 compact, whose
 * bf16 re-staging is exact). Out of place: src and dst describe two caches of the same
 * layout, dtype and vgroup whose arrays must not overlap; dst's arrays are written (its
 * pointers are const only because ma_kv's are). Needs C <= the slots of src (nq packed,
 * nf dense) and of dst. A packed src must have no dense tail (nf == 0: the reference
 * requires a fully quantized cache); paged storage: MA_ERR_UNSUPPORTED.
 * MA_KV_PACKED_CHANNEL: keep indexes KEY GROUPS of kgroup tokens (C groups, n = nq /
 * kgroup): a kept group's key payload and scale/zero rows move with its kgroup value
 * slots, which must be packed back to back in src and dst (svq[2] = D/2, svs[2] =
 * D/vgroup, else MA_ERR_UNSUPPORTED); the dense tail is not touched. This is the group
 * copy of the reference's group-preserving rebuild (cache.py:236-335, copy_groups).
 * kchan, mask and lens are not read; a keep index outside [0, n) writes a zero row (the
 * reference's gather raises).
 * Several layers at once: pass [L*B] as B when the layer axis merges with the batch
 * axis (contiguous [L,B,H,...] caches).                                               */
/* The remap of a group-preserving rebuild (cache.py:236-335): remap [B,H,old_len] int64
 * (contiguous) gets, for every old slot, its slot in the rebuilt cache
 * [groups_before | encoded | groups_after] + residual, or -1 if dropped. Index lists are
 * contiguous [B,H,count] int64, -1 = padding: groups_before / groups_after name key
 * groups of kgroup slots (placed at group 0 and at group g1 + ceil(m/kgroup)), encode
 * names old slots re-encoded in order from slot g1*kgroup, stage old slots staged in
 * order from slot (g1 + ceil(m/kgroup) + g3) * kgroup. Entries outside [0, old_len) are
 * skipped. The lists are applied in that order (groups, encode, stage), so a slot named
 * twice takes the later list's position, as the reference's successive scatters do.
 * B*H above INT_MAX returns MA_ERR_UNSUPPORTED.                                        */
/* The planning of that rebuild after an eviction (runtime/session.py:303-356, the lazy
 * group-preserving compaction of _evict_to): per lane (the flattened [L,B,H] axis) the live
 * entries' physical slots phys [lanes, live] int32 and positions pos [lanes, live] int64
 * (lane strides sphys_spos = {phys, pos}; positions increase along the live axis, as the
 * eviction state keeps them). A key group of kgroup slots below quantized_length with at
 * least `need` live entries is kept whole (need 0: no group is), except the last
 * tail_groups; an entry at or past quantized_length (staged) among the recent_window
 * newest positions stays staged; every other entry is re-encoded. Writes groups_before
 * [lanes, ng] (ng = max(1, quantized_length / kgroup)), encode and stage [lanes, live]
 * (contiguous int64, each list ascending / in position order, padded with -1),
 * counts [lanes, 3] int32 (the three lengths) and maxes [4] int32: the three maxima over
 * lanes -- the widths the reference pads its lists to -- and the number of lanes whose
 * positions do not increase (their lists are not meaningful). ng above 8192 returns
 * MA_ERR_UNSUPPORTED.                                                                  */
MA_API int ma_evict_plan(const int32_t* phys, const int64_t* pos, int lanes, int live, const int64_t sphys_spos[2],
                         int quantized_length, int kgroup, int need, int tail_groups, int recent_window,
                         int64_t* groups_before, int64_t* encode, int64_t* stage, int32_t* counts, int32_t* maxes,
                         void* stream);
MA_API int ma_rebuild_remap(int B, int H, int old_len, int kgroup, const int64_t* groups_before, int g1,
                            const int64_t* encode, int m, const int64_t* groups_after, int g3,
                            const int64_t* stage, int st, int64_t* remap, void* stream);
MA_API int ma_compact_tokens(const ma_kv* src, const ma_kv* dst, int B, int H, int D, const int64_t* keep,
                             int C, const int64_t skeep[2], void* stream);

/* ---- quantize-on-append -------------------------------------------------------------
 * Dense rows x [B,H,n,D] (MA_BF16 or MA_F32, strides over (b, h, slot)) -> 4-bit codes
 * with fp16 scale/zero, as the reference's quantizers compute them in x's dtype
 * (reference.py:58-90 quantize_keys, 182-213 quantize_values; cache.py:484-497 append).
 * group must be 32; D a multiple of 32.
 * ma_quantize_tokens: per token and group of 32 channels -> payload [B,H,n,D/32,16]
 *   (16-byte aligned rows: strides sp over (b, h, slot) in bytes), scale/zero
 *   [B,H,n,D/32] (strides ss over (b, h, slot)); values, or token-mode keys when kchan
 *   ([B,H,D] fp32, strides skc over (b, h)) is given: x / kchan rounded to x's dtype
 *   first (cache.py:491-497).
 * ma_quantize_keys_channel: KIVI keys, per channel and group of 32 tokens (n a multiple
 *   of 32) -> payload [B,H,n/32,D,16] (strides over (b, h, group)), scale/zero
 *   [B,H,n/32,D] (strides over (b, h, group)).
 * ma_key_divisor: token-mode divisor kchan[b,h,d] = sqrt(max(max_t |k[b,h,t,d]|, 1e-4))
 *   (cache.py:488-490).                                                               */
MA_API int ma_quantize_tokens(const void* x, int32_t dtype, int B, int H, int n, int D, const int64_t sx[3],
                              const float* kchan, const int64_t skc[2], int group, uint8_t* payload,
                              const int64_t sp[3], uint16_t* scale, uint16_t* zero, const int64_t ss[3],
                              void* stream);
MA_API int ma_quantize_keys_channel(const void* k, int32_t dtype, int B, int H, int n, int D, const int64_t sk[3],
                                    int group, uint8_t* payload, const int64_t sp[3], uint16_t* scale,
                                    uint16_t* zero, const int64_t ss[3], void* stream);
MA_API int ma_key_divisor(const void* k, int32_t dtype, int B, int H, int n, int D, const int64_t sk[3],
                          float* kchan, const int64_t skc[2], void* stream);

/* ---- KV-head sharding: the head outputs exchanged over NVLink ------------------------
 * Every rank of a KV-head-sharded layer step (shard.py: rank r holds query heads
 * [r Hl, (r+1) Hl), Hl = Hq / world) needs all ranks' outputs; the reference runs
 * independent replicas only (scripts/gpu_queue.sh:1-49), so this has no reference
 * counterpart. Each rank allocates a receive region (ma_peer_alloc, its own device
 * allocation, zeroed, ma_head_gather_region_bytes(B, Hq, T) bytes) and shares it through a
 * CUDA IPC handle (ma_ipc_get_handle / ma_ipc_open_handle, handle of
 * ma_ipc_handle_bytes() bytes; ma_ipc_close_handle, ma_peer_free to release).
 * ma_head_gather: this rank's rows part [B, Hl, T, D] (bf16, strides sp over (b, head, t),
 *   D = 128) go into every rank's region by peer stores from this library's kernel (no
 *   multicast), then the call waits -- bounded by ma_set_peer_wait_ns -- for every rank's
 *   rows in its own region and copies them to out [B, Hq, T, D] (strides so). regions[p]
 *   = rank p's region as mapped in this process (regions[rank] this rank's own). Every
 *   rank makes the same sequence of calls (one process per GPU, all running); the call
 *   counter lives in the workspace (ma_head_gather_workspace() bytes, zeroed once), so a
 *   CUDA graph of the calls replays correctly. A wait that gave up is reported by
 *   ma_workspace_status (MA_ERR_TIMEOUT); out then holds stale rows of the other ranks. */
MA_API size_t ma_head_gather_region_bytes(int B, int Hq, int T);
MA_API size_t ma_head_gather_workspace(void);
MA_API int ma_peer_alloc(size_t bytes, void** ptr);
MA_API int ma_peer_free(void* ptr);
MA_API size_t ma_ipc_handle_bytes(void);
MA_API int ma_ipc_get_handle(void* ptr, void* handle);
MA_API int ma_ipc_open_handle(const void* handle, void** ptr);
MA_API int ma_ipc_close_handle(void* ptr);
MA_API int ma_head_gather(const void* part, const int64_t sp[3], int B, int Hl, int T, int D, int world, int rank,
                          void* const* regions, void* out, const int64_t so[3], void* workspace,
                          size_t workspace_bytes, void* stream);
/* ma_prefix_attention_gather: ma_prefix_attention of this rank's query heads (out [B, Hl, T,
 *   D], q->Hq = Hl) and the head gather of its rows t < Tg in the same launch: the split
 *   merge stores every finished row into every rank's region (regions and gather_ws as for
 *   ma_head_gather; the region sized ma_head_gather_region_bytes(B, Hq, Tg)), the launch's
 *   CTAs wait -- bounded -- for every rank's rows and copy them to gout [B, Hq, Tg, D]
 *   (strides sgo), Hq = world * Hl. When the attention cannot merge in one resident wave
 *   (its plan needs more CTAs than the GPU holds at once, or the prefix is not read by
 *   TMA) the gather runs as ma_head_gather's kernels after it, with the same result. Calls
 *   share gather_ws's counters with ma_head_gather, so the two may alternate. No reference
 *   counterpart (the reference does not shard heads): it fuses the per-layer attention
 *   with the all-gather of head outputs that KV-head sharding adds after it.           */
MA_API int ma_prefix_attention_gather(const ma_rows* q, const ma_kv* kv, int H, const ma_block* cur, float scale,
                                      int causal_block, int q_pos0, int c_pos0, void* out, const int64_t so[3],
                                      float* m_p, float* l_p, float* o_p, void* workspace, size_t workspace_bytes,
                                      int world, int rank, void* const* regions, int Tg, void* gout,
                                      const int64_t sgo[3], void* gather_ws, size_t gather_ws_bytes, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* MASKAHEAD_B200_H */
