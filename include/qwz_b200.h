/*
 * qwz_b200 — C ABI of the B200 (sm_100a) NVFP4/FP8 paged-attention kernels.
 *
 * Every entry point:
 *   - takes plain device pointers, sizes and a cudaStream_t passed as void*;
 *   - enqueues work on that stream and returns without synchronising;
 *   - allocates nothing (workspaces are caller-owned), so calls may be
 *     captured into CUDA graphs;
 *   - returns 0 on success, QWZ_EINVAL for a rejected argument (nothing was
 *     launched) or QWZ_ELAUNCH when a launch failed; qwz_last_error() then
 *     describes the failure (thread-local string).
 * Device-side metadata faults (a logical page beyond the block table, a
 * physical page id outside the pool) skip the affected copy/store and set
 * bits of a device error word that qwz_device_error() reads back.
 *
 * Fixed geometry (the reference pins it, src/qwasar_runtime/xqa.py:318-321):
 * 24 query heads, 4 KV heads, head_dim 256, 256-token pages.
 * NVFP4 cache (engine/forward/attention.py:159-167): codes uint8
 * [P, 256, 4, 128] (even d = low nibble), scales E4M3 [P, 256, 4, 16].
 * Lengths are int32 device words (graph-safe: never read on the host).
 */
#ifndef QWZ_B200_H
#define QWZ_B200_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define QWZ_OK 0
#define QWZ_EINVAL (-1)
#define QWZ_ELAUNCH (-2)

#define QWZ_DTYPE_F16 0
#define QWZ_DTYPE_BF16 1

/* Bits of the device error word. */
#define QWZ_DEVERR_TABLE_RANGE 1
#define QWZ_DEVERR_PAGE_RANGE 2
#define QWZ_DEVERR_SLOT_RANGE 4
#define QWZ_DEVERR_TIMEOUT 8 /* a bounded in-kernel wait gave up */

/* Library version string. */
const char* qwz_version(void);

/* Description of the last error returned on this host thread. */
const char* qwz_last_error(void);

/* Reads (and with clear != 0 resets) the device error word of the current
 * device.  Synchronises the device; for tests and diagnostics only. */
int qwz_device_error(int32_t* out, int32_t clear);

/*
 * NVFP4 KV-page writer.  Replaces the reference's append
 * (src/qwasar_runtime/xqa.py:356-379, ExLlamaV3 `_paged_kv_update_nvfp4_kernel`,
 * same argument order): for i < append_len and each KV head, quantises row i
 * of k and v ([append_len, num_kv_heads, 256], FP16/BF16) into the page
 * block_table[pos / 256] at offset pos % 256, pos = cache_seqlens[0] + i.
 * One E4M3 scale (amax / 6, RNE) per 16 elements; E2M1 codes (RNE of
 * x / scale, saturating at 6).  num_pages bounds the physical page ids.
 */
int qwz_nvfp4_append(const void* k, const void* v, void* k_cache, void* v_cache,
                     void* k_scales, void* v_scales, const int32_t* block_table,
                     const int32_t* cache_seqlens, int32_t table_width, int32_t append_len,
                     int32_t num_kv_heads, int32_t page_size, int32_t head_dim,
                     int32_t num_pages, int32_t dtype, void* stream);

/*
 * Writer for one shard of a sequence-sharded cache: as qwz_nvfp4_append, but
 * block_table entry 0 maps logical page table_page_offset, and rows whose
 * page lies outside [table_page_offset, table_page_offset + table_width) are
 * skipped silently (another rank owns them).  New work: the reference has no
 * multi-GPU path.
 */
int qwz_nvfp4_append_shard(const void* k, const void* v, void* k_cache, void* v_cache,
                           void* k_scales, void* v_scales, const int32_t* block_table,
                           const int32_t* cache_seqlens, int32_t table_width,
                           int32_t table_page_offset, int32_t append_len, int32_t num_pages,
                           int32_t dtype, void* stream);

/*
 * Split-K attention kernel with the reference split ABI
 * (tests/test_attention_kernel_abi.py:13-32): arguments 0..14 in the order
 *   q, k_cache, v_cache, block_table, cache_seqlens, out, partial_o,
 *   partial_ml, k_scales, v_scales, h32, split_len, num_pages_per_seq,
 *   num_splits, sinks
 * then the two trailing pointer slots global_scratch, profile_scratch.
 * For the NVFP4 cache h32 and sinks must be NULL; out is not written (the
 * combine writes it); the trailing slots are reserved and may be NULL.
 *   q            [q_len, 24, 256] FP16/BF16 (q_len 1..8)
 *   cache_seqlens pre-append length; attention covers post = pre + q_len
 *                tokens, row (qi, head) sees tokens <= pre + qi
 *   partial_o    FP32 [q_len, 24, num_splits, 256] (unnormalised O)
 *   partial_ml   FP32 [q_len, 24, num_splits, 2] (m in log2 units of
 *                sm_scale * q.k, l); splits that own no token write m = -inf
 *   split_len    0: the token range is balanced over num_splits on the
 *                device; > 0: fixed tokens per split (multiple of 256)
 *   num_pages_per_seq  entries of the block table row
 *   num_pages    physical pages in the pool (bounds check)
 * Grid = num_splits x 4 KV heads.
 */
int qwz_attn_split(const void* q, const void* k_cache, const void* v_cache,
                   const int32_t* block_table, const int32_t* cache_seqlens, void* out,
                   float* partial_o, float* partial_ml, const void* k_scales,
                   const void* v_scales, const void* h32, int32_t split_len,
                   int32_t num_pages_per_seq, int32_t num_splits, const void* sinks,
                   void* global_scratch, void* profile_scratch, int32_t q_len,
                   int32_t num_pages, float sm_scale, int32_t dtype, void* stream);

/*
 * Combine kernel with the reference combine ABI
 * (tests/test_attention_kernel_abi.py:22-24): partial_o, partial_ml, out,
 * h32, num_splits, sinks.  Writes out [q_len, 24, 256] (FP16/BF16),
 * out = sum_s 2^(m_s - M) O_s / sum_s 2^(m_s - M) l_s.  h32, sinks NULL.
 */
int qwz_attn_combine(const float* partial_o, const float* partial_ml, void* out,
                     const void* h32, int32_t num_splits, const void* sinks, int32_t q_len,
                     int32_t dtype, void* stream);

/*
 * Graph patching of captured split / combine launches.  The reference's
 * decode graphs patch split arguments 3, 4, 11, 12, 13 (block_table,
 * cache_seqlens, split_len, num_pages_per_seq, num_splits) and combine
 * argument 4 (num_splits) between replays
 * (docs/superpowers/specs/2026-09-11-qwasar-attention-kernel.md:66-74,
 * tests/test_attention_kernel_abi.py:25-31).  Here a captured split or
 * combine launch (from qwz_attn_split, qwz_attn_combine or
 * qwz_nvfp4_attend) is one kernel node whose single parameter packs those
 * arguments:
 *   qwz_graph_kernel_nodes  lists the split (QWZ_NODE_SPLIT) or combine
 *                           (QWZ_NODE_COMBINE) nodes of this library in a
 *                           cudaGraph_t, in the graph's node order: up to
 *                           max_nodes handles into nodes, the total in count;
 *   qwz_graph_patch_split   sets the five split arguments of one node, in the
 *                           graph and, if graph_exec is not NULL, in that
 *                           instantiated graph (the split grid follows
 *                           num_splits);
 *   qwz_graph_patch_combine sets num_splits of one combine node that reads
 *                           the split ABI's partial layout.
 * The workspace (partial_o, partial_ml) must hold the new num_splits, and
 * the new block_table / cache_seqlens must stay valid for every later
 * replay.  The pool (k/v caches and scales) cannot be patched.  Do not patch
 * a graph_exec while it is being replayed.
 */
#define QWZ_NODE_SPLIT 0
#define QWZ_NODE_COMBINE 1
int qwz_graph_kernel_nodes(void* graph, int32_t kind, void** nodes, int32_t max_nodes, int32_t* count);
int qwz_graph_patch_split(void* graph, void* graph_exec, void* node, const int32_t* block_table,
                          const int32_t* cache_seqlens, int32_t split_len, int32_t num_pages_per_seq,
                          int32_t num_splits);
int qwz_graph_patch_combine(void* graph, void* graph_exec, void* node, int32_t num_splits);

/*
 * The adapter's decode/verify route in one call: append + split + combine
 * (replaces NVFP4AttentionAdapter._append + _xqa, src/qwasar_runtime/
 * xqa.py:356-379 and 484-554).  k, v: the q_len new rows [q_len, 4, 256];
 * cache_seqlens is the PRE-append length (it is not modified).
 */
int qwz_nvfp4_attend(const void* q, const void* k, const void* v, void* k_cache, void* v_cache,
                     void* k_scales, void* v_scales, const int32_t* block_table,
                     const int32_t* cache_seqlens, void* out, float* partial_o,
                     float* partial_ml, int32_t table_width, int32_t num_pages, int32_t q_len,
                     int32_t num_splits, float sm_scale, int32_t dtype, void* stream);

/*
 * NVFP4 paged prefill attention: q [q_len, 24, 256] (FP16/BF16) over the
 * cache that already holds the q_len new rows (qwz_nvfp4_append first);
 * query position s sees keys j <= cache_seqlens[0] + s (lower-right causal),
 * out [q_len, 24, 256] same type.  Replaces the reference's staged prefill
 * route (src/qwasar_runtime/xqa.py:612-768: gather NVFP4 -> FP16 scratch ->
 * FP8 repage -> PRIMS / SDPA) with one launch that reads the NVFP4 pages
 * directly; the semantics are those of `_flash_prefill` (xqa.py:612-673).
 * No workspace.  Grid = ceil(q_len / 21) x 4 KV heads.
 */
int qwz_nvfp4_prefill(const void* q, const void* k_cache, const void* v_cache, const void* k_scales,
                      const void* v_scales, const int32_t* block_table, const int32_t* cache_seqlens,
                      void* out, int32_t table_width, int32_t num_pages, int32_t q_len, float sm_scale,
                      int32_t dtype, void* stream);

/*
 * Draft-model prefill attention over FP16 K/V rows (no pages, no
 * quantisation): q [q_len, 24, 256] FP16, k and v [kv_len, 4, 256] FP16 with
 * a token stride of k_token_stride / v_token_stride elements (a multiple of
 * 8, >= 1024; head and dim contiguous), out [q_len, 24, 256] FP16.  Query
 * row s sees keys j <= kv_len - q_len + s (bottom-right causal), GQA 6.
 * Replaces engine/forward/draft.py:33-61 `draft_attend` (SDPA for short
 * chunks, `_merge_bottom_right` for a chunk after a past, and the FP8
 * repage + sm120 paged FMHA of draft.py:99-181 for long ones).  Requires
 * 1 <= q_len <= kv_len.  No workspace.
 */
int qwz_draft_prefill(const void* q, const void* k, const void* v, void* out, int32_t q_len, int32_t kv_len,
                      int64_t k_token_stride, int64_t v_token_stride, float sm_scale, void* stream);

/*
 * qwz_nvfp4_attend without a caller-supplied workspace.  No counterpart in
 * the reference: it exists for callers that cannot allocate device memory
 * (an engine that owns every allocation, a fixed memory pool, an FFI that
 * only passes raw input/output pointers).  The split-K partials live in a
 * static device array of 4096 (query row x split) records, 4 MiB + 32 KiB,
 * held by every GPU that loads the library until the process exits.
 * Requests with q_len * 24 * num_splits > 4096 return QWZ_EINVAL.  The first
 * call on a device resolves the array's device address (cudaGetSymbolAddress
 * with that device current) and must come before any stream capture on it;
 * after a cudaDeviceReset the next call resolves it again (likewise outside
 * a capture).
 * Calls share the array and race if they overlap on the GPU: serialise them.
 * Allocates nothing; arguments otherwise as qwz_nvfp4_attend.
 */
int qwz_nvfp4_attend_noalloc(const void* q, const void* k, const void* v, void* k_cache,
                             void* v_cache, void* k_scales, void* v_scales,
                             const int32_t* block_table, const int32_t* cache_seqlens, void* out,
                             int32_t table_width, int32_t num_pages, int32_t q_len,
                             int32_t num_splits, float sm_scale, int32_t dtype, void* stream);

/*
 * Sequence-sharded decode, local half: attention of q over the logical
 * tokens [tok_begin, tok_begin + tok_span) clipped to the post-append length,
 * through a block table whose entry 0 maps logical page tok_begin / 256
 * (tok_begin a multiple of 256).  The local splits are reduced to one
 * record per row: send_buf FP32 [q_len * 24, 258] = (m, l, O[256]).
 * New work; the reference has no multi-GPU path (its engine refuses more
 * than one GPU, src/qwasar_runtime/engine.py:602-610).
 */
int qwz_attn_shard_partial(const void* q, const void* k_cache, const void* v_cache,
                           const void* k_scales, const void* v_scales,
                           const int32_t* block_table, const int32_t* cache_seqlens,
                           float* partial_o, float* partial_ml, float* send_buf,
                           int32_t table_width, int32_t num_pages, int32_t tok_begin,
                           int32_t tok_span, int32_t q_len, int32_t num_splits, float sm_scale,
                           int32_t dtype, void* stream);

/*
 * Sequence-sharded decode, global half: LSE combine of the all-gathered
 * records gathered FP32 [world, q_len * 24, 258] into out [q_len, 24, 256].
 */
int qwz_lse_combine_gathered(const float* gathered, void* out, int32_t world, int32_t q_len,
                             int32_t dtype, void* stream);

/*
 * Sequence-sharded decode over NVLink peer memory (no reference
 * counterpart: the reference is single-GPU).  Each rank owns one exchange
 * buffer of qwz_peer_buffer_bytes(world, q_len) bytes, layout
 *   uint64 [2 (epoch parity), world, q_len * 24, 258], each word an FP32
 *   value (low half) tagged with the epoch of the call that wrote it,
 * allocated zeroed by qwz_peer_alloc, which also returns its 64-byte CUDA
 * IPC handle; the caller exchanges the handles (e.g. torch.distributed) and
 * maps the other ranks' buffers with qwz_peer_open.  These set-up calls
 * allocate and synchronise (once per rank); the per-step calls below do not.
 */
int64_t qwz_peer_buffer_bytes(int32_t world, int32_t q_len);  /* 0 when out of range */
int qwz_peer_alloc(int64_t bytes, void** dev_ptr, uint8_t* ipc_handle);
int qwz_peer_open(const uint8_t* ipc_handle, void** dev_ptr);
int qwz_peer_close(void* peer_ptr);  /* a mapping from qwz_peer_open */
int qwz_peer_free(void* dev_ptr);    /* the rank's own buffer */

/*
 * Shard split with the new rows appended: the split half of
 * qwz_attn_shard_partial (local partials in partial_o / partial_ml) plus
 * k, v [q_len, 4, 256] of the new rows, stored only by the rank whose pages
 * hold them (inside the decode kernel at q_len 1).
 */
int qwz_attn_shard_split(const void* q, const void* k, const void* v, void* k_cache, void* v_cache,
                         void* k_scales, void* v_scales, const int32_t* block_table,
                         const int32_t* cache_seqlens, float* partial_o, float* partial_ml,
                         int32_t table_width, int32_t num_pages, int32_t tok_begin, int32_t tok_span,
                         int32_t q_len, int32_t num_splits, float sm_scale, int32_t dtype, void* stream);

/*
 * Exchange and merge in one kernel: merges this rank's num_splits partials
 * into one (m, l, O) record per query row and stores it into every rank's
 * buffer, each value in a 64-bit word tagged with the epoch of this call (no
 * separate flag: a reader polls the data words until they carry the epoch
 * it waits for).  Once every rank's record is in its own buffer it
 * LSE-merges them in rank order into out [q_len, 24, 256] FP16/BF16 (the
 * same on every rank).  The wait is bounded: after timeout_ns (0: 0.5 s) the
 * kernel sets QWZ_DEVERR_TIMEOUT, merges what has arrived and returns.
 *   peers        HOST array [world] of the buffers' device addresses as this
 *                GPU maps them (its own buffer at [rank])
 *   buffer_bytes the size the buffers were allocated with; must equal
 *                qwz_peer_buffer_bytes(world, q_len) (QWZ_EINVAL otherwise)
 *   epochs       device uint32 [q_len * 24], zeroed once; the kernel counts
 *                calls
 * Every rank must call it the same number of times, with the same q_len.
 */
int qwz_shard_exchange_combine(const float* partial_o, const float* partial_ml, int32_t num_splits,
                               int32_t q_len, const uint64_t* peers, int64_t buffer_bytes, uint32_t* epochs,
                               int32_t rank, int32_t world, void* out, int64_t timeout_ns, int32_t dtype,
                               void* stream);

/*
 * The same for `world` ranks emulated on one GPU in one cooperative launch
 * (rank g's partials at partial_o + g * q_len*24*rank_stride_splits*256 and
 * partial_ml + g * q_len*24*rank_stride_splits*2, its epochs at
 * epochs + g * q_len*24, its output at out + g * q_len*24*256 elements;
 * peers[g] = rank g's buffer on this GPU).
 */
int qwz_shard_exchange_combine_emulated(const float* partial_o, const float* partial_ml,
                                        int64_t rank_stride_splits, int32_t num_splits, int32_t q_len,
                                        const uint64_t* peers, int64_t buffer_bytes, uint32_t* epochs,
                                        void* out, int32_t world, int64_t timeout_ns, int32_t dtype,
                                        void* stream);

/*
 * FP8 shadow-KV draft decode (replaces DecodeAttention.attend,
 * engine/forward/draft_attention.py:93-108): one query row per head,
 *   q      FP16 [1, 1, 24, 256]
 *   k8,v8  E4M3 [capacity, 4, 256] (contiguous, not paged)
 *   k_scale, v_scale FP32 [ceil(capacity/256), 4] per (page, head), or NULL
 *          (scale 1, the reference's `_fp8` shadow)
 *   length int32 [1] on the device: keys [0, length) are attended
 *   part   FP32 [24, splits, 256], stat FP32 [24, splits, 2]
 *   out    FP16 [1, 1, 24, 256]
 */
int qwz_fp8_draft_decode(const void* q, const void* k8, const void* v8, const float* k_scale,
                         const float* v_scale, const int32_t* length, float* part, float* stat,
                         void* out, int32_t splits, int32_t capacity, void* stream);

/*
 * One draft step with the FP8 shadow write fused in: what
 * qwz_fp8_shadow_write(k_new, v_new, k8, v8, k_scale, v_scale, position)
 * followed by qwz_fp8_draft_decode(...) computes, in two launches instead of
 * three (engine/forward/draft.py:359-366 then draft_attention.py:82-108).
 * k_new, v_new FP16 [4, 256]; position int32 [1] on the device, in
 * [0, capacity) (a slot past length is written but not attended).
 */
int qwz_fp8_draft_step(const void* q, const void* k_new, const void* v_new, const int32_t* position, void* k8,
                       void* v8, const float* k_scale, const float* v_scale, const int32_t* length, float* part,
                       float* stat, void* out, int32_t splits, int32_t capacity, void* stream);

/*
 * FP8 shadow write (replaces engine/forward/draft.py:359-366): writes one new
 * row k, v [4, 256] (FP16/BF16) into k8, v8 at slot position[0] as
 * E4M3(clamp(x / scale, +-448)), scale per (page, head) or 1 when NULL.
 */
int qwz_fp8_shadow_write(const void* k, const void* v, void* k8, void* v8, const float* k_scale,
                         const float* v_scale, const int32_t* position, int32_t capacity,
                         int32_t dtype, void* stream);

/*
 * NVFP4 -> FP16 dequant gather in logical order; mirrors the reference
 * oracle kernel `_gather_nvfp4_kernel` (src/qwasar_runtime/xqa.py:73-143)
 * argument for argument: out[b, t, h, :] for t < seq_lens[b]; tokens beyond
 * seq_lens[b] are not written.  head_dim must be a multiple of 16.
 */
int qwz_nvfp4_gather(const void* packed, const void* scales, const int32_t* block_table,
                     const int32_t* seq_lens, void* output, int32_t batch, int32_t max_tokens,
                     int32_t table_width, int32_t n_heads, int32_t head_dim, int32_t page_size,
                     void* stream);

/*
 * K8/V4 cache path: the cache of the reference's Attention64 split/combine
 * slot and of its MTP draft (ExLlamaV3 CacheLayer_quant, k_bits 8, v_bits 4;
 * src/qwasar_runtime/xqa.py:926-961).  Geometry as
 * src/qwasar_bench/prefill_flash.py:32-44 checks it:
 *   k_cache int32 [P, 256, 256], v_cache int32 [P, 256, 128],
 *   k_scales / v_scales FP16 [P, 256, 32].
 * A (token, KV head h, 32-dim block j) holds 32 codes of b bits (8 for K, 4
 * for V) as b bit-plane words (word i = bit i of the codes, bit t = element
 * t) at (h * 8 + j) * b of the token's row, and one FP16 scale at h * 8 + j,
 * in the rotated domain R = H32 / sqrt(32).  The reader is
 *   x_rot = FP16((FP32(c) - (2^(b-1) - 0.5)) * (FP32(s) / 2^(b-1)))
 * (docs/superpowers/specs/2026-09-08-direct-k8v4-attention-design.md:55-61).
 *
 * qwz_k8v4_append  quantises rows k, v [append_len, 4, 256] (FP16/BF16) at
 *                  logical positions cache_seqlens[0] + s: each 32-dim block
 *                  is rotated by the natural-order Hadamard butterfly (FP32),
 *                  s = FP16(max |x_rot|), c = clamp(floor(x_rot / s *
 *                  2^(b-1) + 2^(b-1)), 0, 2^b - 1).
 * qwz_k8v4_split   the split kernel with the reference's 15 + 2 argument
 *                  order (docs/superpowers/specs/2026-09-11-qwasar-attention-
 *                  kernel.md:62-74; same tail as qwz_attn_split): h32 is the
 *                  rotation R, FP32 [32, 32] row-major (required); sinks must
 *                  be NULL.  The partials are in the rotated domain, in the
 *                  layout of qwz_attn_split.  num_pages bounds the pool.
 * qwz_k8v4_combine the combine with the reference combine order: merges the
 *                  partials and writes out = R^T O per 32-dim block.
 * qwz_k8v4_gather  the reader alone: logical tokens [0, length) of one cache
 *                  (bits 8 for K, 4 for V) into FP16 [length, 4, 256],
 *                  rotated domain.
 */
int qwz_k8v4_append(const void* k, const void* v, void* k_cache, void* v_cache, void* k_scales,
                    void* v_scales, const int32_t* block_table, const int32_t* cache_seqlens,
                    int32_t table_width, int32_t num_pages, int32_t append_len, int32_t dtype,
                    void* stream);
int qwz_k8v4_split(const void* q, const void* k_cache, const void* v_cache, const int32_t* block_table,
                   const int32_t* cache_seqlens, void* out, float* partial_o, float* partial_ml,
                   const void* k_scales, const void* v_scales, const void* h32, int32_t split_len,
                   int32_t num_pages_per_seq, int32_t num_splits, const void* sinks, void* global_scratch,
                   void* profile_scratch, int32_t q_len, int32_t num_pages, float sm_scale, int32_t dtype,
                   void* stream);
int qwz_k8v4_combine(const float* partial_o, const float* partial_ml, void* out, const void* h32,
                     int32_t num_splits, const void* sinks, int32_t q_len, int32_t dtype, void* stream);
int qwz_k8v4_gather(const void* words, const void* scales, const int32_t* block_table, int32_t table_width,
                    int32_t num_pages, int32_t length, int32_t bits, void* out, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* QWZ_B200_H */
