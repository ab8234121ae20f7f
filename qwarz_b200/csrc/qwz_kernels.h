// Host-side launch interface of the sm_100a kernels (internal; the public
// C ABI is include/qwz_b200.h).
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>
#include <cuda_fp16.h>
#include <stdint.h>

namespace qwz {

enum : int { kDtypeF16 = 0, kDtypeBF16 = 1 };

// Split-K attention launch (NVFP4 paged decode/verify, FP8 draft decode).
struct alignas(64) SplitParams {
  // TMA descriptors of the NVFP4 pool viewed as 2-D byte tensors
  // [P*256 token rows, 512 B] (codes, 128B swizzle, 128 x 64 box) and
  // [P*256, 64 B] (scales, 16 x 64 box); filled by the host (capi.cu).
  CUtensorMap tm_kc, tm_vc, tm_ks, tm_vs;
  const void* q;                 // [q_len, 24, 256] FP16/BF16
  const uint8_t* k_codes;        // NVFP4: [P,256,4,128] ; FP8: [T,4,256] E4M3
  const uint8_t* v_codes;
  const uint8_t* k_scales;       // NVFP4: [P,256,4,16] E4M3 ; FP8: unused
  const uint8_t* v_scales;
  const float* k_page_scale;     // FP8: [ceil(T/256), 4] FP32 or null (= 1)
  const float* v_page_scale;
  const int32_t* block_table;    // NVFP4: logical page -> physical page
  const int32_t* seqlens;        // device length word [1]
  float* partial_o;              // [R, num_splits, 256]
  float* partial_ml;             // [R, num_splits, 2]  (m in log2 units, l)
  int table_width;               // entries of block_table
  int table_page_offset;         // logical page index of block_table[0]
  int num_pages;                 // physical pages in the NVFP4 pool
  int capacity;                  // FP8: token slots in the store
  int q_len;                     // query rows per head (1..8)
  int len_add;                   // valid length = seqlens[0] + len_add
  int tok_begin;                 // first logical token of this launch (multiple of 256)
  int tok_span;                  // tokens this launch may cover
  int split_len;                 // >0: fixed tokens per split (multiple of 256); 0: balanced
  int num_splits;
  float sm_scale_log2;           // sm_scale * log2(e)
  // Fused append (NVFP4 decode, q_len 1, through qwz_nvfp4_attend): the new
  // K/V row [4, 256] (same type as q) for token seqlens[0]; the CTA owning
  // that token's page quantises it into the pool before reading the page.
  // Null: no append.
  const void* app_k;
  const void* app_v;
  // Fused FP8 shadow write (draft step, qwz_fp8_draft_step): app_k / app_v
  // are FP16 [4, 256] rows for store slot app_slot[0]; the CTA whose stage
  // holds that slot writes it to the store and into its shared-memory copy.
  const int32_t* app_slot;
  // K8/V4 split (k8v4.cu): the rotation R, FP32 [32, 32] row-major; the
  // codes are int32 bit-plane words and the scales FP16.
  const float* h32;
};

// NVFP4 paged prefill attention (attn_prefill.cu): q [q_len, 24, 256] over
// the post-append cache, lower-right causal.  Tensor maps as SplitParams
// but with 64-row boxes.  The dense FP16 source (draft prefill) uses tm_kc /
// tm_vc over K, V [kv_len rows, token stride] with 128-byte x 64-row boxes,
// pre_len instead of seqlens, and no table.
struct alignas(64) PrefillParams {
  CUtensorMap tm_kc, tm_vc, tm_ks, tm_vs;
  const void* q;                 // [q_len, 24, 256] FP16/BF16
  void* out;                     // [q_len, 24, 256] same type
  const int32_t* block_table;
  const int32_t* seqlens;        // pre-append length [1]
  int table_width;
  int num_pages;
  int q_len;
  float sm_scale_log2;
  int pre_len;                   // dense FP16 source: keys before the q_len rows (host)
};

// LSE combine of split partials.  Row r, split s reads
//   m,l at pml[r*ml_row + s*ml_split + {0,1}] and O at po[r*o_row + s*o_split + d].
struct CombineParams {
  const float* po;
  const float* pml;
  long long o_row, o_split, ml_row, ml_split;
  int rows;
  int num_splits;
  void* out;          // final: [rows, 256] FP16/BF16 ; partial: [rows, 258] FP32 (m, l, O)
  const float* h32;   // rotate mode: R, FP32 [32, 32]; out = R^T O per 32-dim block
};

enum : int { kCombineFinal = 0, kCombinePartial = 1, kCombineRotate = 2 };

// K8/V4 writer (k8v4.cu): new rows at logical positions seqlens[0] + s.
struct K8v4AppendParams {
  const void* k;                 // [S, 4, 256] FP16/BF16
  const void* v;
  uint32_t* k_cache;             // [P, 256, 256] bit-plane words
  uint32_t* v_cache;             // [P, 256, 128]
  __half* k_scales;              // [P, 256, 32]
  __half* v_scales;
  const int32_t* block_table;
  const int32_t* seqlens;        // pre-append length [1]
  int table_width;
  int num_pages;
  int append_len;
};

struct AppendParams {
  const void* k;                 // [S, kv_heads, 256] new rows
  const void* v;
  uint8_t* k_cache;              // [P, 256, kv_heads, 128]
  uint8_t* v_cache;
  uint8_t* k_scales;             // [P, 256, kv_heads, 16] E4M3
  uint8_t* v_scales;
  const int32_t* block_table;
  const int32_t* seqlens;        // pre-append length [1]
  int table_width;
  int table_page_offset;
  int append_len;
  int num_kv_heads;
  int num_pages;
  int skip_foreign;              // rows outside this table's pages: skip silently (shards)
};

struct Fp8WriteParams {
  const void* k;                 // [kv_heads, 256] one new row (FP16/BF16)
  const void* v;
  uint8_t* k8;                   // [capacity, kv_heads, 256] E4M3
  uint8_t* v8;
  const float* k_page_scale;     // [pages, kv_heads] or null (= 1)
  const float* v_page_scale;
  const int32_t* position;       // slot to write [1]
  int capacity;
  int num_kv_heads;
};

struct GatherParams {
  const uint8_t* packed;         // [P, page, heads, dim/2]
  const uint8_t* scales;         // [P, page, heads, dim/16] E4M3
  const int32_t* block_table;    // [batch, table_width]
  const int32_t* seq_lens;       // [batch]
  __half* out;                   // [batch, max_tokens, heads, dim]
  int batch, max_tokens, table_width, n_heads, head_dim, page_size;
};

// Sequence-sharded decode: record exchange over peer memory + final merge.
// Arrays are indexed by blockIdx.y (emulated ranks on one GPU) or hold one
// entry (a real rank, rank0 = its rank).
constexpr int kMaxWorld = 8;
struct ExchangeParams {
  const float* po[kMaxWorld];    // [rows, num_splits, 256] split partials of the rank
  const float* pml[kMaxWorld];   // [rows, num_splits, 2]
  uint32_t* epochs[kMaxWorld];   // [rows] call counters of the rank
  void* out[kMaxWorld];          // [rows, 256] FP16/BF16
  uint64_t peers[kMaxWorld];     // exchange buffer of every rank, as this GPU addresses it
  int num_splits;
  int rows;
  int world;
  int rank0;
  unsigned long long timeout_ns; // bound of each rank's wait for the others' records
};

cudaError_t launch_nvfp4_split(const SplitParams& p, int dtype, cudaStream_t stream);
cudaError_t launch_nvfp4_prefill(const PrefillParams& p, int dtype, cudaStream_t stream);
cudaError_t launch_draft_prefill(const PrefillParams& p, cudaStream_t stream);
cudaError_t launch_shard_exchange(const ExchangeParams& p, int emulated, int dtype, cudaStream_t stream);
cudaError_t launch_fp8_split(const SplitParams& p, cudaStream_t stream);
cudaError_t launch_combine(const CombineParams& p, int mode, int dtype, cudaStream_t stream);
cudaError_t launch_nvfp4_append(const AppendParams& p, int dtype, cudaStream_t stream);
cudaError_t launch_fp8_write(const Fp8WriteParams& p, int dtype, cudaStream_t stream);
cudaError_t launch_nvfp4_gather(const GatherParams& p, cudaStream_t stream);
cudaError_t launch_k8v4_split(const SplitParams& p, int dtype, cudaStream_t stream);
cudaError_t launch_k8v4_append(const K8v4AppendParams& p, int dtype, cudaStream_t stream);
cudaError_t launch_k8v4_gather(const uint32_t* words, const __half* scales, const int32_t* table, int width,
                               int num_pages, int length, int bits, __half* out, cudaStream_t stream);

}  // namespace qwz
