// extern "C" entry points declared in include/qwz_b200.h: argument checks,
// launch-parameter packing, error reporting.  Nothing here allocates device
// memory or synchronises, except qwz_device_error (a diagnostic) and the
// peer-buffer set-up calls of the sharded decode (qwz_peer_*, once per rank).

#include "qwz_common.cuh"
#include "qwz_kernels.h"
#include "../../include/qwz_b200.h"

#include <cudaTypedefs.h>

#include <cmath>
#include <cstdio>
#include <cstring>
#include <mutex>
#include <string>

namespace {

thread_local std::string g_last_error;

int fail(int code, const char* fmt, const char* detail = nullptr) {
  char buf[512];
  if (detail)
    std::snprintf(buf, sizeof(buf), fmt, detail);
  else
    std::snprintf(buf, sizeof(buf), "%s", fmt);
  g_last_error = buf;
  return code;
}

int launched(cudaError_t e, const char* what) {
  if (e == cudaSuccess) return QWZ_OK;
  char buf[512];
  std::snprintf(buf, sizeof(buf), "%s: launch failed: %s", what, cudaGetErrorString(e));
  g_last_error = buf;
  return QWZ_ELAUNCH;
}

bool aligned(const void* p, uintptr_t a) { return (reinterpret_cast<uintptr_t>(p) % a) == 0; }

cudaStream_t as_stream(void* s) { return reinterpret_cast<cudaStream_t>(s); }

constexpr float kLog2e = 1.4426950408889634f;

int check_dtype(int32_t dtype) {
  if (dtype != QWZ_DTYPE_F16 && dtype != QWZ_DTYPE_BF16)
    return fail(QWZ_EINVAL, "dtype must be QWZ_DTYPE_F16 (0) or QWZ_DTYPE_BF16 (1)");
  return QWZ_OK;
}

int check_nvfp4_cache(const void* kc, const void* vc, const void* ks, const void* vs,
                      int32_t num_pages) {
  if (!kc || !vc || !ks || !vs)
    return fail(QWZ_EINVAL, "NVFP4 caches and block scales are required (non-null)");
  if (!aligned(kc, 16) || !aligned(vc, 16) || !aligned(ks, 16) || !aligned(vs, 16))
    return fail(QWZ_EINVAL, "NVFP4 caches and scales must be 16-byte aligned");
  if (num_pages <= 0) return fail(QWZ_EINVAL, "num_pages must be positive");
  if ((long long)num_pages * qwz::kPage * qwz::kKvHeads > 0x7fffffffLL)
    return fail(QWZ_EINVAL, "num_pages too large for 32-bit token rows");
  return QWZ_OK;
}

// cuTensorMapEncodeTiled through the runtime's driver entry point (the
// library links only the static CUDA runtime).
PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* f = nullptr;
    cudaDriverEntryPointQueryResult q{};
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &f, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(f);
  });
  return fn;
}

// 2-D uint8 view [rows, row_bytes] of a pool, box box_x bytes x box_y rows.
// Rows of `inner_bytes` used bytes at a stride of `row_stride` bytes.
int encode_rows(CUtensorMap* m, const void* base, uint64_t inner_bytes, uint64_t row_stride, uint64_t rows,
                uint32_t box_x, uint32_t box_y, CUtensorMapSwizzle swizzle) {
  auto fn = encode_fn();
  if (!fn) return fail(QWZ_ELAUNCH, "cuTensorMapEncodeTiled is unavailable from the driver");
  cuuint64_t dims[2] = {inner_bytes, rows};
  cuuint64_t strides[1] = {row_stride};
  cuuint32_t box[2] = {box_x, box_y};
  cuuint32_t elem[2] = {1, 1};
  const CUresult r = fn(m, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<void*>(base), dims, strides,
                        box, elem, CU_TENSOR_MAP_INTERLEAVE_NONE, swizzle,
                        CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return fail(QWZ_EINVAL, "TMA descriptor encoding failed (base, stride or extent)");
  return QWZ_OK;
}

int encode_2d(CUtensorMap* m, const void* base, uint64_t row_bytes, uint64_t rows, uint32_t box_x,
              uint32_t box_y, CUtensorMapSwizzle swizzle) {
  return encode_rows(m, base, row_bytes, row_bytes, rows, box_x, box_y, swizzle);
}

// Descriptors of the NVFP4 pool: codes [P*256, 512 B] (boxes of one head's
// 128 B x box_rows tokens, 128-byte swizzle), scales [P*256, 64 B] (16 B x
// box_rows).  The decode kernel streams whole pages (256 rows), the verify
// kernel 128-token tiles.
int encode_pool(qwz::SplitParams& p, int32_t num_pages, uint32_t box_rows) {
  const uint64_t rows = (uint64_t)num_pages * qwz::kPage;
  int rc = encode_2d(&p.tm_kc, p.k_codes, qwz::kRowBytesCodes, rows, qwz::kCodeBytes, box_rows,
                     CU_TENSOR_MAP_SWIZZLE_128B);
  if (!rc) rc = encode_2d(&p.tm_vc, p.v_codes, qwz::kRowBytesCodes, rows, qwz::kCodeBytes, box_rows,
                          CU_TENSOR_MAP_SWIZZLE_128B);
  if (!rc) rc = encode_2d(&p.tm_ks, p.k_scales, qwz::kRowBytesScales, rows, qwz::kScaleBytes, box_rows,
                          CU_TENSOR_MAP_SWIZZLE_NONE);
  if (!rc) rc = encode_2d(&p.tm_vs, p.v_scales, qwz::kRowBytesScales, rows, qwz::kScaleBytes, box_rows,
                          CU_TENSOR_MAP_SWIZZLE_NONE);
  return rc;
}

int fill_split(qwz::SplitParams& p, const void* q, const void* kc, const void* vc,
               const void* ks, const void* vs, const int32_t* table, const int32_t* seqlens,
               float* po, float* pml, int32_t table_width, int32_t num_pages, int32_t q_len,
               int32_t num_splits, int32_t split_len, float sm_scale) {
  if (!q || !aligned(q, 16)) return fail(QWZ_EINVAL, "q must be a non-null 16-byte aligned pointer");
  int rc = check_nvfp4_cache(kc, vc, ks, vs, num_pages);
  if (rc) return rc;
  if (!table || !seqlens) return fail(QWZ_EINVAL, "block_table and cache_seqlens are required");
  if (!po || !pml || !aligned(po, 16) || !aligned(pml, 8))
    return fail(QWZ_EINVAL, "partial_o (16-byte aligned) and partial_ml are required");
  if (table_width <= 0) return fail(QWZ_EINVAL, "num_pages_per_seq (table width) must be positive");
  if (q_len < 1 || q_len > 8) return fail(QWZ_EINVAL, "q_len must be in 1..8");
  if (num_splits < 1 || num_splits > 65535) return fail(QWZ_EINVAL, "num_splits must be in 1..65535");
  if (split_len < 0 || split_len % qwz::kPage != 0)
    return fail(QWZ_EINVAL, "split_len must be 0 or a positive multiple of 256");
  if (!(sm_scale > 0.f) || !std::isfinite(sm_scale)) return fail(QWZ_EINVAL, "sm_scale must be positive and finite");
  p = qwz::SplitParams{};
  p.q = q;
  p.k_codes = static_cast<const uint8_t*>(kc);
  p.v_codes = static_cast<const uint8_t*>(vc);
  p.k_scales = static_cast<const uint8_t*>(ks);
  p.v_scales = static_cast<const uint8_t*>(vs);
  p.block_table = table;
  p.seqlens = seqlens;
  p.partial_o = po;
  p.partial_ml = pml;
  p.table_width = table_width;
  p.table_page_offset = 0;
  p.num_pages = num_pages;
  p.capacity = 0;
  p.q_len = q_len;
  p.len_add = q_len;
  p.tok_begin = 0;
  p.tok_span = 0x7fffffff;
  p.split_len = split_len;
  p.num_splits = num_splits;
  p.sm_scale_log2 = sm_scale * kLog2e;
  return encode_pool(p, num_pages, q_len == 1 ? qwz::kPage : 128u);
}

qwz::CombineParams split_combine_params(const float* po, const float* pml, int rows, int splits,
                                        void* out) {
  qwz::CombineParams c{};
  c.po = po;
  c.pml = pml;
  c.o_row = (long long)splits * qwz::kHeadDim;
  c.o_split = qwz::kHeadDim;
  c.ml_row = (long long)splits * 2;
  c.ml_split = 2;
  c.rows = rows;
  c.num_splits = splits;
  c.out = out;
  return c;
}

}  // namespace

extern "C" {

const char* qwz_version(void) { return "qwz_b200 0.1 sm_100a"; }

const char* qwz_last_error(void) { return g_last_error.c_str(); }

int qwz_device_error(int32_t* out, int32_t clear) {
  if (!out) return fail(QWZ_EINVAL, "out is null");
  int v = 0;
  cudaError_t e = cudaMemcpyFromSymbol(&v, qwz::g_qwz_device_error, sizeof(int));
  if (e != cudaSuccess) return launched(e, "qwz_device_error");
  *out = v;
  if (clear) {
    const int zero = 0;
    e = cudaMemcpyToSymbol(qwz::g_qwz_device_error, &zero, sizeof(int));
    if (e != cudaSuccess) return launched(e, "qwz_device_error");
  }
  return QWZ_OK;
}

int qwz_nvfp4_append(const void* k, const void* v, void* k_cache, void* v_cache, void* k_scales,
                     void* v_scales, const int32_t* block_table, const int32_t* cache_seqlens,
                     int32_t table_width, int32_t append_len, int32_t num_kv_heads,
                     int32_t page_size, int32_t head_dim, int32_t num_pages, int32_t dtype,
                     void* stream) {
  int rc = check_dtype(dtype);
  if (rc) return rc;
  if (page_size != qwz::kPage || head_dim != qwz::kHeadDim || num_kv_heads != qwz::kKvHeads)
    return fail(QWZ_EINVAL, "NVFP4 writer is pinned to page 256, head_dim 256, 4 KV heads");
  if (!k || !v || !aligned(k, 16) || !aligned(v, 16))
    return fail(QWZ_EINVAL, "k and v must be non-null 16-byte aligned pointers");
  rc = check_nvfp4_cache(k_cache, v_cache, k_scales, v_scales, num_pages);
  if (rc) return rc;
  if (!block_table || !cache_seqlens) return fail(QWZ_EINVAL, "block_table and cache_seqlens are required");
  if (table_width <= 0) return fail(QWZ_EINVAL, "table_width must be positive");
  if (append_len < 0) return fail(QWZ_EINVAL, "append_len must be non-negative");
  qwz::AppendParams p{};
  p.k = k;
  p.v = v;
  p.k_cache = static_cast<uint8_t*>(k_cache);
  p.v_cache = static_cast<uint8_t*>(v_cache);
  p.k_scales = static_cast<uint8_t*>(k_scales);
  p.v_scales = static_cast<uint8_t*>(v_scales);
  p.block_table = block_table;
  p.seqlens = cache_seqlens;
  p.table_width = table_width;
  p.table_page_offset = 0;
  p.append_len = append_len;
  p.num_kv_heads = num_kv_heads;
  p.num_pages = num_pages;
  p.skip_foreign = 0;
  return launched(qwz::launch_nvfp4_append(p, dtype, as_stream(stream)), "qwz_nvfp4_append");
}

int qwz_nvfp4_append_shard(const void* k, const void* v, void* k_cache, void* v_cache,
                           void* k_scales, void* v_scales, const int32_t* block_table,
                           const int32_t* cache_seqlens, int32_t table_width,
                           int32_t table_page_offset, int32_t append_len, int32_t num_pages,
                           int32_t dtype, void* stream) {
  int rc = check_dtype(dtype);
  if (rc) return rc;
  if (!k || !v || !aligned(k, 16) || !aligned(v, 16))
    return fail(QWZ_EINVAL, "k and v must be non-null 16-byte aligned pointers");
  rc = check_nvfp4_cache(k_cache, v_cache, k_scales, v_scales, num_pages);
  if (rc) return rc;
  if (!block_table || !cache_seqlens) return fail(QWZ_EINVAL, "block_table and cache_seqlens are required");
  if (table_width <= 0 || table_page_offset < 0) return fail(QWZ_EINVAL, "bad table width/offset");
  if (append_len < 0) return fail(QWZ_EINVAL, "append_len must be non-negative");
  qwz::AppendParams p{};
  p.k = k;
  p.v = v;
  p.k_cache = static_cast<uint8_t*>(k_cache);
  p.v_cache = static_cast<uint8_t*>(v_cache);
  p.k_scales = static_cast<uint8_t*>(k_scales);
  p.v_scales = static_cast<uint8_t*>(v_scales);
  p.block_table = block_table;
  p.seqlens = cache_seqlens;
  p.table_width = table_width;
  p.table_page_offset = table_page_offset;
  p.append_len = append_len;
  p.num_kv_heads = qwz::kKvHeads;
  p.num_pages = num_pages;
  p.skip_foreign = 1;
  return launched(qwz::launch_nvfp4_append(p, dtype, as_stream(stream)), "qwz_nvfp4_append_shard");
}

int qwz_attn_split(const void* q, const void* k_cache, const void* v_cache,
                   const int32_t* block_table, const int32_t* cache_seqlens, void* out,
                   float* partial_o, float* partial_ml, const void* k_scales, const void* v_scales,
                   const void* h32, int32_t split_len, int32_t num_pages_per_seq,
                   int32_t num_splits, const void* sinks, void* global_scratch,
                   void* profile_scratch, int32_t q_len, int32_t num_pages, float sm_scale,
                   int32_t dtype, void* stream) {
  (void)out;
  (void)global_scratch;
  (void)profile_scratch;
  int rc = check_dtype(dtype);
  if (rc) return rc;
  if (h32 || sinks)
    return fail(QWZ_EINVAL, "h32 and sinks belong to the K8/V4 cache; they must be NULL for NVFP4");
  qwz::SplitParams p;
  rc = fill_split(p, q, k_cache, v_cache, k_scales, v_scales, block_table, cache_seqlens,
                  partial_o, partial_ml, num_pages_per_seq, num_pages, q_len, num_splits,
                  split_len, sm_scale);
  if (rc) return rc;
  return launched(qwz::launch_nvfp4_split(p, dtype, as_stream(stream)), "qwz_attn_split");
}

int qwz_attn_combine(const float* partial_o, const float* partial_ml, void* out, const void* h32,
                     int32_t num_splits, const void* sinks, int32_t q_len, int32_t dtype,
                     void* stream) {
  int rc = check_dtype(dtype);
  if (rc) return rc;
  if (h32 || sinks) return fail(QWZ_EINVAL, "h32 and sinks must be NULL for NVFP4");
  if (!partial_o || !partial_ml || !out) return fail(QWZ_EINVAL, "partial_o, partial_ml and out are required");
  if (!aligned(partial_o, 8) || !aligned(partial_ml, 4)) return fail(QWZ_EINVAL, "misaligned partials");
  if (q_len < 1 || q_len > 8) return fail(QWZ_EINVAL, "q_len must be in 1..8");
  if (num_splits < 1 || num_splits > 65535) return fail(QWZ_EINVAL, "num_splits must be in 1..65535");
  const qwz::CombineParams c =
      split_combine_params(partial_o, partial_ml, q_len * qwz::kQHeads, num_splits, out);
  return launched(qwz::launch_combine(c, qwz::kCombineFinal, dtype, as_stream(stream)), "qwz_attn_combine");
}

int qwz_nvfp4_attend(const void* q, const void* k, const void* v, void* k_cache, void* v_cache,
                     void* k_scales, void* v_scales, const int32_t* block_table,
                     const int32_t* cache_seqlens, void* out, float* partial_o, float* partial_ml,
                     int32_t table_width, int32_t num_pages, int32_t q_len, int32_t num_splits,
                     float sm_scale, int32_t dtype, void* stream) {
  int rc = check_dtype(dtype);
  if (rc) return rc;
  if (!out) return fail(QWZ_EINVAL, "out is required");
  qwz::SplitParams p;
  rc = fill_split(p, q, k_cache, v_cache, k_scales, v_scales, block_table, cache_seqlens,
                  partial_o, partial_ml, table_width, num_pages, q_len, num_splits, 0, sm_scale);
  if (rc) return rc;
  // the split kernel (decode or verify) writes the new rows itself, in the
  // CTAs whose pages hold them, before it reads those pages (one launch fewer)
  if (!k || !v || !aligned(k, 16) || !aligned(v, 16))
    return fail(QWZ_EINVAL, "k and v must be non-null 16-byte aligned pointers");
  p.app_k = k;
  p.app_v = v;
  rc = launched(qwz::launch_nvfp4_split(p, dtype, as_stream(stream)), "qwz_nvfp4_attend(split)");
  if (rc) return rc;
  const qwz::CombineParams c =
      split_combine_params(partial_o, partial_ml, q_len * qwz::kQHeads, num_splits, out);
  return launched(qwz::launch_combine(c, qwz::kCombineFinal, dtype, as_stream(stream)),
                  "qwz_nvfp4_attend(combine)");
}

int qwz_nvfp4_prefill(const void* q, const void* k_cache, const void* v_cache, const void* k_scales,
                      const void* v_scales, const int32_t* block_table, const int32_t* cache_seqlens,
                      void* out, int32_t table_width, int32_t num_pages, int32_t q_len, float sm_scale,
                      int32_t dtype, void* stream) {
  int rc = check_dtype(dtype);
  if (rc) return rc;
  if (!q || !aligned(q, 16) || !out || !aligned(out, 16))
    return fail(QWZ_EINVAL, "q and out must be non-null 16-byte aligned pointers");
  rc = check_nvfp4_cache(k_cache, v_cache, k_scales, v_scales, num_pages);
  if (rc) return rc;
  if (!block_table || !cache_seqlens) return fail(QWZ_EINVAL, "block_table and cache_seqlens are required");
  if (table_width <= 0) return fail(QWZ_EINVAL, "table_width must be positive");
  if (q_len < 1) return fail(QWZ_EINVAL, "q_len must be positive");
  if (!(sm_scale > 0.f) || !std::isfinite(sm_scale)) return fail(QWZ_EINVAL, "sm_scale must be positive and finite");
  qwz::PrefillParams p{};
  p.q = q;
  p.out = out;
  p.block_table = block_table;
  p.seqlens = cache_seqlens;
  p.table_width = table_width;
  p.num_pages = num_pages;
  p.q_len = q_len;
  p.sm_scale_log2 = sm_scale * kLog2e;
  const uint64_t rows = (uint64_t)num_pages * qwz::kPage;
  rc = encode_2d(&p.tm_kc, k_cache, qwz::kRowBytesCodes, rows, qwz::kCodeBytes, 64u, CU_TENSOR_MAP_SWIZZLE_128B);
  if (!rc) rc = encode_2d(&p.tm_vc, v_cache, qwz::kRowBytesCodes, rows, qwz::kCodeBytes, 64u, CU_TENSOR_MAP_SWIZZLE_128B);
  if (!rc) rc = encode_2d(&p.tm_ks, k_scales, qwz::kRowBytesScales, rows, qwz::kScaleBytes, 64u, CU_TENSOR_MAP_SWIZZLE_NONE);
  if (!rc) rc = encode_2d(&p.tm_vs, v_scales, qwz::kRowBytesScales, rows, qwz::kScaleBytes, 64u, CU_TENSOR_MAP_SWIZZLE_NONE);
  if (rc) return rc;
  return launched(qwz::launch_nvfp4_prefill(p, dtype, as_stream(stream)), "qwz_nvfp4_prefill");
}

int qwz_draft_prefill(const void* q, const void* k, const void* v, void* out, int32_t q_len, int32_t kv_len,
                      int64_t k_token_stride, int64_t v_token_stride, float sm_scale, void* stream) {
  if (!q || !aligned(q, 16) || !out || !aligned(out, 16))
    return fail(QWZ_EINVAL, "q and out must be non-null 16-byte aligned pointers");
  if (!k || !v || !aligned(k, 16) || !aligned(v, 16)) return fail(QWZ_EINVAL, "k and v must be non-null 16-byte aligned pointers");
  if (q_len < 1 || kv_len < q_len) return fail(QWZ_EINVAL, "need 1 <= q_len <= kv_len");
  const int64_t row = (int64_t)qwz::kKvHeads * qwz::kHeadDim;
  if (k_token_stride < row || v_token_stride < row || k_token_stride % 8 || v_token_stride % 8 ||
      k_token_stride > (int64_t(1) << 36) || v_token_stride > (int64_t(1) << 36))
    return fail(QWZ_EINVAL, "token strides must be multiples of 8 elements and at least 1024");
  if (!(sm_scale > 0.f) || !std::isfinite(sm_scale)) return fail(QWZ_EINVAL, "sm_scale must be positive and finite");
  qwz::PrefillParams p{};
  p.q = q;
  p.out = out;
  p.q_len = q_len;
  p.pre_len = kv_len - q_len;
  p.sm_scale_log2 = sm_scale * kLog2e;
  // FP16 rows as bytes: [kv_len rows, 2048 B used of the stride], boxes of
  // 128 B (64 head dims) x 64 tokens with the 128-byte swizzle
  int rc = encode_rows(&p.tm_kc, k, (uint64_t)row * 2, (uint64_t)k_token_stride * 2, (uint64_t)kv_len, 128u, 64u,
                       CU_TENSOR_MAP_SWIZZLE_128B);
  if (!rc) rc = encode_rows(&p.tm_vc, v, (uint64_t)row * 2, (uint64_t)v_token_stride * 2, (uint64_t)kv_len, 128u, 64u,
                            CU_TENSOR_MAP_SWIZZLE_128B);
  if (rc) return rc;
  return launched(qwz::launch_draft_prefill(p, as_stream(stream)), "qwz_draft_prefill");
}

int qwz_attn_shard_partial(const void* q, const void* k_cache, const void* v_cache,
                           const void* k_scales, const void* v_scales, const int32_t* block_table,
                           const int32_t* cache_seqlens, float* partial_o, float* partial_ml,
                           float* send_buf, int32_t table_width, int32_t num_pages,
                           int32_t tok_begin, int32_t tok_span, int32_t q_len, int32_t num_splits,
                           float sm_scale, int32_t dtype, void* stream) {
  int rc = check_dtype(dtype);
  if (rc) return rc;
  if (!send_buf || !aligned(send_buf, 8)) return fail(QWZ_EINVAL, "send_buf must be non-null and 8-byte aligned");
  if (tok_begin < 0 || tok_begin % qwz::kPage != 0) return fail(QWZ_EINVAL, "tok_begin must be a non-negative multiple of 256");
  if (tok_span <= 0) return fail(QWZ_EINVAL, "tok_span must be positive");
  qwz::SplitParams p;
  rc = fill_split(p, q, k_cache, v_cache, k_scales, v_scales, block_table, cache_seqlens,
                  partial_o, partial_ml, table_width, num_pages, q_len, num_splits, 0, sm_scale);
  if (rc) return rc;
  p.tok_begin = tok_begin;
  p.tok_span = tok_span;
  p.table_page_offset = tok_begin / qwz::kPage;
  rc = launched(qwz::launch_nvfp4_split(p, dtype, as_stream(stream)), "qwz_attn_shard_partial(split)");
  if (rc) return rc;
  const qwz::CombineParams c =
      split_combine_params(partial_o, partial_ml, q_len * qwz::kQHeads, num_splits, send_buf);
  return launched(qwz::launch_combine(c, qwz::kCombinePartial, dtype, as_stream(stream)),
                  "qwz_attn_shard_partial(combine)");
}

int qwz_lse_combine_gathered(const float* gathered, void* out, int32_t world, int32_t q_len,
                             int32_t dtype, void* stream) {
  int rc = check_dtype(dtype);
  if (rc) return rc;
  if (!gathered || !out || !aligned(gathered, 8)) return fail(QWZ_EINVAL, "gathered (8-byte aligned) and out are required");
  if (world < 1 || world > 65535) return fail(QWZ_EINVAL, "world must be in 1..65535");
  if (q_len < 1 || q_len > 8) return fail(QWZ_EINVAL, "q_len must be in 1..8");
  const int rows = q_len * qwz::kQHeads;
  qwz::CombineParams c{};
  c.po = gathered + 2;
  c.pml = gathered;
  c.o_row = qwz::kHeadDim + 2;
  c.o_split = (long long)rows * (qwz::kHeadDim + 2);
  c.ml_row = qwz::kHeadDim + 2;
  c.ml_split = (long long)rows * (qwz::kHeadDim + 2);
  c.rows = rows;
  c.num_splits = world;
  c.out = out;
  return launched(qwz::launch_combine(c, qwz::kCombineFinal, dtype, as_stream(stream)),
                  "qwz_lse_combine_gathered");
}

// Draft split + combine; k_new / v_new / position set: fused shadow write.
static int fp8_draft(const void* q, const void* k8, const void* v8, const float* k_scale, const float* v_scale,
                     const int32_t* length, float* part, float* stat, void* out, int32_t splits, int32_t capacity,
                     void* stream, const void* k_new, const void* v_new, const int32_t* position, const char* what) {
  if (!q || !aligned(q, 16)) return fail(QWZ_EINVAL, "q must be non-null and 16-byte aligned");
  if (!k8 || !v8 || !aligned(k8, 16) || !aligned(v8, 16)) return fail(QWZ_EINVAL, "k8 and v8 must be non-null and 16-byte aligned");
  if (!length || !part || !stat || !out) return fail(QWZ_EINVAL, "length, part, stat and out are required");
  if (!aligned(part, 16) || !aligned(stat, 8)) return fail(QWZ_EINVAL, "misaligned part/stat");
  if (splits < 1 || splits > 65535) return fail(QWZ_EINVAL, "splits must be in 1..65535");
  if (capacity <= 0 || (long long)capacity * qwz::kKvHeads > 0x7fffffffLL) return fail(QWZ_EINVAL, "capacity out of range");
  qwz::SplitParams p{};
  p.q = q;
  p.k_codes = static_cast<const uint8_t*>(k8);
  p.v_codes = static_cast<const uint8_t*>(v8);
  p.k_page_scale = k_scale;
  p.v_page_scale = v_scale;
  p.seqlens = length;
  p.partial_o = part;
  p.partial_ml = stat;
  p.capacity = capacity;
  p.q_len = 1;
  p.len_add = 0;
  p.tok_begin = 0;
  p.tok_span = capacity;
  p.split_len = 0;
  p.num_splits = splits;
  p.sm_scale_log2 = (1.0f / 16.0f) * kLog2e;
  p.app_k = k_new;
  p.app_v = v_new;
  p.app_slot = position;
  // [capacity, 4 x 256 B] views; boxes of 128 head-dim bytes x 128 tokens.
  const uint64_t row_bytes = (uint64_t)qwz::kKvHeads * qwz::kHeadDim;
  int rc = encode_2d(&p.tm_kc, k8, row_bytes, (uint64_t)capacity, 128, 128, CU_TENSOR_MAP_SWIZZLE_128B);
  if (!rc) rc = encode_2d(&p.tm_vc, v8, row_bytes, (uint64_t)capacity, 128, 128, CU_TENSOR_MAP_SWIZZLE_128B);
  if (rc) return rc;
  rc = launched(qwz::launch_fp8_split(p, as_stream(stream)), what);
  if (rc) return rc;
  const qwz::CombineParams c = split_combine_params(part, stat, qwz::kQHeads, splits, out);
  return launched(qwz::launch_combine(c, qwz::kCombineFinal, QWZ_DTYPE_F16, as_stream(stream)),
                  what);
}

int qwz_fp8_draft_decode(const void* q, const void* k8, const void* v8, const float* k_scale,
                         const float* v_scale, const int32_t* length, float* part, float* stat,
                         void* out, int32_t splits, int32_t capacity, void* stream) {
  return fp8_draft(q, k8, v8, k_scale, v_scale, length, part, stat, out, splits, capacity, stream, nullptr,
                   nullptr, nullptr, "qwz_fp8_draft_decode");
}

int qwz_fp8_draft_step(const void* q, const void* k_new, const void* v_new, const int32_t* position, void* k8,
                       void* v8, const float* k_scale, const float* v_scale, const int32_t* length, float* part,
                       float* stat, void* out, int32_t splits, int32_t capacity, void* stream) {
  if (!k_new || !v_new || !aligned(k_new, 16) || !aligned(v_new, 16))
    return fail(QWZ_EINVAL, "k_new and v_new must be non-null and 16-byte aligned");
  if (!position) return fail(QWZ_EINVAL, "position is required");
  return fp8_draft(q, k8, v8, k_scale, v_scale, length, part, stat, out, splits, capacity, stream, k_new, v_new,
                   position, "qwz_fp8_draft_step");
}

int qwz_fp8_shadow_write(const void* k, const void* v, void* k8, void* v8, const float* k_scale,
                         const float* v_scale, const int32_t* position, int32_t capacity,
                         int32_t dtype, void* stream) {
  int rc = check_dtype(dtype);
  if (rc) return rc;
  if (!k || !v || !aligned(k, 16) || !aligned(v, 16)) return fail(QWZ_EINVAL, "k and v must be non-null and 16-byte aligned");
  if (!k8 || !v8 || !aligned(k8, 8) || !aligned(v8, 8)) return fail(QWZ_EINVAL, "k8 and v8 must be non-null and 8-byte aligned");
  if (!position) return fail(QWZ_EINVAL, "position is required");
  if (capacity <= 0) return fail(QWZ_EINVAL, "capacity must be positive");
  qwz::Fp8WriteParams p{};
  p.k = k;
  p.v = v;
  p.k8 = static_cast<uint8_t*>(k8);
  p.v8 = static_cast<uint8_t*>(v8);
  p.k_page_scale = k_scale;
  p.v_page_scale = v_scale;
  p.position = position;
  p.capacity = capacity;
  p.num_kv_heads = qwz::kKvHeads;
  return launched(qwz::launch_fp8_write(p, dtype, as_stream(stream)), "qwz_fp8_shadow_write");
}

int qwz_nvfp4_gather(const void* packed, const void* scales, const int32_t* block_table,
                     const int32_t* seq_lens, void* output, int32_t batch, int32_t max_tokens,
                     int32_t table_width, int32_t n_heads, int32_t head_dim, int32_t page_size,
                     void* stream) {
  if (!packed || !scales || !block_table || !seq_lens || !output)
    return fail(QWZ_EINVAL, "all pointers are required");
  if (!aligned(packed, 4) || !aligned(output, 16)) return fail(QWZ_EINVAL, "packed must be 4-byte and output 16-byte aligned");
  if (batch < 0 || max_tokens < 0 || table_width <= 0 || n_heads <= 0 || page_size <= 0)
    return fail(QWZ_EINVAL, "sizes must be positive");
  if (head_dim <= 0 || head_dim % 16 != 0) return fail(QWZ_EINVAL, "head_dim must be a positive multiple of 16");
  qwz::GatherParams p{};
  p.packed = static_cast<const uint8_t*>(packed);
  p.scales = static_cast<const uint8_t*>(scales);
  p.block_table = block_table;
  p.seq_lens = seq_lens;
  p.out = static_cast<__half*>(output);
  p.batch = batch;
  p.max_tokens = max_tokens;
  p.table_width = table_width;
  p.n_heads = n_heads;
  p.head_dim = head_dim;
  p.page_size = page_size;
  return launched(qwz::launch_nvfp4_gather(p, as_stream(stream)), "qwz_nvfp4_gather");
}


// ------------------------------------------------ sharded decode over NVLink
int64_t qwz_peer_buffer_bytes(int32_t world, int32_t q_len) {
  if (world < 1 || world > qwz::kMaxWorld || q_len < 1 || q_len > 8) return 0;
  const int64_t rows = (int64_t)q_len * qwz::kQHeads;
  return 2 * (int64_t)world * rows * (qwz::kHeadDim + 2) * 8;  // two epoch-parity halves of tagged words
}

int qwz_peer_alloc(int64_t bytes, void** dev_ptr, uint8_t* ipc_handle) {
  if (bytes <= 0 || !dev_ptr || !ipc_handle) return fail(QWZ_EINVAL, "bytes > 0, dev_ptr and ipc_handle are required");
  void* p = nullptr;
  cudaError_t e = cudaMalloc(&p, (size_t)bytes);
  if (e == cudaSuccess) e = cudaMemset(p, 0, (size_t)bytes);
  if (e == cudaSuccess) e = cudaDeviceSynchronize();
  cudaIpcMemHandle_t h;
  if (e == cudaSuccess) e = cudaIpcGetMemHandle(&h, p);
  if (e != cudaSuccess) {
    if (p) cudaFree(p);
    return launched(e, "qwz_peer_alloc");
  }
  static_assert(sizeof(cudaIpcMemHandle_t) == 64, "64-byte IPC handle");
  std::memcpy(ipc_handle, &h, sizeof(h));
  *dev_ptr = p;
  return QWZ_OK;
}

int qwz_peer_open(const uint8_t* ipc_handle, void** dev_ptr) {
  if (!ipc_handle || !dev_ptr) return fail(QWZ_EINVAL, "ipc_handle and dev_ptr are required");
  cudaIpcMemHandle_t h;
  std::memcpy(&h, ipc_handle, sizeof(h));
  return launched(cudaIpcOpenMemHandle(dev_ptr, h, cudaIpcMemLazyEnablePeerAccess), "qwz_peer_open");
}

int qwz_peer_close(void* peer_ptr) {
  if (!peer_ptr) return fail(QWZ_EINVAL, "peer_ptr is null");
  return launched(cudaIpcCloseMemHandle(peer_ptr), "qwz_peer_close");
}

int qwz_peer_free(void* dev_ptr) {
  if (!dev_ptr) return fail(QWZ_EINVAL, "dev_ptr is null");
  return launched(cudaFree(dev_ptr), "qwz_peer_free");
}

int qwz_attn_shard_split(const void* q, const void* k, const void* v, void* k_cache, void* v_cache,
                         void* k_scales, void* v_scales, const int32_t* block_table,
                         const int32_t* cache_seqlens, float* partial_o, float* partial_ml,
                         int32_t table_width, int32_t num_pages, int32_t tok_begin, int32_t tok_span,
                         int32_t q_len, int32_t num_splits, float sm_scale, int32_t dtype, void* stream) {
  int rc = check_dtype(dtype);
  if (rc) return rc;
  if (tok_begin < 0 || tok_begin % qwz::kPage != 0) return fail(QWZ_EINVAL, "tok_begin must be a non-negative multiple of 256");
  if (tok_span <= 0) return fail(QWZ_EINVAL, "tok_span must be positive");
  if (!k || !v || !aligned(k, 16) || !aligned(v, 16))
    return fail(QWZ_EINVAL, "k and v must be non-null 16-byte aligned pointers");
  qwz::SplitParams p;
  rc = fill_split(p, q, k_cache, v_cache, k_scales, v_scales, block_table, cache_seqlens, partial_o,
                  partial_ml, table_width, num_pages, q_len, num_splits, 0, sm_scale);
  if (rc) return rc;
  p.tok_begin = tok_begin;
  p.tok_span = tok_span;
  p.table_page_offset = tok_begin / qwz::kPage;
  // the shard that owns a new row's page writes it inside the split kernel
  p.app_k = k;
  p.app_v = v;
  return launched(qwz::launch_nvfp4_split(p, dtype, as_stream(stream)), "qwz_attn_shard_split");
}

namespace {
constexpr int64_t kExchangeTimeoutDefaultNs = 500ll * 1000 * 1000;  // 0.5 s
constexpr int64_t kExchangeTimeoutMaxNs = 10ll * 1000 * 1000 * 1000;  // 10 s

int fill_exchange(qwz::ExchangeParams& x, int32_t num_splits, int32_t q_len, const uint64_t* peers,
                  int64_t buffer_bytes, int32_t world, int64_t timeout_ns) {
  if (world < 1 || world > qwz::kMaxWorld) return fail(QWZ_EINVAL, "world must be in 1..8");
  if (q_len < 1 || q_len > 8) return fail(QWZ_EINVAL, "q_len must be in 1..8");
  if (num_splits < 1 || num_splits > 65535) return fail(QWZ_EINVAL, "num_splits must be in 1..65535");
  if (!peers) return fail(QWZ_EINVAL, "peers (host array of buffer addresses) is required");
  // the buffers are laid out for one (world, q_len): any other pair would
  // store past their end or read a stale record of the same epoch
  if (buffer_bytes != qwz_peer_buffer_bytes(world, q_len))
    return fail(QWZ_EINVAL, "buffer_bytes must be qwz_peer_buffer_bytes(world, q_len) of the buffers' allocation");
  if (timeout_ns < 0 || timeout_ns > kExchangeTimeoutMaxNs)
    return fail(QWZ_EINVAL, "timeout_ns must be in 0..1e10 (0: the default 0.5 s)");
  x = qwz::ExchangeParams{};
  x.timeout_ns = (unsigned long long)(timeout_ns == 0 ? kExchangeTimeoutDefaultNs : timeout_ns);
  for (int g = 0; g < world; ++g) {
    if (!peers[g] || peers[g] % 16) return fail(QWZ_EINVAL, "every peer buffer address must be non-null and 16-byte aligned");
    x.peers[g] = peers[g];
  }
  x.num_splits = num_splits;
  x.rows = q_len * qwz::kQHeads;
  x.world = world;
  return QWZ_OK;
}
}  // namespace

int qwz_shard_exchange_combine(const float* partial_o, const float* partial_ml, int32_t num_splits,
                               int32_t q_len, const uint64_t* peers, int64_t buffer_bytes, uint32_t* epochs,
                               int32_t rank, int32_t world, void* out, int64_t timeout_ns, int32_t dtype,
                               void* stream) {
  int rc = check_dtype(dtype);
  if (rc) return rc;
  if (!partial_o || !partial_ml || !epochs || !out) return fail(QWZ_EINVAL, "partials, epochs and out are required");
  qwz::ExchangeParams x;
  rc = fill_exchange(x, num_splits, q_len, peers, buffer_bytes, world, timeout_ns);
  if (rc) return rc;
  if (rank < 0 || rank >= world) return fail(QWZ_EINVAL, "rank must be in 0..world-1");
  x.po[0] = partial_o;
  x.pml[0] = partial_ml;
  x.epochs[0] = epochs;
  x.out[0] = out;
  x.rank0 = rank;
  return launched(qwz::launch_shard_exchange(x, 0, dtype, as_stream(stream)), "qwz_shard_exchange_combine");
}

int qwz_shard_exchange_combine_emulated(const float* partial_o, const float* partial_ml,
                                        int64_t rank_stride_splits, int32_t num_splits, int32_t q_len,
                                        const uint64_t* peers, int64_t buffer_bytes, uint32_t* epochs,
                                        void* out, int32_t world, int64_t timeout_ns, int32_t dtype,
                                        void* stream) {
  int rc = check_dtype(dtype);
  if (rc) return rc;
  if (!partial_o || !partial_ml || !epochs || !out) return fail(QWZ_EINVAL, "partials, epochs and out are required");
  qwz::ExchangeParams x;
  rc = fill_exchange(x, num_splits, q_len, peers, buffer_bytes, world, timeout_ns);
  if (rc) return rc;
  if (rank_stride_splits < num_splits) return fail(QWZ_EINVAL, "rank_stride_splits must be >= num_splits");
  const int64_t rows = (int64_t)q_len * qwz::kQHeads;
  const size_t esize = 2;  // FP16 / BF16
  for (int g = 0; g < world; ++g) {
    x.po[g] = partial_o + (size_t)g * rows * rank_stride_splits * qwz::kHeadDim;
    x.pml[g] = partial_ml + (size_t)g * rows * rank_stride_splits * 2;
    x.epochs[g] = epochs + (size_t)g * rows;
    x.out[g] = static_cast<uint8_t*>(out) + (size_t)g * rows * qwz::kHeadDim * esize;
  }
  x.rank0 = 0;
  return launched(qwz::launch_shard_exchange(x, 1, dtype, as_stream(stream)),
                  "qwz_shard_exchange_combine_emulated");
}

}  // extern "C"
