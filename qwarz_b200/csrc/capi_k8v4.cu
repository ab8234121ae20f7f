// C ABI of the K8/V4 cache path (k8v4.cu): the writer, the split and the
// rotating combine of the reference's Attention64 slot, which keeps the same
// 15-argument split order and the combine order
// (docs/superpowers/specs/2026-09-11-qwasar-attention-kernel.md:62-74), and
// the reader used by the parity tests.  Part of the single translation unit
// qwz_b200.cu; it uses the argument checks and TMA helpers of capi.cu.

#include "qwz_common.cuh"
#include "qwz_kernels.h"
#include "../../include/qwz_b200.h"

namespace {

int check_k8v4_cache(const void* kc, const void* vc, const void* ks, const void* vs, int32_t num_pages) {
  if (!kc || !vc || !ks || !vs) return fail(QWZ_EINVAL, "K8/V4 caches and scales are required (non-null)");
  if (!aligned(kc, 16) || !aligned(vc, 16) || !aligned(ks, 16) || !aligned(vs, 16))
    return fail(QWZ_EINVAL, "K8/V4 caches and scales must be 16-byte aligned");
  if (num_pages <= 0) return fail(QWZ_EINVAL, "num_pages must be positive");
  if ((long long)num_pages * qwz::kPage > 0x7fffffffLL) return fail(QWZ_EINVAL, "num_pages too large");
  return QWZ_OK;
}

int check_h32(const void* h32) {
  if (!h32 || !aligned(h32, 16))
    return fail(QWZ_EINVAL, "h32 (the FP32 [32, 32] rotation) is required and must be 16-byte aligned");
  return QWZ_OK;
}

}  // namespace

extern "C" {

int qwz_k8v4_append(const void* k, const void* v, void* k_cache, void* v_cache, void* k_scales,
                    void* v_scales, const int32_t* block_table, const int32_t* cache_seqlens,
                    int32_t table_width, int32_t num_pages, int32_t append_len, int32_t dtype,
                    void* stream) {
  int rc = check_dtype(dtype);
  if (rc) return rc;
  rc = check_k8v4_cache(k_cache, v_cache, k_scales, v_scales, num_pages);
  if (rc) return rc;
  if (!k || !v || !aligned(k, 2) || !aligned(v, 2)) return fail(QWZ_EINVAL, "k and v rows are required");
  if (!block_table || !cache_seqlens) return fail(QWZ_EINVAL, "block_table and cache_seqlens are required");
  if (table_width <= 0) return fail(QWZ_EINVAL, "table_width must be positive");
  if (append_len < 0 || append_len > 65535) return fail(QWZ_EINVAL, "append_len must be in 0..65535");
  qwz::K8v4AppendParams p{};
  p.k = k;
  p.v = v;
  p.k_cache = static_cast<uint32_t*>(k_cache);
  p.v_cache = static_cast<uint32_t*>(v_cache);
  p.k_scales = static_cast<__half*>(k_scales);
  p.v_scales = static_cast<__half*>(v_scales);
  p.block_table = block_table;
  p.seqlens = cache_seqlens;
  p.table_width = table_width;
  p.num_pages = num_pages;
  p.append_len = append_len;
  return launched(qwz::launch_k8v4_append(p, dtype, as_stream(stream)), "qwz_k8v4_append");
}

int qwz_k8v4_split(const void* q, const void* k_cache, const void* v_cache, const int32_t* block_table,
                   const int32_t* cache_seqlens, void* out, float* partial_o, float* partial_ml,
                   const void* k_scales, const void* v_scales, const void* h32, int32_t split_len,
                   int32_t num_pages_per_seq, int32_t num_splits, const void* sinks, void* global_scratch,
                   void* profile_scratch, int32_t q_len, int32_t num_pages, float sm_scale, int32_t dtype,
                   void* stream) {
  (void)out;
  (void)global_scratch;
  (void)profile_scratch;
  int rc = check_dtype(dtype);
  if (rc) return rc;
  if (sinks) return fail(QWZ_EINVAL, "attention sinks are not supported (sinks must be NULL)");
  rc = check_h32(h32);
  if (rc) return rc;
  if (!q || !aligned(q, 16)) return fail(QWZ_EINVAL, "q must be a non-null 16-byte aligned pointer");
  rc = check_k8v4_cache(k_cache, v_cache, k_scales, v_scales, num_pages);
  if (rc) return rc;
  if (!block_table || !cache_seqlens) return fail(QWZ_EINVAL, "block_table and cache_seqlens are required");
  if (!partial_o || !partial_ml || !aligned(partial_o, 16) || !aligned(partial_ml, 8))
    return fail(QWZ_EINVAL, "partial_o (16-byte aligned) and partial_ml are required");
  if (num_pages_per_seq <= 0) return fail(QWZ_EINVAL, "num_pages_per_seq (table width) must be positive");
  if (q_len < 1 || q_len > 8) return fail(QWZ_EINVAL, "q_len must be in 1..8");
  if (num_splits < 1 || num_splits > 65535) return fail(QWZ_EINVAL, "num_splits must be in 1..65535");
  if (split_len < 0 || split_len % qwz::kPage != 0)
    return fail(QWZ_EINVAL, "split_len must be 0 or a positive multiple of 256");
  if (!(sm_scale > 0.f) || !std::isfinite(sm_scale)) return fail(QWZ_EINVAL, "sm_scale must be positive and finite");
  qwz::SplitParams p{};
  p.q = q;
  p.k_codes = static_cast<const uint8_t*>(k_cache);
  p.v_codes = static_cast<const uint8_t*>(v_cache);
  p.k_scales = static_cast<const uint8_t*>(k_scales);
  p.v_scales = static_cast<const uint8_t*>(v_scales);
  p.h32 = static_cast<const float*>(h32);
  p.block_table = block_table;
  p.seqlens = cache_seqlens;
  p.partial_o = partial_o;
  p.partial_ml = partial_ml;
  p.table_width = num_pages_per_seq;
  p.table_page_offset = 0;
  p.num_pages = num_pages;
  p.q_len = q_len;
  p.len_add = q_len;
  p.tok_begin = 0;
  p.tok_span = 0x7fffffff;
  p.split_len = split_len;
  p.num_splits = num_splits;
  p.sm_scale_log2 = sm_scale * kLog2e;
  // [P*256 token rows] views: K words 1024 B, V words 512 B, scales 64 B;
  // boxes of 128 tokens x (128 B of K or V words | 16 B of one head's scales)
  const uint64_t rows = (uint64_t)num_pages * qwz::kPage;
  rc = encode_2d(&p.tm_kc, k_cache, 1024, rows, 128u, 128u, CU_TENSOR_MAP_SWIZZLE_128B);
  if (!rc) rc = encode_2d(&p.tm_vc, v_cache, 512, rows, 128u, 128u, CU_TENSOR_MAP_SWIZZLE_128B);
  if (!rc) rc = encode_2d(&p.tm_ks, k_scales, 64, rows, 16u, 128u, CU_TENSOR_MAP_SWIZZLE_NONE);
  if (!rc) rc = encode_2d(&p.tm_vs, v_scales, 64, rows, 16u, 128u, CU_TENSOR_MAP_SWIZZLE_NONE);
  if (rc) return rc;
  return launched(qwz::launch_k8v4_split(p, dtype, as_stream(stream)), "qwz_k8v4_split");
}

int qwz_k8v4_combine(const float* partial_o, const float* partial_ml, void* out, const void* h32,
                     int32_t num_splits, const void* sinks, int32_t q_len, int32_t dtype, void* stream) {
  int rc = check_dtype(dtype);
  if (rc) return rc;
  if (sinks) return fail(QWZ_EINVAL, "attention sinks are not supported (sinks must be NULL)");
  rc = check_h32(h32);
  if (rc) return rc;
  if (!partial_o || !partial_ml || !out) return fail(QWZ_EINVAL, "partial_o, partial_ml and out are required");
  if (!aligned(partial_o, 8) || !aligned(partial_ml, 4)) return fail(QWZ_EINVAL, "misaligned partials");
  if (q_len < 1 || q_len > 8) return fail(QWZ_EINVAL, "q_len must be in 1..8");
  if (num_splits < 1 || num_splits > 65535) return fail(QWZ_EINVAL, "num_splits must be in 1..65535");
  qwz::CombineParams c = split_combine_params(partial_o, partial_ml, q_len * qwz::kQHeads, num_splits, out);
  c.h32 = static_cast<const float*>(h32);
  return launched(qwz::launch_combine(c, qwz::kCombineRotate, dtype, as_stream(stream)), "qwz_k8v4_combine");
}

int qwz_k8v4_gather(const void* words, const void* scales, const int32_t* block_table, int32_t table_width,
                    int32_t num_pages, int32_t length, int32_t bits, void* out, void* stream) {
  if (!words || !scales || !block_table || !out) return fail(QWZ_EINVAL, "words, scales, block_table and out are required");
  if (!aligned(words, 4) || !aligned(scales, 2) || !aligned(out, 2))
    return fail(QWZ_EINVAL, "words must be 4-byte aligned, scales and out 2-byte aligned");
  if (bits != 4 && bits != 8) return fail(QWZ_EINVAL, "bits must be 8 (K) or 4 (V)");
  if (table_width <= 0 || num_pages <= 0 || length < 0) return fail(QWZ_EINVAL, "bad table width, pool or length");
  if ((long long)length > (long long)table_width * qwz::kPage)
    return fail(QWZ_EINVAL, "length exceeds the pages the table maps");
  return launched(qwz::launch_k8v4_gather(static_cast<const uint32_t*>(words), static_cast<const __half*>(scales),
                                          block_table, table_width, num_pages, length, bits,
                                          static_cast<__half*>(out), as_stream(stream)),
                  "qwz_k8v4_gather");
}

}  // extern "C"
