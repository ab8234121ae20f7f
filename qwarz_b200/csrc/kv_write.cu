// KV writers and the NVFP4 dequant gather, sm_100a.
//
// nvfp4_append_kernel replaces the NVFP4 page writer the reference calls at
// src/qwasar_runtime/xqa.py:356-379 (ExLlamaV3 `_paged_kv_update_nvfp4_kernel`,
// not vendored).  For new row i < append_len and KV head h it writes token
// pos = cache_seqlens[0] + i into page block_table[pos / 256] at offset
// pos % 256, with the block quantisation of nvfp4_quant.cuh.
//
// fp8_write_kernel replaces the FP8 shadow write of engine/forward/draft.py:
// 359-366 (`_fp8`: clamp to +-448, cast to E4M3, draft.py:209-210) with an
// optional per-(page, head) scale: e = E4M3(clamp(x / scale, +-448)), sign
// kept (so it is bit-identical to torch's cast when scale == 1).
//
// nvfp4_gather_kernel mirrors the reference oracle dequant
// `_gather_nvfp4_kernel` (xqa.py:73-143) using the same conversion path as
// the attention kernels, so a bit-exact check of it validates their dequant.

#include "nvfp4_quant.cuh"
#include "qwz_kernels.h"

namespace qwz {

using namespace quant;

// grid (append_len, num_kv_heads), block 64: warp 0 writes K, warp 1 writes V.
template <typename T>
__global__ void __launch_bounds__(64) nvfp4_append_kernel(const AppendParams p) {
  const int i = blockIdx.x, h = blockIdx.y;
  const int tensor = threadIdx.x >> 5, lane = threadIdx.x & 31;
  griddep_wait();               // the new rows come from the previous kernel
  griddep_launch_dependents();  // the attention kernel may begin its launch
  const int pos = __ldg(p.seqlens) + i;
  const int lp = (pos >> 8) - p.table_page_offset;
  if (pos < 0 || lp < 0 || lp >= p.table_width) {
    if (threadIdx.x == 0 && !p.skip_foreign) flag_error(kErrTableRange);
    return;
  }
  const int pp = __ldg(p.block_table + lp);
  if (pp < 0 || pp >= p.num_pages) {
    if (threadIdx.x == 0) flag_error(kErrPageRange);
    return;
  }
  const int off = pos & (kPage - 1);
  const T* src = reinterpret_cast<const T*>(tensor ? p.v : p.k) + ((size_t)i * p.num_kv_heads + h) * kHeadDim;
  const size_t row = ((size_t)pp * kPage + off) * p.num_kv_heads + h;
  quantize_row_lane<T>(src, (tensor ? p.v_cache : p.k_cache) + row * kCodeBytes,
                       (tensor ? p.v_scales : p.k_scales) + row * kScaleBytes, lane);
}

// grid (num_kv_heads), block 64: warp 0 writes K, warp 1 writes V.
template <typename T>
__global__ void __launch_bounds__(64) fp8_write_kernel(const Fp8WriteParams p) {
  const int h = blockIdx.x;
  const int tensor = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int slot = __ldg(p.position);
  if (slot < 0 || slot >= p.capacity) {
    if (threadIdx.x == 0) flag_error(kErrSlotRange);
    return;
  }
  const float* ps = tensor ? p.v_page_scale : p.k_page_scale;
  const float scale = ps ? __ldg(ps + (slot >> 8) * p.num_kv_heads + h) : 1.f;
  const T* src = reinterpret_cast<const T*>(tensor ? p.v : p.k) + (size_t)h * kHeadDim + lane * 8;
  const uint2 e = fp8_shadow8<T>(src, scale);
  uint8_t* dst = (tensor ? p.v8 : p.k8) + ((size_t)slot * p.num_kv_heads + h) * kHeadDim + lane * 8;
  *reinterpret_cast<uint2*>(dst) = e;
}

// One warp per (batch, token, head); lane handles 8 head-dim elements per
// 256-wide pass.
__global__ void __launch_bounds__(128) nvfp4_gather_kernel(const GatherParams p) {
  const long long unit = (long long)blockIdx.x * 4 + (threadIdx.x >> 5);
  const long long total = (long long)p.batch * p.max_tokens * p.n_heads;
  if (unit >= total) return;
  const int lane = threadIdx.x & 31;
  const int head = (int)(unit % p.n_heads);
  const long long bt = unit / p.n_heads;
  const int batch = (int)(bt / p.max_tokens), token = (int)(bt % p.max_tokens);
  if (token >= __ldg(p.seq_lens + batch)) return;
  const int lp = token / p.page_size, off = token - lp * p.page_size;
  if (lp >= p.table_width) {
    if (lane == 0) flag_error(kErrTableRange);
    return;
  }
  const int pp = __ldg(p.block_table + (size_t)batch * p.table_width + lp);
  const size_t row = ((size_t)pp * p.page_size + off) * p.n_heads + head;
  const uint8_t* codes = p.packed + row * (p.head_dim / 2);
  const uint8_t* sc = p.scales + row * (p.head_dim / 16);
  __half* out = p.out + ((size_t)(batch * (long long)p.max_tokens + token) * p.n_heads + head) * p.head_dim;
  for (int d0 = lane * 8; d0 < p.head_dim; d0 += 256) {
    uint32_t w = *reinterpret_cast<const uint32_t*>(codes + d0 / 2);
    // The reference negates with 0 - magnitude, so code 8 is +0: clear the
    // sign bit of every zero-magnitude nibble before the hardware convert.
    const uint32_t mag = w & 0x77777777u;
    const uint32_t nonzero = (mag | (mag >> 1) | (mag >> 2)) & 0x11111111u;
    w = mag | (w & (nonzero << 3));
    uint32_t h[4];
    e2m1x8_to_f16x2x4(w, h);
    const uint32_t sb = sc[d0 / 16];
    uint32_t s2, unused;
    e4m3x4_to_f16x2x2(sb | (sb << 8), s2, unused);
    uint4 v;
    v.x = hmul2_u32(h[0], s2);
    v.y = hmul2_u32(h[1], s2);
    v.z = hmul2_u32(h[2], s2);
    v.w = hmul2_u32(h[3], s2);
    *reinterpret_cast<uint4*>(out + d0) = v;
  }
}

cudaError_t launch_nvfp4_append(const AppendParams& p, int dtype, cudaStream_t stream) {
  if (p.append_len <= 0) return cudaSuccess;
  const dim3 grid(p.append_len, p.num_kv_heads);
  if (dtype == kDtypeBF16) return launch_pdl(nvfp4_append_kernel<__nv_bfloat16>, grid, dim3(64), 0, stream, p);
  return launch_pdl(nvfp4_append_kernel<__half>, grid, dim3(64), 0, stream, p);
}

cudaError_t launch_fp8_write(const Fp8WriteParams& p, int dtype, cudaStream_t stream) {
  dim3 grid(p.num_kv_heads);
  if (dtype == kDtypeBF16)
    fp8_write_kernel<__nv_bfloat16><<<grid, 64, 0, stream>>>(p);
  else
    fp8_write_kernel<__half><<<grid, 64, 0, stream>>>(p);
  return cudaGetLastError();
}

cudaError_t launch_nvfp4_gather(const GatherParams& p, cudaStream_t stream) {
  const long long units = (long long)p.batch * p.max_tokens * p.n_heads;
  if (units <= 0) return cudaSuccess;
  const long long blocks = (units + 3) / 4;
  if (blocks > 0x7fffffffLL) return cudaErrorInvalidValue;
  nvfp4_gather_kernel<<<(unsigned)blocks, 128, 0, stream>>>(p);
  return cudaGetLastError();
}

}  // namespace qwz
