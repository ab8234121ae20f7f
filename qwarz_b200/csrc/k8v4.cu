// K8/V4 quantised-cache attention for sm_100a: the writer, the format policy
// with which the tcgen05 split kernel of attn_verify_tc.cu reads this cache
// (decode and verify, q_len 1..8), and the reader used by the parity tests.
//
// The cache is ExLlamaV3's CacheLayer_quant with 8-bit K and 4-bit V, the
// MTP draft cache the reference selects in src/qwasar_runtime/xqa.py:926-961
// and the cache of its Attention64 split/combine slot
// (docs/superpowers/specs/2026-09-11-qwasar-attention-kernel.md:62-74).
//   k_cache int32 [P, 256, 256]   v_cache int32 [P, 256, 128]
//   k_scales / v_scales FP16 [P, 256, 32]   (src/qwasar_bench/prefill_flash.py:32-44)
// Each (token, KV head, 32-dim block) holds 32 codes of b bits (b = 8 for K,
// 4 for V) in the rotated domain R = H32 / sqrt(32), stored as b bit-plane
// words (word i = bit i of the 32 codes, bit t = element t) at
// (head * 8 + block) * b of the token's row, with one FP16 scale at
// head * 8 + block.  The reader is the reference's formula
// (docs/superpowers/specs/2026-09-08-direct-k8v4-attention-design.md:57):
//   x_rot = FP16((FP32(c) - (2^(b-1) - 0.5)) * (FP32(s) / 2^(b-1)))
// computed here in FP32, where the product is exact, and rounded once.
//
// Attention runs in the rotated domain (spec :61): the split kernel rotates
// the queries with the caller's h32 matrix (FP32 [32, 32], R) and writes
// rotated partials; the combine merges them and restores the output with R^T.

#include "qwz_common.cuh"
#include "qwz_kernels.h"
#include "attn_common.cuh"

#include <math_constants.h>

namespace qwz {

using namespace detail;

namespace k8v4 {

constexpr int kBlock = 32;
constexpr int kBlocks = kHeadDim / kBlock;               // 8 per head
constexpr int kKBits = 8, kVBits = 4;
constexpr int kKWords = kKvHeads * kBlocks * kKBits;     // 256 words a token
constexpr int kVWords = kKvHeads * kBlocks * kVBits;     // 128
constexpr int kScales = kKvHeads * kBlocks;              // 32 FP16 a token

constexpr int kTile = 128;                               // tokens a tile of the split kernel
constexpr int kKHalf = kTile * 128;                      // 16 KB: blocks 0-3 or 4-7 of a head
constexpr int kVBox = kTile * 128;                       // 16 KB
constexpr int kSBox = kTile * 16;                        // 2 KB: 8 scales of a head
static_assert((2 * kKHalf + kSBox) % 1024 == 0 && (kVBox + kSBox) % 1024 == 0,
              "tiles stay 1024-byte aligned for the swizzled boxes");

constexpr float kInvSqrt32 = 0.17677669529663687f;

// Whether h32 is exactly the natural-order Hadamard matrix (every entry
// +-1/sqrt(32) in FP32 with the sign (-1)^popcount(i & j)): the threads of
// the CTA (nthreads of them) test 1024 / nthreads entries each; the caller
// reduces the answer over the CTA.
QWZ_DEVINL bool h32_is_hadamard(const float* h32, int tid, int nthreads) {
  bool had = true;
  for (int i = tid; i < 1024; i += nthreads) {
    const int ri = i >> 5, cj = i & 31;
    had &= __ldg(h32 + i) == ((__popc(ri & cj) & 1) ? -kInvSqrt32 : kInvSqrt32);
  }
  return had;
}

// Two code bytes of x (sel 0x4140: bytes 0, 1; 0x4342: bytes 2, 3) as the
// FP16 pair (1024 + c0, 1024 + c1).
QWZ_DEVINL uint32_t codes_h2(uint32_t x, uint32_t sel) { return __byte_perm(x, 0x64646464u, sel); }

// The reader on an FP16 pair of codes h = (1024 + c): (c - 2^(b-1)) exactly,
// then one fused multiply-add by s' = s / 2^(b-1) and s' / 2, a single
// rounding of (c - 2^(b-1) + 0.5) * s'.  Equal to the FP32 reader whenever
// s' and s' / 2 are normal FP16 numbers (the callers check the scales).
QWZ_DEVINL uint32_t deq_h2(uint32_t h, uint32_t base, uint32_t s2, uint32_t hs2) {
  uint32_t d;
  asm("{\n sub.rn.f16x2 %0, %1, %2;\n fma.rn.f16x2 %0, %0, %3, %4;\n}\n"
      : "=&r"(d) : "r"(h), "r"(base), "r"(s2), "r"(hs2));
  return d;
}
QWZ_DEVINL uint32_t hmul2_bits(uint32_t a, uint32_t b) {
  uint32_t d;
  asm("mul.rn.f16x2 %0, %1, %2;\n" : "=r"(d) : "r"(a), "r"(b));
  return d;
}
// FP16 scale bits for which s / 2^(b-1) and s / 2^b are normal: s >= 2^-6
// (K, b = 8) or s >= 2^-10 (V, b = 4), and finite.
constexpr uint32_t kKFastMin = 0x2400u, kVFastMin = 0x1400u, kHalfInf = 0x7C00u;

// The reader for one code: (c - mid) * (s / 2^(b-1)), exact in FP32.
QWZ_DEVINL float deq(uint32_t code, float mid, float sm) { return (static_cast<float>(code) - mid) * sm; }

QWZ_DEVINL float half_bits_to_float(uint32_t h) {
  return __half2float(__ushort_as_half(static_cast<unsigned short>(h)));
}

// Physical page of logical token t (-1 and an error bit if the table or the
// pool does not cover it).
QWZ_DEVINL int page_of(const int32_t* table, int width, int num_pages, int t) {
  const int lp = t >> 8;
  if (lp < 0 || lp >= width) {
    flag_error(kErrTableRange);
    return -1;
  }
  const int pp = __ldg(table + lp);
  if (pp < 0 || pp >= num_pages) {
    flag_error(kErrPageRange);
    return -1;
  }
  return pp;
}

}  // namespace k8v4

// --------------------------------------------------------------- writer
// One CTA per new row s and KV head: warps 0-7 quantise the 8 K blocks,
// warps 8-15 the 8 V blocks.  Lane t holds element t of its block.  The
// rotation is the natural-order fast Walsh-Hadamard butterfly in FP32 (five
// stages: x_i + x_(i+s) where bit s of i is clear, x_(i-s) - x_i where it is
// set), then the factor 1/sqrt(32); s = FP16(max |x_rot|) (at most 65504);
// c = clamp(floor(x_rot / s * 2^(b-1) + 2^(b-1)), 0, 2^b - 1), or 2^(b-1)
// when s = 0, the bin whose midpoint the reader returns.  Each operation is
// one IEEE FP32 operation (no contraction), so the result is reproducible.
template <typename T>
__global__ void __launch_bounds__(512) k8v4_append_kernel(K8v4AppendParams p) {
  using namespace k8v4;
  griddep_wait();               // the rows and the length may come from the previous kernel
  griddep_launch_dependents();  // the split may begin its launch (it waits for this grid to finish)
  const int s = blockIdx.x, h = blockIdx.y;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const bool is_v = warp >= kBlocks;
  const int j = warp & (kBlocks - 1);
  const int pos = __ldg(p.seqlens) + s;
  const int pp = page_of(p.block_table, p.table_width, p.num_pages, pos);
  if (pp < 0) return;
  const long long row = (long long)pp * kPage + (pos & (kPage - 1));
  const T* src = reinterpret_cast<const T*>(is_v ? p.v : p.k) + ((size_t)s * kKvHeads + h) * kHeadDim + j * kBlock;
  static_assert(sizeof(T) == 2, "FP16 or BF16 rows");
  const unsigned short raw = reinterpret_cast<const unsigned short*>(src)[lane];
  float x = InTraits<T>::to_float2((uint32_t)raw).x;
#pragma unroll
  for (int st = 1; st < kBlock; st <<= 1) {
    const float o = __shfl_xor_sync(0xffffffffu, x, st);
    x = (lane & st) ? __fsub_rn(o, x) : __fadd_rn(x, o);
  }
  x = __fmul_rn(x, kInvSqrt32);
  float amax = fabsf(x);
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
  amax = fminf(amax, 65504.f);
  const __half s16 = __float2half_rn(amax);
  const float sf = __half2float(s16);
  const int bits = is_v ? kVBits : kKBits;
  const float m = is_v ? 8.f : 128.f;
  uint32_t c = (uint32_t)m;
  if (sf > 0.f) {
    const float u = __fadd_rn(__fmul_rn(__fdiv_rn(x, sf), m), m);
    const float f = floorf(u);
    c = f <= 0.f ? 0u : (f >= 2.f * m - 1.f ? (uint32_t)(2.f * m - 1.f) : (uint32_t)f);
  }
  uint32_t mine = 0u;
#pragma unroll
  for (int i = 0; i < kKBits; ++i) {
    const uint32_t w = __ballot_sync(0xffffffffu, (c >> i) & 1u);
    if (lane == i) mine = w;
  }
  const int blk = h * kBlocks + j;
  if (lane < bits) {
    uint32_t* dst = is_v ? p.v_cache + row * kVWords : p.k_cache + row * kKWords;
    dst[blk * bits + lane] = mine;
  }
  if (lane == 0) (is_v ? p.v_scales : p.k_scales)[row * kScales + blk] = s16;
}

// --------------------------------------------------------------- reader
// Logical tokens [0, length) of one cache (K: bits 8, V: bits 4) dequantised
// into FP16 [length, 4, 256], rotated domain.  One thread per element.
__global__ void __launch_bounds__(256) k8v4_gather_kernel(const uint32_t* __restrict__ words,
                                                         const __half* __restrict__ scales,
                                                         const int32_t* __restrict__ table, int width,
                                                         int num_pages, int length, int bits,
                                                         __half* __restrict__ out) {
  using namespace k8v4;
  const long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= (long long)length * kKvHeads * kHeadDim) return;
  const int t = (int)(i / (kKvHeads * kHeadDim));
  const int hd = (int)(i % (kKvHeads * kHeadDim));
  const int blk = hd / kBlock, e = hd % kBlock;
  const int pp = page_of(table, width, num_pages, t);
  if (pp < 0) {
    out[i] = __float2half_rn(0.f);
    return;
  }
  const long long row = (long long)pp * kPage + (t & (kPage - 1));
  const int wpt = kKvHeads * kBlocks * bits;
  uint32_t c = 0u;
  for (int b = 0; b < bits; ++b) c |= ((__ldg(words + row * wpt + blk * bits + b) >> e) & 1u) << b;
  const float m = (float)(1 << (bits - 1));
  const float sf = __half2float(scales[row * kScales + blk]);
  out[i] = __float2half_rn(deq(c, m - 0.5f, sf * (1.f / m)));
}

// -------------------------------------- split: the tcgen05 kernel's policy
namespace k8v4 {

// 8 x 8 bit transpose of each byte column of 8 plane words (three rounds of
// block swaps: 4 x 4, 2 x 2, 1 x 1).  Before, bit j of byte m of word i is
// plane i of dim 8m + j; after, byte m of word j is the code of dim 8m + j.
QWZ_DEVINL void transpose8(uint32_t (&w)[8]) {
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const uint32_t t = ((w[i] >> 4) ^ w[i + 4]) & 0x0F0F0F0Fu;
    w[i + 4] ^= t;
    w[i] ^= t << 4;
  }
#pragma unroll
  for (int i = 0; i < 8; i += 4)
#pragma unroll
    for (int k = 0; k < 2; ++k) {
      const uint32_t t = ((w[i + k] >> 2) ^ w[i + k + 2]) & 0x33333333u;
      w[i + k + 2] ^= t;
      w[i + k] ^= t << 2;
    }
#pragma unroll
  for (int i = 0; i < 8; i += 2) {
    const uint32_t t = ((w[i] >> 1) ^ w[i + 1]) & 0x55555555u;
    w[i + 1] ^= t;
    w[i] ^= t << 1;
  }
}

// K position of dim p of a block in the tile order the verify's unpacking
// produces (word j of the transpose holds dims j, j + 8, j + 16, j + 24; the
// f16x2 word 2j + h holds dims j + 16h and j + 16h + 8), and its inverse.
QWZ_DEVINL int vt_pos(int p) { return 4 * (p & 7) + 2 * ((p >> 4) & 1) + ((p >> 3) & 1); }
QWZ_DEVINL int vt_dim(int l) { return (l >> 2) + 8 * (l & 1) + 16 * ((l >> 1) & 1); }

// One block's 32 codes (words w after transpose8) as 16 f16x2 words in the
// tile order, (c - 2^(b-1) + 0.5) * s / 2^(b-1): one fma.rn.f16x2 per pair
// when s / 2^(b-1) and half of it are normal FP16 numbers (or s is 0), the
// FP32 reader otherwise.
template <int BITS>
QWZ_DEVINL void block_values(const uint32_t (&w)[8], uint32_t hscale, uint32_t (&r)[16]) {
  constexpr uint32_t kMin = BITS == 8 ? kKFastMin : kVFastMin;
  constexpr uint32_t kBase = BITS == 8 ? 0x64806480u : 0x64086408u;  // 1024 + 2^(b-1)
  constexpr uint32_t kF = BITS == 8 ? 0x20002000u : 0x30003000u;     // 2^-(b-1)
  constexpr uint32_t kH = BITS == 8 ? 0x1C001C00u : 0x2C002C00u;     // 2^-b
  if (hscale == 0u || (hscale >= kMin && hscale < kHalfInf)) {
    const uint32_t pr = __byte_perm(hscale, hscale, 0x1010);
    const uint32_t s2 = hmul2_bits(pr, kF), hs2 = hmul2_bits(pr, kH);
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      r[2 * j] = deq_h2(codes_h2(w[j], 0x4140u), kBase, s2, hs2);
      r[2 * j + 1] = deq_h2(codes_h2(w[j], 0x4342u), kBase, s2, hs2);
    }
  } else {
    const float mid = BITS == 8 ? 127.5f : 7.5f;
    const float sm = half_bits_to_float(hscale) * (BITS == 8 ? (1.f / 128.f) : 0.125f);
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const uint32_t x = w[j];
      r[2 * j] = pack_half2(deq(x & 0xff, mid, sm), deq((x >> 8) & 0xff, mid, sm));
      r[2 * j + 1] = pack_half2(deq((x >> 16) & 0xff, mid, sm), deq(x >> 24, mid, sm));
    }
  }
}

}  // namespace k8v4

// The K8/V4 cache in the tcgen05 verify kernel: a K tile is two 128-byte-
// swizzled boxes of bit planes (blocks 0-3 and 4-7 of the head) and one box
// of FP16 scales (34 KB), a V tile one swizzled box of planes and one of
// scales (18 KB); two tiles of each in flight.  A math thread owns whole
// blocks of its token, so it transposes the bit planes of a block at once
// and hands the values in the tile order of vt_pos; Q is rotated and laid out
// in the same order, and O^T's rows come back to the head's order in the
// epilogue.
struct VtK8v4 {
  static constexpr int kKStages = 2, kVStages = 2;
  static constexpr int kKStage = 2 * k8v4::kKHalf + k8v4::kSBox;
  static constexpr int kVStage = k8v4::kVBox + k8v4::kSBox;
  static constexpr int kBlocksPerPart = k8v4::kBlocks / kVtParts;

  QWZ_DEVINL static void issue(bool is_k, const SplitParams& p, uint32_t dst, int kvh, int y, uint32_t bar) {
    if (is_k) {
      tma_load_2d(dst, &p.tm_kc, kvh * 256, y, bar);
      tma_load_2d(dst + k8v4::kKHalf, &p.tm_kc, kvh * 256 + 128, y, bar);
      tma_load_2d(dst + 2 * k8v4::kKHalf, &p.tm_ks, kvh * 16, y, bar);
    } else {
      tma_load_2d(dst, &p.tm_vc, kvh * 128, y, bar);
      tma_load_2d(dst + k8v4::kVBox, &p.tm_vs, kvh * 16, y, bar);
    }
  }
  template <class Put>
  QWZ_DEVINL static void dequant_k(uint32_t st, int tt, int u, Put put) {
#pragma unroll
    for (int c = 0; c < kBlocksPerPart; ++c) {
      const int b = kBlocksPerPart * u + c;
      const uint32_t half = st + (b >> 2) * k8v4::kKHalf;
      const int c0 = 2 * (b & 3);
      const uint4 a0 = lds128(half + swz128(tt, c0)), a1 = lds128(half + swz128(tt, c0 + 1));
      uint32_t w[8] = {a0.x, a0.y, a0.z, a0.w, a1.x, a1.y, a1.z, a1.w};
      k8v4::transpose8(w);
      uint32_t r[16];
      k8v4::block_values<8>(w, lds16(st + 2 * k8v4::kKHalf + tt * 16 + 2 * b), r);
      put(b, r);
    }
  }
  template <class Put>
  QWZ_DEVINL static void dequant_v(uint32_t st, int tt, int u, bool zero, Put put) {
#pragma unroll
    for (int c = 0; c < kBlocksPerPart; ++c) {
      const int b = kBlocksPerPart * u + c;
      const uint4 a = lds128(st + swz128(tt, b));
      uint32_t w[8] = {a.x, a.y, a.z, a.w, 0u, 0u, 0u, 0u};
      k8v4::transpose8(w);
      uint32_t r[16];
      k8v4::block_values<4>(w, zero ? 0u : lds16(st + k8v4::kVBox + tt * 16 + 2 * b), r);
      put(b, r);
    }
  }
  // Q_rot rows of this KV head (R q per block: the butterfly when h32 is the
  // natural-order Hadamard matrix, else 32 multiply-adds), each scaled by a
  // power of two, FP16, at K position 32 b + vt_pos(p) of the K-major atoms.
  template <typename T, int N>
  QWZ_DEVINL static void stage(const SplitParams& p, int kvh, uint32_t qbase, float* rowfac, bool had, int mw,
                               int lane) {
    using namespace k8v4;
    float rrow[kBlock];
    if (!had) {
#pragma unroll
      for (int jj = 0; jj < kBlock; ++jj) rrow[jj] = __ldg(p.h32 + lane * kBlock + jj);
    }
    const int pos = vt_pos(lane);
    for (int r = mw; r < N; r += kVtMathWarps) {
      const int qi = r / kGroup, hg = r - qi * kGroup;
      float xr[kBlocks];
      float amax = 0.f;
      if (qi < p.q_len) {
        const T* row = reinterpret_cast<const T*>(p.q) + ((size_t)qi * kQHeads + kvh * kGroup + hg) * kHeadDim;
#pragma unroll
        for (int b = 0; b < kBlocks; ++b) {
          const unsigned short raw = reinterpret_cast<const unsigned short*>(row)[b * kBlock + lane];
          xr[b] = InTraits<T>::to_float2((uint32_t)raw).x;
        }
        if (had) {
#pragma unroll
          for (int b = 0; b < kBlocks; ++b) {
            float x = xr[b];
#pragma unroll
            for (int stp = 1; stp < kBlock; stp <<= 1) {
              const float o = __shfl_xor_sync(0xffffffffu, x, stp);
              x = (lane & stp) ? o - x : x + o;
            }
            xr[b] = x * kInvSqrt32;
          }
        } else {
          float xin[kBlocks];
#pragma unroll
          for (int b = 0; b < kBlocks; ++b) {
            xin[b] = xr[b];
            xr[b] = 0.f;
          }
#pragma unroll
          for (int jj = 0; jj < kBlock; ++jj)
#pragma unroll
            for (int b = 0; b < kBlocks; ++b) xr[b] = fmaf(rrow[jj], __shfl_sync(0xffffffffu, xin[b], jj), xr[b]);
        }
#pragma unroll
        for (int b = 0; b < kBlocks; ++b) amax = fmaxf(amax, fabsf(xr[b]));
      } else {
#pragma unroll
        for (int b = 0; b < kBlocks; ++b) xr[b] = 0.f;
      }
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
      const float sc = pow2_row_scale(amax);
#pragma unroll
      for (int b = 0; b < kBlocks; ++b) {
        const int dl = b * kBlock + pos;  // K position of this lane's dim
        const uint32_t addr = qbase + (dl >> 6) * (N * 128) + r * 128 + ((((dl & 63) >> 3) ^ (r & 7)) << 4) + (dl & 7) * 2;
        const __half hv = __float2half_rn(xr[b] * sc);
        asm volatile("st.shared.u16 [%0], %1;\n" ::"r"(addr), "h"(__half_as_ushort(hv)));
      }
      // padding rows (zero Q) keep a positive factor so masked scores stay -inf
      if (lane == 0) rowfac[r] = qi < p.q_len ? p.sm_scale_log2 / sc : p.sm_scale_log2;
    }
  }
  QWZ_DEVINL static bool rotation_check(const SplitParams& p, int tid) {
    return __syncthreads_and(k8v4::h32_is_hadamard(p.h32, tid, kVtWarps * 32)) != 0;
  }
  QWZ_DEVINL static int o_dim(int d) { return (d & ~31) + k8v4::vt_dim(d & 31); }
  // rows are appended by qwz_k8v4_append (the split is never given app_k)
  template <typename T>
  QWZ_DEVINL static void append_row(const SplitParams&, int, int, int, int, int) {}
};

cudaError_t launch_k8v4_split(const SplitParams& p, int dtype, cudaStream_t stream) {
  if (dtype == kDtypeBF16) return launch_verify_tc<__nv_bfloat16, VtK8v4>(p, stream);
  return launch_verify_tc<__half, VtK8v4>(p, stream);
}

cudaError_t launch_k8v4_append(const K8v4AppendParams& p, int dtype, cudaStream_t stream) {
  if (p.append_len <= 0) return cudaSuccess;
  const dim3 grid(p.append_len, kKvHeads), block(512);
  if (dtype == kDtypeBF16) return launch_pdl(k8v4_append_kernel<__nv_bfloat16>, grid, block, 0, stream, p);
  return launch_pdl(k8v4_append_kernel<__half>, grid, block, 0, stream, p);
}

cudaError_t launch_k8v4_gather(const uint32_t* words, const __half* scales, const int32_t* table, int width,
                               int num_pages, int length, int bits, __half* out, cudaStream_t stream) {
  const long long n = (long long)length * kKvHeads * kHeadDim;
  if (n <= 0) return cudaSuccess;
  const unsigned blocks = (unsigned)((n + 255) / 256);
  k8v4_gather_kernel<<<blocks, 256, 0, stream>>>(words, scales, table, width, num_pages, length, bits, out);
  return cudaGetLastError();
}

}  // namespace qwz
