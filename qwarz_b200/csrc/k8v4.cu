// K8/V4 quantised-cache attention for sm_100a: the writer, the split-K
// decode / verify kernel and the reader used by the parity tests.
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
// Attention runs in the rotated domain (spec :61): the split kernels rotate
// the queries with the caller's h32 matrix (FP32 [32, 32], R) and write
// rotated partials; the combine merges them and restores the output with R^T.
//
// Decode (q_len 1), k8v4_decode16_kernel: one CTA per (split, KV head), two
// groups of 8 warps take the even and the odd 128-token stages of the split
// from a 4-slot TMA ring (K as two 128-byte-swizzled halves, V swizzled, the
// FP16 scales unswizzled; 52 KB a stage) that a producer warp refills.  For
// each stage a group runs:
//   QK   warp w takes tokens 16w..16w+15 and every query row of the head
//        group: S^T = K Q^T with mma.sync m16n8k16, the K A-fragments
//        unpacked straight from the bit planes (a thread's 8 dims q + 4k of a
//        block come out of the 8 planes with one rotate and one masked merge
//        per plane) and Q B-fragments by ldmatrix;
//   max  the group's row maxima meet in shared memory (one barrier), every
//        warp derives the same running max, P = 2^(S - m) goes to shared
//        memory in FP16 (second barrier);
//   PV   warp w owns the 32 dims of block w for all 128 tokens:
//        O^T[d x rows] += V^T P^T, the V A-fragments unpacked from the 4 bit
//        planes (dims g + 8k), P^T by ldmatrix.trans.
// The running max and O rescale are per row and need no further exchange,
// because the PV accumulator's columns are the same rows as the QK
// accumulator's columns in every thread; the two groups merge at the end.
//
// Verify (q_len 2..8): the tcgen05 verify kernel of attn_verify_tc.cu with
// the VtK8v4 format policy below (whole-block bit transposes by the math
// threads, Q in the matching dim order).

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
constexpr int kKRowBytes = kKWords * 4;                  // 1024
constexpr int kVRowBytes = kVWords * 4;                  // 512
constexpr int kScaleRowBytes = kScales * 2;              // 64

constexpr int kStage = 128;                              // tokens a stage
constexpr int kSlots = 3;
constexpr int kWarps = 8;
constexpr int kKHalf = kStage * 128;                     // 16 KB: blocks 0-3 or 4-7 of a head
constexpr int kVBox = kStage * 128;                      // 16 KB
constexpr int kSBox = kStage * 16;                       // 2 KB: 8 scales of a head
constexpr int kStageBytes = 2 * kKHalf + kVBox + 2 * kSBox;  // 53,248
static_assert(kStageBytes % 1024 == 0, "stages stay 1024-byte aligned for the swizzled boxes");

constexpr float kInvSqrt32 = 0.17677669529663687f;

// Codes of the 8 dims q + 4k (k = 0..7) of one K block from its 8 plane
// words.  Rotating plane i right by q - i moves bit q + 4k to i + 4k, so
// planes 0-3 and 4-7 gather into two words of nibbles (one rotate and one
// masked merge per plane), which two merges turn into bytes:
//   lo byte b = code of dim q + 8b,   hi byte b = code of dim q + 8b + 4.
QWZ_DEVINL void k_codes(const uint4& w0, const uint4& w1, int q, uint32_t& lo, uint32_t& hi) {
  const uint32_t w[8] = {w0.x, w0.y, w0.z, w0.w, w1.x, w1.y, w1.z, w1.w};
  uint32_t ca = 0u, cb = 0u;
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    ca |= __funnelshift_r(w[i], w[i], q - i) & (0x11111111u << i);
    cb |= __funnelshift_r(w[i + 4], w[i + 4], q - i) & (0x11111111u << i);
  }
  lo = (ca & 0x0F0F0F0Fu) | ((cb << 4) & 0xF0F0F0F0u);
  hi = ((ca >> 4) & 0x0F0F0F0Fu) | (cb & 0xF0F0F0F0u);
}

// Codes of the dims g + 8k (k = 0..3) of one V block (4 plane words): byte k.
QWZ_DEVINL uint32_t v_codes(const uint4& w, int g) {
  return (__funnelshift_r(w.x, w.x, g) & 0x01010101u) | (__funnelshift_r(w.y, w.y, g - 1) & 0x02020202u) |
         (__funnelshift_r(w.z, w.z, g - 2) & 0x04040404u) | (__funnelshift_r(w.w, w.w, g - 3) & 0x08080808u);
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
  griddep_wait();
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

// ----------------------------------------------------------- split kernel
namespace k8v4 {

// Per-thread row state of the split: rows nt * 8 + 2 q4 + {0, 1} of the head
// group (row r = 6 qi + hg; rows past 6 q_len are padding), the O^T
// accumulator of the thread's dims of the warp's block, and the visibility
// limit of each row.
template <int NT>
struct RowState {
  float m_run[NT][2], l_run[NT][2], fac[NT][2];
  float o[2][NT][4];
  int lim[NT][2];
};

// A barrier over the 8 warps (256 threads) that share one stage: a named
// barrier per stage group.
struct StageBar {
  int id;
  QWZ_DEVINL void sync() const { asm volatile("bar.sync %0, 256;\n" ::"r"(id) : "memory"); }
  QWZ_DEVINL bool any(bool v) const {
    uint32_t r;
    asm volatile(
        "{\n .reg .pred p, q;\n setp.ne.u32 p, %1, 0;\n bar.red.or.pred q, %2, 256, p;\n"
        " selp.u32 %0, 1, 0, q;\n}\n"
        : "=r"(r)
        : "r"((uint32_t)v), "r"(id)
        : "memory");
    return r != 0;
  }
};

// Q_rot = R q for the 6 q_len rows of KV head kvh (row r = 6 qi + hg), FP16,
// each row scaled by a power of two (its factor sm_scale*log2e/scale goes to
// rowfac[r]), written at K position 32 b + L(lane) of the row in the order
// k_codes hands a thread its dims: dim p = q + 8 (2 h + e) + 4 t of a block
// <-> position 16 t + 8 h + 2 q + e; 16-byte chunks swizzled by row.  When
// h32 is exactly the natural-order Hadamard matrix (every entry
// +-1/sqrt(32) in FP32 with the sign (-1)^popcount(i & j)) the rotation is
// the five-stage butterfly, else 32 multiply-adds per element with the
// lane's row of R read from global memory.  `had` is that test's result.
template <typename T>
QWZ_DEVINL void stage_q_rot(const SplitParams& p, int kvh, int rows_padded, uint8_t* qsm, float* rowfac, bool had,
                            int warp, int nwarps, int lane) {
  const T* qsrc = reinterpret_cast<const T*>(p.q);
  float rrow[kBlock];  // R[lane][j]
  if (!had) {
#pragma unroll
    for (int jj = 0; jj < kBlock; ++jj) rrow[jj] = __ldg(p.h32 + lane * kBlock + jj);
  }
  const int pl = 16 * ((lane >> 2) & 1) + 8 * (lane >> 4) + 2 * (lane & 3) + ((lane >> 3) & 1);
  for (int r = warp; r < rows_padded; r += nwarps) {
    const int qi = r / kGroup, hg = r % kGroup;
    float xr[kBlocks];
    float amax = 0.f;
    if (qi < p.q_len) {
      const T* row = qsrc + ((size_t)qi * kQHeads + kvh * kGroup + hg) * kHeadDim;
#pragma unroll
      for (int b = 0; b < kBlocks; ++b) {
        const unsigned short bits = reinterpret_cast<const unsigned short*>(row)[b * kBlock + lane];
        xr[b] = InTraits<T>::to_float2((uint32_t)bits).x;
      }
      if (had) {
#pragma unroll
        for (int b = 0; b < kBlocks; ++b) {
          float x = xr[b];
#pragma unroll
          for (int st = 1; st < kBlock; st <<= 1) {
            const float o = __shfl_xor_sync(0xffffffffu, x, st);
            x = (lane & st) ? o - x : x + o;
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
    __half* qrow = reinterpret_cast<__half*>(qsm + r * 512);
#pragma unroll
    for (int b = 0; b < kBlocks; ++b) {
      const int d = b * kBlock + pl;
      const int chunk = d >> 3;
      qrow[(((chunk ^ (r & 7)) << 3) | (d & 7))] = __float2half_rn(xr[b] * sc);
    }
    if (lane == 0) rowfac[r] = p.sm_scale_log2 / sc;
  }
}

// Whether h32 is exactly the natural-order Hadamard matrix: the threads of
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

template <int NT>
QWZ_DEVINL void init_rows(RowState<NT>& rs, const float* rowfac, int q4, int q_len, int tok_end, int len_all) {
  const int qmax = q_len - 1;
#pragma unroll
  for (int nt = 0; nt < NT; ++nt) {
#pragma unroll
    for (int e = 0; e < 2; ++e) {
      rs.m_run[nt][e] = -CUDART_INF_F;
      rs.l_run[nt][e] = 0.f;
      rs.fac[nt][e] = rowfac[nt * 8 + 2 * q4 + e];
      const int qi = min((nt * 8 + 2 * q4 + e) / kGroup, qmax);
      rs.lim[nt][e] = min(tok_end, len_all - (qmax - qi));
    }
#pragma unroll
    for (int mt = 0; mt < 2; ++mt)
#pragma unroll
      for (int e = 0; e < 4; ++e) rs.o[mt][nt][e] = 0.f;
  }
}

// One 128-token stage for the 8 warps of a stage group (warp = 0..7 within
// the group): QK, the group's row maxima through red[8 warps][R] (one
// barrier), P into pbase, the rescale, a second barrier, PV.  Returns false
// when any thread of the group reports !ok at the first barrier (every
// thread of the group then returns false).
template <int NT>
QWZ_DEVINL bool run_stage(RowState<NT>& rs, uint32_t st, uint32_t qbase, uint32_t pbase, float* red, int t0,
                          bool sok, bool ok, int warp, int lane, StageBar bar) {
  constexpr int R = NT * 8;
  constexpr int kPRow = (NT | 1) * 16;  // P^T row bytes (odd chunk count: conflict-free ldmatrix)
  const int g = lane >> 2, q4 = lane & 3;
  const uint32_t kst = st, vst = st + 2 * kKHalf, ksc = vst + kVBox, vsc = ksc + kSBox;

  // -------------------------------------------------------------- QK
  float s[NT][4];
#pragma unroll
  for (int nt = 0; nt < NT; ++nt)
#pragma unroll
    for (int e = 0; e < 4; ++e) s[nt][e] = 0.f;
  const int r0 = 16 * warp + g, r1 = r0 + 8;  // token rows of the stage
#pragma unroll 2
  for (int j = 0; j < kBlocks; ++j) {
    const uint32_t half = kst + (j >> 2) * kKHalf;
    const int c0 = 2 * (j & 3);
    const uint4 a0 = lds128(half + swz128(r0, c0)), a1 = lds128(half + swz128(r0, c0 + 1));
    const uint4 b0 = lds128(half + swz128(r1, c0)), b1 = lds128(half + swz128(r1, c0 + 1));
    uint32_t lo0, hi0, lo1, hi1;
    k_codes(a0, a1, q4, lo0, hi0);
    k_codes(b0, b1, q4, lo1, hi1);
    const uint32_t h0 = lds16(ksc + r0 * 16 + 2 * j), h1 = lds16(ksc + r1 * 16 + 2 * j);
    // A fragments of k-steps 2j (af[0..3]) and 2j+1 (af[4..7]), in the dim
    // order stage_q_rot writes Q in
    uint32_t af[8];
    const uint32_t src[4] = {lo0, lo1, hi0, hi1};
    if (__all_sync(0xffffffffu, h0 >= kKFastMin && h0 < kHalfInf && h1 >= kKFastMin && h1 < kHalfInf)) {
      const uint32_t p0 = __byte_perm(h0, h0, 0x1010), p1 = __byte_perm(h1, h1, 0x1010);
      const uint32_t s0 = hmul2_bits(p0, 0x20002000u), hs0 = hmul2_bits(p0, 0x1C001C00u);  // s/128, s/256
      const uint32_t s1 = hmul2_bits(p1, 0x20002000u), hs1 = hmul2_bits(p1, 0x1C001C00u);
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        const bool odd = k & 1;
        af[2 * k] = deq_h2(codes_h2(src[k], 0x4140u), 0x64806480u, odd ? s1 : s0, odd ? hs1 : hs0);
        af[2 * k + 1] = deq_h2(codes_h2(src[k], 0x4342u), 0x64806480u, odd ? s1 : s0, odd ? hs1 : hs0);
      }
    } else {  // a scale too small for the FP16 path: the FP32 reader
      const float sm0 = half_bits_to_float(h0) * (1.f / 128.f), sm1 = half_bits_to_float(h1) * (1.f / 128.f);
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        const float sm = (k & 1) ? sm1 : sm0;
        const uint32_t x = src[k];
        af[2 * k] = pack_half2(deq(x & 0xff, 127.5f, sm), deq((x >> 8) & 0xff, 127.5f, sm));
        af[2 * k + 1] = pack_half2(deq((x >> 16) & 0xff, 127.5f, sm), deq(x >> 24, 127.5f, sm));
      }
    }
#pragma unroll
    for (int nt = 0; nt < NT; ++nt) {
      // B fragments of k-steps 2j, 2j+1: Q rows nt*8.., chunks 4j..4j+3
      const int qr = nt * 8 + (lane & 7);
      const int ch = 4 * j + (lane >> 3);
      uint32_t q0, q1, q2, q3;
      ldmatrix_x4(q0, q1, q2, q3, qbase + qr * 512 + ((ch ^ (qr & 7)) << 4));
      mma_16816(s[nt], af[0], af[2], af[1], af[3], q0, q1);
      mma_16816(s[nt], af[4], af[6], af[5], af[7], q2, q3);
    }
  }

  // ---------------------------------------------------- stage maxima
  const int tok0 = t0 + r0, tok1 = t0 + r1;
#pragma unroll
  for (int nt = 0; nt < NT; ++nt) {
#pragma unroll
    for (int e = 0; e < 2; ++e) {
      const float x0 = (sok && tok0 < rs.lim[nt][e]) ? s[nt][e] * rs.fac[nt][e] : -CUDART_INF_F;
      const float x1 = (sok && tok1 < rs.lim[nt][e]) ? s[nt][2 + e] * rs.fac[nt][e] : -CUDART_INF_F;
      s[nt][e] = x0;
      s[nt][2 + e] = x1;
      float mx = fmaxf(x0, x1);
      mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 4));
      mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 8));
      mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 16));
      if (g == 0) red[warp * R + nt * 8 + 2 * q4 + e] = mx;
    }
  }
  if (bar.any(!ok)) return false;  // every thread of the group leaves together

  // ----------------------------------------- running max, P, rescale
  // P is rounded to FP16 for the PV product; the row sums l add the same
  // rounded values, so numerator and denominator use identical weights.
#pragma unroll
  for (int nt = 0; nt < NT; ++nt) {
    float pe[2][2];  // [row e][token r0 / r1]
#pragma unroll
    for (int e = 0; e < 2; ++e) {
      const int rr = nt * 8 + 2 * q4 + e;
      float mx = red[rr];
#pragma unroll
      for (int w = 1; w < kWarps; ++w) mx = fmaxf(mx, red[w * R + rr]);
      const float mnew = fmaxf(rs.m_run[nt][e], mx);
      const float alpha = rs.m_run[nt][e] == -CUDART_INF_F ? 0.f : exp2_approx(rs.m_run[nt][e] - mnew);
      const float mu = mnew == -CUDART_INF_F ? 0.f : mnew;
      rs.m_run[nt][e] = mnew;
      pe[e][0] = exp2_approx(s[nt][e] - mu);
      pe[e][1] = exp2_approx(s[nt][2 + e] - mu);
      rs.l_run[nt][e] *= alpha;
#pragma unroll
      for (int mt = 0; mt < 2; ++mt) {
        rs.o[mt][nt][e] *= alpha;
        rs.o[mt][nt][2 + e] *= alpha;
      }
    }
    // P^T[token][row]: (r0, rows 2q4, 2q4+1) and (r1, ...)
    const uint32_t h0 = pack_half2(pe[0][0], pe[1][0]), h1 = pack_half2(pe[0][1], pe[1][1]);
    const float2 f0 = __half22float2(*reinterpret_cast<const __half2*>(&h0));
    const float2 f1 = __half22float2(*reinterpret_cast<const __half2*>(&h1));
    rs.l_run[nt][0] += f0.x + f1.x;
    rs.l_run[nt][1] += f0.y + f1.y;
    sts32(pbase + r0 * kPRow + (nt * 8 + 2 * q4) * 2, h0);
    sts32(pbase + r1 * kPRow + (nt * 8 + 2 * q4) * 2, h1);
  }
  bar.sync();

  // -------------------------------------------------------------- PV
#pragma unroll 2
  for (int kk = 0; kk < kStage / 16; ++kk) {
    const int ta = 16 * kk + 2 * q4;  // tokens ta, ta+1, ta+8, ta+9
    const uint4 w0 = lds128(vst + swz128(ta, warp)), w1 = lds128(vst + swz128(ta + 1, warp));
    const uint4 w2 = lds128(vst + swz128(ta + 8, warp)), w3 = lds128(vst + swz128(ta + 9, warp));
    const uint32_t c0 = v_codes(w0, g), c1 = v_codes(w1, g), c2 = v_codes(w2, g), c3 = v_codes(w3, g);
    const uint32_t hs0 = lds16(vsc + ta * 16 + 2 * warp), hs1 = lds16(vsc + (ta + 1) * 16 + 2 * warp);
    const uint32_t hs2 = lds16(vsc + (ta + 8) * 16 + 2 * warp), hs3 = lds16(vsc + (ta + 9) * 16 + 2 * warp);
    // av[m-tile][reg]: m-tile 0 = dims g, g+8 (bytes 0, 1), m-tile 1 = dims
    // g+16, g+24 (bytes 2, 3); regs (dim lo, tokens ta,ta+1), (dim hi,
    // ta,ta+1), (dim lo, ta+8,ta+9), (dim hi, ta+8,ta+9)
    uint32_t av[2][4];
    if (__all_sync(0xffffffffu, hs0 >= kVFastMin && hs0 < kHalfInf && hs1 >= kVFastMin && hs1 < kHalfInf &&
                                    hs2 >= kVFastMin && hs2 < kHalfInf && hs3 >= kVFastMin && hs3 < kHalfInf)) {
      const uint32_t p01 = hs0 | (hs1 << 16), p23 = hs2 | (hs3 << 16);
      const uint32_t s01 = hmul2_bits(p01, 0x30003000u), h01 = hmul2_bits(p01, 0x2C002C00u);  // s/8, s/16
      const uint32_t s23 = hmul2_bits(p23, 0x30003000u), h23 = hmul2_bits(p23, 0x2C002C00u);
      const uint32_t u01 = __byte_perm(c0, c1, 0x5140), v01 = __byte_perm(c0, c1, 0x7362);
      const uint32_t u23 = __byte_perm(c2, c3, 0x5140), v23 = __byte_perm(c2, c3, 0x7362);
      av[0][0] = deq_h2(codes_h2(u01, 0x4140u), 0x64086408u, s01, h01);
      av[0][1] = deq_h2(codes_h2(u01, 0x4342u), 0x64086408u, s01, h01);
      av[0][2] = deq_h2(codes_h2(u23, 0x4140u), 0x64086408u, s23, h23);
      av[0][3] = deq_h2(codes_h2(u23, 0x4342u), 0x64086408u, s23, h23);
      av[1][0] = deq_h2(codes_h2(v01, 0x4140u), 0x64086408u, s01, h01);
      av[1][1] = deq_h2(codes_h2(v01, 0x4342u), 0x64086408u, s01, h01);
      av[1][2] = deq_h2(codes_h2(v23, 0x4140u), 0x64086408u, s23, h23);
      av[1][3] = deq_h2(codes_h2(v23, 0x4342u), 0x64086408u, s23, h23);
    } else {  // a scale too small for the FP16 path: the FP32 reader
      const float s0 = half_bits_to_float(hs0) * 0.125f, s1 = half_bits_to_float(hs1) * 0.125f;
      const float s2 = half_bits_to_float(hs2) * 0.125f, s3 = half_bits_to_float(hs3) * 0.125f;
#pragma unroll
      for (int mt = 0; mt < 2; ++mt)
#pragma unroll
        for (int hi = 0; hi < 2; ++hi) {
          const int sh = 8 * (2 * mt + hi);
          av[mt][hi] = pack_half2(deq((c0 >> sh) & 0xff, 7.5f, s0), deq((c1 >> sh) & 0xff, 7.5f, s1));
          av[mt][2 + hi] = pack_half2(deq((c2 >> sh) & 0xff, 7.5f, s2), deq((c3 >> sh) & 0xff, 7.5f, s3));
        }
    }
    // P^T B fragments: tokens 16kk..+15, n-tiles by pairs (x4.trans)
#pragma unroll
    for (int nt = 0; nt < NT; nt += 2) {
      uint32_t b0, b1, b2 = 0u, b3 = 0u;
      const int trow = 16 * kk + (lane & 7) + ((lane >> 3) & 1) * 8;
      if (nt + 1 < NT) {
        const int ch = nt + (lane >> 4);
        asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];\n"
                     : "=r"(b0), "=r"(b1), "=r"(b2), "=r"(b3)
                     : "r"(pbase + trow * kPRow + ch * 16));
      } else {
        asm volatile("ldmatrix.sync.aligned.m8n8.x2.trans.shared.b16 {%0,%1}, [%2];\n"
                     : "=r"(b0), "=r"(b1)
                     : "r"(pbase + trow * kPRow + nt * 16));
      }
      mma_16816(rs.o[0][nt], av[0][0], av[0][1], av[0][2], av[0][3], b0, b1);
      mma_16816(rs.o[1][nt], av[1][0], av[1][1], av[1][2], av[1][3], b0, b1);
      if (nt + 1 < NT) {
        mma_16816(rs.o[0][nt + 1], av[0][0], av[0][1], av[0][2], av[0][3], b2, b3);
        mma_16816(rs.o[1][nt + 1], av[1][0], av[1][1], av[1][2], av[1][3], b2, b3);
      }
    }
  }
  return true;
}

// The l of each row summed over the lanes and warps of a group into red_l
// (one barrier of the group inside), then the partial records: m in log2
// units, l, and the unnormalised O^T of the thread's dims.  `fine` false
// (a timeout) or l = 0 (no visible key) writes the empty record.
template <int NT>
QWZ_DEVINL void group_l(const RowState<NT>& rs, float* red_l, int warp, int lane) {
  constexpr int R = NT * 8;
  const int g = lane >> 2, q4 = lane & 3;
#pragma unroll
  for (int nt = 0; nt < NT; ++nt)
#pragma unroll
    for (int e = 0; e < 2; ++e) {
      float l = rs.l_run[nt][e];
      l += __shfl_xor_sync(0xffffffffu, l, 4);
      l += __shfl_xor_sync(0xffffffffu, l, 8);
      l += __shfl_xor_sync(0xffffffffu, l, 16);
      if (g == 0) red_l[warp * R + nt * 8 + 2 * q4 + e] = l;
    }
}

// The sum over the warps of red_l for each of the thread's rows.
template <int NT>
QWZ_DEVINL void row_totals(const float* red_l, int lane, float (&lrow)[NT][2]) {
  constexpr int R = NT * 8;
  const int q4 = lane & 3;
#pragma unroll
  for (int nt = 0; nt < NT; ++nt)
#pragma unroll
    for (int e = 0; e < 2; ++e) {
      float l = 0.f;
#pragma unroll
      for (int w = 0; w < kWarps; ++w) l += red_l[w * R + nt * 8 + 2 * q4 + e];
      lrow[nt][e] = l;
    }
}

template <int NT>
QWZ_DEVINL void write_partials(const SplitParams& p, const RowState<NT>& rs, const float (&lrow)[NT][2], bool fine,
                               int split, int kvh, int warp, int lane) {
  const int g = lane >> 2, q4 = lane & 3;
  const int rows = kGroup * p.q_len;
#pragma unroll
  for (int nt = 0; nt < NT; ++nt)
#pragma unroll
    for (int e = 0; e < 2; ++e) {
      const int rr = nt * 8 + 2 * q4 + e;
      if (rr >= rows) continue;
      const float l = lrow[nt][e];
      const bool live = fine && l > 0.f;
      const size_t Rg = (size_t)(rr / kGroup) * kQHeads + kvh * kGroup + rr % kGroup;
      const size_t base = Rg * p.num_splits + split;
      if (warp == 0 && g == 0) {
        p.partial_ml[base * 2 + 0] = live ? rs.m_run[nt][e] : -CUDART_INF_F;
        p.partial_ml[base * 2 + 1] = live ? l : 0.f;
      }
      float* dst = p.partial_o + base * kHeadDim + warp * kBlock;
#pragma unroll
      for (int mt = 0; mt < 2; ++mt) {
        dst[16 * mt + g] = live ? rs.o[mt][nt][e] : 0.f;
        dst[16 * mt + g + 8] = live ? rs.o[mt][nt][2 + e] : 0.f;
      }
    }
}

}  // namespace k8v4

// Decode (q_len 1) with twice the warps: two groups of 8 warps take the
// even and the odd 128-token stages of the split, each with its own online
// softmax, from a 4-slot ring that a producer warp (warp 16) refills as a
// group releases a slot; the groups' (m, l, O) merge in shared memory at the
// end.  The K8/V4 unpacking is latency-bound at 8 warps per SM; 16 give the
// schedulers twice the independent work.
namespace k8v4 {
constexpr int kD16Slots = 4;
struct D16Layout {
  static constexpr int kRing = 0;
  static constexpr int kQ = kD16Slots * kStageBytes;     // Q_rot FP16 [8][256]
  static constexpr int kP = kQ + 8 * 512;                // P^T per group [128 tok][16 B]
  static constexpr int kRed = kP + 2 * kStage * 16;      // row maxima [group][8 warps][8]
  static constexpr int kRedL = kRed + 2 * kWarps * 8 * 4;
  static constexpr int kRowFac = kRedL + 2 * kWarps * 8 * 4;
  static constexpr int kMerge = kRowFac + 8 * 4;         // group 1's m, l [8] each
  static constexpr int kBars = kMerge + 2 * 8 * 4;       // full[4], empty[4]
  static constexpr int kStageOk = kBars + 16 * kD16Slots;
  static constexpr int kBytes = kStageOk + 4 * kD16Slots + 1024;
  static_assert(kQ % 1024 == 0 && kP % 16 == 0 && kBars % 8 == 0, "layout alignment");
  static_assert(kBytes <= 227 * 1024, "shared memory of one CTA");
};
}  // namespace k8v4

template <typename T>
__global__ void __launch_bounds__(544, 1) k8v4_decode16_kernel(const __grid_constant__ SplitParams p) {
  using namespace k8v4;
  using L = D16Layout;
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const uint32_t sb = smem_u32(smem);
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int q4 = lane & 3;
  const int split = blockIdx.x, kvh = blockIdx.y;
  const int grp = warp >> 3, gw = warp & 7;  // stage group, warp within it (warp 16: producer)
  float* rowfac = reinterpret_cast<float*>(smem + L::kRowFac);
  float* merge = reinterpret_cast<float*>(smem + L::kMerge);
  int* stage_ok = reinterpret_cast<int*>(smem + L::kStageOk);
  const uint32_t full = sb + L::kBars, empty = full + 8 * kD16Slots;

  if (tid == 0) {
    for (int i = 0; i < kD16Slots; ++i) {
      mbar_init(full + 8 * i, 1);
      mbar_init(empty + 8 * i, kWarps);
    }
    mbar_fence_init();
    tma_prefetch_desc(&p.tm_kc);
    tma_prefetch_desc(&p.tm_vc);
    tma_prefetch_desc(&p.tm_ks);
    tma_prefetch_desc(&p.tm_vs);
  }
  griddep_wait();  // the length, the table, the cache and q may come from the previous kernel
  const StageRange rg = stage_range<kStage>(p, split);
  const int len_all = __ldg(p.seqlens) + p.len_add;
  __syncthreads();

  bool ok = true;
  int done = 0;  // stages this thread's group finished
  if (warp == 2 * kWarps) {
    // ------------------------------------------------------------ producer
    // The whole warp takes part in every CTA-wide barrier (lane 0 does the
    // issuing, the warp reconverges before each barrier).
    int issued = 0;
    auto issue = [&](int i) {
      const int slot = i % kD16Slots;
      const uint32_t bar = full + 8 * slot;
      const int t0 = p.tok_begin + (rg.st_lo + i) * kStage;
      const int pp = page_of(p.block_table, p.table_width, p.num_pages, t0);
      stage_ok[slot] = pp >= 0;
      if (pp < 0) {
        mbar_arrive(bar);  // nothing to load: the stage is masked as a whole
        return;
      }
      const int y = pp * kPage + (t0 & (kPage - 1));
      const uint32_t dst = sb + L::kRing + slot * kStageBytes;
      mbar_arrive_expect_tx(bar, kStageBytes);
      tma_load_2d(dst, &p.tm_kc, kvh * 256, y, bar);
      tma_load_2d(dst + kKHalf, &p.tm_kc, kvh * 256 + 128, y, bar);
      tma_load_2d(dst + 2 * kKHalf, &p.tm_vc, kvh * 128, y, bar);
      tma_load_2d(dst + 2 * kKHalf + kVBox, &p.tm_ks, kvh * 16, y, bar);
      tma_load_2d(dst + 2 * kKHalf + kVBox + kSBox, &p.tm_vs, kvh * 16, y, bar);
    };
    if (lane == 0)
      for (; issued < min(kD16Slots, rg.n_st); ++issued) issue(issued);
    __syncwarp();
    (void)__syncthreads_and(h32_is_hadamard(p.h32, tid, 544));  // (A)
    __syncthreads();                                             // (B) Q staged
    if (lane == 0) {
      for (; issued < rg.n_st; ++issued) {
        // slot i % 4 was last used by stage i - 4 (the same group): wait
        // until that group's 8 warps have released it
        if (!mbar_wait(empty + 8 * (issued % kD16Slots), ((issued / kD16Slots) - 1) & 1)) {
          flag_error(kErrTimeout);
          break;
        }
        issue(issued);
      }
      // never leave with copies in flight: the last slots' fills have landed
      for (int i = max(issued - kD16Slots, 0); i < issued; ++i)
        if (!mbar_wait(full + 8 * (i % kD16Slots), (i / kD16Slots) & 1)) flag_error(kErrTimeout);
    }
    __syncwarp();
    griddep_launch_dependents();
    __syncthreads();  // (C)
    __syncthreads();  // (D)
    __syncthreads();  // (E)
    __syncthreads();  // (F)
    return;
  }
  const bool had = __syncthreads_and(h32_is_hadamard(p.h32, tid, 544)) != 0;
  stage_q_rot<T>(p, kvh, 8, smem + L::kQ, rowfac, had, warp, 2 * kWarps, lane);
  __syncthreads();

  RowState<1> rs;
  init_rows<1>(rs, rowfac, q4, p.q_len, rg.tok_end, len_all);
  float* red = reinterpret_cast<float*>(smem + L::kRed) + grp * kWarps * 8;
  float* red_l = reinterpret_cast<float*>(smem + L::kRedL) + grp * kWarps * 8;
  const uint32_t pbase = sb + L::kP + grp * kStage * 16;
  const StageBar bar{1 + grp};
  int mine = 0;  // stages of this group
  for (int i = grp; i < rg.n_st; i += 2, ++mine) {
    const int slot = i % kD16Slots;
    ok &= mbar_wait(full + 8 * slot, (i / kD16Slots) & 1);
    const int t0 = p.tok_begin + (rg.st_lo + i) * kStage;
    const bool fine = run_stage<1>(rs, sb + L::kRing + slot * kStageBytes, sb + L::kQ, pbase, red, t0,
                                   stage_ok[slot] != 0, ok, gw, lane, bar);
    if (!fine) break;
    __syncwarp();
    if (lane == 0) mbar_arrive(empty + 8 * slot);  // this warp is done with the slot
    done = mine + 1;
  }
  const int expect = rg.n_st > grp ? (rg.n_st - grp + 1) / 2 : 0;
  const bool fine = ok && done == expect;
  if (!fine) flag_error(kErrTimeout);
  griddep_launch_dependents();
  __syncthreads();  // (C) every group done; the producer's copies have all landed
  group_l<1>(rs, red_l, gw, lane);
  __syncthreads();  // (D) both groups' l are in red_l; the ring is idle

  // merge group 1 into group 0: group 1 leaves its m, l and O in the ring
  float* o1 = reinterpret_cast<float*>(smem + L::kRing);  // [8 warps][32 lanes][8]
  float lrow[1][2];
  row_totals<1>(red_l, lane, lrow);
  if (grp == 1) {
    if (gw == 0 && (lane >> 2) == 0) {
#pragma unroll
      for (int e = 0; e < 2; ++e) {
        merge[2 * q4 + e] = fine ? rs.m_run[0][e] : -CUDART_INF_F;
        merge[8 + 2 * q4 + e] = fine ? lrow[0][e] : 0.f;
      }
    }
    float* dst = o1 + (gw * 32 + lane) * 8;
#pragma unroll
    for (int mt = 0; mt < 2; ++mt)
#pragma unroll
      for (int e = 0; e < 4; ++e) dst[mt * 4 + e] = rs.o[mt][0][e];
  }
  __syncthreads();  // (E)
  if (grp == 0) {
    const float* src = o1 + (gw * 32 + lane) * 8;
#pragma unroll
    for (int e = 0; e < 2; ++e) {
      const int rr = 2 * q4 + e;
      const float la = lrow[0][e];
      const float ma = fine ? rs.m_run[0][e] : -CUDART_INF_F;
      const float mb = merge[rr], lb = merge[8 + rr];
      const float M = fmaxf(ma, mb);
      const float wa = (ma == -CUDART_INF_F || la == 0.f) ? 0.f : exp2_approx(ma - M);
      const float wb = (mb == -CUDART_INF_F || lb == 0.f) ? 0.f : exp2_approx(mb - M);
      rs.m_run[0][e] = M;
      lrow[0][e] = wa * la + wb * lb;
#pragma unroll
      for (int mt = 0; mt < 2; ++mt) {
        rs.o[mt][0][e] = wa * rs.o[mt][0][e] + wb * src[mt * 4 + e];
        rs.o[mt][0][2 + e] = wa * rs.o[mt][0][2 + e] + wb * src[mt * 4 + 2 + e];
      }
    }
    write_partials<1>(p, rs, lrow, true, split, kvh, gw, lane);
  }
  __syncthreads();  // (F)
}

// ------------------------------------------------ tcgen05 verify (q_len 2..8)
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
  static constexpr bool kRotated = true;
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
};

template <typename T>
static cudaError_t launch_k8v4_decode16_t(const SplitParams& p, cudaStream_t stream) {
  auto kern = k8v4_decode16_kernel<T>;
  const int smem = k8v4::D16Layout::kBytes;
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
  if (e != cudaSuccess) return e;
  return launch_pdl(kern, dim3(p.num_splits, kKvHeads), dim3(544), (size_t)smem, stream, p);
}

cudaError_t launch_k8v4_split(const SplitParams& p, int dtype, cudaStream_t stream) {
  const int nt = (kGroup * p.q_len + 7) / 8;
  if (nt == 1) {
    if (dtype == kDtypeBF16) return launch_k8v4_decode16_t<__nv_bfloat16>(p, stream);
    return launch_k8v4_decode16_t<__half>(p, stream);
  }
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
