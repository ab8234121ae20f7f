// NVFP4 paged MTP verify (q_len 2..8) on the fifth-generation tensor cores
// (tcgen05: accumulators in tensor memory), sm_100a.
//
// Replaces the q_len > 1 XQA launch of src/qwasar_runtime/xqa.py:484-554
// (MTP verify: q_len query rows per head, lower-right causal, xqa.py:662)
// behind the split ABI of tests/test_attention_kernel_abi.py:13-32.
//
// CTA = one KV head x one split (a run of pages), 19 warps:
//   warp 0      TMA producer of K tiles (codes + scales, 18 KB per 128
//               tokens) into a 3-deep ring;
//   warp 1      TMEM owner (512 columns) and MMA issuer (one thread);
//   warp 2      TMA producer of V tiles into a 2-deep ring;
//   warps 3-18  sixteen math warps: warp w serves TMEM lane quadrant
//               q = w % 4 and quarter u = (w - 3) / 4 of the work (a quarter
//               of the head dim for K and V, of the score columns for the
//               softmax), four warps per scheduler to hide the TMEM,
//               shared-memory and barrier latencies.
// Per 128-token tile i (tokens on the MMA M dimension, head-dim d):
//   K(i)    math: E2M1 x E4M3 -> FP16 (exact) into TMEM as the A operand,
//           lane = token, column = d pair (32x32b stores, thread = token);
//   QK(i)   MMA:  S^T[128 tok x N] = K Q^T into one of two S buffers, N =
//           6 q_len rounded up to 16, Q in shared memory (K-major, 128-byte
//           swizzle, rows scaled by a power of two so BF16 queries convert
//           to FP16 exactly);
//   soft(i) math: base-2 online softmax on S^T (thread = token, packed
//           f32x2 arithmetic): the reference max of a column only moves when
//           a score exceeds it by kLazy (then O is rescaled in TMEM); P in
//           FP16, the PV operand precision of the reference's XQA kernel;
//   V(i)    math: V -> FP16 rows [token][d] in shared memory (the MN-major A
//           operand of PV), P -> [token][N] (the MN-major B operand);
//   PV(i)   MMA:  O^T[256 d x N] += V^T P^T, two M=128 halves of d.
// Order: the math warps dequantise K(i+1) as soon as S(i) is read, so
// QK(i+1) is queued ahead of PV(i); they write V(i) and P(i) only after
// PV(i-1) has finished with the single V and P buffers, which by then it
// long has.  The epilogue writes one (m, l, O) record per query row and
// split, the layout lse_combine_kernel reads.  Every wait is bounded; the math warps decide timeouts
// collectively at a per-tile vote, so named barriers never wait for a warp
// that left.

#include "attn_common.cuh"
#include "nvfp4_quant.cuh"
#include "tc_common.cuh"

namespace qwz {

using namespace detail;

#ifndef QWZ_VT_MATH_WARPS
#define QWZ_VT_MATH_WARPS 16
#endif
constexpr int kVtMathWarps = QWZ_VT_MATH_WARPS;            // 8 or 16
constexpr int kVtMath0 = 3;                                // first math warp
constexpr int kVtWarps = kVtMath0 + kVtMathWarps;
constexpr int kVtParts = kVtMathWarps / 4;                 // math warps per TMEM lane quadrant
static_assert(kVtParts == 2 || kVtParts == 4, "8 or 16 math warps");
constexpr int kVtKStages = 3, kVtVStages = 2;
constexpr int kVtTile = 128;
constexpr int kVtCodeBox = kVtTile * kCodeBytes;           // 16 KB
constexpr int kVtScaleBox = kVtTile * kScaleBytes;         // 2 KB
constexpr int kVtHalfStage = kVtCodeBox + kVtScaleBox;     // 18 KB (K or V of one tile)
constexpr int kVtPidCache = 512;
// TMEM columns: K (A of QK) | S^T buffer 0 | S^T buffer 1 | O^T halves
constexpr uint32_t kTmK = 0, kTmS = 128, kTmO = 256;
constexpr uint32_t kTmCols = 512;

template <int N, class F>
struct VtLayout {
  static constexpr int kKRing = 0;                                      // K tiles (NVFP4: 3 x 18 KB)
  static constexpr int kVRing = kKRing + F::kKStages * F::kKStage;      // V tiles (NVFP4: 2 x 18 KB)
  static constexpr int kVf = (kVRing + F::kVStages * F::kVStage + 1023) / 1024 * 1024;  // V FP16: [2h+a][128 tok][128 B]
  static constexpr int kQ = kVf + 4 * 16384;                         // Q: 4 k-atoms [N x 128 B]
  static constexpr int kPAtoms = (N + 63) / 64;                      // P: n-atoms [128 tok][128 B]
  static constexpr int kP = kQ + N * 512;
  static constexpr int kBars = kP + kPAtoms * 16384;
  // kfull[3] kempty[3] vfull[2] vempty[2] kready pvready s[2] o (15 x 8 B)
  static constexpr int kMeta = kBars + 128;
  static constexpr int kRowfac = kMeta + 32;                         // stage ends, tmem, abort, fin
  static constexpr int kAlpha = kRowfac + 4 * N;
  static constexpr int kMref = kAlpha + 4 * N;
  static constexpr int kWred = kMref + 4 * N;                        // [parts][4 q][N / parts]
  static constexpr int kPid = kWred + 4 * 4 * N;
  static constexpr int kBytes = kPid + 4 * kVtPidCache + 1024;
  static_assert(kVRing + F::kVStages * F::kVStage <= kVf && kVf % 1024 == 0, "ring / V layout");
  static_assert(kQ % 1024 == 0 && kP % 1024 == 0 && kBars % 1024 == 0, "operand atoms are 1024-byte aligned");
  static_assert(8 * (2 * F::kKStages + 2 * F::kVStages + 5) <= 128 && (kMeta + 24) % 8 == 0,
                "mbarriers are 8-byte aligned");
  static_assert(kRowfac % 16 == 0, "row factors are read as float4");
};

namespace {

// Named barrier 1: exactly the kVtMathWarps math warps take part.
constexpr int kVtMathThreads = kVtMathWarps * 32;
QWZ_DEVINL void math_bar() { asm volatile("bar.sync 1, %0;\n" ::"n"(kVtMathThreads) : "memory"); }
QWZ_DEVINL bool math_bar_or(bool v) {
  uint32_t r;
  asm volatile(
      "{\n .reg .pred p, q;\n setp.ne.u32 p, %1, 0;\n bar.red.or.pred q, 1, %2, p;\n"
      " selp.u32 %0, 1, 0, q;\n}\n"
      : "=r"(r)
      : "r"((uint32_t)v), "n"(kVtMathThreads)
      : "memory");
  return r != 0;
}
QWZ_DEVINL uint2 lds64(uint32_t addr) {
  uint2 v;
  asm volatile("ld.shared.v2.u32 {%0,%1}, [%2];\n" : "=r"(v.x), "=r"(v.y) : "r"(addr));
  return v;
}
QWZ_DEVINL float warp_max(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, shfl_xor(v, o));
  return v;
}
QWZ_DEVINL float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += shfl_xor(v, o);
  return v;
}

// tcgen05.ld writes its registers asynchronously; after tcgen05.wait::ld,
// route them through an empty asm so no use is scheduled above the wait.
template <int NC>
QWZ_DEVINL void regs_ready(float (&v)[NC]) {
#pragma unroll
  for (int c = 0; c < NC; ++c) asm volatile("" : "+f"(v[c])::"memory");
}
template <int NC>
QWZ_DEVINL void regs_ready(uint32_t (&v)[NC]) {
#pragma unroll
  for (int c = 0; c < NC; ++c) asm volatile("" : "+r"(v[c])::"memory");
}

// TMEM loads of NC (multiple of 8) consecutive columns into v.
template <int NC>
QWZ_DEVINL void ld_cols(uint32_t taddr, float (&v)[NC]) {
  static_assert(NC % 4 == 0, "4-column granularity");
#pragma unroll
  for (int c = 0; c + 16 <= NC; c += 16) {
    uint32_t r[16];
    tc::ld_32x32b_x16(taddr + c, r);
#pragma unroll
    for (int j = 0; j < 16; ++j) v[c + j] = __uint_as_float(r[j]);
  }
  constexpr int c8 = NC / 16 * 16;
  if constexpr (NC - c8 >= 8) {
    uint32_t r[8];
    tc::ld_32x32b_x8(taddr + c8, r);
#pragma unroll
    for (int j = 0; j < 8; ++j) v[c8 + j] = __uint_as_float(r[j]);
  }
  if constexpr (NC % 8 == 4) {
    uint32_t r[4];
    tc::ld_32x32b_x4(taddr + NC - 4, r);
#pragma unroll
    for (int j = 0; j < 4; ++j) v[NC - 4 + j] = __uint_as_float(r[j]);
  }
}

// TMEM stores of NC (multiple of 4) consecutive columns from v.
template <int NC>
QWZ_DEVINL void st_cols(uint32_t taddr, const float (&v)[NC]) {
#pragma unroll
  for (int c = 0; c + 16 <= NC; c += 16) {
    uint32_t r[16];
#pragma unroll
    for (int j = 0; j < 16; ++j) r[j] = __float_as_uint(v[c + j]);
    tc::st_32x32b_x16(taddr + c, r);
  }
  constexpr int c8 = NC / 16 * 16;
  if constexpr (NC - c8 >= 8) {
    uint32_t r[8];
#pragma unroll
    for (int j = 0; j < 8; ++j) r[j] = __float_as_uint(v[c8 + j]);
    tc::st_32x32b_x8(taddr + c8, r);
  }
  if constexpr (NC % 8 == 4) {
    uint32_t r[4];
#pragma unroll
    for (int j = 0; j < 4; ++j) r[j] = __float_as_uint(v[NC - 4 + j]);
    tc::st_32x32b_x4(taddr + NC - 4, r);
  }
}

// Q rows of this KV head into the K-major operand, scaled per row by a power
// of two (FP16-exact), and the per-row score factor sm_scale*log2e/scale.
template <typename T, int N>
QWZ_DEVINL void stage_q(const SplitParams& p, int kvh, uint32_t qbase, float* rowfac, int mw, int lane) {
  constexpr int kRows = (N + kVtMathWarps - 1) / kVtMathWarps;  // rows of this warp
  uint4 raw[kRows];
#pragma unroll
  for (int j = 0; j < kRows; ++j) {  // all loads first: one memory latency, not kRows
    const int r = mw + j * kVtMathWarps, qi = r / kGroup, hg = r - qi * kGroup;
    raw[j] = make_uint4(0u, 0u, 0u, 0u);
    if (r < N && qi < p.q_len)
      raw[j] = __ldg(reinterpret_cast<const uint4*>(reinterpret_cast<const T*>(p.q) +
                                                    ((size_t)qi * kQHeads + kvh * kGroup + hg) * kHeadDim) + lane);
  }
#pragma unroll
  for (int j = 0; j < kRows; ++j) {
    const int r = mw + j * kVtMathWarps, qi = r / kGroup;
    if (r >= N) break;
    const uint32_t w[4] = {raw[j].x, raw[j].y, raw[j].z, raw[j].w};
    float amax = 0.f;
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const float2 f = InTraits<T>::to_float2(w[i]);
      amax = fmaxf(amax, fmaxf(fabsf(f.x), fabsf(f.y)));
    }
    amax = warp_max(amax);
    const float sc = pow2_row_scale(amax);
    uint32_t h[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const float2 f = InTraits<T>::to_float2(w[i]);
      h[i] = pack_half2(f.x * sc, f.y * sc);
    }
    // d = 8 lane .. +7: k-atom lane / 8, 16-byte chunk lane % 8 of row r
    sts128(qbase + (lane >> 3) * (N * 128) + r * 128 + (((lane & 7) ^ (r & 7)) << 4), h[0], h[1], h[2], h[3]);
    // padding rows (zero Q) keep a positive factor so masked scores stay -inf
    if (lane == 0) rowfac[r] = qi < p.q_len ? p.sm_scale_log2 / sc : p.sm_scale_log2;
  }
}

// Head-dim part u (d in [D u, D u + D), D = 256 / kVtParts) of token row tt
// of a K or V tile (code chunks kCh u .. kCh u + kCh - 1 of 32 values each,
// 128-byte swizzle, and their 2 kCh scales) as f16x2 words in d order,
// handed to put(g, r16) per code chunk g.  `zero` (rows at or past the valid
// end) makes every value 0.
template <class Put>
QWZ_DEVINL void dequant_row_part(uint32_t codes, uint32_t scales, int tt, int u, bool zero, Put put) {
  constexpr int kCh = 8 / kVtParts;
  uint32_t spair[kCh];
  if constexpr (kCh == 2) {
    uint32_t sc = lds32(scales + tt * kScaleBytes + 4 * u);
    if (zero) sc = 0u;
    e4m3x4_to_f16x2x2(sc, spair[0], spair[1]);
  } else {
    uint2 sc = lds64(scales + tt * kScaleBytes + 8 * u);
    if (zero) sc = make_uint2(0u, 0u);
    e4m3x4_to_f16x2x2(sc.x, spair[0], spair[1]);
    e4m3x4_to_f16x2x2(sc.y, spair[2], spair[3]);
  }
#pragma unroll
  for (int c = 0; c < kCh; ++c) {
    const int g = kCh * u + c;
    const uint4 w = lds128(codes + tt * kCodeBytes + ((g ^ (tt & 7)) << 4));
    const uint32_t wv[4] = {w.x, w.y, w.z, w.w};
    const uint32_t sA = __byte_perm(spair[c], 0, 0x1010), sB = __byte_perm(spair[c], 0, 0x3232);
    uint32_t r[16];
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      uint32_t hv[4];
      e2m1x8_to_f16x2x4(wv[j], hv);
      const uint32_t sc2 = j < 2 ? sA : sB;
#pragma unroll
      for (int e = 0; e < 4; ++e) r[4 * j + e] = hmul2_u32(hv[e], sc2);
    }
    put(g, r);
  }
}

// Packed f32x2 arithmetic (one instruction for two lanes of work).
QWZ_DEVINL void ffma2(float& d0, float& d1, float a0, float a1, float b0, float b1, float c0, float c1) {
  uint64_t d;
  asm("{\n .reg .b64 a, b, c;\n mov.b64 a, {%1, %2};\n mov.b64 b, {%3, %4};\n mov.b64 c, {%5, %6};\n"
      " fma.rn.f32x2 %0, a, b, c;\n}\n"
      : "=l"(d)
      : "f"(a0), "f"(a1), "f"(b0), "f"(b1), "f"(c0), "f"(c1));
  asm("mov.b64 {%0, %1}, %2;\n" : "=f"(d0), "=f"(d1) : "l"(d));
}
QWZ_DEVINL void fadd2(float& a0, float& a1, float b0, float b1) {
  uint64_t d;
  asm("{\n .reg .b64 a, b;\n mov.b64 a, {%1, %2};\n mov.b64 b, {%3, %4};\n add.rn.f32x2 %0, a, b;\n}\n"
      : "=l"(d)
      : "f"(a0), "f"(a1), "f"(b0), "f"(b1));
  asm("mov.b64 {%0, %1}, %2;\n" : "=f"(a0), "=f"(a1) : "l"(d));
}
QWZ_DEVINL float fmax3(float a, float b, float c) {
  float d;
  asm("max.f32 %0, %1, %2, %3;\n" : "=f"(d) : "f"(a), "f"(b), "f"(c));
  return d;
}

QWZ_DEVINL void sts64(uint32_t addr, uint32_t a, uint32_t b) {
  asm volatile("st.shared.v2.u32 [%0], {%1,%2};\n" ::"r"(addr), "r"(a), "r"(b));
}

}  // namespace

// The NVFP4 cache: a K or V tile is one 128-token box of E2M1 codes (128 B
// a row, 128-byte swizzle) and one of E4M3 scales (16 B a row).
struct VtNvfp4 {
  static constexpr int kKStages = kVtKStages, kVStages = kVtVStages;
  static constexpr int kKStage = kVtHalfStage, kVStage = kVtHalfStage;
  QWZ_DEVINL static void issue(bool is_k, const SplitParams& p, uint32_t dst, int kvh, int y, uint32_t bar) {
    tma_load_2d(dst, is_k ? &p.tm_kc : &p.tm_vc, kvh * kCodeBytes, y, bar);
    tma_load_2d(dst + kVtCodeBox, is_k ? &p.tm_ks : &p.tm_vs, kvh * kScaleBytes, y, bar);
  }
  template <class Put>
  QWZ_DEVINL static void dequant_k(uint32_t st, int tt, int u, Put put) {
    dequant_row_part(st, st + kVtCodeBox, tt, u, false, put);
  }
  template <class Put>
  QWZ_DEVINL static void dequant_v(uint32_t st, int tt, int u, bool zero, Put put) {
    dequant_row_part(st, st + kVtCodeBox, tt, u, zero, put);
  }
  template <typename T, int N>
  QWZ_DEVINL static void stage(const SplitParams& p, int kvh, uint32_t qbase, float* rowfac, bool, int mw,
                               int lane) {
    stage_q<T, N>(p, kvh, qbase, rowfac, mw, lane);
  }
  QWZ_DEVINL static bool rotation_check(const SplitParams&, int) { return true; }
  QWZ_DEVINL static int o_dim(int d) { return d; }  // the V tile's d order is the head's
  // The fused append: new row s (at logical position pos) of K (tensor 0)
  // or V (1) for KV head kvh, quantised by one warp into the pool and fenced
  // for the TMA reads that follow (the rule of nvfp4_append_kernel).
  template <typename T>
  QWZ_DEVINL static void append_row(const SplitParams& p, int pos, int s, int kvh, int tensor, int lane) {
    const int pp = lookup_page(p, pos, lane == 0 && tensor == 0);
    if (pp < 0) return;
    const size_t row = ((size_t)pp * kPage + (pos & (kPage - 1))) * kKvHeads + kvh;
    const T* src = reinterpret_cast<const T*>(tensor ? p.app_v : p.app_k) + ((size_t)s * kKvHeads + kvh) * kHeadDim;
    uint8_t* codes = const_cast<uint8_t*>(tensor ? p.v_codes : p.k_codes) + row * kCodeBytes;
    uint8_t* scales = const_cast<uint8_t*>(tensor ? p.v_scales : p.k_scales) + row * kScaleBytes;
    quant::quantize_row_lane<T>(src, codes, scales, lane);
    __threadfence();
    fence_proxy_async_global();
  }
};

template <typename T, int N, class F>
__global__ void __launch_bounds__(kVtWarps * 32, 1)
    verify_tc_kernel(const __grid_constant__ SplitParams p) {
  using L = VtLayout<N, F>;
  extern __shared__ __align__(1024) uint8_t smem[];
  const uint32_t sraw = smem_u32(smem);
  const uint32_t sb = (sraw + 1023u) & ~1023u;
  uint8_t* sg = smem + (sb - sraw);
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int split = blockIdx.x, kvh = blockIdx.y;
  const uint32_t bar_kfull = sb + L::kBars, bar_kempty = bar_kfull + 8 * F::kKStages;
  const uint32_t bar_vfull = bar_kempty + 8 * F::kKStages, bar_vempty = bar_vfull + 8 * F::kVStages;
  const uint32_t bar_kready = bar_vempty + 8 * F::kVStages, bar_pv = bar_kready + 8;
  const uint32_t bar_s = bar_pv + 8, bar_o = bar_s + 16;  // bar_s: one per S buffer
  int* kstage_end = reinterpret_cast<int*>(sg + L::kMeta);  // [F::kKStages]
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(sg + L::kMeta + 16);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(sg + L::kMeta + 20);
  const uint32_t bar_fin = sb + L::kMeta + 24;  // the MMA thread's last commit
  float* rowfac = reinterpret_cast<float*>(sg + L::kRowfac);
  float* alpha_s = reinterpret_cast<float*>(sg + L::kAlpha);
  float* mref_s = reinterpret_cast<float*>(sg + L::kMref);
  float* wred = reinterpret_cast<float*>(sg + L::kWred);
  int* pid = reinterpret_cast<int*>(sg + L::kPid);

  if (tid == 0) {
#pragma unroll
    for (int s = 0; s < F::kKStages; ++s) {
      mbar_init(bar_kfull + 8 * s, 1);
      mbar_init(bar_kempty + 8 * s, kVtMathWarps);
    }
#pragma unroll
    for (int s = 0; s < F::kVStages; ++s) {
      mbar_init(bar_vfull + 8 * s, 1);
      mbar_init(bar_vempty + 8 * s, kVtMathWarps);
    }
    mbar_init(bar_kready, kVtMathWarps);
    mbar_init(bar_pv, kVtMathWarps);
    mbar_init(bar_s, 1);
    mbar_init(bar_s + 8, 1);
    mbar_init(bar_o, 1);
    mbar_init(bar_fin, 1);
    *abort_flag = 0;
    mbar_fence_init();
  }
  if (warp == 1) {
    tc::tmem_alloc(sb + L::kMeta + 16, kTmCols);
    tc::tmem_relinquish();
  }
  // barriers and tensor memory are set up while the previous kernel drains;
  // global memory (lengths, table, Q, pages) only after it completes
  griddep_wait();
  // tile-granular split bounds: a split may start or end mid-page, which
  // evens out the splits (at 32K, 7 tiles at most instead of 4 pages = 8)
  const StageRange rg = stage_range<kVtTile>(p, split);
  const int n_tiles = rg.n_st;
  const int page0 = rg.st_lo >> 1;  // this split's first page (pages from tok_begin)
  const int n_pages = n_tiles > 0 ? ((rg.st_lo + n_tiles + 1) >> 1) - page0 : 0;
  const int len_all = __ldg(p.seqlens) + p.len_add;  // causal limits use the whole sequence
  if (warp == 0) {
    for (int i = lane; i < min(n_pages, kVtPidCache); i += 32)
      pid[i] = lookup_page(p, p.tok_begin + (page0 + i) * kPage, true);
  }
  const bool had = F::rotation_check(p, tid);  // the K8/V4 rotation test (a CTA-wide barrier)
  if (p.app_k != nullptr && warp >= kVtMath0) {
    // fused append: the q_len new rows that fall in this CTA's tiles, one
    // warp per (row, K or V), written and fenced before any tile is loaded
    const int first = p.tok_begin + rg.st_lo * kVtTile, last = first + n_tiles * kVtTile;
    const int pre = len_all - p.len_add;
    for (int task = warp - kVtMath0; task < 2 * p.q_len; task += kVtMathWarps) {
      const int srow = task >> 1, pos = pre + srow;
      if (pos >= first && pos < last) F::template append_row<T>(p, pos, srow, kvh, task & 1, lane);
    }
  }
  tc::fence_before();
  __syncthreads();  // barriers, the TMEM base, the page ids and appended rows are in place
  tc::fence_after();
  const uint32_t tbase = *tmem_slot;

  if (warp == 0 || warp == 2) {
    // ----------------------------------------------- producers (K: 0, V: 2)
    const bool is_k = warp == 0;
    const int nst = is_k ? F::kKStages : F::kVStages;
    const int stage_bytes = is_k ? F::kKStage : F::kVStage;
    const uint32_t ring = sb + (is_k ? L::kKRing : L::kVRing);
    const uint32_t full = is_k ? bar_kfull : bar_vfull, empty = is_k ? bar_kempty : bar_vempty;
    const CUtensorMap* tm_c = is_k ? &p.tm_kc : &p.tm_vc;
    const CUtensorMap* tm_s = is_k ? &p.tm_ks : &p.tm_vs;
    if (lane == 0 && n_tiles > 0) {
      tma_prefetch_desc(tm_c);
      tma_prefetch_desc(tm_s);
      int issued = 0;
      for (int i = 0; i < n_tiles; ++i) {
        const int s = i % nst;
        if (*abort_flag) break;
        if (i >= nst && !mbar_wait(empty + 8 * s, ((i / nst) - 1) & 1)) {
          flag_error(kErrTimeout);
          *abort_flag = 1;
          break;
        }
        const int gt = rg.st_lo + i, k = (gt >> 1) - page0;  // tile from tok_begin, page of this split
        const int t0 = p.tok_begin + gt * kVtTile;
        const int pp = k < kVtPidCache ? pid[k] : lookup_page(p, t0, is_k);
        if (is_k) kstage_end[s] = pp >= 0 ? rg.tok_end : t0;  // released by the arrive below
        const uint32_t fb = full + 8 * s;
        issued = i + 1;
        if (pp < 0) {  // bad page id: no copy; the math warps mask the tile
          mbar_arrive(fb);
          continue;
        }
        mbar_arrive_expect_tx(fb, stage_bytes);
        const uint32_t dst = ring + s * stage_bytes;
        const int y = pp * kPage + kVtTile * (gt & 1);
        F::issue(is_k, p, dst, kvh, y, fb);
      }
      // never leave with copies in flight (only reachable after an abort)
      for (int i = max(issued - nst, 0); i < issued; ++i)
        if (!mbar_wait(full + 8 * (i % nst), (i / nst) & 1)) flag_error(kErrTimeout);
    }
  } else if (warp == 1) {
    // ----------------------------------------------------------------- MMA
    if (lane == 0 && n_tiles > 0) {
      constexpr uint32_t idesc_qk = tc::idesc_f16_f32(128, N);
      constexpr uint32_t idesc_pv = tc::idesc_f16_f32(128, N, true, true);
      // Descriptors are built once; a K step adds its byte offset / 16 to the
      // start-address field (addresses stay below 256 KB, so no carry).  The
      // issuing thread shares its scheduler with four math warps: every
      // instruction it saves between two MMAs keeps the tensor pipe fed.
      const uint64_t dq = tc::smem_desc_k128(sb + L::kQ);
      const uint64_t dv = tc::smem_desc_mn128(sb + L::kVf, 16384, 1024);
      const uint64_t dp = tc::smem_desc_mn128(sb + L::kP, 16384, 1024);
      const uint32_t tk = tbase + kTmK, ts = tbase + kTmS, to = tbase + kTmO;
      auto qk = [&](int j) -> bool {
        if (!mbar_wait(bar_kready, j & 1)) return false;
        tc::fence_after();
        const uint32_t d = ts + 64 * (j & 1);
#pragma unroll
        for (int ks = 0; ks < 16; ++ks)
          tc::mma_ts(d, tk + 8 * ks, dq + (uint64_t)(((ks >> 2) * (N * 128) + (ks & 3) * 32) >> 4), idesc_qk,
                     ks > 0);
        tc::commit(bar_s + 8 * (j & 1));
        return true;
      };
      bool fine = qk(0);
      for (int i = 0; fine && i < n_tiles; ++i) {
        if (*abort_flag) break;
        if (i + 1 < n_tiles && !(fine = qk(i + 1))) break;
        if (!(fine = mbar_wait(bar_pv, i & 1))) break;
        tc::fence_after();
#pragma unroll
        for (int h = 0; h < 2; ++h) {
#pragma unroll
          for (int ks = 0; ks < 8; ++ks)
            tc::mma_ss(to + N * h, dv + (uint64_t)((2 * h * 16384 + ks * 2048) >> 4),
                       dp + (uint64_t)((ks * 2048) >> 4), idesc_pv, (i > 0 || ks > 0));
        }
        tc::commit(bar_o);
      }
      if (!fine) {
        flag_error(kErrTimeout);
        *abort_flag = 1;
      }
      // never leave with MMAs in flight: one more commit covers every
      // tcgen05.mma issued so far
      tc::commit(bar_fin);
      if (!mbar_wait(bar_fin, 0)) flag_error(kErrTimeout);
    }
  } else {
    // ---------------------------------------------------------------- math
    constexpr int NP = N / kVtParts;      // score columns of this warp
    constexpr int NO = 2 * N / kVtParts;  // O^T columns this warp rescales and stores
    static_assert(NP % 4 == 0, "P is stored in 8-byte pieces");
    const int q = warp & 3, u = (warp - kVtMath0) >> 2;
    const int ohalf = u & 1, ocol = (u >> 1) * NO;  // this warp's M half of O^T and first column
    const uint32_t lane_base = (uint32_t)(32 * q) << 16;
    const int tt = 32 * q + lane;  // this thread's token row of K, V, S^T and P
    const float* fac = rowfac + NP * u;
    // nm = -(reference max); kMFloor stands for "no score yet": finite, so a
    // masked score (-inf) stays -inf and a real one exceeds it by far more
    // than kLazy
    constexpr float kMFloor = -1e30f;
    float lsum[NP], nm[NP];
#pragma unroll
    for (int c = 0; c < NP; ++c) {
      lsum[c] = 0.f;
      nm[c] = -kMFloor;
    }
    bool ok = true;

    // Q while the producers' first tiles are in flight; QK(0) waits for
    // kready(0), which every math warp arrives at only after staging its rows
    F::template stage<T, N>(p, kvh, sb + L::kQ, rowfac, had, warp - kVtMath0, lane);
    fence_proxy_async_smem();  // Q is read by the tensor core
    math_bar();                // every row's score factor is written before a softmax reads it

    // K(j) -> TMEM, thread = token tt, head-dim part u (columns 16 g ..);
    // returns the tile's valid end, read before the ring slot is released
    auto do_k = [&](int j) -> int {
      const int s = j % F::kKStages;
      ok &= mbar_wait(bar_kfull + 8 * s, (j / F::kKStages) & 1);
      const int end = kstage_end[s];
      const uint32_t st = sb + L::kKRing + s * F::kKStage;
      const uint32_t col = tbase + lane_base + kTmK;
      F::dequant_k(st, tt, u,
                       [&](int g, const uint32_t (&r)[16]) { tc::st_32x32b_x16(col + 16 * g, r); });
      __syncwarp();
      if (lane == 0) mbar_arrive(bar_kempty + 8 * s);
      tc::wait_st();
      tc::fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(bar_kready);
      return end;
    };

    int vend_next = n_tiles > 0 ? do_k(0) : 0;
    int done_tiles = 0;
    for (int i = 0; i < n_tiles; ++i) {
      const int sbuf = i & 1;
      ok &= mbar_wait(bar_s + 8 * sbuf, (i >> 1) & 1);
      tc::fence_after();
      const int t0 = p.tok_begin + (rg.st_lo + i) * kVtTile;
      const int vend = vend_next;

      float x[NP];
      ld_cols<NP>(tbase + lane_base + kTmS + 64 * sbuf + NP * u, x);
      tc::wait_ld();
      regs_ready(x);
      // S(i) is read and QK(i) is done: the K buffer takes K(i+1) now
      if (i + 1 < n_tiles) vend_next = do_k(i + 1);

      // ------------------------------------------------------- softmax(i)
      // causal / length mask only on tiles that reach the end
      if (t0 + kVtTile > min(vend, len_all - (p.q_len - 1))) {
        const int tok = t0 + tt;
#pragma unroll
        for (int c = 0; c < NP; ++c) {
          const int qi = min((NP * u + c) / kGroup, p.q_len - 1);
          if (tok >= min(vend, len_all - (p.q_len - 1 - qi))) x[c] = -CUDART_INF_F;
        }
      }
      // y = x * factor - max (base-2 units), two columns per instruction
      float y[NP];
      float ymax = -CUDART_INF_F;
#pragma unroll
      for (int c = 0; c < NP; c += 4) {
        const float4 f = *reinterpret_cast<const float4*>(fac + c);
        ffma2(y[c], y[c + 1], x[c], x[c + 1], f.x, f.y, nm[c], nm[c + 1]);
        ffma2(y[c + 2], y[c + 3], x[c + 2], x[c + 3], f.z, f.w, nm[c + 2], nm[c + 3]);
        ymax = fmax3(ymax, y[c], y[c + 1]);
        ymax = fmax3(ymax, y[c + 2], y[c + 3]);
      }
      const bool need = ymax > kLazy;
      const bool bad = !ok || *abort_flag;
      if (math_bar_or(need || bad)) {
        if (math_bar_or(bad)) {
          if (tid == kVtMath0 * 32) *abort_flag = 1;
          flag_error(kErrTimeout);
          break;
        }
        // move the reference max of every column to this tile's max
#pragma unroll
        for (int c = 0; c < NP; ++c) {
          const float mx = warp_max(x[c]);
          if (lane == 0) wred[(u * 4 + q) * NP + c] = mx;
        }
        math_bar();
#pragma unroll
        for (int c = 0; c < NP; ++c) {
          float tm = wred[(u * 4) * NP + c];
#pragma unroll
          for (int qq = 1; qq < 4; ++qq) tm = fmaxf(tm, wred[(u * 4 + qq) * NP + c]);
          const float mold = -nm[c];
          const float mnew = fmaxf(mold, tm * fac[c]);  // factor > 0
          const float alpha = exp2_approx(mold - mnew);  // 0 from kMFloor
          lsum[c] *= alpha;
          nm[c] = -mnew;
          y[c] = fmaf(x[c], fac[c], -mnew);
          if (q == 0 && lane == 0) alpha_s[NP * u + c] = alpha;
        }
        math_bar();
        if (i > 0) {  // this warp's block of O^T (M half, column range), after PV(i-1)
          ok &= mbar_wait(bar_o, (i - 1) & 1);
          tc::fence_after();
          const uint32_t oc = tbase + lane_base + kTmO + N * ohalf + ocol;
          float ov[NO];
          ld_cols<NO>(oc, ov);
          tc::wait_ld();
          regs_ready(ov);
#pragma unroll
          for (int j = 0; j < NO; ++j) ov[j] *= alpha_s[ocol + j];
          st_cols<NO>(oc, ov);
        }
        math_bar();  // alpha_s / wred are rewritten by the next slow tile
      }
      uint32_t hw[NP / 2];
#pragma unroll
      for (int j = 0; j < NP / 2; ++j) {
        const float p0 = exp2_approx(y[2 * j]), p1 = exp2_approx(y[2 * j + 1]);
        fadd2(lsum[2 * j], lsum[2 * j + 1], p0, p1);
        hw[j] = pack_half2(p0, p1);
      }

      // ------------------------------ V(i) and P(i) after PV(i-1) is done
      if (i > 0) ok &= mbar_wait(bar_o, (i - 1) & 1);
      {
        const int s = i % F::kVStages;
        ok &= mbar_wait(bar_vfull + 8 * s, (i / F::kVStages) & 1);
        const uint32_t st = sb + L::kVRing + s * F::kVStage;
        const uint32_t vrow = sb + L::kVf + tt * 128;
        F::dequant_v(st, tt, u, t0 + tt >= vend, [&](int g, const uint32_t (&r)[16]) {
          // d = 32g + 8j .. +7: atom g / 2 (64 d), 16-byte chunk 4 (g % 2) + j of the row
#pragma unroll
          for (int j = 0; j < 4; ++j)
            sts128(vrow + (g >> 1) * 16384 + (((4 * (g & 1) + j) ^ (tt & 7)) << 4), r[4 * j], r[4 * j + 1],
                   r[4 * j + 2], r[4 * j + 3]);
        });
        __syncwarp();
        if (lane == 0) mbar_arrive(bar_vempty + 8 * s);
      }
      {
        const uint32_t prow = sb + L::kP + tt * 128;  // N <= 64: one atom
        if constexpr (NP % 8 == 0) {
#pragma unroll
          for (int c = 0; c < NP; c += 8) {
            const int n = NP * u + c;
            sts128(prow + (((n >> 3) ^ (tt & 7)) << 4), hw[c / 2], hw[c / 2 + 1], hw[c / 2 + 2], hw[c / 2 + 3]);
          }
        } else {
#pragma unroll
          for (int c = 0; c < NP; c += 4) {
            const int n = NP * u + c;
            sts64(prow + (((n >> 3) ^ (tt & 7)) << 4) + (n & 4) * 2, hw[c / 2], hw[c / 2 + 1]);
          }
        }
      }
      fence_proxy_async_smem();  // V and P are read by the tensor core
      tc::wait_st();
      tc::fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(bar_pv);
      done_tiles = i + 1;
    }

    // ------------------------------------------------------------ epilogue
    const bool have_o = done_tiles == n_tiles && n_tiles > 0 && !*abort_flag &&
                        mbar_wait(bar_o, (n_tiles - 1) & 1);
    tc::fence_after();
#pragma unroll
    for (int c = 0; c < NP; ++c) {
      const float lw = warp_sum(lsum[c]);
      if (lane == 0) wred[(u * 4 + q) * NP + c] = lw;
      if (q == 0 && lane == 0) mref_s[NP * u + c] = -nm[c];
    }
    math_bar();
    const int rows = kGroup * p.q_len;
    if (q == 0 && lane < NP && NP * u + lane < rows) {
      const int r = NP * u + lane;
      float l = 0.f;
#pragma unroll
      for (int qq = 0; qq < 4; ++qq) l += wred[(u * 4 + qq) * NP + lane];
      if (!have_o) l = 0.f;
      const size_t R = (size_t)(r / kGroup) * kQHeads + kvh * kGroup + r % kGroup;
      const size_t base = R * p.num_splits + split;
      p.partial_ml[base * 2 + 0] = l > 0.f ? mref_s[r] : -CUDART_INF_F;  // no key: empty split
      p.partial_ml[base * 2 + 1] = l;
    }
    {
      const int d = F::o_dim(128 * ohalf + tt);  // O^T lane tt of M half ohalf
      float o[NO];
      if (have_o) {
        ld_cols<NO>(tbase + lane_base + kTmO + N * ohalf + ocol, o);
        tc::wait_ld();
        regs_ready(o);
      }
#pragma unroll
      for (int j = 0; j < NO; ++j) {
        const int r = ocol + j;
        if (r < rows) {
          const size_t R = (size_t)(r / kGroup) * kQHeads + kvh * kGroup + r % kGroup;
          p.partial_o[(R * p.num_splits + split) * kHeadDim + d] = have_o ? o[j] : 0.f;
        }
      }
    }
  }

  griddep_launch_dependents();  // the combine may begin its launch
  tc::fence_before();
  __syncthreads();
  if (warp == 1) {
    tc::fence_after();
    tc::tmem_dealloc(tbase, kTmCols);
  }
}

template <typename T, int N, class F>
cudaError_t launch_verify_tc_n(const SplitParams& p, cudaStream_t stream) {
  using L = VtLayout<N, F>;
  static_assert(L::kBytes <= 227 * 1024, "shared memory");
  static_assert(kTmO + 4 * N <= kTmCols && kTmS + 64 + N <= kTmO, "tensor memory columns");
  auto kernel = verify_tc_kernel<T, N, F>;
  cudaError_t e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, L::kBytes);
  if (e != cudaSuccess) return e;
  return launch_pdl(kernel, dim3(p.num_splits, kKvHeads), dim3(kVtWarps * 32), L::kBytes, stream, p);
}

template <typename T, class F = VtNvfp4>
cudaError_t launch_verify_tc(const SplitParams& p, cudaStream_t stream) {
  const int rows = kGroup * p.q_len;
  if (rows <= 16) return launch_verify_tc_n<T, 16, F>(p, stream);
  if (rows <= 32) return launch_verify_tc_n<T, 32, F>(p, stream);
  if (rows <= 48) return launch_verify_tc_n<T, 48, F>(p, stream);
  return cudaErrorInvalidValue;
}

}  // namespace qwz
