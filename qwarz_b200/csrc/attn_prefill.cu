// NVFP4 paged prefill attention (q_len > 8), sm_100a, tcgen05 with the
// accumulators in tensor memory.
//
// Replaces the reference's staged prefill route (src/qwasar_runtime/
// xqa.py:612-768: gather NVFP4 -> FP16 scratch -> FP8 repage -> PRIMS /
// SDPA) with one kernel that reads the NVFP4 pages directly.  Semantics are
// the reference's `_flash_prefill` (xqa.py:612-673): after the q_len new
// rows are appended, query position s of every head sees the keys
// j <= pre + s (lower-right causal, `causal_lower_right(S, total)`), GQA
// with 6 query heads per KV head, softmax in FP32.
//
// CTA = one KV head x 21 query positions: their 6 x 21 = 126 (position,
// head) rows are the M = 128 rows of the MMAs (2 padding rows).  The CTA
// streams 64-token KV tiles from token 0 to the last row's causal limit.
// 14 warps:
//   warps 0-3   softmax and epilogue, thread = row (TMEM lane): the row max,
//               the lazy rescale of the row's O and the row sum stay inside
//               the thread, with no cross-warp vote;
//   warp 4      TMA producer: K and V codes + scales of a tile (2 x 9 KB)
//               into 3-deep rings;
//   warp 5      TMEM owner (512 columns) and MMA issuer (one thread);
//   warps 6-9   dequant K, warps 10-13 dequant V: a tile -> FP16
//               [64 tok][256 d] in shared memory (4 head-dim atoms of 64 tok
//               x 128 B, 128-byte swizzle), thread = (token, half of d).  The
//               same bytes are the K-major B operand of QK and the MN-major
//               B operand of PV.  K has two buffers, so K(j+1) is written
//               while QK(j) reads K(j); V has one, written once PV(j-1) is
//               done.
// Per tile j:
//   QK(j)  S[128 rows x 64 tok] = Q K^T, A = Q (K-major in shared memory,
//          rows scaled by a power of two so they convert to FP16 exactly),
//          B = K(j); into one of two S buffers in TMEM;
//   soft   base-2 online softmax per row (packed f32x2 arithmetic; the
//          mask only on tiles that cross a row's causal limit); P in FP16
//          (the reference's PV operand precision) written to TMEM as the A
//          operand of PV;
//   PV(j)  O[128 x 256] += P V(j), A = P from TMEM, B = V(j) MN-major.
// The MMA thread issues QK(j+1) ahead of PV(j).  Every wait
// is bounded; a role that times out raises the abort flag and the others
// leave at their next wait.
//
// The same kernel, instantiated with kDense, is the draft model's prefill
// (engine/forward/draft.py:33-61 `draft_attend`: bottom-right causal
// attention of q_len FP16 rows over an FP16 K/V of kv_len rows, which the
// reference runs as SDPA, or as an FP8 repage + sm120 paged FMHA for long
// chunks, draft.py:99-181).  Here the K and V rows are read in place.

#include "attn_common.cuh"
#include "tc_common.cuh"

namespace qwz {

using namespace detail;

constexpr int kPfPos = 21;                             // query positions per CTA
constexpr int kPfRows = 128;                           // MMA M (126 rows used)
constexpr int kPfTok = 64;                             // KV tokens per tile
constexpr int kPfStages = 3;                           // TMA ring depth (tiles)
constexpr int kPfSoftWarps = 4;                        // warps 0-3
constexpr int kPfProd = 4;                             // TMA producer warp
constexpr int kPfMma = 5;                              // TMEM owner + MMA issuer
constexpr int kPfDq0 = 6;                              // first dequant warp (K: 6-9, V: 10-13)
constexpr int kPfDqWarps = 4;                          // per tensor
constexpr int kPfWarps = kPfDq0 + 2 * kPfDqWarps;      // 14
constexpr int kPfPidCache = 512;                       // table entries staged in smem
constexpr int kPfTileBytes = 4 * kPfTok * 128;         // one FP16 tile: 4 d-atoms [64 tok x 128 B]
// shared memory, offsets from the 1024-byte aligned base
constexpr int kPfQ = 0;                                // Q: 4 k-atoms [128 rows x 128 B]
constexpr int kPfK = kPfQ + 4 * kPfRows * 128;         // two K tiles FP16
constexpr int kPfV = kPfK + 2 * kPfTileBytes;          // one V tile FP16
constexpr int kPfCodeBox = kPfTok * kCodeBytes;        // 8 KB
constexpr int kPfScaleBox = kPfTok * kScaleBytes;      // 1 KB
constexpr int kPfStage = kPfCodeBox + kPfScaleBox;     // 9 KB
constexpr int kPfKRing = kPfV + kPfTileBytes;
constexpr int kPfVRing = kPfKRing + kPfStages * kPfStage;
constexpr int kPfBars = kPfVRing + kPfStages * kPfStage;
// kfull[3] kempty[3] vfull[3] vempty[3] kready[2] kfree[2] sfull[2]
// sfree[2] vready pready pvdone fin
constexpr int kPfNumBars = 4 * kPfStages + 12;
constexpr int kPfMeta = kPfBars + 8 * kPfNumBars;      // TMEM base, abort flag
constexpr int kPfRowfac = kPfMeta + 16;                // [128] row score factors
constexpr int kPfPid = kPfRowfac + 4 * kPfRows;        // [kPfPidCache] page ids
constexpr int kPfSmem = kPfPid + 4 * kPfPidCache + 1024;
static_assert(kPfKRing % 1024 == 0 && kPfVRing % 1024 == 0 && kPfStage % 1024 == 0,
              "TMA destinations with the 128-byte swizzle are 1024-byte aligned");
static_assert(kPfBars % 8 == 0 && kPfRowfac % 16 == 0 && kPfPid % 4 == 0, "alignment");
static_assert(kPfSmem <= 227 * 1024, "shared memory");
static_assert(kPfV + 2 * kPfTileBytes <= kPfBars, "dense source: the second V tile reuses the code rings");
// tensor-memory columns: S buffers 0 and 1, P (FP16 pairs), O
constexpr uint32_t kPfTmS = 0, kPfTmP = 128, kPfTmO = 256, kPfTmCols = 512;

namespace {

enum PfBar : int {
  kBarKFull = 0,
  kBarKEmpty = kPfStages,
  kBarVFull = 2 * kPfStages,
  kBarVEmpty = 3 * kPfStages,
  kBarKReady = 4 * kPfStages,  // two (per K buffer)
  kBarKFree = kBarKReady + 2,   // two
  kBarSFull = kBarKFree + 2,    // two
  kBarSFree = kBarSFull + 2,  // two
  kBarVReady = kBarSFree + 2,
  kBarPReady,
  kBarPvDone,
  kBarFin,
};
static_assert(kBarFin + 1 == kPfNumBars, "barrier count");

// Packed f32x2 arithmetic (one instruction for two lanes of work) and the
// 3-input max.
QWZ_DEVINL void pf_ffma2(float& d0, float& d1, float a0, float a1, float b, float c) {
  uint64_t d;
  asm("{\n .reg .b64 a, b, c;\n mov.b64 a, {%1, %2};\n mov.b64 b, {%3, %3};\n mov.b64 c, {%4, %4};\n"
      " fma.rn.f32x2 %0, a, b, c;\n}\n"
      : "=l"(d)
      : "f"(a0), "f"(a1), "f"(b), "f"(c));
  asm("mov.b64 {%0, %1}, %2;\n" : "=f"(d0), "=f"(d1) : "l"(d));
}
QWZ_DEVINL void pf_fadd2(float& a0, float& a1, float b0, float b1) {
  uint64_t d;
  asm("{\n .reg .b64 a, b;\n mov.b64 a, {%1, %2};\n mov.b64 b, {%3, %4};\n add.rn.f32x2 %0, a, b;\n}\n"
      : "=l"(d)
      : "f"(a0), "f"(a1), "f"(b0), "f"(b1));
  asm("mov.b64 {%0, %1}, %2;\n" : "=f"(a0), "=f"(a1) : "l"(d));
}
QWZ_DEVINL float pf_fmax3(float a, float b, float c) {
  float d;
  asm("max.f32 %0, %1, %2, %3;\n" : "=f"(d) : "f"(a), "f"(b), "f"(c));
  return d;
}

// Half u0/2 of token row tt (head-dim atoms u0 and u0 + 1: code chunks
// 2u0 .. 2u0+3, scales 4u0 .. 4u0+7) -> FP16.  Every shared-memory load is
// issued before the first convert, so their latencies overlap.
QWZ_DEVINL void pf_dequant_half(uint32_t codes, uint32_t scales, uint32_t out, int tt, int u0, bool zero) {
  uint32_t s0, s1;
  asm volatile("ld.shared.v2.u32 {%0,%1}, [%2];\n" : "=r"(s0), "=r"(s1) : "r"(scales + tt * kScaleBytes + 4 * u0));
  uint4 w[4];
#pragma unroll
  for (int c = 0; c < 4; ++c) w[c] = lds128(codes + tt * kCodeBytes + (((2 * u0 + c) ^ (tt & 7)) << 4));
  if (zero) s0 = s1 = 0u;
  uint32_t h[4];
  e4m3x4_to_f16x2x2(s0, h[0], h[1]);
  e4m3x4_to_f16x2x2(s1, h[2], h[3]);
#pragma unroll
  for (int c = 0; c < 4; ++c) {  // code chunk 2u0 + c: head dim 32 (2u0 + c) .. +31
    const uint32_t wv[4] = {w[c].x, w[c].y, w[c].z, w[c].w};
    const uint32_t row = out + (u0 + (c >> 1)) * (kPfTok * 128) + tt * 128;
#pragma unroll
    for (int j = 0; j < 4; ++j) {  // 8 values: scale 2c + j / 2 of the eight
      const int b = 2 * c + (j >> 1);
      const uint32_t s2 = __byte_perm(h[b >> 1], 0, (b & 1) ? 0x3232 : 0x1010);
      uint32_t hv[4];
      e2m1x8_to_f16x2x4(wv[j], hv);
      sts128(row + (((4 * (c & 1) + j) ^ (tt & 7)) << 4), hmul2_u32(hv[0], s2), hmul2_u32(hv[1], s2),
             hmul2_u32(hv[2], s2), hmul2_u32(hv[3], s2));
    }
  }
}

template <int NC>
QWZ_DEVINL void pf_regs_ready(float (&v)[NC]) {
#pragma unroll
  for (int c = 0; c < NC; ++c) asm volatile("" : "+f"(v[c])::"memory");
}

}  // namespace

// kDense = false: the NVFP4 paged cache (dequant warps 6-13).
// kDense = true: FP16 K, V [kv_len, 4, 256] rows (the draft model's cache);
// the producer's TMA writes the tiles straight into the FP16 operand layout,
// K and V both double-buffered, and warps 6-13 are not launched.
template <typename T, bool kDense>
__global__ void __launch_bounds__(kPfWarps * 32, 1) prefill_attn_kernel(const __grid_constant__ PrefillParams p) {
  constexpr int kWarps = kDense ? kPfDq0 : kPfWarps;
  extern __shared__ __align__(1024) uint8_t smem[];
  const uint32_t sraw = smem_u32(smem);
  const uint32_t sb = (sraw + 1023u) & ~1023u;
  uint8_t* sg = smem + (sb - sraw);
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int blk = blockIdx.x, kvh = blockIdx.y;
  const uint32_t bars = sb + kPfBars;
  auto bar = [&](int i) -> uint32_t { return bars + 8u * (uint32_t)i; };
  volatile int* abort_flag = reinterpret_cast<volatile int*>(sg + kPfMeta + 4);
  float* rowfac = reinterpret_cast<float*>(sg + kPfRowfac);
  int* pid = reinterpret_cast<int*>(sg + kPfPid);

  if (tid == 0) {
    // dense: KReady[b] / VFull[b] complete on the TMA bytes, VEmpty[b] on
    // the PV commit that read V buffer b
#pragma unroll
    for (int s = 0; s < kPfStages; ++s) {
      mbar_init(bar(kBarKFull + s), 1);
      mbar_init(bar(kBarKEmpty + s), kDense ? 1 : kPfDqWarps);
      mbar_init(bar(kBarVFull + s), 1);
      mbar_init(bar(kBarVEmpty + s), kDense ? 1 : kPfDqWarps);
    }
    mbar_init(bar(kBarKReady), kDense ? 1 : kPfDqWarps);
    mbar_init(bar(kBarKReady + 1), kDense ? 1 : kPfDqWarps);
    mbar_init(bar(kBarKFree), 1);
    mbar_init(bar(kBarKFree + 1), 1);
    mbar_init(bar(kBarSFull), 1);
    mbar_init(bar(kBarSFull + 1), 1);
    mbar_init(bar(kBarSFree), kPfSoftWarps);
    mbar_init(bar(kBarSFree + 1), kPfSoftWarps);
    mbar_init(bar(kBarVReady), kPfDqWarps);
    mbar_init(bar(kBarPReady), kPfSoftWarps);
    mbar_init(bar(kBarPvDone), 1);
    mbar_init(bar(kBarFin), 1);
    *abort_flag = 0;
    mbar_fence_init();
  }
  if (warp == kPfMma) {
    tc::tmem_alloc(sb + kPfMeta, kPfTmCols);
    tc::tmem_relinquish();
  }
  griddep_wait();  // barriers and tensor memory are set up while the previous kernel drains

  const int pre = kDense ? p.pre_len : __ldg(p.seqlens);
  const int S = p.q_len;
  const int L = pre + S;                          // post-append length
  const int pos0 = blk * kPfPos;
  const int npos = min(kPfPos, S - pos0);         // >= 1 by the grid size
  const int lim_max = pre + pos0 + npos;          // tokens the CTA's last position sees
  const int n_tiles = (lim_max + kPfTok - 1) / kPfTok;

  // the pages of the tiles, staged once
  if constexpr (!kDense) {
    const int n_pg = min((lim_max + kPage - 1) / kPage, min(p.table_width, kPfPidCache));
    for (int i = tid; i < n_pg; i += kWarps * 32) {
      const int pp = __ldg(p.block_table + i);
      pid[i] = (pp >= 0 && pp < p.num_pages) ? pp : -1;
    }
  }
  // Q rows -> K-major FP16 operand, row r = (position r / 6, head r % 6),
  // scaled by a power of two (exact for BF16 and FP16 inputs)
  for (int r = warp; r < kPfRows; r += kWarps) {
    const int pos = pos0 + r / kGroup;
    const bool valid = r < kGroup * kPfPos && pos < S;
    uint32_t w[4] = {0u, 0u, 0u, 0u};
    if (valid) {
      const uint4 v = __ldg(reinterpret_cast<const uint4*>(reinterpret_cast<const T*>(p.q) +
                                                           ((size_t)pos * kQHeads + kvh * kGroup + r % kGroup) *
                                                               kHeadDim) +
                            lane);
      w[0] = v.x; w[1] = v.y; w[2] = v.z; w[3] = v.w;
    }
    float amax = 0.f;
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const float2 f = InTraits<T>::to_float2(w[i]);
      amax = fmaxf(amax, fmaxf(fabsf(f.x), fabsf(f.y)));
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) amax = fmaxf(amax, shfl_xor(amax, o));
    const float sc = pow2_row_scale(amax);
    uint32_t h[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const float2 f = InTraits<T>::to_float2(w[i]);
      h[i] = pack_half2(f.x * sc, f.y * sc);
    }
    // d = 8 lane .. +7: k-atom lane / 8, 16-byte chunk lane % 8 of row r
    sts128(sb + kPfQ + (lane >> 3) * (kPfRows * 128) + r * 128 + (((lane & 7) ^ (r & 7)) << 4), h[0], h[1],
           h[2], h[3]);
    if (lane == 0) rowfac[r] = valid ? p.sm_scale_log2 / sc : p.sm_scale_log2;
  }
  fence_proxy_async_smem();  // Q is read by the tensor core
  tc::fence_before();
  __syncthreads();
  tc::fence_after();
  const uint32_t tbase = *reinterpret_cast<volatile uint32_t*>(sg + kPfMeta);

  if (kDense && warp == kPfProd) {
    // ------------------------------------- TMA producer, dense FP16 rows
    // tile i -> K buffer i & 1 and V buffer i & 1: four boxes of 64 tokens
    // x 128 B (64 head dims) each, 128-byte swizzle = the operand layout.
    // Rows past kv_len read as zeros.
    if (lane == 0 && n_tiles > 0) {
      tma_prefetch_desc(&p.tm_kc);
      tma_prefetch_desc(&p.tm_vc);
      int issued_k = 0, issued_v = 0;
      for (int i = 0; i < n_tiles; ++i) {
        const int b = i & 1;
        const uint32_t ph = ((i - 2) >> 1) & 1;
        if (*abort_flag) break;
        if (i >= 2 && !mbar_wait(bar(kBarKFree + b), ph)) {  // QK(i-2) read K buffer b
          flag_error(kErrTimeout);
          *abort_flag = 1;
          break;
        }
        const uint32_t kr = bar(kBarKReady + b);
        mbar_arrive_expect_tx(kr, kPfTileBytes);
#pragma unroll
        for (int a = 0; a < 4; ++a)
          tma_load_2d(sb + kPfK + b * kPfTileBytes + a * (kPfTok * 128), &p.tm_kc,
                      kvh * (kHeadDim * 2) + a * 128, i * kPfTok, kr);
        issued_k = i + 1;
        if (i >= 2 && !mbar_wait(bar(kBarVEmpty + b), ph)) {  // PV(i-2) read V buffer b
          flag_error(kErrTimeout);
          *abort_flag = 1;
          break;
        }
        const uint32_t vr = bar(kBarVFull + b);
        mbar_arrive_expect_tx(vr, kPfTileBytes);
#pragma unroll
        for (int a = 0; a < 4; ++a)
          tma_load_2d(sb + kPfV + b * kPfTileBytes + a * (kPfTok * 128), &p.tm_vc,
                      kvh * (kHeadDim * 2) + a * 128, i * kPfTok, vr);
        issued_v = i + 1;
      }
      // never leave with copies in flight (only reachable after an abort)
      for (int i = max(issued_k - 2, 0); i < issued_k; ++i)
        if (!mbar_wait(bar(kBarKReady + (i & 1)), (i >> 1) & 1)) flag_error(kErrTimeout);
      for (int i = max(issued_v - 2, 0); i < issued_v; ++i)
        if (!mbar_wait(bar(kBarVFull + (i & 1)), (i >> 1) & 1)) flag_error(kErrTimeout);
    }
  } else if (warp == kPfProd) {
    // -------------------------------------------------------- TMA producer
    if (lane == 0 && n_tiles > 0) {
      tma_prefetch_desc(&p.tm_kc);
      tma_prefetch_desc(&p.tm_vc);
      tma_prefetch_desc(&p.tm_ks);
      tma_prefetch_desc(&p.tm_vs);
      int issued = 0;
      for (int i = 0; i < n_tiles; ++i) {
        const int s = i % kPfStages;
        if (*abort_flag) break;
        if (i >= kPfStages) {
          const uint32_t ph = ((i / kPfStages) - 1) & 1;
          if (!mbar_wait(bar(kBarKEmpty + s), ph) || !mbar_wait(bar(kBarVEmpty + s), ph)) {
            flag_error(kErrTimeout);
            *abort_flag = 1;
            break;
          }
        }
        const int t0 = i * kPfTok;
        const int lp = t0 >> 8;
        int pp = -1;
        if (lp < p.table_width) {
          pp = lp < kPfPidCache ? pid[lp] : __ldg(p.block_table + lp);
          if (pp >= p.num_pages) pp = -1;
        }
        issued = i + 1;
        const uint32_t kf = bar(kBarKFull + s), vf = bar(kBarVFull + s);
        if (pp < 0) {  // bad table entry: no copy (the tile's bytes are stale)
          flag_error(lp < p.table_width ? kErrPageRange : kErrTableRange);
          mbar_arrive(kf);
          mbar_arrive(vf);
          continue;
        }
        const int y = pp * kPage + (t0 & (kPage - 1));
        const uint32_t kd = sb + kPfKRing + s * kPfStage, vd = sb + kPfVRing + s * kPfStage;
        mbar_arrive_expect_tx(kf, kPfStage);
        tma_load_2d(kd, &p.tm_kc, kvh * kCodeBytes, y, kf);
        tma_load_2d(kd + kPfCodeBox, &p.tm_ks, kvh * kScaleBytes, y, kf);
        mbar_arrive_expect_tx(vf, kPfStage);
        tma_load_2d(vd, &p.tm_vc, kvh * kCodeBytes, y, vf);
        tma_load_2d(vd + kPfCodeBox, &p.tm_vs, kvh * kScaleBytes, y, vf);
      }
      // never leave with copies in flight (only reachable after an abort)
      for (int i = max(issued - kPfStages, 0); i < issued; ++i) {
        const uint32_t ph = (i / kPfStages) & 1;
        if (!mbar_wait(bar(kBarKFull + i % kPfStages), ph) || !mbar_wait(bar(kBarVFull + i % kPfStages), ph))
          flag_error(kErrTimeout);
      }
    }
  } else if (warp == kPfMma) {
    // ------------------------------------------------------------------ MMA
    if (lane == 0 && n_tiles > 0) {
      constexpr uint32_t idesc_qk = tc::idesc_f16_f32(kPfRows, kPfTok);
      constexpr uint32_t idesc_pv = tc::idesc_f16_f32(kPfRows, kHeadDim, /*b_mn_major=*/true);
      const uint64_t dq = tc::smem_desc_k128(sb + kPfQ);
      const uint64_t dk0 = tc::smem_desc_k128(sb + kPfK);
      const uint64_t dv = tc::smem_desc_mn128(sb + kPfV, kPfTok * 128, 1024);
      bool fine = true;
      auto qk = [&](int j) -> bool {
        if (!mbar_wait(bar(kBarKReady + (j & 1)), (j >> 1) & 1)) return false;
        if (j >= 2 && !mbar_wait(bar(kBarSFree + (j & 1)), ((j - 2) >> 1) & 1)) return false;
        tc::fence_after();
        const uint32_t d = tbase + kPfTmS + 64u * (j & 1);
        const uint64_t dk = dk0 + (uint64_t)(((j & 1) * kPfTileBytes) >> 4);
#pragma unroll
        for (int ks = 0; ks < kHeadDim / 16; ++ks)
          tc::mma_ss(d, dq + (uint64_t)(((ks >> 2) * (kPfRows * 128) + (ks & 3) * 32) >> 4),
                     dk + (uint64_t)(((ks >> 2) * (kPfTok * 128) + (ks & 3) * 32) >> 4), idesc_qk, ks > 0);
        tc::commit(bar(kBarSFull + (j & 1)));
        tc::commit(bar(kBarKFree + (j & 1)));
        return true;
      };
      auto pv = [&](int j) -> bool {
        if (!mbar_wait(bar(kBarPReady), j & 1)) return false;
        if (kDense ? !mbar_wait(bar(kBarVFull + (j & 1)), (j >> 1) & 1) : !mbar_wait(bar(kBarVReady), j & 1))
          return false;
        tc::fence_after();
        const uint64_t dvj = kDense ? dv + (uint64_t)(((j & 1) * kPfTileBytes) >> 4) : dv;
#pragma unroll
        for (int kk = 0; kk < kPfTok / 16; ++kk)
          tc::mma_ts(tbase + kPfTmO, tbase + kPfTmP + 8u * kk, dvj + (uint64_t)((kk * 2048) >> 4), idesc_pv,
                     (j > 0 || kk > 0) ? 1u : 0u);
        tc::commit(bar(kBarPvDone));
        if (kDense) tc::commit(bar(kBarVEmpty + (j & 1)));
        return true;
      };
      fine = qk(0);
      for (int j = 0; fine && j < n_tiles; ++j) {
        if (*abort_flag) break;
        if (j + 1 < n_tiles && !(fine = qk(j + 1))) break;
        fine = pv(j);
      }
      if (!fine) {
        flag_error(kErrTimeout);
        *abort_flag = 1;
      }
      // never leave with MMAs in flight
      tc::commit(bar(kBarFin));
      if (!mbar_wait(bar(kBarFin), 0)) flag_error(kErrTimeout);
    }
  } else if (!kDense && warp >= kPfDq0) {
    // ------------------------------------------------- dequant (K or V)
    const bool is_k = warp < kPfDq0 + kPfDqWarps;
    const int t = (warp - kPfDq0 - (is_k ? 0 : kPfDqWarps)) * 32 + lane;
    const int tt = t >> 1, u0 = 2 * (t & 1);  // token row of the tile, first of two head-dim atoms
    bool ok = true;
    for (int i = 0; i < n_tiles; ++i) {
      const int s = i % kPfStages;
      const bool stale = i * kPfTok + tt >= L;
      ok &= mbar_wait(bar((is_k ? kBarKFull : kBarVFull) + s), (i / kPfStages) & 1);
      if (is_k) {
        if (i >= 2) ok &= mbar_wait(bar(kBarKFree + (i & 1)), ((i - 2) >> 1) & 1);  // QK(i-2) read the buffer
      } else {
        if (i >= 1) ok &= mbar_wait(bar(kBarPvDone), (i - 1) & 1);  // PV(i-1) read the V buffer
      }
      if (__any_sync(kFull, !ok || *abort_flag)) break;  // the whole warp leaves together
      const uint32_t ring = sb + (is_k ? kPfKRing : kPfVRing) + s * kPfStage;
      const uint32_t dst = sb + (is_k ? kPfK + (i & 1) * kPfTileBytes : kPfV);
      pf_dequant_half(ring, ring + kPfCodeBox, dst, tt, u0, stale);
      fence_proxy_async_smem();
      __syncwarp();
      if (lane == 0) {
        mbar_arrive(bar((is_k ? kBarKEmpty : kBarVEmpty) + s));
        mbar_arrive(bar(is_k ? kBarKReady + (i & 1) : kBarVReady));
      }
    }
    if (__any_sync(kFull, !ok) && lane == 0) {
      flag_error(kErrTimeout);
      *abort_flag = 1;
    }
  } else {
    // ------------------------------------------------- softmax (thread = row)
    // tcgen05.ld / st / wait are warp-collective (.sync.aligned): every
    // branch around them below is decided by a warp vote.
    const int r = 32 * warp + lane;
    const int pos = pos0 + r / kGroup;
    const bool valid = r < kGroup * kPfPos && pos < S;
    const int limit = valid ? pre + pos + 1 : 1;  // keys j < limit are visible
    const float fac = rowfac[r];
    const uint32_t lane_base = (uint32_t)(32 * warp) << 16;
    float m_ref = -CUDART_INF_F, la = 0.f, lb = 0.f;  // the row sum in two halves (packed adds)
    bool ok = true;
    int done = 0;
    for (int j = 0; j < n_tiles; ++j) {
      ok &= mbar_wait(bar(kBarSFull + (j & 1)), (j >> 1) & 1);
      if (__any_sync(kFull, !ok || *abort_flag)) break;
      tc::fence_after();
      float x[kPfTok];
#pragma unroll
      for (int c = 0; c < kPfTok; c += 16) {
        uint32_t rr[16];
        tc::ld_32x32b_x16(tbase + lane_base + kPfTmS + 64u * (j & 1) + c, rr);
#pragma unroll
        for (int e = 0; e < 16; ++e) x[c + e] = __uint_as_float(rr[e]);
      }
      tc::wait_ld();
      pf_regs_ready(x);
      tc::fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(bar(kBarSFree + (j & 1)));  // QK(j+2) may overwrite this buffer

      const int t0 = j * kPfTok;
      if (!__all_sync(kFull, t0 + kPfTok <= limit)) {  // a diagonal tile: keys past the row's limit
#pragma unroll
        for (int c = 0; c < kPfTok; ++c) x[c] = (t0 + c < limit) ? x[c] : -CUDART_INF_F;
      }
      // raw row max (fac > 0, so the scaled max is the max scaled)
      float mr = -CUDART_INF_F;
#pragma unroll
      for (int c = 0; c < kPfTok; c += 2) mr = pf_fmax3(mr, x[c], x[c + 1]);
      const float mt = mr * fac;
      // the row's reference max moves only by more than 2^kLazy
      const bool need = mt > m_ref + kLazy;
      const float m_new = need ? mt : m_ref;
      const float alpha = (need && m_ref != -CUDART_INF_F) ? exp2_approx(m_ref - m_new) : 1.f;
      const float mu = m_new == -CUDART_INF_F ? 0.f : m_new;
      la *= alpha;
      lb *= alpha;
      uint32_t pw[kPfTok / 2];
#pragma unroll
      for (int c = 0; c < kPfTok / 2; ++c) {
        float p0, p1;
        pf_ffma2(p0, p1, x[2 * c], x[2 * c + 1], fac, -mu);  // base-2 score minus the reference max
        p0 = exp2_approx(p0);
        p1 = exp2_approx(p1);
        pf_fadd2(la, lb, p0, p1);
        pw[c] = pack_half2(p0, p1);
      }
      m_ref = m_new;
      // O and the P buffer are free once PV(j-1) is done
      if (j > 0) {
        ok &= mbar_wait(bar(kBarPvDone), (j - 1) & 1);
        if (__any_sync(kFull, !ok)) break;
        tc::fence_after();
        if (__any_sync(kFull, alpha != 1.f)) {  // lanes whose max did not move scale by 1
#pragma unroll 1
          for (int c = 0; c < kHeadDim; c += 16) {
            uint32_t rr[16];
            tc::ld_32x32b_x16(tbase + lane_base + kPfTmO + c, rr);
            tc::wait_ld();
#pragma unroll
            for (int e = 0; e < 16; ++e) rr[e] = __float_as_uint(__uint_as_float(rr[e]) * alpha);
            tc::st_32x32b_x16(tbase + lane_base + kPfTmO + c, rr);
          }
        }
      }
#pragma unroll
      for (int c = 0; c < kPfTok / 2; c += 16) {
        uint32_t rr[16];
#pragma unroll
        for (int e = 0; e < 16; ++e) rr[e] = pw[c + e];
        tc::st_32x32b_x16(tbase + lane_base + kPfTmP + c, rr);
      }
      tc::wait_st();
      tc::fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(bar(kBarPReady));
      done = j + 1;
    }
    if (__any_sync(kFull, !ok) && lane == 0) {
      flag_error(kErrTimeout);
      *abort_flag = 1;
    }
    // ------------------------------------------------------------ epilogue
    // (warp-uniform: all lanes load O, the rows that exist store it)
    bool have_o = done == n_tiles && n_tiles > 0 && !*abort_flag;
    have_o = __all_sync(kFull, have_o);
    if (have_o) have_o = __all_sync(kFull, mbar_wait(bar(kBarPvDone), (n_tiles - 1) & 1));
    tc::fence_after();
    {
      T* out = reinterpret_cast<T*>(p.out) + ((size_t)(valid ? pos : 0) * kQHeads + kvh * kGroup + r % kGroup) * kHeadDim;
      const float l = la + lb;
      const float inv = (have_o && l > 0.f) ? 1.f / l : 0.f;
#pragma unroll 1
      for (int c = 0; c < kHeadDim; c += 16) {
        uint32_t rr[16];
        if (have_o) {
          tc::ld_32x32b_x16(tbase + lane_base + kPfTmO + c, rr);
          tc::wait_ld();
        } else {
#pragma unroll
          for (int e = 0; e < 16; ++e) rr[e] = 0u;
        }
        if (!valid) continue;
        uint32_t packed[8];
#pragma unroll
        for (int e = 0; e < 8; ++e) {
          const T a = InTraits<T>::from_float(__uint_as_float(rr[2 * e]) * inv);
          const T b = InTraits<T>::from_float(__uint_as_float(rr[2 * e + 1]) * inv);
          packed[e] = (uint32_t)(*reinterpret_cast<const uint16_t*>(&a)) |
                      ((uint32_t)(*reinterpret_cast<const uint16_t*>(&b)) << 16);
        }
        uint4* dst = reinterpret_cast<uint4*>(out + c);
        dst[0] = make_uint4(packed[0], packed[1], packed[2], packed[3]);
        dst[1] = make_uint4(packed[4], packed[5], packed[6], packed[7]);
      }
    }
  }

  griddep_launch_dependents();
  tc::fence_before();
  __syncthreads();
  if (warp == kPfMma) {
    tc::fence_after();
    tc::tmem_dealloc(tbase, kPfTmCols);
  }
}

cudaError_t launch_nvfp4_prefill(const PrefillParams& p, int dtype, cudaStream_t stream) {
  if (p.q_len <= 0) return cudaSuccess;
  auto kernel = dtype == kDtypeBF16 ? prefill_attn_kernel<__nv_bfloat16, false> : prefill_attn_kernel<__half, false>;
  cudaError_t e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, kPfSmem);
  if (e != cudaSuccess) return e;
  const dim3 grid((unsigned)((p.q_len + kPfPos - 1) / kPfPos), kKvHeads);
  return launch_pdl(kernel, grid, dim3(kPfWarps * 32), kPfSmem, stream, p);
}

cudaError_t launch_draft_prefill(const PrefillParams& p, cudaStream_t stream) {
  if (p.q_len <= 0) return cudaSuccess;
  auto kernel = prefill_attn_kernel<__half, true>;
  cudaError_t e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, kPfSmem);
  if (e != cudaSuccess) return e;
  const dim3 grid((unsigned)((p.q_len + kPfPos - 1) / kPfPos), kKvHeads);
  return launch_pdl(kernel, grid, dim3(kPfDq0 * 32), kPfSmem, stream, p);
}

}  // namespace qwz
