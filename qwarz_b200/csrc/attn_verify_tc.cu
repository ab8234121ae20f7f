// NVFP4 paged MTP verify (q_len 2..8) on the fifth-generation tensor cores
// (tcgen05: operands and accumulators in tensor memory), sm_100a.
//
// Replaces the q_len > 1 XQA launch of src/qwasar_runtime/xqa.py:484-554
// (MTP verify: q_len query rows per head, lower-right causal, xqa.py:662)
// behind the split ABI of tests/test_attention_kernel_abi.py:13-32.
//
// CTA = one KV head x one split (a run of pages), 10 warps:
//   warp 0     TMA producer: 128-token stages (codes + scales of K and V,
//              36 KB) into a 4-deep ring (full / empty mbarriers);
//   warp 1     TMEM owner (512 columns) and MMA issuer (one thread);
//   warps 2-9  eight math warps: warp w serves TMEM lane quadrant q = w % 4
//              and half h = (w - 2) / 4 of the work.
// Per 128-token tile:
//   1. math: K (E2M1 x E4M3 -> FP16, exact) into TMEM as the A operand,
//      lane = token, column = head-dim pair (32x32b stores, thread = token);
//   2. MMA:  S^T[128 tok x N] = K Q^T, N = 6 q_len rounded up to 16, Q in
//      shared memory (K-major, 128-byte swizzle, rows scaled by a power of
//      two so BF16 queries convert to FP16 exactly);
//   3. math: V^T into TMEM, lane = head-dim (two M=128 halves), column =
//      token pair, built in mma-fragment registers and written with 16x256b
//      stores; tokens inside each 16-token step are permuted (kperm) and the
//      head-dim order on the lanes is d = 32g + 2x + e (see vt_lane_d);
//   4. math: base-2 online softmax on S^T (thread = token): the reference
//      max of a column only moves when a score exceeds it by kLazy (then O
//      is rescaled in TMEM); P = hi + lo in FP16 is written to shared
//      memory as the K-major operand [2N rows (hi | lo) x 128 tokens];
//   5. MMA:  O^T[256 d x 2N] += V^T [P_hi | P_lo]^T (one MMA per M half and
//      16-token step reads V^T once for both halves of P).
// The epilogue adds the hi and lo halves of O^T and writes one (m, l, O)
// record per query row and split, the layout lse_combine_kernel reads.
// Every wait is bounded; the math warps decide timeouts collectively at a
// per-tile vote, so named barriers never wait for a warp that left.

#include "attn_common.cuh"
#include "tc_common.cuh"

namespace qwz {

using namespace detail;

constexpr int kVtWarps = 10;
constexpr int kVtStages = 4;
constexpr int kVtTile = 128;
constexpr int kVtCodeBox = kVtTile * kCodeBytes;                         // 16 KB
constexpr int kVtScaleBox = kVtTile * kScaleBytes;                       // 2 KB
constexpr int kVtStageBytes = 2 * kVtCodeBox + 2 * kVtScaleBox;          // 36 KB
constexpr int kVtPidCache = 512;
// TMEM columns: K (A of QK) | V^T halves (A of PV) | S^T | O^T halves
constexpr uint32_t kTmK = 0, kTmV = 128, kTmS = 256, kTmO = 320;
constexpr uint32_t kTmCols = 512;

template <int N>
struct VtLayout {
  static constexpr int kQ = kVtStages * kVtStageBytes;      // Q operand: 4 k-atoms [N x 128 B]
  static constexpr int kP = kQ + N * 512;                   // P operand: 2 k-atoms [2N x 128 B]
  static constexpr int kBars = kP + 2 * N * 256;            // full[4] empty[4] k pv s o
  static constexpr int kMeta = kBars + 8 * (2 * kVtStages + 4);  // stage_end[4], tmem, abort
  static constexpr int kRowfac = kMeta + 32;                // [N]
  static constexpr int kAlpha = kRowfac + 4 * N;            // [N]
  static constexpr int kMref = kAlpha + 4 * N;              // [N]
  static constexpr int kWred = kMref + 4 * N;               // [2 h][4 q][N / 2]
  static constexpr int kPid = kWred + 4 * 4 * N;            // [kVtPidCache]
  static constexpr int kBytes = kPid + 4 * kVtPidCache + 1024;
};

namespace {

// Position of token t (0..15) of a 16-token step inside the PV K order that
// the 16x256b V^T stores produce: column 2c holds tokens (2c, 2c+1) of the
// step, column 2c+1 tokens (2c+8, 2c+9) (c = lane % 4).
QWZ_DEVINL int kperm(int t) { return 4 * ((t & 7) >> 1) + 2 * (t >> 3) + (t & 1); }

// Head-dim index held by V^T / O^T lane L of M half h.
QWZ_DEVINL int vt_lane_d(int L, int h) {
  const int x = 8 * h + (L >> 4), g = L & 7, e = (L >> 3) & 1;
  return 32 * g + 2 * x + e;
}

QWZ_DEVINL void math_bar() { asm volatile("bar.sync 1, 256;\n" ::: "memory"); }
QWZ_DEVINL bool math_bar_or(bool v) {
  uint32_t r;
  asm volatile(
      "{\n .reg .pred p, q;\n setp.ne.u32 p, %1, 0;\n bar.red.or.pred q, 1, 256, p;\n"
      " selp.u32 %0, 1, 0, q;\n}\n"
      : "=r"(r)
      : "r"((uint32_t)v)
      : "memory");
  return r != 0;
}
QWZ_DEVINL uint2 lds64(uint32_t addr) {
  uint2 v;
  asm volatile("ld.shared.v2.u32 {%0,%1}, [%2];\n" : "=r"(v.x), "=r"(v.y) : "r"(addr));
  return v;
}
QWZ_DEVINL void sts16(uint32_t addr, uint32_t v) {
  asm volatile("st.shared.u16 [%0], %1;\n" ::"r"(addr), "h"((unsigned short)v));
}
QWZ_DEVINL void sts128(uint32_t addr, uint32_t a, uint32_t b, uint32_t c, uint32_t d) {
  asm volatile("st.shared.v4.u32 [%0], {%1,%2,%3,%4};\n" ::"r"(addr), "r"(a), "r"(b), "r"(c), "r"(d));
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

// TMEM loads of n (multiple of 8) consecutive columns into v.
template <int NC>
QWZ_DEVINL void ld_cols(uint32_t taddr, float (&v)[NC]) {
  static_assert(NC % 8 == 0, "8-column granularity");
#pragma unroll
  for (int c = 0; c + 16 <= NC; c += 16) {
    uint32_t r[16];
    tc::ld_32x32b_x16(taddr + c, r);
#pragma unroll
    for (int j = 0; j < 16; ++j) v[c + j] = __uint_as_float(r[j]);
  }
  if constexpr (NC % 16 == 8) {
    uint32_t r[8];
    tc::ld_32x32b_x8(taddr + NC - 8, r);
#pragma unroll
    for (int j = 0; j < 8; ++j) v[NC - 8 + j] = __uint_as_float(r[j]);
  }
}

// Q rows of this KV head into the K-major operand, scaled per row by a power
// of two (FP16-exact), and the per-row score factor sm_scale*log2e/scale.
template <typename T, int N>
QWZ_DEVINL void stage_q(const SplitParams& p, int kvh, uint32_t qbase, float* rowfac, int mw, int lane) {
  for (int r = mw; r < N; r += 8) {
    const int qi = r / kGroup, hg = r - qi * kGroup;
    uint32_t w[4] = {0u, 0u, 0u, 0u};
    if (qi < p.q_len) {
      const uint4 v = __ldg(reinterpret_cast<const uint4*>(reinterpret_cast<const T*>(p.q) +
                                                           ((size_t)qi * kQHeads + kvh * kGroup + hg) * kHeadDim) + lane);
      w[0] = v.x; w[1] = v.y; w[2] = v.z; w[3] = v.w;
    }
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
    if (lane == 0) rowfac[r] = qi < p.q_len ? p.sm_scale_log2 / sc : 0.f;
  }
}

}  // namespace

template <typename T, int N>
__global__ void __launch_bounds__(kVtWarps * 32, 1)
    nvfp4_verify_tc_kernel(const __grid_constant__ SplitParams p) {
  using L = VtLayout<N>;
  constexpr int NH = N / 2;
  extern __shared__ __align__(1024) uint8_t smem[];
  const uint32_t sraw = smem_u32(smem);
  const uint32_t sb = (sraw + 1023u) & ~1023u;
  uint8_t* sg = smem + (sb - sraw);
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int split = blockIdx.x, kvh = blockIdx.y;
  const uint32_t bar_full = sb + L::kBars, bar_empty = bar_full + 8 * kVtStages;
  const uint32_t bar_k = bar_empty + 8 * kVtStages, bar_pv = bar_k + 8, bar_s = bar_pv + 8, bar_o = bar_s + 8;
  int* stage_end = reinterpret_cast<int*>(sg + L::kMeta);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(sg + L::kMeta + 16);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(sg + L::kMeta + 20);
  float* rowfac = reinterpret_cast<float*>(sg + L::kRowfac);
  float* alpha_s = reinterpret_cast<float*>(sg + L::kAlpha);
  float* mref_s = reinterpret_cast<float*>(sg + L::kMref);
  float* wred = reinterpret_cast<float*>(sg + L::kWred);
  int* pid = reinterpret_cast<int*>(sg + L::kPid);

  const StageRange rg = stage_range<kPage>(p, split);
  const int n_tiles = 2 * rg.n_st;
  const int len_all = __ldg(p.seqlens) + p.len_add;  // causal limits use the whole sequence

  if (tid == 0) {
#pragma unroll
    for (int s = 0; s < kVtStages; ++s) {
      mbar_init(bar_full + 8 * s, 1);
      mbar_init(bar_empty + 8 * s, 8);
    }
    mbar_init(bar_k, 8);
    mbar_init(bar_pv, 8);
    mbar_init(bar_s, 1);
    mbar_init(bar_o, 1);
    *abort_flag = 0;
    mbar_fence_init();
  }
  if (warp == 1) {
    tc::tmem_alloc(sb + L::kMeta + 16, kTmCols);
    tc::tmem_relinquish();
  }
  if (warp == 0) {
    for (int i = lane; i < min(rg.n_st, kVtPidCache); i += 32)
      pid[i] = lookup_page(p, p.tok_begin + (rg.st_lo + i) * kPage, true);
  }
  if (warp >= 2) {
    stage_q<T, N>(p, kvh, sb + L::kQ, rowfac, warp - 2, lane);
    fence_proxy_async_smem();  // Q is read by the tensor core
  }
  tc::fence_before();
  __syncthreads();
  tc::fence_after();
  const uint32_t tbase = *tmem_slot;

  if (warp == 0) {
    // ------------------------------------------------------------ producer
    if (lane == 0 && n_tiles > 0) {
      tma_prefetch_desc(&p.tm_kc);
      tma_prefetch_desc(&p.tm_vc);
      tma_prefetch_desc(&p.tm_ks);
      tma_prefetch_desc(&p.tm_vs);
      int issued = 0;
      for (int i = 0; i < n_tiles; ++i) {
        const int s = i % kVtStages;
        if (*abort_flag) break;
        if (i >= kVtStages && !mbar_wait(bar_empty + 8 * s, ((i / kVtStages) - 1) & 1)) {
          flag_error(kErrTimeout);
          *abort_flag = 1;
          break;
        }
        const int k = i >> 1;
        const int t0 = p.tok_begin + (rg.st_lo + k) * kPage + kVtTile * (i & 1);
        const int pp = k < kVtPidCache ? pid[k] : lookup_page(p, t0, true);
        stage_end[s] = pp >= 0 ? rg.tok_end : t0;  // released by the arrive below
        const uint32_t fb = bar_full + 8 * s;
        issued = i + 1;
        if (pp < 0) {  // bad page id: no copy; the math warps mask the tile
          mbar_arrive(fb);
          continue;
        }
        mbar_arrive_expect_tx(fb, kVtStageBytes);
        const uint32_t dst = sb + s * kVtStageBytes;
        const int y = pp * kPage + kVtTile * (i & 1);
        tma_load_2d(dst, &p.tm_kc, kvh * kCodeBytes, y, fb);
        tma_load_2d(dst + kVtCodeBox, &p.tm_vc, kvh * kCodeBytes, y, fb);
        tma_load_2d(dst + 2 * kVtCodeBox, &p.tm_ks, kvh * kScaleBytes, y, fb);
        tma_load_2d(dst + 2 * kVtCodeBox + kVtScaleBox, &p.tm_vs, kvh * kScaleBytes, y, fb);
      }
      // never leave with copies in flight (only reachable after an abort)
      for (int i = max(issued - kVtStages, 0); i < issued; ++i)
        if (!mbar_wait(bar_full + 8 * (i % kVtStages), (i / kVtStages) & 1)) flag_error(kErrTimeout);
    }
  } else if (warp == 1) {
    // ----------------------------------------------------------------- MMA
    if (lane == 0 && n_tiles > 0) {
      constexpr uint32_t idesc_qk = tc::idesc_f16_f32(128, N);
      constexpr uint32_t idesc_pv = tc::idesc_f16_f32(128, 2 * N);
      int committed = 0;
      for (int i = 0; i < n_tiles; ++i) {
        if (*abort_flag) break;
        if (!mbar_wait(bar_k, i & 1)) {
          flag_error(kErrTimeout);
          *abort_flag = 1;
          break;
        }
        tc::fence_after();
#pragma unroll
        for (int ks = 0; ks < 16; ++ks)
          tc::mma_ts(tbase + kTmS, tbase + kTmK + 8 * ks,
                     tc::smem_desc_k128(sb + L::kQ + (ks >> 2) * (N * 128) + (ks & 3) * 32), idesc_qk, ks > 0);
        tc::commit(bar_s);
        if (!mbar_wait(bar_pv, i & 1)) {
          flag_error(kErrTimeout);
          *abort_flag = 1;
          break;
        }
        tc::fence_after();
#pragma unroll
        for (int h = 0; h < 2; ++h) {
#pragma unroll
          for (int ks = 0; ks < 8; ++ks)
            tc::mma_ts(tbase + kTmO + 2 * N * h, tbase + kTmV + 64 * h + 8 * ks,
                       tc::smem_desc_k128(sb + L::kP + (ks >> 2) * (2 * N * 128) + (ks & 3) * 32), idesc_pv,
                       (i > 0 || ks > 0));
        }
        tc::commit(bar_o);
        committed = i + 1;
      }
      if (*abort_flag && committed > 0 && !mbar_wait(bar_o, (committed - 1) & 1)) flag_error(kErrTimeout);
    }
  } else {
    // ---------------------------------------------------------------- math
    const int q = warp & 3, h = (warp - 2) >> 2;
    const int g = lane >> 2, qd = lane & 3;
    const uint32_t lane_base = (uint32_t)(32 * q) << 16;
    float lsum[NH], mreg[NH];
#pragma unroll
    for (int c = 0; c < NH; ++c) {
      lsum[c] = 0.f;
      mreg[c] = -CUDART_INF_F;
    }
    bool ok = true;
    int done_tiles = 0;
    for (int i = 0; i < n_tiles; ++i) {
      const int s = i % kVtStages;
      const uint32_t st = sb + s * kVtStageBytes;
      ok &= mbar_wait(bar_full + 8 * s, (i / kVtStages) & 1);
      const int t0 = p.tok_begin + (rg.st_lo + (i >> 1)) * kPage + kVtTile * (i & 1);
      const int vend = stage_end[s];

      // (1) K -> TMEM, thread = token tt, head-dim half h
      {
        const int tt = 32 * q + lane;
        const uint2 sc = lds64(st + 2 * kVtCodeBox + tt * kScaleBytes + 8 * h);
        uint32_t s01, s23, s45, s67;
        e4m3x4_to_f16x2x2(sc.x, s01, s23);
        e4m3x4_to_f16x2x2(sc.y, s45, s67);
        const uint32_t spair[4] = {s01, s23, s45, s67};
#pragma unroll
        for (int c = 0; c < 4; ++c) {
          const uint4 w = lds128(st + tt * kCodeBytes + (((4 * h + c) ^ (tt & 7)) << 4));
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
          tc::st_32x32b_x16(tbase + lane_base + kTmK + 64 * h + 16 * c, r);
        }
      }
      tc::wait_st();
      tc::fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(bar_k);

      // (3) V^T -> TMEM after PV of the previous tile
      if (i > 0) ok &= mbar_wait(bar_o, (i - 1) & 1);
      tc::fence_after();
      {
        const uint32_t vcode = st + kVtCodeBox, vscale = st + 2 * kVtCodeBox + kVtScaleBox;
        const int lo = 8 * h + 2 * q;                // byte of m-tile x0 = 8h + 2q within chunk g
        const bool tail = t0 + kVtTile > vend;
#pragma unroll 2
        for (int b = 0; b < 8; ++b) {
          const int ta = 16 * b + 2 * qd;
          const uint32_t va = lds16(vcode + ta * kCodeBytes + ((g ^ (ta & 7)) << 4) + lo);
          const uint32_t vb = lds16(vcode + (ta + 1) * kCodeBytes + ((g ^ ((ta + 1) & 7)) << 4) + lo);
          const uint32_t vc = lds16(vcode + (ta + 8) * kCodeBytes + ((g ^ ((ta + 8) & 7)) << 4) + lo);
          const uint32_t vd = lds16(vcode + (ta + 9) * kCodeBytes + ((g ^ ((ta + 9) & 7)) << 4) + lo);
          uint32_t sa = lds8(vscale + ta * kScaleBytes + 2 * g + h);
          uint32_t sbb = lds8(vscale + (ta + 1) * kScaleBytes + 2 * g + h);
          uint32_t sc = lds8(vscale + (ta + 8) * kScaleBytes + 2 * g + h);
          uint32_t sd = lds8(vscale + (ta + 9) * kScaleBytes + 2 * g + h);
          if (tail) {  // stale rows past the end add 0
            if (t0 + ta >= vend) sa = 0;
            if (t0 + ta + 1 >= vend) sbb = 0;
            if (t0 + ta + 8 >= vend) sc = 0;
            if (t0 + ta + 9 >= vend) sd = 0;
          }
          uint32_t sab, scd;
          e4m3x4_to_f16x2x2(sa | (sbb << 8) | (sc << 16) | (sd << 24), sab, scd);
          // byte j of X / Y: tokens (ta, ta+1) then (ta+8, ta+9), m-tiles x0, x0+1
          const uint32_t xab = (va & 0x0F0Fu) | ((vb & 0x0F0Fu) << 4);
          const uint32_t yab = ((va >> 4) & 0x0F0Fu) | (vb & 0xF0F0u);
          const uint32_t xcd = (vc & 0x0F0Fu) | ((vd & 0x0F0Fu) << 4);
          const uint32_t ycd = ((vc >> 4) & 0x0F0Fu) | (vd & 0xF0F0u);
          uint32_t hx[4], hy[4];
          e2m1x8_to_f16x2x4(xab | (xcd << 16), hx);
          e2m1x8_to_f16x2x4(yab | (ycd << 16), hy);
          const uint32_t col = tbase + kTmV + 64 * h + 8 * b;
          tc::st_16x256b(col + lane_base, hmul2_u32(hx[0], sab), hmul2_u32(hx[2], scd), hmul2_u32(hy[0], sab),
                         hmul2_u32(hy[2], scd));
          tc::st_16x256b(col + lane_base + (16u << 16), hmul2_u32(hx[1], sab), hmul2_u32(hx[3], scd),
                         hmul2_u32(hy[1], sab), hmul2_u32(hy[3], scd));
        }
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(bar_empty + 8 * s);  // stage read completely

      // (4) softmax on S^T
      ok &= mbar_wait(bar_s, i & 1);
      tc::fence_after();
      float x[NH];
      ld_cols<NH>(tbase + lane_base + kTmS + NH * h, x);
      tc::wait_ld();
      const int tok = t0 + 32 * q + lane;
      bool need = false;
#pragma unroll
      for (int c = 0; c < NH; ++c) {
        const int r = NH * h + c;
        const int qi = min(r / kGroup, p.q_len - 1);
        const int limit = min(vend, len_all - (p.q_len - 1 - qi));
        x[c] = tok < limit ? x[c] * rowfac[r] : -CUDART_INF_F;
        need |= x[c] > mreg[c] + kLazy;
      }
      const bool bad = !ok || *abort_flag;
      if (math_bar_or(need || bad)) {
        if (math_bar_or(bad)) {
          if (tid == 64) *abort_flag = 1;
          flag_error(kErrTimeout);
          break;
        }
        // move the reference max of every column to this tile's max
#pragma unroll
        for (int c = 0; c < NH; ++c) {
          const float mx = warp_max(x[c]);
          if (lane == 0) wred[(h * 4 + q) * NH + c] = mx;
        }
        math_bar();
#pragma unroll
        for (int c = 0; c < NH; ++c) {
          float tm = wred[(h * 4) * NH + c];
#pragma unroll
          for (int qq = 1; qq < 4; ++qq) tm = fmaxf(tm, wred[(h * 4 + qq) * NH + c]);
          const float mnew = fmaxf(mreg[c], tm);
          const float alpha = mreg[c] == -CUDART_INF_F ? 0.f : exp2_approx(mreg[c] - mnew);
          lsum[c] *= alpha;
          mreg[c] = mnew;
          if (q == 0 && lane == 0) alpha_s[NH * h + c] = alpha;
        }
        math_bar();
        if (i > 0) {  // O^T of this quadrant and half, both P halves
#pragma unroll
          for (int c0 = 0; c0 < 2 * N; c0 += 16) {
            uint32_t r[16];
            tc::ld_32x32b_x16(tbase + lane_base + kTmO + 2 * N * h + c0, r);
            tc::wait_ld();
#pragma unroll
            for (int j = 0; j < 16; ++j)
              r[j] = __float_as_uint(__uint_as_float(r[j]) * alpha_s[(c0 + j) % N]);
            tc::st_32x32b_x16(tbase + lane_base + kTmO + 2 * N * h + c0, r);
          }
        }
        math_bar();  // alpha_s / wred are rewritten by the next slow tile
      }
      // P = hi + lo into the K-major operand, token tt at position kperm
      {
        const int tt = 32 * q + lane;
        const int k = 16 * (tt >> 4) + kperm(tt & 15);
        const uint32_t pk = sb + L::kP + (k >> 6) * (2 * N * 128) + ((k & 63) * 2 & 15);
        const int chunk = ((k & 63) * 2) >> 4;
#pragma unroll
        for (int c = 0; c < NH; ++c) {
          const float mu = mreg[c] == -CUDART_INF_F ? 0.f : mreg[c];
          const float pv = exp2_approx(x[c] - mu);
          lsum[c] += pv;
          const __half hi = __float2half_rn(pv);
          const __half lo = __float2half_rn(pv - __half2float(hi));
          const int r = NH * h + c, r2 = N + r;
          sts16(pk + r * 128 + ((chunk ^ (r & 7)) << 4), __half_as_ushort(hi));
          sts16(pk + r2 * 128 + ((chunk ^ (r2 & 7)) << 4), __half_as_ushort(lo));
        }
      }
      tc::wait_st();
      fence_proxy_async_smem();
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
    for (int c = 0; c < NH; ++c) {
      const float lw = warp_sum(lsum[c]);
      if (lane == 0) wred[(h * 4 + q) * NH + c] = lw;
      if (q == 0 && lane == 0) mref_s[NH * h + c] = have_o ? mreg[c] : -CUDART_INF_F;
    }
    math_bar();
    const int rows = kGroup * p.q_len;
    if (q == 0 && lane < NH && NH * h + lane < rows) {
      const int r = NH * h + lane;
      float l = 0.f;
#pragma unroll
      for (int qq = 0; qq < 4; ++qq) l += wred[(h * 4 + qq) * NH + lane];
      const size_t R = (size_t)(r / kGroup) * kQHeads + kvh * kGroup + r % kGroup;
      const size_t base = R * p.num_splits + split;
      p.partial_ml[base * 2 + 0] = mref_s[r];
      p.partial_ml[base * 2 + 1] = have_o ? l : 0.f;
    }
    const int d = vt_lane_d(32 * q + lane, h);
#pragma unroll
    for (int c0 = 0; c0 < N; c0 += 8) {
      uint32_t hi[8], lo[8];
      if (have_o) {
        tc::ld_32x32b_x8(tbase + lane_base + kTmO + 2 * N * h + c0, hi);
        tc::ld_32x32b_x8(tbase + lane_base + kTmO + 2 * N * h + N + c0, lo);
        tc::wait_ld();
      }
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        const int r = c0 + j;
        if (r < rows) {
          const size_t R = (size_t)(r / kGroup) * kQHeads + kvh * kGroup + r % kGroup;
          const float o = have_o ? __uint_as_float(hi[j]) + __uint_as_float(lo[j]) : 0.f;
          p.partial_o[(R * p.num_splits + split) * kHeadDim + d] = o;
        }
      }
    }
  }

  tc::fence_before();
  __syncthreads();
  if (warp == 1) {
    tc::fence_after();
    tc::tmem_dealloc(tbase, kTmCols);
  }
}

template <typename T, int N>
cudaError_t launch_verify_tc_n(const SplitParams& p, cudaStream_t stream) {
  using L = VtLayout<N>;
  static_assert(L::kBytes <= 227 * 1024, "shared memory");
  static_assert(kTmO + 4 * N <= kTmCols, "tensor memory columns");
  auto kernel = nvfp4_verify_tc_kernel<T, N>;
  cudaError_t e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, L::kBytes);
  if (e != cudaSuccess) return e;
  dim3 grid(p.num_splits, kKvHeads);
  kernel<<<grid, kVtWarps * 32, L::kBytes, stream>>>(p);
  return cudaGetLastError();
}

template <typename T>
cudaError_t launch_verify_tc(const SplitParams& p, cudaStream_t stream) {
  const int rows = kGroup * p.q_len;
  if (rows <= 16) return launch_verify_tc_n<T, 16>(p, stream);
  if (rows <= 32) return launch_verify_tc_n<T, 32>(p, stream);
  if (rows <= 48) return launch_verify_tc_n<T, 48>(p, stream);
  return cudaErrorInvalidValue;
}

}  // namespace qwz
