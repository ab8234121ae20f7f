// NVFP4 paged MTP verify (q_len 2..8) on the fifth-generation tensor cores
// (tcgen05: accumulators in tensor memory), sm_100a.
//
// Replaces the q_len > 1 XQA launch of src/qwasar_runtime/xqa.py:484-554
// (MTP verify: q_len query rows per head, lower-right causal, xqa.py:662)
// behind the split ABI of tests/test_attention_kernel_abi.py:13-32.
//
// CTA = one KV head x one split (a run of pages), 11 warps:
//   warp 0      TMA producer of K tiles (codes + scales, 18 KB per 128
//               tokens) into a 3-deep ring;
//   warp 1      TMEM owner (512 columns) and MMA issuer (one thread);
//   warp 2      TMA producer of V tiles into a 2-deep ring;
//   warps 3-10  eight math warps: warp w serves TMEM lane quadrant q = w % 4
//               and half h = (w - 3) / 4 of the work.
// Per 128-token tile i (tokens on the MMA M dimension, head-dim d):
//   K(i)    math: E2M1 x E4M3 -> FP16 (exact) into TMEM as the A operand,
//           lane = token, column = d pair (32x32b stores, thread = token);
//   QK(i)   MMA:  S^T[128 tok x N] = K Q^T into one of two S buffers, N =
//           6 q_len rounded up to 16, Q in shared memory (K-major, 128-byte
//           swizzle, rows scaled by a power of two so BF16 queries convert
//           to FP16 exactly);
//   soft(i) math: base-2 online softmax on S^T (thread = token): the
//           reference max of a column only moves when a score exceeds it by
//           kLazy (then O is rescaled in TMEM); P = hi + lo in FP16;
//   V(i)    math: V -> FP16 rows [token][d] in shared memory (the MN-major A
//           operand of PV), P -> [token][hi | lo] (the MN-major B operand);
//   PV(i)   MMA:  O^T[256 d x 2N] += V^T [P_hi | P_lo]^T, two M=128 halves
//           of d, V^T read once for both halves of P.
// Order: the math warps dequantise K(i+1) as soon as S(i) is read, so
// QK(i+1) is queued ahead of PV(i); they write V(i) and P(i) only after
// PV(i-1) has finished with the single V and P buffers, which by then it
// long has.  The epilogue adds the hi and lo halves of O^T and writes one
// (m, l, O) record per query row and split, the layout lse_combine_kernel
// reads.  Every wait is bounded; the math warps decide timeouts
// collectively at a per-tile vote, so named barriers never wait for a warp
// that left.

#include "attn_common.cuh"
#include "tc_common.cuh"

namespace qwz {

using namespace detail;

constexpr int kVtWarps = 11;
constexpr int kVtMath0 = 3;                                // first math warp
constexpr int kVtKStages = 3, kVtVStages = 2;
constexpr int kVtTile = 128;
constexpr int kVtCodeBox = kVtTile * kCodeBytes;           // 16 KB
constexpr int kVtScaleBox = kVtTile * kScaleBytes;         // 2 KB
constexpr int kVtHalfStage = kVtCodeBox + kVtScaleBox;     // 18 KB (K or V of one tile)
constexpr int kVtPidCache = 512;
// TMEM columns: K (A of QK) | S^T buffer 0 | S^T buffer 1 | O^T halves
constexpr uint32_t kTmK = 0, kTmS = 128, kTmO = 256;
constexpr uint32_t kTmCols = 512;

template <int N>
struct VtLayout {
  static constexpr int kKRing = 0;                                   // 3 x 18 KB
  static constexpr int kVRing = kKRing + kVtKStages * kVtHalfStage;  // 2 x 18 KB
  static constexpr int kVf = 92160;                                  // V FP16: [2h+a][128 tok][128 B]
  static constexpr int kQ = kVf + 4 * 16384;                         // Q: 4 k-atoms [N x 128 B]
  static constexpr int kPAtoms = (2 * N + 63) / 64;                  // P: n-atoms [128 tok][128 B]
  static constexpr int kP = kQ + N * 512;
  static constexpr int kBars = kP + kPAtoms * 16384;
  // kfull[3] kempty[3] vfull[2] vempty[2] kready pvready s[2] o (15 x 8 B)
  static constexpr int kMeta = kBars + 128;
  static constexpr int kRowfac = kMeta + 32;                         // stage ends, tmem, abort, fin
  static constexpr int kAlpha = kRowfac + 4 * N;
  static constexpr int kMref = kAlpha + 4 * N;
  static constexpr int kWred = kMref + 4 * N;                        // [2 h][4 q][N / 2]
  static constexpr int kPid = kWred + 4 * 4 * N;
  static constexpr int kBytes = kPid + 4 * kVtPidCache + 1024;
  static_assert(kVRing + kVtVStages * kVtHalfStage <= kVf && kVf % 1024 == 0, "ring / V layout");
  static_assert(kQ % 1024 == 0 && kP % 1024 == 0 && kBars % 1024 == 0, "operand atoms are 1024-byte aligned");
  static_assert(8 * (2 * kVtKStages + 2 * kVtVStages + 5) <= 128 && (kMeta + 24) % 8 == 0,
                "mbarriers are 8-byte aligned");
  static_assert(kRowfac % 16 == 0, "row factors are read as float4");
};

namespace {

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

// TMEM loads of NC (multiple of 8) consecutive columns into v.
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

// Head-dim half h of token row tt of a K or V tile (the 64 code bytes of
// chunks 4h..4h+3, 128-byte swizzle, and their 8 scales) as f16x2 words in
// d order, handed to put(c, r16) per 32 values (code chunk c).  `zero`
// (rows at or past the valid end) makes every value 0.
template <class Put>
QWZ_DEVINL void dequant_row_half(uint32_t codes, uint32_t scales, int tt, int h, bool zero, Put put) {
  uint2 sc = lds64(scales + tt * kScaleBytes + 8 * h);
  if (zero) sc = make_uint2(0u, 0u);
  uint32_t s01, s23, s45, s67;
  e4m3x4_to_f16x2x2(sc.x, s01, s23);
  e4m3x4_to_f16x2x2(sc.y, s45, s67);
  const uint32_t spair[4] = {s01, s23, s45, s67};
#pragma unroll
  for (int c = 0; c < 4; ++c) {
    const uint4 w = lds128(codes + tt * kCodeBytes + (((4 * h + c) ^ (tt & 7)) << 4));
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
    put(c, r);
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
  const uint32_t bar_kfull = sb + L::kBars, bar_kempty = bar_kfull + 8 * kVtKStages;
  const uint32_t bar_vfull = bar_kempty + 8 * kVtKStages, bar_vempty = bar_vfull + 8 * kVtVStages;
  const uint32_t bar_kready = bar_vempty + 8 * kVtVStages, bar_pv = bar_kready + 8;
  const uint32_t bar_s = bar_pv + 8, bar_o = bar_s + 16;  // bar_s: one per S buffer
  int* kstage_end = reinterpret_cast<int*>(sg + L::kMeta);  // [kVtKStages]
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(sg + L::kMeta + 16);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(sg + L::kMeta + 20);
  const uint32_t bar_fin = sb + L::kMeta + 24;  // the MMA thread's last commit
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
    for (int s = 0; s < kVtKStages; ++s) {
      mbar_init(bar_kfull + 8 * s, 1);
      mbar_init(bar_kempty + 8 * s, 8);
    }
#pragma unroll
    for (int s = 0; s < kVtVStages; ++s) {
      mbar_init(bar_vfull + 8 * s, 1);
      mbar_init(bar_vempty + 8 * s, 8);
    }
    mbar_init(bar_kready, 8);
    mbar_init(bar_pv, 8);
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
  if (warp == 0) {
    for (int i = lane; i < min(rg.n_st, kVtPidCache); i += 32)
      pid[i] = lookup_page(p, p.tok_begin + (rg.st_lo + i) * kPage, true);
  }
  if (warp >= kVtMath0) {
    stage_q<T, N>(p, kvh, sb + L::kQ, rowfac, warp - kVtMath0, lane);
    fence_proxy_async_smem();  // Q is read by the tensor core
  }
  tc::fence_before();
  __syncthreads();
  tc::fence_after();
  const uint32_t tbase = *tmem_slot;

  if (warp == 0 || warp == 2) {
    // ----------------------------------------------- producers (K: 0, V: 2)
    const bool is_k = warp == 0;
    const int nst = is_k ? kVtKStages : kVtVStages;
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
        const int k = i >> 1;
        const int t0 = p.tok_begin + (rg.st_lo + k) * kPage + kVtTile * (i & 1);
        const int pp = k < kVtPidCache ? pid[k] : lookup_page(p, t0, is_k);
        if (is_k) kstage_end[s] = pp >= 0 ? rg.tok_end : t0;  // released by the arrive below
        const uint32_t fb = full + 8 * s;
        issued = i + 1;
        if (pp < 0) {  // bad page id: no copy; the math warps mask the tile
          mbar_arrive(fb);
          continue;
        }
        mbar_arrive_expect_tx(fb, kVtHalfStage);
        const uint32_t dst = ring + s * kVtHalfStage;
        const int y = pp * kPage + kVtTile * (i & 1);
        tma_load_2d(dst, tm_c, kvh * kCodeBytes, y, fb);
        tma_load_2d(dst + kVtCodeBox, tm_s, kvh * kScaleBytes, y, fb);
      }
      // never leave with copies in flight (only reachable after an abort)
      for (int i = max(issued - nst, 0); i < issued; ++i)
        if (!mbar_wait(full + 8 * (i % nst), (i / nst) & 1)) flag_error(kErrTimeout);
    }
  } else if (warp == 1) {
    // ----------------------------------------------------------------- MMA
    if (lane == 0 && n_tiles > 0) {
      constexpr uint32_t idesc_qk = tc::idesc_f16_f32(128, N);
      constexpr uint32_t idesc_pv = tc::idesc_f16_f32(128, 2 * N, true, true);
      auto qk = [&](int j) -> bool {
        if (!mbar_wait(bar_kready, j & 1)) return false;
        tc::fence_after();
#pragma unroll
        for (int ks = 0; ks < 16; ++ks)
          tc::mma_ts(tbase + kTmS + 64 * (j & 1), tbase + kTmK + 8 * ks,
                     tc::smem_desc_k128(sb + L::kQ + (ks >> 2) * (N * 128) + (ks & 3) * 32), idesc_qk, ks > 0);
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
            tc::mma_ss(tbase + kTmO + 2 * N * h,
                       tc::smem_desc_mn128(sb + L::kVf + 2 * h * 16384 + ks * 2048, 16384, 1024),
                       tc::smem_desc_mn128(sb + L::kP + ks * 2048, 16384, 1024), idesc_pv, (i > 0 || ks > 0));
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
    const int q = warp & 3, h = (warp - kVtMath0) >> 2;
    const uint32_t lane_base = (uint32_t)(32 * q) << 16;
    const int tt = 32 * q + lane;  // this thread's token row of K, V, S^T and P
    float lsum[NH], mreg[NH];
#pragma unroll
    for (int c = 0; c < NH; ++c) {
      lsum[c] = 0.f;
      mreg[c] = -CUDART_INF_F;
    }
    bool ok = true;

    // K(j) -> TMEM, thread = token tt, head-dim half h (columns 64h ..);
    // returns the tile's valid end, read before the ring slot is released
    auto do_k = [&](int j) -> int {
      const int s = j % kVtKStages;
      ok &= mbar_wait(bar_kfull + 8 * s, (j / kVtKStages) & 1);
      const int end = kstage_end[s];
      const uint32_t st = sb + L::kKRing + s * kVtHalfStage;
      const uint32_t col = tbase + lane_base + kTmK + 64 * h;
      dequant_row_half(st, st + kVtCodeBox, tt, h, false,
                       [&](int c, const uint32_t (&r)[16]) { tc::st_32x32b_x16(col + 16 * c, r); });
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
      const int t0 = p.tok_begin + (rg.st_lo + (i >> 1)) * kPage + kVtTile * (i & 1);
      const int vend = vend_next;

      float x[NH];
      ld_cols<NH>(tbase + lane_base + kTmS + 64 * sbuf + NH * h, x);
      tc::wait_ld();
      // S(i) is read and QK(i) is done: the K buffer takes K(i+1) now
      if (i + 1 < n_tiles) vend_next = do_k(i + 1);

      // ------------------------------------------------------- softmax(i)
#pragma unroll
      for (int c = 0; c < NH; c += 4) {
        const float4 f = *reinterpret_cast<const float4*>(rowfac + NH * h + c);
        x[c] *= f.x;
        x[c + 1] *= f.y;
        x[c + 2] *= f.z;
        x[c + 3] *= f.w;
      }
      // causal / length mask only on tiles that reach the end
      if (t0 + kVtTile > min(vend, len_all - (p.q_len - 1))) {
        const int tok = t0 + tt;
#pragma unroll
        for (int c = 0; c < NH; ++c) {
          const int qi = min((NH * h + c) / kGroup, p.q_len - 1);
          if (tok >= min(vend, len_all - (p.q_len - 1 - qi))) x[c] = -CUDART_INF_F;
        }
      }
      bool need = false;
#pragma unroll
      for (int c = 0; c < NH; ++c) need |= x[c] > mreg[c] + kLazy;
      const bool bad = !ok || *abort_flag;
      if (math_bar_or(need || bad)) {
        if (math_bar_or(bad)) {
          if (tid == kVtMath0 * 32) *abort_flag = 1;
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
        if (i > 0) {  // O^T of this quadrant and half, both P halves, after PV(i-1)
          ok &= mbar_wait(bar_o, (i - 1) & 1);
          tc::fence_after();
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
      uint32_t hw[NH / 2], lw[NH / 2];
#pragma unroll
      for (int j = 0; j < NH / 2; ++j) {
        const float m0 = mreg[2 * j] == -CUDART_INF_F ? 0.f : mreg[2 * j];
        const float m1 = mreg[2 * j + 1] == -CUDART_INF_F ? 0.f : mreg[2 * j + 1];
        const float p0 = exp2_approx(x[2 * j] - m0), p1 = exp2_approx(x[2 * j + 1] - m1);
        lsum[2 * j] += p0;
        lsum[2 * j + 1] += p1;
        hw[j] = pack_half2(p0, p1);
        const float2 hf = __half22float2(*reinterpret_cast<const __half2*>(&hw[j]));
        lw[j] = pack_half2(p0 - hf.x, p1 - hf.y);
      }

      // ------------------------------ V(i) and P(i) after PV(i-1) is done
      if (i > 0) ok &= mbar_wait(bar_o, (i - 1) & 1);
      {
        const int s = i % kVtVStages;
        ok &= mbar_wait(bar_vfull + 8 * s, (i / kVtVStages) & 1);
        const uint32_t st = sb + L::kVRing + s * kVtHalfStage;
        const uint32_t vrow = sb + L::kVf + 2 * h * 16384 + tt * 128;
        dequant_row_half(st, st + kVtCodeBox, tt, h, t0 + tt >= vend, [&](int c, const uint32_t (&r)[16]) {
          // d = 128h + 32c + 8j .. +7: atom 2h + c/2, 16-byte chunk 4(c%2) + j
#pragma unroll
          for (int j = 0; j < 4; ++j)
            sts128(vrow + (c >> 1) * 16384 + (((4 * (c & 1) + j) ^ (tt & 7)) << 4), r[4 * j], r[4 * j + 1],
                   r[4 * j + 2], r[4 * j + 3]);
        });
        __syncwarp();
        if (lane == 0) mbar_arrive(bar_vempty + 8 * s);
      }
      {
        const uint32_t prow = sb + L::kP + tt * 128;
#pragma unroll
        for (int c = 0; c < NH; c += 8) {
          const int nh = NH * h + c, nl = N + NH * h + c;  // first column of the 16-byte chunk
          sts128(prow + (nh >> 6) * 16384 + ((((nh & 63) >> 3) ^ (tt & 7)) << 4), hw[c / 2], hw[c / 2 + 1],
                 hw[c / 2 + 2], hw[c / 2 + 3]);
          sts128(prow + (nl >> 6) * 16384 + ((((nl & 63) >> 3) ^ (tt & 7)) << 4), lw[c / 2], lw[c / 2 + 1],
                 lw[c / 2 + 2], lw[c / 2 + 3]);
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
    const int d = 128 * h + tt;  // O^T lane tt of M half h
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
  static_assert(kTmO + 4 * N <= kTmCols && kTmS + 64 + N <= kTmO, "tensor memory columns");
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
