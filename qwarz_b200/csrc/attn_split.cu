// Split-K paged attention over the NVFP4 one-level KV cache (decode and MTP
// verify) and over the FP8 shadow KV of the MTP draft, for sm_100a.
//
// Replaces, behind the reference's split/combine ABI
// (tests/test_attention_kernel_abi.py:13-55), the FlashInfer XQA launch of
// src/qwasar_runtime/xqa.py:484-554 (q_len <= 8 over NVFP4 pages) and the
// Triton draft split-K of engine/forward/draft_attention.py:23-61.
//
// Work decomposition.  One CTA owns one KV head and one contiguous chunk of
// 64-token stages.  Stages are staged global->shared with 16-byte cp.async
// into a multi-buffer ring (XOR-swizzled rows, so every fragment load below
// is bank-conflict free).  Dequantisation happens in registers straight into
// mma.sync fragments: codes -> f16 with the hardware E2M1/E4M3 converts and
// one f16x2 multiply by the block scale (exact: an E2M1 value times an E4M3
// scale has at most 6 significant bits and lies inside the FP16 range).
//
// Decode (q_len = 1): tokens are the MMA M dimension and the 6 GQA heads
// (padded to 8) the N dimension, so one warp holds the whole 256 x 8 output
// tile of its head group in registers and never exchanges data with other
// warps until the epilogue.  S^T comes out with tokens on rows; movmatrix
// turns it into the P^T B-fragment of the PV product.  The head-dim
// contraction of QK uses a permuted d order (k-step s of lane quad q covers
// d = 64q + 4s + {0..3}) so every A fragment register is one code byte.
//
// Verify (q_len 2..8, 6*q_len rows): phase 1 splits the 64-token stage by
// tokens (warp w: tokens 16w..16w+15, full head dim, Q from shared memory by
// ldmatrix), phase 2 splits the head dim (warp w: d in [64w, 64w+64)) so the
// 48 x 256 FP32 output tile fits in registers.  The column maxima and P
// (FP16) cross phases through shared memory.
//
// Online softmax is base-2 with lazy rescaling: the reference maximum of a
// column only moves when a tile exceeds it by more than 2^8, so p <= 256 and
// the O rescale is rare.  Partials are (m, l, O) with O unnormalised and m in
// log2 units of sm_scale * q.k.

#include "attn_common.cuh"

namespace qwz {

using namespace detail;

// =====================================================================
// NVFP4 verify, q_len 2..8 (rows = 6 * q_len <= 8 * NT).
// =====================================================================
template <typename T, int NT, int NST>
__global__ void __launch_bounds__(128, 2) nvfp4_verify_kernel(const SplitParams p) {
  constexpr int WARPS = 4, ST = 64;
  constexpr int CODE_TILE = ST * kCodeBytes;
  constexpr int SCALE_TILE = ST * kScaleBytes;
  constexpr int STAGE_BYTES = 2 * CODE_TILE + 2 * SCALE_TILE;
  constexpr int NCOL = 8 * NT;
  constexpr int Q_OFF = NST * STAGE_BYTES;
  constexpr int P_OFF = Q_OFF + NCOL * 512;
  constexpr int P_BYTES = 2 * NCOL * 128;  // hi and lo halves of P, [NCOL][64] FP16 each
  constexpr int CM_OFF = P_OFF + 2 * P_BYTES;
  constexpr int CF_OFF = CM_OFF + 2 * WARPS * NCOL * 4;
  extern __shared__ __align__(1024) uint8_t smem[];
  const uint32_t sbase = smem_u32(smem);
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31, g = lane >> 2, qd = lane & 3;
  const int split = blockIdx.x, kvh = blockIdx.y;
  const int ncol_real = p.q_len * kGroup;

  const StageRange rg = stage_range<ST>(p, split);
  const int L_pre = __ldg(p.seqlens) + p.len_add - p.q_len;

  float* colmax = reinterpret_cast<float*>(smem + CM_OFF);  // [2][WARPS][NCOL]
  float* colfac = reinterpret_cast<float*>(smem + CF_OFF);  // [NCOL]

  // ---------------- Q -> shared (FP16, permuted d order, swizzled rows)
  {
    const T* q = reinterpret_cast<const T*>(p.q);
    for (int c = warp; c < NCOL; c += WARPS) {
      uint4 raw = make_uint4(0u, 0u, 0u, 0u);
      if (c < ncol_real) {
        const int qi = c / kGroup, hg = c - qi * kGroup;
        const int row = qi * kQHeads + kvh * kGroup + hg;
        raw = __ldg(reinterpret_cast<const uint4*>(q + (size_t)row * kHeadDim) + lane);
      }
      const uint32_t rw[4] = {raw.x, raw.y, raw.z, raw.w};
      float amax = 0.f;
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const float2 f = InTraits<T>::to_float2(rw[i]);
        amax = fmaxf(amax, fmaxf(fabsf(f.x), fabsf(f.y)));
      }
#pragma unroll
      for (int off = 1; off < 32; off <<= 1) amax = fmaxf(amax, shfl_xor(amax, off));
      const float sc = pow2_row_scale(amax);
      uint32_t h[4];
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const float2 f = InTraits<T>::to_float2(rw[i]);
        h[i] = pack_half2(f.x * sc, f.y * sc);
      }
      // lane holds d = 8*lane .. 8*lane+7: quad q = lane/8, k-steps s0, s0+1.
      const int qq = lane >> 3, s0 = 2 * (lane & 7);
#pragma unroll
      for (int hs = 0; hs < 2; ++hs) {
        const int s = s0 + hs;
        // d = 64q + 4s + {0,1} -> logical k {2q, 2q+1} (chunk 2s);
        // d = 64q + 4s + {2,3} -> logical k {2q+8, 2q+9} (chunk 2s+1).
        const uint32_t rowb = sbase + Q_OFF + c * 512;
        sts32(rowb + (((2 * s) ^ (c & 7)) << 4) + 4 * qq, h[2 * hs]);
        sts32(rowb + (((2 * s + 1) ^ (c & 7)) << 4) + 4 * qq, h[2 * hs + 1]);
      }
      if (lane == 0) colfac[c] = (c < ncol_real) ? p.sm_scale_log2 / sc : 0.f;
    }
  }

  float o[4][NT][4];
#pragma unroll
  for (int j = 0; j < 4; ++j)
#pragma unroll
    for (int n = 0; n < NT; ++n) o[j][n][0] = o[j][n][1] = o[j][n][2] = o[j][n][3] = 0.f;
  float mref[NT][2], lpart[NT][2];
#pragma unroll
  for (int n = 0; n < NT; ++n) {
    mref[n][0] = mref[n][1] = -CUDART_INF_F;
    lpart[n][0] = lpart[n][1] = 0.f;
  }

  auto issue = [&](int k) {
    const int t0 = p.tok_begin + (rg.st_lo + k) * ST;
    const uint32_t slot = sbase + (k % NST) * STAGE_BYTES;
    const int pp = lookup_page(p, t0, tid == 0);
    const size_t rowbase = (size_t)(pp < 0 ? 0 : pp) * kPage + (t0 & (kPage - 1));
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const int idx = tid + (i & 3) * (2 * ST);
      const int row = idx >> 3, ch = idx & 7;
      const bool ok = pp >= 0 && (t0 + row) < rg.tok_end;
      const uint8_t* base = (i < 4) ? p.k_codes : p.v_codes;
      const uint8_t* src = ok ? base + ((rowbase + row) * kKvHeads + kvh) * kCodeBytes + ch * 16 : base;
      cp_async16(slot + (i >> 2) * CODE_TILE + swz128(row, ch), src, ok ? 16u : 0u);
    }
    {
      const int tensor = tid >= ST ? 1 : 0;
      const int row = tid - tensor * ST;
      const bool ok = pp >= 0 && (t0 + row) < rg.tok_end;
      const uint8_t* base = tensor ? p.v_scales : p.k_scales;
      const uint8_t* src = ok ? base + ((rowbase + row) * kKvHeads + kvh) * kScaleBytes : base;
      cp_async16(slot + 2 * CODE_TILE + tensor * SCALE_TILE + row * 16, src, ok ? 16u : 0u);
    }
  };

#pragma unroll
  for (int k = 0; k < NST - 1; ++k) {
    if (k < rg.n_st) issue(k);
    cp_async_commit();
  }

  for (int k = 0; k < rg.n_st; ++k) {
    cp_async_wait<NST - 2>();
    __syncthreads();
    if (k + NST - 1 < rg.n_st) issue(k + NST - 1);
    cp_async_commit();

    const uint32_t slot = sbase + (k % NST) * STAGE_BYTES;
    const int buf = k & 1;
    const int tw0 = p.tok_begin + (rg.st_lo + k) * ST + 16 * warp;

    // ---------------- phase 1: S^T for tokens 16w..16w+15, all columns
    float s[NT][4];
#pragma unroll
    for (int n = 0; n < NT; ++n) s[n][0] = s[n][1] = s[n][2] = s[n][3] = 0.f;
    {
      const int r0 = 16 * warp + g, r1 = r0 + 8;
      uint32_t kw0[8], kw1[8];
      const uint4 a = lds128(slot + swz128(r0, 2 * qd));
      const uint4 b = lds128(slot + swz128(r0, 2 * qd + 1));
      const uint4 c = lds128(slot + swz128(r1, 2 * qd));
      const uint4 d = lds128(slot + swz128(r1, 2 * qd + 1));
      kw0[0] = a.x; kw0[1] = a.y; kw0[2] = a.z; kw0[3] = a.w;
      kw0[4] = b.x; kw0[5] = b.y; kw0[6] = b.z; kw0[7] = b.w;
      kw1[0] = c.x; kw1[1] = c.y; kw1[2] = c.z; kw1[3] = c.w;
      kw1[4] = d.x; kw1[5] = d.y; kw1[6] = d.z; kw1[7] = d.w;
      uint32_t sc0[4], sc1[4];
      scales_bcast4(lds32(slot + 2 * CODE_TILE + r0 * 16 + 4 * qd), sc0);
      scales_bcast4(lds32(slot + 2 * CODE_TILE + r1 * 16 + 4 * qd), sc1);
      const int mi = lane >> 3, ri = lane & 7;
#pragma unroll
      for (int w8 = 0; w8 < 8; ++w8) {
        uint32_t h0[4], h1[4];
        e2m1x8_to_f16x2x4(kw0[w8], h0);
        e2m1x8_to_f16x2x4(kw1[w8], h1);
        const uint32_t s0 = sc0[w8 >> 1], s1 = sc1[w8 >> 1];
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          h0[j] = hmul2_u32(h0[j], s0);
          h1[j] = hmul2_u32(h1[j], s1);
        }
#pragma unroll
        for (int hs = 0; hs < 2; ++hs) {
          const int ks = 2 * w8 + hs;
#pragma unroll
          for (int np = 0; np < NT / 2; ++np) {
            const int cc = 8 * (2 * np + (mi >> 1)) + ri;
            const int chunk = 2 * ks + (mi & 1);
            uint32_t b00, b01, b10, b11;
            ldmatrix_x4(b00, b01, b10, b11, sbase + Q_OFF + cc * 512 + ((chunk ^ ri) << 4));
            mma_16816(s[2 * np], h0[2 * hs], h1[2 * hs], h0[2 * hs + 1], h1[2 * hs + 1], b00, b01);
            mma_16816(s[2 * np + 1], h0[2 * hs], h1[2 * hs], h0[2 * hs + 1], h1[2 * hs + 1], b10, b11);
          }
          if (NT & 1) {
            const int cc = 8 * (NT - 1) + ri;
            const int chunk = 2 * ks + (mi & 1);
            uint32_t b0, b1;
            ldmatrix_x2(b0, b1, sbase + Q_OFF + cc * 512 + ((chunk ^ ri) << 4));
            mma_16816(s[NT - 1], h0[2 * hs], h1[2 * hs], h0[2 * hs + 1], h1[2 * hs + 1], b0, b1);
          }
        }
      }
    }

    // scale, mask (causal inside the window, end of sequence), column max
    const bool tail = (tw0 + 15 > L_pre) || (tw0 + 16 > rg.tok_end);
    float cm[NT][2];
#pragma unroll
    for (int n = 0; n < NT; ++n) {
      const int c0 = 8 * n + 2 * qd;
      const float2 f = *reinterpret_cast<const float2*>(colfac + c0);
      s[n][0] *= f.x;
      s[n][1] *= f.y;
      s[n][2] *= f.x;
      s[n][3] *= f.y;
      if (tail) {
        const int ta = tw0 + g, tb = ta + 8;
#pragma unroll
        for (int jj = 0; jj < 2; ++jj) {
          const int c = c0 + jj;
          if (c < ncol_real) {
            const int lim = L_pre + c / kGroup;  // last visible token (inclusive)
            if (ta > lim || ta >= rg.tok_end) s[n][jj] = -CUDART_INF_F;
            if (tb > lim || tb >= rg.tok_end) s[n][2 + jj] = -CUDART_INF_F;
          }
        }
      }
      cm[n][0] = fmaxf(s[n][0], s[n][2]);
      cm[n][1] = fmaxf(s[n][1], s[n][3]);
#pragma unroll
      for (int off = 4; off < 32; off <<= 1) {
        cm[n][0] = fmaxf(cm[n][0], shfl_xor(cm[n][0], off));
        cm[n][1] = fmaxf(cm[n][1], shfl_xor(cm[n][1], off));
      }
    }
    float* cmw = colmax + (buf * WARPS + warp) * NCOL;
    if (g == 0) {
#pragma unroll
      for (int n = 0; n < NT; ++n)
        *reinterpret_cast<float2*>(cmw + 8 * n + 2 * qd) = make_float2(cm[n][0], cm[n][1]);
    }
    __syncthreads();
    bool need = false;
#pragma unroll
    for (int n = 0; n < NT; ++n) {
#pragma unroll
      for (int jj = 0; jj < 2; ++jj) {
        const int c = 8 * n + 2 * qd + jj;
        float tm = colmax[(buf * WARPS + 0) * NCOL + c];
#pragma unroll
        for (int w = 1; w < WARPS; ++w) tm = fmaxf(tm, colmax[(buf * WARPS + w) * NCOL + c]);
        cm[n][jj] = tm;
        need |= tm > mref[n][jj] + kLazy;
      }
    }
    const bool rescale = __any_sync(kFull, need);
    float alpha[NT][2];
#pragma unroll
    for (int n = 0; n < NT; ++n) {
#pragma unroll
      for (int jj = 0; jj < 2; ++jj) {
        alpha[n][jj] = 1.f;
        if (rescale) {
          const float nm = fmaxf(mref[n][jj], cm[n][jj]);
          alpha[n][jj] = (nm == -CUDART_INF_F) ? 1.f : exp2_approx(mref[n][jj] - nm);
          mref[n][jj] = nm;
          lpart[n][jj] *= alpha[n][jj];
        }
      }
    }
    const uint32_t pbuf = sbase + P_OFF + buf * P_BYTES;
#pragma unroll
    for (int n = 0; n < NT; ++n) {
      const float mu0 = (mref[n][0] == -CUDART_INF_F) ? 0.f : mref[n][0];
      const float mu1 = (mref[n][1] == -CUDART_INF_F) ? 0.f : mref[n][1];
      const float p0 = exp2_approx(s[n][0] - mu0), p1 = exp2_approx(s[n][1] - mu1);
      const float p2 = exp2_approx(s[n][2] - mu0), p3 = exp2_approx(s[n][3] - mu1);
      lpart[n][0] += p0 + p2;
      lpart[n][1] += p1 + p3;
      const PFrag pf = p_fragments(p0, p1, p2, p3);
      const int col = 8 * n + g;
      const int tl0 = 16 * warp + 2 * qd;  // token (local to the stage) of hi0/lo0; hi1/lo1 are +8
      const uint32_t a0 = col * 128 + (((tl0 >> 3) ^ (col & 7)) << 4) + (tl0 & 7) * 2;
      const uint32_t a1 = col * 128 + ((((tl0 + 8) >> 3) ^ (col & 7)) << 4) + (tl0 & 7) * 2;
      sts32(pbuf + a0, pf.hi0);
      sts32(pbuf + a1, pf.hi1);
      sts32(pbuf + NCOL * 128 + a0, pf.lo0);
      sts32(pbuf + NCOL * 128 + a1, pf.lo1);
    }
    __syncthreads();

    // ---------------- phase 2: O^T[d in 64w..64w+63] += V^T P^T
    if (rescale) {
#pragma unroll
      for (int j = 0; j < 4; ++j)
#pragma unroll
        for (int n = 0; n < NT; ++n) {
          o[j][n][0] *= alpha[n][0];
          o[j][n][1] *= alpha[n][1];
          o[j][n][2] *= alpha[n][0];
          o[j][n][3] *= alpha[n][1];
        }
    }
    const uint32_t vbase = slot + CODE_TILE;
    const uint32_t vsb = slot + 2 * CODE_TILE + SCALE_TILE + 4 * warp + (g >> 1);
    const int vchunk = 2 * warp + (g >> 2);
    const int vword = (g & 3) * 4;
    const int mi = lane >> 3, ri = lane & 7;
#pragma unroll
    for (int kk = 0; kk < 4; ++kk) {
      const int ta = 16 * kk + 2 * qd;
      const uint32_t Wa = lds32(vbase + ta * 128 + ((vchunk ^ (ta & 7)) << 4) + vword);
      const uint32_t Wb = lds32(vbase + (ta + 1) * 128 + ((vchunk ^ ((ta + 1) & 7)) << 4) + vword);
      const uint32_t Wc = lds32(vbase + (ta + 8) * 128 + ((vchunk ^ ((ta + 8) & 7)) << 4) + vword);
      const uint32_t Wd = lds32(vbase + (ta + 9) * 128 + ((vchunk ^ ((ta + 9) & 7)) << 4) + vword);
      const uint32_t sa8 = lds8(vsb + ta * 16), sb8 = lds8(vsb + (ta + 1) * 16);
      const uint32_t sc8 = lds8(vsb + (ta + 8) * 16), sd8 = lds8(vsb + (ta + 9) * 16);
      uint32_t spab, spcd, unused;
      e4m3x4_to_f16x2x2(sa8 | (sb8 << 8), spab, unused);
      e4m3x4_to_f16x2x2(sc8 | (sd8 << 8), spcd, unused);
      const uint32_t xab = (Wa & 0x0F0F0F0Fu) | ((Wb << 4) & 0xF0F0F0F0u);
      const uint32_t yab = ((Wa >> 4) & 0x0F0F0F0Fu) | (Wb & 0xF0F0F0F0u);
      const uint32_t xcd = (Wc & 0x0F0F0F0Fu) | ((Wd << 4) & 0xF0F0F0F0u);
      const uint32_t ycd = ((Wc >> 4) & 0x0F0F0F0Fu) | (Wd & 0xF0F0F0F0u);
      uint32_t hxab[4], hyab[4], hxcd[4], hycd[4];
      e2m1x8_to_f16x2x4(xab, hxab);
      e2m1x8_to_f16x2x4(yab, hyab);
      e2m1x8_to_f16x2x4(xcd, hxcd);
      e2m1x8_to_f16x2x4(ycd, hycd);
      uint32_t av[4][4];
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        av[j][0] = hmul2_u32(hxab[j], spab);
        av[j][1] = hmul2_u32(hyab[j], spab);
        av[j][2] = hmul2_u32(hxcd[j], spcd);
        av[j][3] = hmul2_u32(hycd[j], spcd);
      }
#pragma unroll
      for (int part = 0; part < 2; ++part) {  // P hi, then P lo
        const uint32_t pb = pbuf + part * (NCOL * 128);
        uint32_t bfr[NT][2];
#pragma unroll
        for (int np = 0; np < NT / 2; ++np) {
          const int cc = 8 * (2 * np + (mi >> 1)) + ri;
          const int chunk = 2 * kk + (mi & 1);
          ldmatrix_x4(bfr[2 * np][0], bfr[2 * np][1], bfr[2 * np + 1][0], bfr[2 * np + 1][1],
                      pb + cc * 128 + ((chunk ^ (cc & 7)) << 4));
        }
        if (NT & 1) {
          const int cc = 8 * (NT - 1) + ri;
          const int chunk = 2 * kk + (mi & 1);
          ldmatrix_x2(bfr[NT - 1][0], bfr[NT - 1][1], pb + cc * 128 + ((chunk ^ (cc & 7)) << 4));
        }
#pragma unroll
        for (int j = 0; j < 4; ++j)
#pragma unroll
          for (int n = 0; n < NT; ++n)
            mma_16816(o[j][n], av[j][0], av[j][1], av[j][2], av[j][3], bfr[n][0], bfr[n][1]);
      }
    }
  }

  cp_async_wait<0>();
  __syncthreads();
  // l: reduce over the 8 row-lanes, then over warps (token split of phase 1).
  float* lred = colmax;  // [WARPS][NCOL]
#pragma unroll
  for (int n = 0; n < NT; ++n) {
#pragma unroll
    for (int jj = 0; jj < 2; ++jj) {
      float v = lpart[n][jj];
#pragma unroll
      for (int off = 4; off < 32; off <<= 1) v += shfl_xor(v, off);
      lpart[n][jj] = v;
    }
  }
  if (g == 0) {
#pragma unroll
    for (int n = 0; n < NT; ++n)
      *reinterpret_cast<float2*>(lred + warp * NCOL + 8 * n + 2 * qd) =
          make_float2(lpart[n][0], lpart[n][1]);
  }
  __syncthreads();
#pragma unroll
  for (int n = 0; n < NT; ++n) {
#pragma unroll
    for (int jj = 0; jj < 2; ++jj) {
      const int c = 8 * n + 2 * qd + jj;
      if (c >= ncol_real) continue;
      const int qi = c / kGroup, hg = c - qi * kGroup;
      const size_t R = (size_t)qi * kQHeads + kvh * kGroup + hg;
      const size_t base = R * p.num_splits + split;
      float* dst = p.partial_o + base * kHeadDim + 64 * warp + 8 * g;
      *reinterpret_cast<float4*>(dst) =
          make_float4(o[0][n][jj], o[0][n][2 + jj], o[1][n][jj], o[1][n][2 + jj]);
      *reinterpret_cast<float4*>(dst + 4) =
          make_float4(o[2][n][jj], o[2][n][2 + jj], o[3][n][jj], o[3][n][2 + jj]);
      if (warp == 0 && g == 0) {
        float ls = 0.f;
#pragma unroll
        for (int w = 0; w < WARPS; ++w) ls += lred[w * NCOL + c];
        p.partial_ml[base * 2 + 0] = mref[n][jj];
        p.partial_ml[base * 2 + 1] = ls;
      }
    }
  }
}

// =====================================================================
// launchers
// =====================================================================
namespace {

template <typename K>
cudaError_t set_smem(K kernel, int bytes) {
  return cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
}

template <typename T, int NT>
cudaError_t launch_verify_nt(const SplitParams& p, cudaStream_t stream) {
  constexpr int NST = 3, ST = 64, NCOL = 8 * NT, WARPS = 4;
  const int stage = 2 * ST * kCodeBytes + 2 * ST * kScaleBytes;
  const int bytes = NST * stage + NCOL * 512 + 2 * 2 * NCOL * 128 + 2 * WARPS * NCOL * 4 + NCOL * 4;
  auto kernel = nvfp4_verify_kernel<T, NT, NST>;
  cudaError_t e = set_smem(kernel, bytes);
  if (e != cudaSuccess) return e;
  dim3 grid(p.num_splits, kKvHeads);
  kernel<<<grid, 128, bytes, stream>>>(p);
  return cudaGetLastError();
}

template <typename T>
cudaError_t launch_verify(const SplitParams& p, cudaStream_t stream) {
  const int nt = (p.q_len * kGroup + 7) / 8;
  switch (nt) {
    case 1:
    case 2: return launch_verify_nt<T, 2>(p, stream);
    case 3: return launch_verify_nt<T, 3>(p, stream);
    case 4: return launch_verify_nt<T, 4>(p, stream);
    case 5: return launch_verify_nt<T, 5>(p, stream);
    case 6: return launch_verify_nt<T, 6>(p, stream);
    default: return cudaErrorInvalidValue;
  }
}

}  // namespace

cudaError_t launch_nvfp4_split(const SplitParams& p, int dtype, cudaStream_t stream) {
  if (p.q_len == 1) {
    return dtype == kDtypeBF16 ? launch_nvfp4_decode<__nv_bfloat16>(p, stream)
                               : launch_nvfp4_decode<__half>(p, stream);
  }
  return dtype == kDtypeBF16 ? launch_verify<__nv_bfloat16>(p, stream)
                             : launch_verify<__half>(p, stream);
}

}  // namespace qwz
