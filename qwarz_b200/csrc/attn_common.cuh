// Device helpers shared by the split-K attention kernels (decode, verify,
// FP8 draft): Q fragment loading, stage partitioning, page lookup, the
// base-2 online softmax with lazy rescaling, the FP16 P fragments and
// the cross-warp (m, l, O) merge of the decode layout.
#pragma once

#include "qwz_common.cuh"
#include "qwz_kernels.h"

#include <math_constants.h>

namespace qwz {
namespace detail {


constexpr float kLazy = 8.0f;
constexpr unsigned kFull = 0xffffffffu;

QWZ_DEVINL float shfl_xor(float v, int m) { return __shfl_xor_sync(kFull, v, m); }

// Four E4M3 scale bytes -> four broadcast f16x2 (s_i, s_i).
QWZ_DEVINL void scales_bcast4(uint32_t ks, uint32_t (&sc)[4]) {
  uint32_t h01, h23;
  e4m3x4_to_f16x2x2(ks, h01, h23);
  sc[0] = __byte_perm(h01, 0, 0x1010);
  sc[1] = __byte_perm(h01, 0, 0x3232);
  sc[2] = __byte_perm(h23, 0, 0x1010);
  sc[3] = __byte_perm(h23, 0, 0x3232);
}

// Power-of-two factor that brings a row amax into [2^14, 2^15), so a BF16
// (or FP16) query row converts to FP16 without overflow and, apart from
// elements below amax * 2^-24, exactly.  Returns the factor.
QWZ_DEVINL float pow2_row_scale(float amax) {
  int e = 0;
  if (amax > 0.f && amax < CUDART_INF_F) frexpf(amax, &e);
  int k = 15 - e;
  k = k > 120 ? 120 : (k < -120 ? -120 : k);
  return ldexpf(1.0f, k);
}

// Decode-layout Q fragments.  Lane (g, q) holds row g of the head group,
// d in [64q, 64q+64) as 32 f16x2 words; rows 6,7 are zero padding.
template <typename T>
QWZ_DEVINL void load_q_decode(const T* q, int row, int qd, float sm_scale_log2,
                              uint32_t (&qf)[32], float& cf0, float& cf1) {
  if (row >= 0) {
    const uint4* src = reinterpret_cast<const uint4*>(q + (size_t)row * kHeadDim + 64 * qd);
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const uint4 v = __ldg(src + i);
      qf[4 * i + 0] = v.x;
      qf[4 * i + 1] = v.y;
      qf[4 * i + 2] = v.z;
      qf[4 * i + 3] = v.w;
    }
  } else {
#pragma unroll
    for (int i = 0; i < 32; ++i) qf[i] = 0u;
  }
  float amax = 0.f;
#pragma unroll
  for (int i = 0; i < 32; ++i) {
    const float2 f = InTraits<T>::to_float2(qf[i]);
    amax = fmaxf(amax, fmaxf(fabsf(f.x), fabsf(f.y)));
  }
  amax = fmaxf(amax, shfl_xor(amax, 1));
  amax = fmaxf(amax, shfl_xor(amax, 2));
  const float sc = pow2_row_scale(amax);
#pragma unroll
  for (int i = 0; i < 32; ++i) {
    const float2 f = InTraits<T>::to_float2(qf[i]);
    qf[i] = pack_half2(f.x * sc, f.y * sc);
  }
  const float rowfac = sm_scale_log2 / sc;
  const int lane = threadIdx.x & 31;
  (void)lane;
  cf0 = __shfl_sync(kFull, rowfac, 4 * (2 * qd));
  cf1 = __shfl_sync(kFull, rowfac, 4 * (2 * qd + 1));
}

// Token range of this split, in stages of ST tokens.
struct StageRange {
  int tok_end;  // exclusive end of the valid tokens (post-append length clipped)
  int st_lo;
  int n_st;
};

template <int ST>
QWZ_DEVINL StageRange stage_range(const SplitParams& p, int split) {
  StageRange r;
  const int L = __ldg(p.seqlens) + p.len_add;
  const long long end = (long long)p.tok_begin + (long long)p.tok_span;
  r.tok_end = (int)min((long long)L, end);
  const int n_tok = max(r.tok_end - p.tok_begin, 0);
  const int total = (n_tok + ST - 1) / ST;
  int lo, hi;
  if (p.split_len > 0) {
    const int per = p.split_len / ST;
    lo = split * per;
    hi = min(lo + per, total);
  } else {
    lo = (int)(((long long)split * total) / p.num_splits);
    hi = (int)(((long long)(split + 1) * total) / p.num_splits);
  }
  r.st_lo = lo;
  r.n_st = max(hi - lo, 0);
  return r;
}

// Physical page of the 256-token page holding logical token t, or -1.
QWZ_DEVINL int lookup_page(const SplitParams& p, int t, bool report) {
  const int lp = (t >> 8) - p.table_page_offset;
  if (lp < 0 || lp >= p.table_width) {
    if (report) flag_error(kErrTableRange);
    return -1;
  }
  const int pp = __ldg(p.block_table + lp);
  if (pp < 0 || pp >= p.num_pages) {
    if (report) flag_error(kErrPageRange);
    return -1;
  }
  return pp;
}

// P (FP32) as the FP16 B-fragments of the PV product: P is rounded to FP16
// once, the precision of the PV operand in the reference's XQA kernel
// (the S^T c-fragment is transposed into the P^T b-fragment by movmatrix).
struct PFrag {
  uint32_t hi0, hi1;
};

QWZ_DEVINL PFrag p_fragments(float p0, float p1, float p2, float p3) {
  PFrag f;
  f.hi0 = movmatrix_trans(pack_half2(p0, p1));
  f.hi1 = movmatrix_trans(pack_half2(p2, p3));
  return f;
}

// One online-softmax step on a 16-token x 8-column S^T fragment.
// t: scaled scores (c-fragment), overwritten with p; returns P^T fragments.
QWZ_DEVINL PFrag softmax_step_decode(float (&t)[4], float& m0, float& m1, float& l0,
                                     float& l1, float (&o)[16][4]) {
  float mx0 = fmaxf(t[0], t[2]);
  float mx1 = fmaxf(t[1], t[3]);
#pragma unroll
  for (int off = 4; off < 32; off <<= 1) {
    mx0 = fmaxf(mx0, shfl_xor(mx0, off));
    mx1 = fmaxf(mx1, shfl_xor(mx1, off));
  }
  const bool need = (mx0 > m0 + kLazy) || (mx1 > m1 + kLazy);
  if (__any_sync(kFull, need)) {
    const float n0 = fmaxf(m0, mx0), n1 = fmaxf(m1, mx1);
    const float a0 = (n0 == -CUDART_INF_F) ? 1.f : exp2_approx(m0 - n0);
    const float a1 = (n1 == -CUDART_INF_F) ? 1.f : exp2_approx(m1 - n1);
    m0 = n0;
    m1 = n1;
    l0 *= a0;
    l1 *= a1;
#pragma unroll
    for (int j = 0; j < 16; ++j) {
      o[j][0] *= a0;
      o[j][1] *= a1;
      o[j][2] *= a0;
      o[j][3] *= a1;
    }
  }
  const float mu0 = (m0 == -CUDART_INF_F) ? 0.f : m0;
  const float mu1 = (m1 == -CUDART_INF_F) ? 0.f : m1;
  const float p0 = exp2_approx(t[0] - mu0), p1 = exp2_approx(t[1] - mu1);
  const float p2 = exp2_approx(t[2] - mu0), p3 = exp2_approx(t[3] - mu1);
  l0 += p0 + p2;
  l1 += p1 + p3;
  t[0] = p0;
  t[1] = p1;
  t[2] = p2;
  t[3] = p3;
  return p_fragments(p0, p1, p2, p3);
}

// Shared-memory bytes of decode_epilogue for WARPS warps: per warp 16
// m-tile rows of 32 lane float4s padded to 33 (writes conflict-free, reads
// at most 2-way), then (m, l) per warp and column, then the merge weights.
constexpr int kEpiRowF4 = 33;
constexpr int epilogue_smem_bytes(int warps) {
  return warps * 16 * kEpiRowF4 * 16 + warps * 8 * 2 * 4 + 8 * warps * 4;
}

// Cross-warp merge of decode-layout (m, l, O) and the partial store.
// dinv(d, g, j) gives the lane row g and m-tile j whose accumulator row
// holds head-dim d (the even member of the pair d, d+1 sits in c0/c1, the
// odd one in c2/c3).  Summation order over warps is fixed.
template <int WARPS, class DInv>
QWZ_DEVINL void decode_epilogue(const SplitParams& p, uint8_t* smem, int split, int kvh,
                                float m0, float m1, float l0, float l1,
                                const float (&o)[16][4], DInv dinv) {
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31, g = lane >> 2, qd = lane & 3;
#pragma unroll
  for (int off = 4; off < 32; off <<= 1) {
    l0 += shfl_xor(l0, off);
    l1 += shfl_xor(l1, off);
  }
  float4* red = reinterpret_cast<float4*>(smem);                       // [WARPS][16][33]
  float* mlred = reinterpret_cast<float*>(red + WARPS * 16 * kEpiRowF4);  // [WARPS][8][2]
  float* wts = mlred + WARPS * 16;                                      // [8 cols][WARPS]
#pragma unroll
  for (int j = 0; j < 16; ++j)
    red[(warp * 16 + j) * kEpiRowF4 + lane] = make_float4(o[j][0], o[j][1], o[j][2], o[j][3]);
  if (g == 0) {
    mlred[(warp * 8 + 2 * qd) * 2 + 0] = m0;
    mlred[(warp * 8 + 2 * qd) * 2 + 1] = l0;
    mlred[(warp * 8 + 2 * qd + 1) * 2 + 0] = m1;
    mlred[(warp * 8 + 2 * qd + 1) * 2 + 1] = l1;
  }
  __syncthreads();
  if (tid < kGroup) {  // per column: CTA max, warp weights, l
    const int col = tid;
    float M = -CUDART_INF_F;
#pragma unroll
    for (int w = 0; w < WARPS; ++w) M = fmaxf(M, mlred[(w * 8 + col) * 2]);
    float ls = 0.f;
#pragma unroll
    for (int w = 0; w < WARPS; ++w) {
      const float mw = mlred[(w * 8 + col) * 2];
      const float wt = (mw == -CUDART_INF_F) ? 0.f : exp2_approx(mw - M);
      wts[col * WARPS + w] = wt;
      ls += wt * mlred[(w * 8 + col) * 2 + 1];
    }
    const size_t base = (size_t)(kvh * kGroup + col) * p.num_splits + split;
    p.partial_ml[base * 2 + 0] = M;
    p.partial_ml[base * 2 + 1] = ls;
  }
  __syncthreads();
  const float* rf = reinterpret_cast<const float*>(red);
  for (int idx = tid; idx < kGroup * kHeadDim; idx += blockDim.x) {
    const int col = idx >> 8, d = idx & 255;
    int gg, j;
    dinv(d, gg, j);
    const int src = ((j * kEpiRowF4) + 4 * gg + (col >> 1)) * 4 + (col & 1) + 2 * (d & 1);
    float acc = 0.f;
#pragma unroll
    for (int w = 0; w < WARPS; ++w) acc += wts[col * WARPS + w] * rf[w * 16 * kEpiRowF4 * 4 + src];
    const size_t base = (size_t)(kvh * kGroup + col) * p.num_splits + split;
    p.partial_o[base * kHeadDim + d] = acc;
  }
}


}  // namespace detail
}  // namespace qwz
