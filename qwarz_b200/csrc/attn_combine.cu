// Log-sum-exp combine of split-K partials (m, l, O) for sm_100a.
//
// Semantics follow the reference merge (engine/forward/draft_attention.py:64-79
// `_merge_kernel`, and the two-region merge of engine/forward/draft.py:68-83):
// w_s = 2^(m_s - max_s m_s), empty splits (m = -inf) weigh 0,
// out = sum_s w_s O_s / sum_s w_s l_s.  m is in log2 units here.
//
// One CTA per output row: 8 groups of 32 lanes stride over the splits, each
// lane owns 8 contiguous head-dim elements; the groups are reduced in shared
// memory in a fixed order, so the result is deterministic.  Up to 64 splits
// a row's loads are all issued in one batch (one L2 round trip, not one per
// split), and the next kernel in the stream may begin its launch as soon as
// the combine starts (programmatic dependent launch).  The same kernel
// reduces a shard's local splits to one (m, l, O) record (partial mode) and
// combines the all-gathered records of the sequence-sharded decode.  In
// rotate mode (the K8/V4 cache, whose partials are in the rotated domain
// R = H32 / sqrt(32)) the merged row is restored as out = R^T O per 32-dim
// block, R being the caller's h32 matrix.

#include "qwz_common.cuh"
#include "qwz_kernels.h"

#include <math_constants.h>

namespace qwz {

template <typename TOut, int MODE>
__global__ void __launch_bounds__(256) lse_combine_kernel(const CombineParams p) {
  constexpr int GROUPS = 8;
  constexpr int J = 8;  // splits per group held in registers (64 per row in one batch)
  __shared__ float red_o[GROUPS][kHeadDim];
  __shared__ float red_l[GROUPS];
  __shared__ float red_m[GROUPS];
  const int row = blockIdx.x;
  const int tid = threadIdx.x, grp = tid >> 5, lane = tid & 31;
  constexpr int kRotPitch = 33;
  __shared__ float rot_h[MODE == kCombineRotate ? 32 * kRotPitch : 1];
  __shared__ float rot_v[MODE == kCombineRotate ? kHeadDim : 1];
  if constexpr (MODE == kCombineRotate) {
    // the rotation is a constant input, not written by the split kernel: it
    // is read while the split drains
    for (int k = tid; k < 1024; k += 256) rot_h[(k >> 5) * kRotPitch + (k & 31)] = __ldg(p.h32 + k);
  }
  griddep_wait();               // the partials come from the previous kernel
  griddep_launch_dependents();  // the next kernel may begin its launch
  const float* ml = p.pml + (long long)row * p.ml_row;
  const float* po = p.po + (long long)row * p.o_row + lane * 8;
  const int S = p.num_splits;

  float acc[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
  float ls = 0.f, M = -CUDART_INF_F;
  if (S <= GROUPS * J) {
    // one batch: every (m, l) and O slice of the group's splits, then the
    // row maximum, then the weighted sums from registers
    float mv[J], lv[J], ov[J][8];
#pragma unroll
    for (int j = 0; j < J; ++j) {
      const int s = grp + GROUPS * j;
      mv[j] = -CUDART_INF_F;
      lv[j] = 0.f;
#pragma unroll
      for (int i = 0; i < 8; ++i) ov[j][i] = 0.f;
      if (s < S) {
        mv[j] = __ldcg(ml + (long long)s * p.ml_split);
        lv[j] = __ldcg(ml + (long long)s * p.ml_split + 1);
        const float* src = po + (long long)s * p.o_split;
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          const float2 v = __ldcg(reinterpret_cast<const float2*>(src + 2 * i));
          ov[j][2 * i] = v.x;
          ov[j][2 * i + 1] = v.y;
        }
      }
    }
    float mloc = -CUDART_INF_F;
#pragma unroll
    for (int j = 0; j < J; ++j) mloc = fmaxf(mloc, mv[j]);
    if (lane == 0) red_m[grp] = mloc;
    __syncthreads();
    M = red_m[0];
#pragma unroll
    for (int i = 1; i < GROUPS; ++i) M = fmaxf(M, red_m[i]);
    if (M != -CUDART_INF_F) {
#pragma unroll
      for (int j = 0; j < J; ++j) {  // empty splits (m = -inf, O = 0) weigh 0
        const float w = mv[j] == -CUDART_INF_F ? 0.f : exp2_approx(mv[j] - M);
        ls += w * lv[j];
#pragma unroll
        for (int i = 0; i < 8; ++i) acc[i] += w * ov[j][i];
      }
    }
  } else {
    for (int s = tid; s < S; s += 256) M = fmaxf(M, __ldcg(ml + (long long)s * p.ml_split));
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) M = fmaxf(M, __shfl_xor_sync(0xffffffffu, M, off));
    if (lane == 0) red_m[grp] = M;
    __syncthreads();
    M = red_m[0];
#pragma unroll
    for (int i = 1; i < GROUPS; ++i) M = fmaxf(M, red_m[i]);
    if (M != -CUDART_INF_F) {
      for (int s = grp; s < S; s += GROUPS) {
        const float m = __ldcg(ml + (long long)s * p.ml_split);
        if (m == -CUDART_INF_F) continue;
        const float w = exp2_approx(m - M);
        ls += w * __ldcg(ml + (long long)s * p.ml_split + 1);
        const float* src = po + (long long)s * p.o_split;
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          const float2 v = __ldcg(reinterpret_cast<const float2*>(src + 2 * i));
          acc[2 * i] += w * v.x;
          acc[2 * i + 1] += w * v.y;
        }
      }
    }
  }
#pragma unroll
  for (int i = 0; i < 8; ++i) red_o[grp][lane * 8 + i] = acc[i];
  if (lane == 0) red_l[grp] = ls;
  __syncthreads();

  const int d = tid;
  float o = 0.f, L = 0.f;
#pragma unroll
  for (int i = 0; i < GROUPS; ++i) {
    o += red_o[i][d];
    L += red_l[i];
  }
  if constexpr (MODE == kCombineFinal) {
    TOut* out = reinterpret_cast<TOut*>(p.out) + (long long)row * kHeadDim;
    out[d] = InTraits<TOut>::from_float(L > 0.f ? o / L : 0.f);
  } else if constexpr (MODE == kCombineRotate) {
    rot_v[d] = L > 0.f ? o / L : 0.f;
    __syncthreads();
    // out_i = sum_j R[j][i] O_j within the block (a warp is one block)
    const int b = d >> 5, i = d & 31;
    float acc = 0.f;
#pragma unroll
    for (int j = 0; j < 32; ++j) acc = fmaf(rot_h[j * kRotPitch + i], rot_v[b * 32 + j], acc);
    TOut* out = reinterpret_cast<TOut*>(p.out) + (long long)row * kHeadDim;
    out[d] = InTraits<TOut>::from_float(acc);
  } else {
    float* out = reinterpret_cast<float*>(p.out) + (long long)row * (kHeadDim + 2);
    out[2 + d] = o;
    if (d == 0) {
      out[0] = M;
      out[1] = L;
    }
  }
}

cudaError_t launch_combine(const CombineParams& p, int mode, int dtype, cudaStream_t stream) {
  if (p.rows <= 0) return cudaSuccess;
  // the launch overlaps the split kernel's tail; the kernel reads the
  // partials only after griddep_wait()
  const dim3 grid(p.rows), block(256);
  if (mode == kCombinePartial) return launch_pdl(lse_combine_kernel<float, kCombinePartial>, grid, block, 0, stream, p);
  if (mode == kCombineRotate) {
    if (dtype == kDtypeBF16) return launch_pdl(lse_combine_kernel<__nv_bfloat16, kCombineRotate>, grid, block, 0, stream, p);
    return launch_pdl(lse_combine_kernel<__half, kCombineRotate>, grid, block, 0, stream, p);
  }
  if (dtype == kDtypeBF16) return launch_pdl(lse_combine_kernel<__nv_bfloat16, kCombineFinal>, grid, block, 0, stream, p);
  return launch_pdl(lse_combine_kernel<__half, kCombineFinal>, grid, block, 0, stream, p);
}

}  // namespace qwz
