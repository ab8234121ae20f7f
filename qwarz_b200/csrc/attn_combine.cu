// Log-sum-exp combine of split-K partials (m, l, O) for sm_100a.
//
// Semantics follow the reference merge (engine/forward/draft_attention.py:64-79
// `_merge_kernel`, and the two-region merge of engine/forward/draft.py:68-83):
// w_s = 2^(m_s - max_s m_s), empty splits (m = -inf) weigh 0,
// out = sum_s w_s O_s / sum_s w_s l_s.  m is in log2 units here.
//
// One CTA per output row: 8 groups of 32 lanes stride over the splits, each
// lane owns 8 contiguous head-dim elements; the groups are reduced in shared
// memory in a fixed order, so the result is deterministic.  The same kernel
// reduces a shard's local splits to one (m, l, O) record (partial mode) and
// combines the all-gathered records of the sequence-sharded decode.

#include "qwz_common.cuh"
#include "qwz_kernels.h"

#include <math_constants.h>

namespace qwz {

template <typename TOut, int MODE>
__global__ void __launch_bounds__(256) lse_combine_kernel(const CombineParams p) {
  constexpr int GROUPS = 8;
  __shared__ float red_o[GROUPS][kHeadDim];
  __shared__ float red_l[GROUPS];
  __shared__ float red_m[GROUPS];
  const int row = blockIdx.x;
  const int tid = threadIdx.x, grp = tid >> 5, lane = tid & 31;
  const float* ml = p.pml + (long long)row * p.ml_row;
  const float* po = p.po + (long long)row * p.o_row + lane * 8;

  float M = -CUDART_INF_F;
  for (int s = tid; s < p.num_splits; s += 256) M = fmaxf(M, ml[(long long)s * p.ml_split]);
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) M = fmaxf(M, __shfl_xor_sync(0xffffffffu, M, off));
  if (lane == 0) red_m[grp] = M;
  __syncthreads();
  M = red_m[0];
#pragma unroll
  for (int i = 1; i < GROUPS; ++i) M = fmaxf(M, red_m[i]);

  float acc[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
  float ls = 0.f;
  if (M != -CUDART_INF_F) {
    for (int s = grp; s < p.num_splits; s += GROUPS) {
      const float m = ml[(long long)s * p.ml_split];
      if (m == -CUDART_INF_F) continue;
      const float w = exp2_approx(m - M);
      ls += w * ml[(long long)s * p.ml_split + 1];
      const float* src = po + (long long)s * p.o_split;
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const float2 v = *reinterpret_cast<const float2*>(src + 2 * i);
        acc[2 * i] += w * v.x;
        acc[2 * i + 1] += w * v.y;
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
  dim3 grid(p.rows);
  if (mode == kCombinePartial) {
    lse_combine_kernel<float, kCombinePartial><<<grid, 256, 0, stream>>>(p);
  } else if (dtype == kDtypeBF16) {
    lse_combine_kernel<__nv_bfloat16, kCombineFinal><<<grid, 256, 0, stream>>>(p);
  } else {
    lse_combine_kernel<__half, kCombineFinal><<<grid, 256, 0, stream>>>(p);
  }
  return cudaGetLastError();
}

}  // namespace qwz
