// Sequence-sharded decode: the record exchange and the final LSE merge fused
// into one kernel over NVLink peer memory (no reference counterpart; the
// reference is single-GPU, src/qwasar_runtime/engine.py:602-610).
//
// Every rank owns an exchange buffer of identical layout:
//   records u64 [2][world][rows][258]: (m, l, O[256]) of rank src at
//   [e & 1][src], each value in the low 32 bits of a word whose high 32 bits
//   carry the epoch e of the call that wrote it.  Alternating halves by
//   epoch parity means a rank that runs ahead to call e+1 never overwrites a
//   call-e record a slower rank has yet to read (reaching call e+2 needs the
//   slower rank's call-e+1 record, written after its call e finished).
// A 64-bit aligned store reaches the peer as one unit, so the value and its
// epoch arrive together and the reader polls the data itself: there is no
// separate flag and no system-scope fence (the low-latency protocol of small
// collectives).  CTA r of rank g:
//   1. merges rank g's num_splits partials of row r (split order fixed) into
//      one (m, l, O) record;
//   2. stores it, tagged with e = this row's call count, into every rank's
//      buffer at [g][r] (stores into the peers' memory);
//   3. reads the world records of row r from its own buffer, all ranks'
//      words in one batch of loads per poll, until every word carries epoch
//      e (bounded by globaltimer, p.timeout_ns for the whole row: a timeout
//      sets kErrTimeout and merges the records that did arrive), and merges
//      them in rank order, so every rank writes the same output.
// Epochs count calls per row on every rank (a device word per row, advanced
// by the kernel), so repeated launches and CUDA-graph replays need no reset.
// With fewer GPUs than ranks the kernel runs all ranks in one cooperative
// launch (blockIdx.y = rank, buffers on one GPU), so ranks that wait on one
// another are always co-resident.

#include "qwz_common.cuh"
#include "qwz_kernels.h"

#include <math_constants.h>

namespace qwz {

namespace {

constexpr int kRecWords = kHeadDim + 2;                         // m, l, O[256]

QWZ_DEVINL uint64_t global_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}
QWZ_DEVINL void st_tagged(uint64_t* p, float v, uint32_t e) {
  const uint64_t w = (uint64_t)__float_as_uint(v) | ((uint64_t)e << 32);
  asm volatile("st.relaxed.sys.global.u64 [%0], %1;" ::"l"(p), "l"(w) : "memory");
}
QWZ_DEVINL uint64_t ld_tagged(const uint64_t* p) {
  uint64_t w;
  asm volatile("ld.relaxed.sys.global.u64 %0, [%1];" : "=l"(w) : "l"(p) : "memory");
  return w;
}
}  // namespace

template <typename TOut>
__global__ void __launch_bounds__(256) shard_exchange_kernel(const ExchangeParams p) {
  constexpr int GROUPS = 8;
  __shared__ float red_o[GROUPS][kHeadDim];
  __shared__ float red_l[GROUPS];
  __shared__ float red_m[GROUPS];
  __shared__ uint32_t s_epoch;
  const int r = blockIdx.x, y = blockIdx.y, rank = p.rank0 + y;
  const int tid = threadIdx.x, grp = tid >> 5, lane = tid & 31;
  const int S = p.num_splits, rows = p.rows;

  griddep_wait();               // the split partials come from the previous kernel
  griddep_launch_dependents();  // the next kernel may begin its launch
  // ---------------------------------------------- 1. this rank's record
  const float* ml = p.pml[y] + (size_t)r * S * 2;
  const float* po = p.po[y] + (size_t)r * S * kHeadDim + lane * 8;
  if (tid == 0) s_epoch = p.epochs[y][r] + 1u;
  float acc[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
  float ls = 0.f, M = -CUDART_INF_F;
  constexpr int J = 8;  // splits per group held in registers (64 per row in one batch)
  if (S <= GROUPS * J) {
    // one batch of loads: the group's (m, l) and O slices, then the row max
    float mv[J], lv[J];
    float4 oa[J], ob[J];
#pragma unroll
    for (int j = 0; j < J; ++j) {
      const int s = grp + GROUPS * j;
      mv[j] = -CUDART_INF_F;
      lv[j] = 0.f;
      oa[j] = ob[j] = make_float4(0.f, 0.f, 0.f, 0.f);
      if (s < S) {
        const float2 v = __ldcg(reinterpret_cast<const float2*>(ml) + s);
        mv[j] = v.x;
        lv[j] = v.y;
        oa[j] = __ldcg(reinterpret_cast<const float4*>(po + (size_t)s * kHeadDim));
        ob[j] = __ldcg(reinterpret_cast<const float4*>(po + (size_t)s * kHeadDim + 4));
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
        acc[0] += w * oa[j].x; acc[1] += w * oa[j].y; acc[2] += w * oa[j].z; acc[3] += w * oa[j].w;
        acc[4] += w * ob[j].x; acc[5] += w * ob[j].y; acc[6] += w * ob[j].z; acc[7] += w * ob[j].w;
      }
    }
  } else {
    for (int s = tid; s < S; s += 256) M = fmaxf(M, ml[2 * s]);
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) M = fmaxf(M, __shfl_xor_sync(0xffffffffu, M, off));
    if (lane == 0) red_m[grp] = M;
    __syncthreads();
    M = red_m[0];
#pragma unroll
    for (int i = 1; i < GROUPS; ++i) M = fmaxf(M, red_m[i]);
    if (M != -CUDART_INF_F) {
#pragma unroll 4
      for (int s = grp; s < S; s += GROUPS) {  // empty splits (m = -inf, O = 0) weigh 0
        const float m = ml[2 * s];
        const float w = m == -CUDART_INF_F ? 0.f : exp2_approx(m - M);
        ls += w * ml[2 * s + 1];
        const float4 a = *reinterpret_cast<const float4*>(po + (size_t)s * kHeadDim);
        const float4 b = *reinterpret_cast<const float4*>(po + (size_t)s * kHeadDim + 4);
        acc[0] += w * a.x; acc[1] += w * a.y; acc[2] += w * a.z; acc[3] += w * a.w;
        acc[4] += w * b.x; acc[5] += w * b.y; acc[6] += w * b.z; acc[7] += w * b.w;
      }
    }
  }
#pragma unroll
  for (int i = 0; i < 8; ++i) red_o[grp][lane * 8 + i] = acc[i];
  if (lane == 0) red_l[grp] = ls;
  __syncthreads();
  float o = 0.f, L = 0.f;
#pragma unroll
  for (int i = 0; i < GROUPS; ++i) {
    o += red_o[i][tid];
    L += red_l[i];
  }
  const uint32_t e = s_epoch;

  // ------------------------------------------- 2. store it on every rank
  const size_t half = (size_t)(e & 1u) * p.world * rows * kRecWords;
  const size_t rec = half + ((size_t)rank * rows + r) * kRecWords;
  for (int g = 0; g < p.world; ++g) {
    uint64_t* dst = reinterpret_cast<uint64_t*>(p.peers[g]) + rec;
    st_tagged(dst + 2 + tid, o, e);
    if (tid == 0) {
      st_tagged(dst, M, e);
      st_tagged(dst + 1, L, e);
    }
  }

  // --------------------------------------- 3. wait for all, merge, write
  // Every rank's three words of this thread are loaded in one batch (the
  // loads are independent, so they are in flight together: one round trip
  // per poll, not one per rank); only the words whose epoch is still old
  // are loaded again.
  const uint64_t* local = reinterpret_cast<const uint64_t*>(p.peers[rank]);
  const uint64_t t0 = global_ns();
  bool ok = true;
  float mg[kMaxWorld], lg[kMaxWorld], og[kMaxWorld];
  uint64_t wm[kMaxWorld], wl[kMaxWorld], wo[kMaxWorld];
  uint32_t pending = 0u;  // bit g: rank g's words are not all of epoch e yet
#pragma unroll
  for (int g = 0; g < kMaxWorld; ++g) {
    wm[g] = wl[g] = wo[g] = 0ull;
    if (g < p.world) pending |= 1u << g;
  }
  for (int i = 0; pending; ++i) {
#pragma unroll
    for (int g = 0; g < kMaxWorld; ++g) {
      if (pending & (1u << g)) {
        const uint64_t* src = local + half + ((size_t)g * rows + r) * kRecWords;
        wm[g] = ld_tagged(src);
        wl[g] = ld_tagged(src + 1);
        wo[g] = ld_tagged(src + 2 + tid);
      }
    }
#pragma unroll
    for (int g = 0; g < kMaxWorld; ++g) {
      if ((pending & (1u << g)) && (uint32_t)(wm[g] >> 32) == e && (uint32_t)(wl[g] >> 32) == e &&
          (uint32_t)(wo[g] >> 32) == e)
        pending &= ~(1u << g);
    }
    if (pending && (i & 63) == 63) {
      if (global_ns() - t0 > p.timeout_ns) {
        ok = false;
        break;
      }
      __nanosleep(32);
    }
  }
#pragma unroll
  for (int g = 0; g < kMaxWorld; ++g) {
    // ranks whose record never arrived merge as empty (m = -inf)
    const bool have = g < p.world && !(pending & (1u << g));
    mg[g] = have ? __uint_as_float((uint32_t)wm[g]) : -CUDART_INF_F;
    lg[g] = have ? __uint_as_float((uint32_t)wl[g]) : 0.f;
    og[g] = have ? __uint_as_float((uint32_t)wo[g]) : 0.f;
  }
  if (!ok) flag_error(kErrTimeout);
  float Mg = -CUDART_INF_F;
#pragma unroll
  for (int g = 0; g < kMaxWorld; ++g) Mg = fmaxf(Mg, mg[g]);
  float on = 0.f, ln = 0.f;
  if (Mg != -CUDART_INF_F) {
#pragma unroll
    for (int g = 0; g < kMaxWorld; ++g) {
      if (g >= p.world || mg[g] == -CUDART_INF_F) continue;
      const float w = exp2_approx(mg[g] - Mg);
      ln += w * lg[g];
      on += w * og[g];
    }
  }
  TOut* out = reinterpret_cast<TOut*>(p.out[y]) + (size_t)r * kHeadDim;
  out[tid] = InTraits<TOut>::from_float(ln > 0.f ? on / ln : 0.f);
  if (tid == 0) p.epochs[y][r] = e;
}

cudaError_t launch_shard_exchange(const ExchangeParams& p, int emulated, int dtype, cudaStream_t stream) {
  if (p.rows <= 0) return cudaSuccess;
  dim3 grid(p.rows, emulated ? p.world : 1);
  void* args[] = {const_cast<ExchangeParams*>(&p)};
  auto kernel = dtype == kDtypeBF16 ? (const void*)shard_exchange_kernel<__nv_bfloat16>
                                    : (const void*)shard_exchange_kernel<__half>;
  if (emulated)  // ranks that wait on one another must be co-resident
    return cudaLaunchCooperativeKernel(kernel, grid, dim3(256), args, 0, stream);
  // one real rank: launched with programmatic stream serialisation (the
  // kernel reads the split partials only after griddep_wait())
  if (dtype == kDtypeBF16) return launch_pdl(shard_exchange_kernel<__nv_bfloat16>, grid, dim3(256), 0, stream, p);
  return launch_pdl(shard_exchange_kernel<__half>, grid, dim3(256), 0, stream, p);
}

}  // namespace qwz
