// FP8 (E4M3) shadow-KV draft decode, q_len = 1, sm_100a.
//
// Replaces the Triton split-K draft decode of
// engine/forward/draft_attention.py:23-61 (`_partial_kernel`; the merge is
// lse_combine_kernel).  K/V are contiguous E4M3 [T, 4, 256] (the MTP draft's
// shadow store, engine/forward/draft.py:266-296), with an optional FP32
// scale per (256-token page, KV head); the reference's scale is 1.
//
// Pipeline as in attn_decode.cu: CTA = one KV head x one split (or, when
// the splits are too few to give every SM a CTA, one share of a split whose
// cluster of CTAs merges through distributed shared memory), 8 warps;
// each 128-token stage arrives by TMA as four boxes (K and V, head-dim halves
// d < 128 and d >= 128, [128 tokens x 128 B] with the 128-byte swizzle; 64 KB)
// into a 3-deep ring; the last warp to release a slot issues the next stage
// into it and publishes the stage's page scales in shared memory (a stage
// never straddles a page: the token range starts at 0).  Warp w owns tokens
// 16w..16w+15 of a stage (one mma.sync tile).
//   QK: lane quad q covers bytes [32q, 32q+32) of both halves, so k-step s
//       < 8 is d = 32q + 4s + {0..3} and s >= 8 is d = 128 + 32q + 4(s-8) +
//       {0..3}; each A register is a byte pair through cvt.rn.f16x2.e4m3x2.
//   PV: lane row g covers chunk g of both halves (d = 16g + {0..15} and
//       128 + 16g + {0..15}); tokens are paired with prmt before the convert.
// The K scale multiplies S, the V scale multiplies P (FP16, as the
// reference's Triton draft kernel feeds its PV dot).
//
// Fused shadow write (qwz_fp8_draft_step): the new FP16 K/V row for store
// slot app_slot[0] (engine/forward/draft.py:359-366, done there by two
// index_copy_ before the attention) is converted by the warp that owns the
// slot's row in its stage, right after the stage lands: it writes the E4M3
// bytes to the store and over the stale row in shared memory, so one launch
// replaces the write kernel and the attention reads the new row.

#include "attn_common.cuh"
#include "nvfp4_quant.cuh"

namespace qwz {

using namespace detail;

constexpr int kDrWarps = 8;
constexpr int kDrStages = 3;
constexpr int kDrTokens = kDrWarps * 16;                  // 128 tokens per stage
constexpr int kDrHalf = kDrTokens * 128;                  // one [128 x 128 B] box, 16 KB
constexpr int kDrStageBytes = 4 * kDrHalf;                // K lo/hi, V lo/hi: 64 KB
constexpr int kDrMetaBytes = 8 * kDrStages + 16 * kDrStages;
constexpr int kDrSmemBytes = kDrStages * kDrStageBytes + kDrMetaBytes + 1024;

namespace {

struct DrMeta {
  int released[kDrStages];
  int last_issued[kDrStages];
  float kscale[kDrStages];
  float vscale[kDrStages];
};

// Q fragments in the draft layout (see the file comment).
QWZ_DEVINL void load_q_draft(const __half* q, int row, int qd, float sm_scale_log2, uint32_t (&qf)[32],
                             float& cf0, float& cf1) {
  if (row >= 0) {
    const uint4* lo = reinterpret_cast<const uint4*>(q + (size_t)row * kHeadDim + 32 * qd);
    const uint4* hi = reinterpret_cast<const uint4*>(q + (size_t)row * kHeadDim + 128 + 32 * qd);
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const uint4 a = __ldg(lo + i), b = __ldg(hi + i);
      qf[4 * i + 0] = a.x; qf[4 * i + 1] = a.y; qf[4 * i + 2] = a.z; qf[4 * i + 3] = a.w;
      qf[16 + 4 * i + 0] = b.x; qf[16 + 4 * i + 1] = b.y; qf[16 + 4 * i + 2] = b.z; qf[16 + 4 * i + 3] = b.w;
    }
  } else {
#pragma unroll
    for (int i = 0; i < 32; ++i) qf[i] = 0u;
  }
  float amax = 0.f;
#pragma unroll
  for (int i = 0; i < 32; ++i) {
    const float2 f = InTraits<__half>::to_float2(qf[i]);
    amax = fmaxf(amax, fmaxf(fabsf(f.x), fabsf(f.y)));
  }
  amax = fmaxf(amax, shfl_xor(amax, 1));
  amax = fmaxf(amax, shfl_xor(amax, 2));
  const float sc = pow2_row_scale(amax);
#pragma unroll
  for (int i = 0; i < 32; ++i) {
    const float2 f = InTraits<__half>::to_float2(qf[i]);
    qf[i] = pack_half2(f.x * sc, f.y * sc);
  }
  const float rowfac = sm_scale_log2 / sc;
  cf0 = __shfl_sync(0xffffffffu, rowfac, 4 * (2 * qd));
  cf1 = __shfl_sync(0xffffffffu, rowfac, 4 * (2 * qd + 1));
}

// Lane l's 8 bytes (d = 8l..8l+7) of the new K and V rows of head kvh at
// store slot `slot`: into the store and, when stage != 0, over row r of that
// shared-memory stage (half l / 16, 16-byte chunk (l % 16) / 2).
QWZ_DEVINL void fp8_shadow_patch(const SplitParams& p, int slot, int kvh, int lane, float ks, float vs,
                                 uint32_t stage, int r) {
  const __half* kn = reinterpret_cast<const __half*>(p.app_k) + kvh * kHeadDim + 8 * lane;
  const __half* vn = reinterpret_cast<const __half*>(p.app_v) + kvh * kHeadDim + 8 * lane;
  const uint2 kb = quant::fp8_shadow8<__half>(kn, ks);
  const uint2 vb = quant::fp8_shadow8<__half>(vn, vs);
  const size_t off = ((size_t)slot * kKvHeads + kvh) * kHeadDim + 8 * lane;
  *reinterpret_cast<uint2*>(const_cast<uint8_t*>(p.k_codes) + off) = kb;
  *reinterpret_cast<uint2*>(const_cast<uint8_t*>(p.v_codes) + off) = vb;
  if (stage != 0u) {
    const uint32_t a = stage + (lane >> 4) * kDrHalf + swz128(r, (lane & 15) >> 1) + 8 * (lane & 1);
    asm volatile("st.shared.v2.u32 [%0], {%1, %2};\n" ::"r"(a), "r"(kb.x), "r"(kb.y) : "memory");
    asm volatile("st.shared.v2.u32 [%0], {%1, %2};\n" ::"r"(a + 2 * kDrHalf), "r"(vb.x), "r"(vb.y) : "memory");
  }
}

QWZ_DEVINL void issue_stage(const SplitParams& p, DrMeta* meta, const StageRange& rg, int k, int slot,
                            uint32_t sbase, uint32_t bar_full, int kvh) {
  const int t0 = p.tok_begin + (rg.st_lo + k) * kDrTokens;
  const int page = t0 >> 8;
  meta->last_issued[slot] = k;
  meta->kscale[slot] = p.k_page_scale ? __ldg(p.k_page_scale + page * kKvHeads + kvh) : 1.f;
  meta->vscale[slot] = p.v_page_scale ? __ldg(p.v_page_scale + page * kKvHeads + kvh) : 1.f;
  const uint32_t fb = bar_full + 8 * slot;
  mbar_arrive_expect_tx(fb, kDrStageBytes);
  const uint32_t dst = sbase + slot * kDrStageBytes;
  const int x = kvh * kHeadDim;
  tma_load_2d(dst, &p.tm_kc, x, t0, fb);
  tma_load_2d(dst + kDrHalf, &p.tm_kc, x + 128, t0, fb);
  tma_load_2d(dst + 2 * kDrHalf, &p.tm_vc, x, t0, fb);
  tma_load_2d(dst + 3 * kDrHalf, &p.tm_vc, x + 128, t0, fb);
}

// ---------------------------------------------------------------- clusters
QWZ_DEVINL int cluster_rank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;\n" : "=r"(r));
  return (int)r;
}
QWZ_DEVINL int cluster_size() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_nctarank;\n" : "=r"(r));
  return (int)r;
}
// Every thread of every CTA of the cluster; orders the shared-memory writes
// before the barrier with the peers' reads after it.
QWZ_DEVINL void cluster_sync() {
  asm volatile("barrier.cluster.arrive.release.aligned;\nbarrier.cluster.wait.acquire.aligned;\n" ::: "memory");
}
QWZ_DEVINL float ld_peer_f32(const float* local, int rank) {
  uint32_t a;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;\n" : "=r"(a) : "r"(smem_u32(local)), "r"(rank));
  float v;
  asm volatile("ld.shared::cluster.f32 %0, [%1];\n" : "=f"(v) : "r"(a) : "memory");
  return v;
}

// The cluster form of decode_epilogue: a chunk (split) is streamed by the
// csize CTAs of one cluster, each over a contiguous share of its stages.
// Each CTA merges its warps (the same fixed-order rule) into an (M, l, O)
// record in its own shared memory; rank 0 then merges the ranks' records
// in rank order (weights exp2(M_r - M), 0 for an empty share) through
// distributed shared memory and stores the chunk's partial.
constexpr int kDrMaxCluster = 4;
constexpr int kDrEpiBytes = (epilogue_smem_bytes(kDrWarps) + 15) / 16 * 16;  // then the cluster record
template <int WARPS, class DInv>
QWZ_DEVINL void draft_epilogue_cluster(const SplitParams& p, uint8_t* smem, int split, int kvh, int crank,
                                       int csize, float m0, float m1, float l0, float l1,
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
  static_assert(WARPS == kDrWarps, "the record follows the draft kernel's epilogue area");
  float* ofin = reinterpret_cast<float*>(smem + kDrEpiBytes);           // [6][256]
  float* mlfin = ofin + kGroup * kHeadDim;                              // [6][2]
  float* wfin = mlfin + 2 * kGroup;                                     // [6][kDrMaxCluster]
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
  if (tid < kGroup) {
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
    mlfin[2 * col] = M;
    mlfin[2 * col + 1] = ls;
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
    ofin[idx] = acc;
  }
  cluster_sync();  // every rank's record is in its shared memory
  if (crank == 0) {
    if (tid < kGroup) {
      const int col = tid;
      float mr[kDrMaxCluster];
      float M = -CUDART_INF_F;
      for (int r = 0; r < csize; ++r) {
        mr[r] = r == 0 ? mlfin[2 * col] : ld_peer_f32(mlfin + 2 * col, r);
        M = fmaxf(M, mr[r]);
      }
      float ls = 0.f;
      for (int r = 0; r < csize; ++r) {
        const float wt = (mr[r] == -CUDART_INF_F) ? 0.f : exp2_approx(mr[r] - M);
        wfin[col * kDrMaxCluster + r] = wt;
        ls += wt * (r == 0 ? mlfin[2 * col + 1] : ld_peer_f32(mlfin + 2 * col + 1, r));
      }
      const size_t base = (size_t)(kvh * kGroup + col) * p.num_splits + split;
      p.partial_ml[base * 2 + 0] = M;
      p.partial_ml[base * 2 + 1] = ls;
    }
    __syncthreads();
    for (int idx = tid; idx < kGroup * kHeadDim; idx += blockDim.x) {
      const int col = idx >> 8, d = idx & 255;
      float acc = wfin[col * kDrMaxCluster] * ofin[idx];
      for (int r = 1; r < csize; ++r) acc += wfin[col * kDrMaxCluster + r] * ld_peer_f32(ofin + idx, r);
      const size_t base = (size_t)(kvh * kGroup + col) * p.num_splits + split;
      p.partial_o[base * kHeadDim + d] = acc;
    }
  }
  cluster_sync();  // a peer's shared memory stays until rank 0 has read it
}

}  // namespace

// Launched with programmatic stream serialisation: barriers are set up while
// the previous kernel drains, global memory is read after griddep_wait().
// kCluster: the grid's x is split x cluster size, and the CTAs of a cluster
// share the split's stages (contiguous shares, merged in the epilogue).
template <bool kCluster>
__global__ void __launch_bounds__(kDrWarps * 32, 1) fp8_draft_kernel(const __grid_constant__ SplitParams p) {
  extern __shared__ __align__(1024) uint8_t smem[];
  const uint32_t sraw = smem_u32(smem);
  const uint32_t sbase = (sraw + 1023u) & ~1023u;
  uint8_t* sgen = smem + (sbase - sraw);
  const uint32_t bar_full = sbase + kDrStages * kDrStageBytes;
  DrMeta* meta = reinterpret_cast<DrMeta*>(sgen + kDrStages * kDrStageBytes + 8 * kDrStages);
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31, g = lane >> 2, qd = lane & 3;
  const int crank = kCluster ? cluster_rank() : 0, csize = kCluster ? cluster_size() : 1;
  const int split = blockIdx.x / csize, kvh = blockIdx.y;

  if (tid == 0) {
#pragma unroll
    for (int s = 0; s < kDrStages; ++s) {
      mbar_init(bar_full + 8 * s, 1);
      meta->released[s] = 0;
      meta->last_issued[s] = -1;
    }
    mbar_fence_init();
  }
  griddep_wait();  // shared-memory set-up overlaps the previous kernel
  StageRange rg = stage_range<kDrTokens>(p, split);
  if (kCluster) {  // this rank's contiguous share of the split's stages
    const int a = rg.n_st * crank / csize, b = rg.n_st * (crank + 1) / csize;
    rg.st_lo += a;
    rg.n_st = b - a;
  }
  int slot_new = -1;  // fused shadow write: the store slot, while a stage of this CTA may hold it
  if (p.app_k != nullptr) {
    slot_new = __ldg(p.app_slot);
    if (slot_new < 0 || slot_new >= p.capacity) {
      if (split == 0 && crank == 0 && kvh == 0 && tid == 0) flag_error(kErrSlotRange);
      slot_new = -1;
    } else if (slot_new >= rg.tok_end) {  // past the attended keys: split 0 writes the store only
      if (split == 0 && crank == 0 && warp == 0) {
        const int pg = slot_new >> 8;
        fp8_shadow_patch(p, slot_new, kvh, lane, p.k_page_scale ? __ldg(p.k_page_scale + pg * kKvHeads + kvh) : 1.f,
                         p.v_page_scale ? __ldg(p.v_page_scale + pg * kKvHeads + kvh) : 1.f, 0u, 0);
      }
      slot_new = -1;
    }
  }
  __syncthreads();
  if (tid == 0 && rg.n_st > 0) {
    tma_prefetch_desc(&p.tm_kc);
    tma_prefetch_desc(&p.tm_vc);
    for (int k = 0; k < min(rg.n_st, kDrStages); ++k) issue_stage(p, meta, rg, k, k, sbase, bar_full, kvh);
  }

  float o[16][4];
#pragma unroll
  for (int j = 0; j < 16; ++j) o[j][0] = o[j][1] = o[j][2] = o[j][3] = 0.f;
  float m0 = -CUDART_INF_F, m1 = -CUDART_INF_F, l0 = 0.f, l1 = 0.f;
  uint32_t qf[32];
  float cf0, cf1;
  load_q_draft(reinterpret_cast<const __half*>(p.q), g < kGroup ? kvh * kGroup + g : -1, qd,
               p.sm_scale_log2, qf, cf0, cf1);

  int slot = 0;
  uint32_t phase = 0;
  const int r0 = 16 * warp + g, r1 = r0 + 8;
  const int ra = 16 * warp + 2 * qd;
  for (int k = 0; k < rg.n_st; ++k) {
    if (!mbar_wait(bar_full + 8 * slot, phase)) {
      flag_error(kErrTimeout);
      break;
    }
    const uint32_t st = sbase + slot * kDrStageBytes;
    const int t0 = p.tok_begin + (rg.st_lo + k) * kDrTokens;
    const int valid_end = rg.tok_end;
    const float kscale = meta->kscale[slot], vscale = meta->vscale[slot];
    const int tw0 = t0 + 16 * warp;
    if (slot_new >= tw0 && slot_new < tw0 + 16) {  // this warp alone reads the slot's row
      fp8_shadow_patch(p, slot_new, kvh, lane, kscale, vscale, st, slot_new - t0);
      __syncwarp();
    }

    // ---------------- S^T = K Q^T
    float sa[4] = {0.f, 0.f, 0.f, 0.f}, sb[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
    for (int c = 0; c < 4; ++c) {  // chunks 2q, 2q+1 of half 0, then of half 1
      const uint32_t half = st + (c >> 1) * kDrHalf;
      const int ch = 2 * qd + (c & 1);
      const uint4 a = lds128(half + swz128(r0, ch));
      const uint4 b = lds128(half + swz128(r1, ch));
      const uint32_t A[4] = {a.x, a.y, a.z, a.w};
      const uint32_t B[4] = {b.x, b.y, b.z, b.w};
#pragma unroll
      for (int w = 0; w < 4; ++w) {
        const int ks = 4 * c + w;
        uint32_t a0, a2, a1, a3;
        e4m3x4_to_f16x2x2(A[w], a0, a2);
        e4m3x4_to_f16x2x2(B[w], a1, a3);
        if (w & 1)
          mma_16816(sb, a0, a1, a2, a3, qf[2 * ks], qf[2 * ks + 1]);
        else
          mma_16816(sa, a0, a1, a2, a3, qf[2 * ks], qf[2 * ks + 1]);
      }
    }
    const float f0 = cf0 * kscale, f1 = cf1 * kscale;
    float t[4] = {(sa[0] + sb[0]) * f0, (sa[1] + sb[1]) * f1, (sa[2] + sb[2]) * f0,
                  (sa[3] + sb[3]) * f1};
    const bool tail = tw0 + 16 > valid_end;
    if (tail) {
      if (tw0 + g >= valid_end) t[0] = t[1] = -CUDART_INF_F;
      if (tw0 + g + 8 >= valid_end) t[2] = t[3] = -CUDART_INF_F;
    }
    PFrag pf = softmax_step_decode(t, m0, m1, l0, l1, o);
    if (vscale != 1.f) pf = p_fragments(t[0] * vscale, t[1] * vscale, t[2] * vscale, t[3] * vscale);

    // ---------------- O^T += V^T P^T  (stale rows past the end are zeroed)
    const bool za = tail && t0 + ra >= valid_end, zb = tail && t0 + ra + 1 >= valid_end;
    const bool zc = tail && t0 + ra + 8 >= valid_end, zd = tail && t0 + ra + 9 >= valid_end;
#pragma unroll
    for (int half = 0; half < 2; ++half) {
      const uint32_t vh = st + (2 + half) * kDrHalf;
      const uint4 va = lds128(vh + swz128(ra, g));
      const uint4 vb = lds128(vh + swz128(ra + 1, g));
      const uint4 vc = lds128(vh + swz128(ra + 8, g));
      const uint4 vd = lds128(vh + swz128(ra + 9, g));
      uint32_t VA[4] = {va.x, va.y, va.z, va.w};
      uint32_t VB[4] = {vb.x, vb.y, vb.z, vb.w};
      uint32_t VC[4] = {vc.x, vc.y, vc.z, vc.w};
      uint32_t VD[4] = {vd.x, vd.y, vd.z, vd.w};
      if (tail) {
#pragma unroll
        for (int w = 0; w < 4; ++w) {
          if (za) VA[w] = 0u;
          if (zb) VB[w] = 0u;
          if (zc) VC[w] = 0u;
          if (zd) VD[w] = 0u;
        }
      }
#pragma unroll
      for (int w = 0; w < 4; ++w) {
#pragma unroll
        for (int pr = 0; pr < 2; ++pr) {
          const uint32_t sel = pr ? 0x7362u : 0x5140u;
          uint32_t a0, a1, a2, a3;
          e4m3x4_to_f16x2x2(__byte_perm(VA[w], VB[w], sel), a0, a1);
          e4m3x4_to_f16x2x2(__byte_perm(VC[w], VD[w], sel), a2, a3);
          mma_16816(o[8 * half + 2 * w + pr], a0, a1, a2, a3, pf.hi0, pf.hi1);
        }
      }
    }

    __syncwarp();
    if (lane == 0) {
      __threadfence_block();
      if (atomicAdd(&meta->released[slot], 1) == kDrWarps - 1) {
        meta->released[slot] = 0;
        if (k + kDrStages < rg.n_st) {
          fence_proxy_async_smem();
          issue_stage(p, meta, rg, k + kDrStages, slot, sbase, bar_full, kvh);
        }
      }
    }
    if (++slot == kDrStages) {
      slot = 0;
      phase ^= 1u;
    }
  }

  __syncthreads();
  if (tid == 0) {
#pragma unroll
    for (int s = 0; s < kDrStages; ++s) {
      const int k = meta->last_issued[s];
      if (k >= 0 && !mbar_wait(bar_full + 8 * s, (k / kDrStages) & 1)) flag_error(kErrTimeout);
    }
  }
  __syncthreads();
  griddep_launch_dependents();
  auto dinv = [](int d, int& gg, int& j) {
    gg = (d & 127) >> 4;
    j = ((d >> 7) << 3) + ((d & 15) >> 1);
  };
  if constexpr (kCluster)
    draft_epilogue_cluster<kDrWarps>(p, smem, split, kvh, crank, csize, m0, m1, l0, l1, o, dinv);
  else
    decode_epilogue<kDrWarps>(p, smem, split, kvh, m0, m1, l0, l1, o, dinv);
}

namespace {

int sm_count_of_current_device() {
  static int cached[64] = {0};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return 0;
  if (cached[dev] == 0) cudaDeviceGetAttribute(&cached[dev], cudaDevAttrMultiProcessorCount, dev);
  return cached[dev];
}

}  // namespace

// With fewer chunks than the SMs can hold (the reference's 16 chunks are 64
// CTAs on 148 SMs), each chunk is streamed by a cluster of up to four CTAs,
// so every SM pulls pages; the chunk count, the workspace and the combine
// are unchanged.
cudaError_t launch_fp8_split(const SplitParams& p, cudaStream_t stream) {
  static_assert(kDrEpiBytes + 4 * (kGroup * kHeadDim + 2 * kGroup + kGroup * kDrMaxCluster) <=
                    kDrStages * kDrStageBytes,
                "epilogue reuses the ring");
  const int sms = sm_count_of_current_device();
  int cl = sms > 0 ? sms / (p.num_splits * kKvHeads) : 1;
  cl = cl < 1 ? 1 : (cl > kDrMaxCluster ? kDrMaxCluster : cl);
  if (cl == 3) cl = 2;  // cluster sizes that tile a GPC's SM pairs
  if (cl == 1) {
    cudaError_t e = cudaFuncSetAttribute(fp8_draft_kernel<false>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         kDrSmemBytes);
    if (e != cudaSuccess) return e;
    return launch_pdl(fp8_draft_kernel<false>, dim3(p.num_splits, kKvHeads), dim3(kDrWarps * 32), kDrSmemBytes,
                      stream, p);
  }
  cudaError_t e = cudaFuncSetAttribute(fp8_draft_kernel<true>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       kDrSmemBytes);
  if (e != cudaSuccess) return e;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(p.num_splits * cl, kKvHeads);
  cfg.blockDim = dim3(kDrWarps * 32);
  cfg.dynamicSmemBytes = kDrSmemBytes;
  cfg.stream = stream;
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  attr[1].id = cudaLaunchAttributeClusterDimension;
  attr[1].val.clusterDim.x = cl;
  attr[1].val.clusterDim.y = 1;
  attr[1].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 2;
  return cudaLaunchKernelEx(&cfg, fp8_draft_kernel<true>, p);
}

}  // namespace qwz
