// NVFP4 paged decode (q_len = 1), sm_100a: one 256-token page per pipeline
// stage, streamed by TMA, dequantised in registers into mma.sync fragments.
//
// Replaces the q_len = 1 XQA launch of src/qwasar_runtime/xqa.py:484-554
// behind the split ABI of tests/test_attention_kernel_abi.py:13-32.
//
// CTA = one KV head x one contiguous run of pages (a split), 8 warps.  Each
// page of the head's slice arrives as four TMA boxes ([256 tokens x 128 B]
// codes of K and V with the 128-byte swizzle, [256 x 16 B] scales; 72 KB)
// in a 3-deep ring; a full mbarrier per slot tracks the bytes.  There is no
// producer warp: thread 0 issues the first three pages, and afterwards the
// last warp to release a slot (a shared-memory counter) issues the next page
// into it, so no warp ever waits for a slot to drain.  The block-table row
// (up to kDecPidCache entries) is staged in shared memory up front, loaded
// in parallel with the sequence length.  (Measured on B200: separate K/V
// barriers per slot, or issuing page 0 ahead of pages 1-2, do not pay.)
// Warp w owns tokens 32w..32w+31 of every page as two independent 16-token
// MMA tiles (A: +0..15, B: +16..31), which gives each warp two dependency
// chains to interleave and one softmax update per 32 tokens.  Layout per
// tile:
//   QK  S^T[16 tok x 8 heads] = K[16 x 256] Q^T, tokens on M, the 6 GQA
//       heads (padded to 8) on N, lane quad q's k-step s covering
//       d = 64q + 4s + {0..3} so each A register is one code byte;
//   PV  O^T[256 x 8] += V^T P^T, m-tile j row g <-> d = 32g + 2j (+1),
//       P^T from movmatrix of the S^T fragment, P in FP16 (the PV operand
//       precision of the reference's XQA kernel; measured on B200 the hi + lo
//       split it replaced cost 10 % at 262K for one extra MMA per tile).
// Waits are bounded (kErrTimeout instead of a hang).
//
// The kernel is launched with programmatic stream serialisation: a CTA sets
// up its shared memory and barriers while the previous kernel in the stream
// drains, reads nothing from global memory before griddep_wait(), and lets
// the combine launch begin once its page loop is done.

#include "attn_common.cuh"
#include "nvfp4_quant.cuh"

namespace qwz {

using namespace detail;

constexpr int kDecWarps = 8;                                   // warps per CTA
constexpr int kDecStages = 3;                                  // ring depth (pages)
constexpr int kDecPidCache = 1024;                             // page ids staged in smem
constexpr int kDecCodeTile = kPage * kCodeBytes;               // 32 KB
constexpr int kDecScaleTile = kPage * kScaleBytes;             // 4 KB
constexpr int kDecStageBytes = 2 * kDecCodeTile + 2 * kDecScaleTile;
// ring | full barriers | per-slot release counters, page ends, last issued
// page | table row
constexpr int kDecMetaBytes = 8 * kDecStages + 16 * kDecStages;
constexpr int kDecSmemBytes = kDecStages * kDecStageBytes + kDecMetaBytes + 4 * kDecPidCache + 1024;

namespace {

// One 16-token tile's QK: raw S^T fragment (4 floats).
QWZ_DEVINL void qk_tile(uint32_t codes, uint32_t scales, int r0, int qd, const uint32_t (&qf)[32],
                        float (&s)[4]) {
  uint32_t kw0[8], kw1[8];
  const int r1 = r0 + 8;
  {
    const uint4 a = lds128(codes + swz128(r0, 2 * qd));
    const uint4 b = lds128(codes + swz128(r0, 2 * qd + 1));
    const uint4 c = lds128(codes + swz128(r1, 2 * qd));
    const uint4 d = lds128(codes + swz128(r1, 2 * qd + 1));
    kw0[0] = a.x; kw0[1] = a.y; kw0[2] = a.z; kw0[3] = a.w;
    kw0[4] = b.x; kw0[5] = b.y; kw0[6] = b.z; kw0[7] = b.w;
    kw1[0] = c.x; kw1[1] = c.y; kw1[2] = c.z; kw1[3] = c.w;
    kw1[4] = d.x; kw1[5] = d.y; kw1[6] = d.z; kw1[7] = d.w;
  }
  uint32_t sc0[4], sc1[4];
  scales_bcast4(lds32(scales + r0 * 16 + 4 * qd), sc0);
  scales_bcast4(lds32(scales + r1 * 16 + 4 * qd), sc1);
  float sa[4] = {0.f, 0.f, 0.f, 0.f}, sb[4] = {0.f, 0.f, 0.f, 0.f};
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
    mma_16816(sa, h0[0], h1[0], h0[1], h1[1], qf[4 * w8 + 0], qf[4 * w8 + 1]);
    mma_16816(sb, h0[2], h1[2], h0[3], h1[3], qf[4 * w8 + 2], qf[4 * w8 + 3]);
  }
#pragma unroll
  for (int i = 0; i < 4; ++i) s[i] = sa[i] + sb[i];
}

// V^T fragments of one 16-token tile: tokens ra, ra+1, ra+8, ra+9 (ra = tile
// base + 2q), head-dim slice [32g, 32g+32).  Scales of rows at or past
// `valid_end` (absolute tokens from t_ra) are zeroed so stale bytes add 0.
struct VTile {
  uint32_t a[4], b[4], c[4], d[4];
  uint32_t sab0, sab1, scd0, scd1;
};

QWZ_DEVINL void v_tile_load(uint32_t codes, uint32_t scales, int ra, int g, bool tail, int t_ra,
                            int valid_end, VTile& v) {
  const uint4 va = lds128(codes + swz128(ra, g));
  const uint4 vb = lds128(codes + swz128(ra + 1, g));
  const uint4 vc = lds128(codes + swz128(ra + 8, g));
  const uint4 vd = lds128(codes + swz128(ra + 9, g));
  v.a[0] = va.x; v.a[1] = va.y; v.a[2] = va.z; v.a[3] = va.w;
  v.b[0] = vb.x; v.b[1] = vb.y; v.b[2] = vb.z; v.b[3] = vb.w;
  v.c[0] = vc.x; v.c[1] = vc.y; v.c[2] = vc.z; v.c[3] = vc.w;
  v.d[0] = vd.x; v.d[1] = vd.y; v.d[2] = vd.z; v.d[3] = vd.w;
  const uint32_t sp = scales + 2 * g;
  uint32_t sa16 = lds16(sp + ra * 16), sb16 = lds16(sp + (ra + 1) * 16);
  uint32_t sc16 = lds16(sp + (ra + 8) * 16), sd16 = lds16(sp + (ra + 9) * 16);
  if (tail) {
    if (t_ra >= valid_end) sa16 = 0;
    if (t_ra + 1 >= valid_end) sb16 = 0;
    if (t_ra + 8 >= valid_end) sc16 = 0;
    if (t_ra + 9 >= valid_end) sd16 = 0;
  }
  e4m3x4_to_f16x2x2(__byte_perm(sa16, sb16, 0x5140), v.sab0, v.sab1);
  e4m3x4_to_f16x2x2(__byte_perm(sc16, sd16, 0x5140), v.scd0, v.scd1);
}

// O^T[m-tiles 4*w4 .. 4*w4+3] += V^T P^T for one tile.
QWZ_DEVINL void pv_tile_word(const VTile& v, int w4, const PFrag& pf, float (&o)[16][4]) {
  const uint32_t xab = (v.a[w4] & 0x0F0F0F0Fu) | ((v.b[w4] << 4) & 0xF0F0F0F0u);
  const uint32_t yab = ((v.a[w4] >> 4) & 0x0F0F0F0Fu) | (v.b[w4] & 0xF0F0F0F0u);
  const uint32_t xcd = (v.c[w4] & 0x0F0F0F0Fu) | ((v.d[w4] << 4) & 0xF0F0F0F0u);
  const uint32_t ycd = ((v.c[w4] >> 4) & 0x0F0F0F0Fu) | (v.d[w4] & 0xF0F0F0F0u);
  uint32_t hxab[4], hyab[4], hxcd[4], hycd[4];
  e2m1x8_to_f16x2x4(xab, hxab);
  e2m1x8_to_f16x2x4(yab, hyab);
  e2m1x8_to_f16x2x4(xcd, hxcd);
  e2m1x8_to_f16x2x4(ycd, hycd);
  const uint32_t sab = w4 < 2 ? v.sab0 : v.sab1;
  const uint32_t scd = w4 < 2 ? v.scd0 : v.scd1;
#pragma unroll
  for (int kk = 0; kk < 4; ++kk) {
    const uint32_t a0 = hmul2_u32(hxab[kk], sab), a1 = hmul2_u32(hyab[kk], sab);
    const uint32_t a2 = hmul2_u32(hxcd[kk], scd), a3 = hmul2_u32(hycd[kk], scd);
    mma_16816(o[4 * w4 + kk], a0, a1, a2, a3, pf.hi0, pf.hi1);
  }
}

}  // namespace

namespace {

// Ring metadata in shared memory (after the stages).
struct DecMeta {
  int released[kDecStages];     // warps done with the slot's current page
  int page_end[kDecStages];     // valid token end of the slot's page
  int last_issued[kDecStages];  // CTA page index last issued into the slot
};

// Physical page of the CTA's k-th page (-1 when the id is bad).  pid[]
// holds the first min(table_width, kDecPidCache) entries of the table row.
QWZ_DEVINL int cta_page(const SplitParams& p, const int* pid, const StageRange& rg, int k) {
  const int t = p.tok_begin + (rg.st_lo + k) * kPage;
  const int lp = (t >> 8) - p.table_page_offset;
  if (lp < 0 || lp >= min(p.table_width, kDecPidCache)) return lookup_page(p, t, true);
  const int pp = pid[lp];
  if (pp < 0 || pp >= p.num_pages) {
    flag_error(kErrPageRange);
    return -1;
  }
  return pp;
}

// TMA of the CTA's k-th page into ring slot `slot` (one thread).
QWZ_DEVINL void issue_page(const SplitParams& p, const int* pid, DecMeta* meta, const StageRange& rg,
                           int k, int slot, uint32_t sbase, uint32_t bar_full, int kvh) {
  const int t0 = p.tok_begin + (rg.st_lo + k) * kPage;
  const int pp = cta_page(p, pid, rg, k);
  meta->page_end[slot] = pp >= 0 ? rg.tok_end : t0;  // released by the arrive below
  meta->last_issued[slot] = k;
  const uint32_t fb = bar_full + 8 * slot;
  if (pp < 0) {  // bad page id: no copy; consumers mask the whole page
    mbar_arrive(fb);
    return;
  }
  mbar_arrive_expect_tx(fb, kDecStageBytes);
  const uint32_t dst = sbase + slot * kDecStageBytes;
  const int y = pp * kPage;
  tma_load_2d(dst, &p.tm_kc, kvh * kCodeBytes, y, fb);
  tma_load_2d(dst + kDecCodeTile, &p.tm_vc, kvh * kCodeBytes, y, fb);
  tma_load_2d(dst + 2 * kDecCodeTile, &p.tm_ks, kvh * kScaleBytes, y, fb);
  tma_load_2d(dst + 2 * kDecCodeTile + kDecScaleTile, &p.tm_vs, kvh * kScaleBytes, y, fb);
}

// Fused append of the new row: warp kDecWarps-2 writes K, kDecWarps-1 V,
// for this CTA's KV head, then fences so the page's TMA read sees the bytes
// (the same page lookup and error reporting as nvfp4_append_kernel).
template <typename T>
QWZ_DEVINL void fused_append(const SplitParams& p, int pos, int kvh, int warp, int lane) {
  const int tensor = warp - (kDecWarps - 2);
  const int pp = lookup_page(p, pos, lane == 0 && tensor == 0);
  if (pp < 0) return;
  const size_t row = ((size_t)pp * kPage + (pos & (kPage - 1))) * kKvHeads + kvh;
  const T* src = reinterpret_cast<const T*>(tensor ? p.app_v : p.app_k) + (size_t)kvh * kHeadDim;
  uint8_t* codes = const_cast<uint8_t*>(tensor ? p.v_codes : p.k_codes) + row * kCodeBytes;
  uint8_t* scales = const_cast<uint8_t*>(tensor ? p.v_scales : p.k_scales) + row * kScaleBytes;
  quant::quantize_row_lane<T>(src, codes, scales, lane);
  __threadfence();
  fence_proxy_async_global();
}

}  // namespace

template <typename T>
__global__ void __launch_bounds__(kDecWarps * 32, 1)
    nvfp4_decode_kernel(const __grid_constant__ SplitParams p) {
  extern __shared__ __align__(1024) uint8_t smem[];
  // TMA boxes with the 128-byte swizzle need 1024-byte aligned destinations
  const uint32_t sraw = smem_u32(smem);
  const uint32_t sbase = (sraw + 1023u) & ~1023u;
  uint8_t* sgen = smem + (sbase - sraw);
  const uint32_t bar_full = sbase + kDecStages * kDecStageBytes;
  DecMeta* meta = reinterpret_cast<DecMeta*>(sgen + kDecStages * kDecStageBytes + 8 * kDecStages);
  int* pid = reinterpret_cast<int*>(sgen + kDecStages * kDecStageBytes + kDecMetaBytes);
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31, g = lane >> 2, qd = lane & 3;
  const int split = blockIdx.x, kvh = blockIdx.y;

  // shared-memory set-up overlaps the previous kernel; global reads wait
  if (tid == 0) {
#pragma unroll
    for (int s = 0; s < kDecStages; ++s) {
      mbar_init(bar_full + 8 * s, 1);
      meta->released[s] = 0;
      meta->last_issued[s] = -1;
    }
    mbar_fence_init();
    tma_prefetch_desc(&p.tm_kc);
    tma_prefetch_desc(&p.tm_vc);
    tma_prefetch_desc(&p.tm_ks);
    tma_prefetch_desc(&p.tm_vs);
  }
  griddep_wait();

  // the table row is loaded while the length is in flight
  constexpr int kRowPerThread = kDecPidCache / (kDecWarps * 32);
  const int n_cached = min(p.table_width, kDecPidCache);
  int row[kRowPerThread];
#pragma unroll
  for (int r = 0; r < kRowPerThread; ++r) {
    const int i = tid + r * kDecWarps * 32;
    row[r] = i < n_cached ? __ldg(p.block_table + i) : -1;
  }
  const StageRange rg = stage_range<kPage>(p, split);
#pragma unroll
  for (int r = 0; r < kRowPerThread; ++r) {
    const int i = tid + r * kDecWarps * 32;
    if (i < n_cached) pid[i] = row[r];
  }
  // fused append: the new row's page is this CTA's page k_app (its last)
  int k_app = -1, app_pos = 0;
  if (p.app_k != nullptr) {
    app_pos = __ldg(p.seqlens);
    const int st = (app_pos - p.tok_begin) >> 8;
    if (app_pos >= p.tok_begin && st >= rg.st_lo && st < rg.st_lo + rg.n_st) k_app = st - rg.st_lo;
  }
  const bool app_warp = k_app >= 0 && warp >= kDecWarps - 2;
  if (app_warp && k_app < kDecStages) fused_append<T>(p, app_pos, kvh, warp, lane);  // before the first issue
  __syncthreads();
  if (tid == 0 && rg.n_st > 0) {
    for (int k = 0; k < min(rg.n_st, kDecStages); ++k)
      issue_page(p, pid, meta, rg, k, k, sbase, bar_full, kvh);
  }
  // A later page is issued by the last releaser of an iteration these two
  // warps reach only after writing (release: __threadfence_block + atomic).
  if (app_warp && k_app >= kDecStages) fused_append<T>(p, app_pos, kvh, warp, lane);

  float o[16][4];
#pragma unroll
  for (int j = 0; j < 16; ++j) o[j][0] = o[j][1] = o[j][2] = o[j][3] = 0.f;
  float m0 = -CUDART_INF_F, m1 = -CUDART_INF_F, l0 = 0.f, l1 = 0.f;
  uint32_t qf[32];
  float cf0 = 0.f, cf1 = 0.f;
  load_q_decode<T>(reinterpret_cast<const T*>(p.q), g < kGroup ? kvh * kGroup + g : -1, qd,
                   p.sm_scale_log2, qf, cf0, cf1);

  int slot = 0;
  uint32_t phase = 0;
  const int rA = 32 * warp + g;          // tile A rows rA, rA+8; tile B rows rA+16, rA+24
  const int vA = 32 * warp + 2 * qd;     // tile A V rows vA, +1, +8, +9; tile B +16
  for (int k = 0; k < rg.n_st; ++k) {
    if (!mbar_wait(bar_full + 8 * slot, phase)) {
      flag_error(kErrTimeout);
      break;
    }
    const uint32_t st = sbase + slot * kDecStageBytes;
    const int t0 = p.tok_begin + (rg.st_lo + k) * kPage;
    const int valid_end = meta->page_end[slot];
    const int tw = t0 + 32 * warp;
    const bool tail = tw + 32 > valid_end;

    // ---------------- S^T for both tiles
    float sA[4], sB[4];
    qk_tile(st, st + 2 * kDecCodeTile, rA, qd, qf, sA);
    qk_tile(st, st + 2 * kDecCodeTile, rA + 16, qd, qf, sB);
    float t[8] = {sA[0] * cf0, sA[1] * cf1, sA[2] * cf0, sA[3] * cf1,
                  sB[0] * cf0, sB[1] * cf1, sB[2] * cf0, sB[3] * cf1};
    if (tail) {
      if (tw + g >= valid_end) t[0] = t[1] = -CUDART_INF_F;
      if (tw + g + 8 >= valid_end) t[2] = t[3] = -CUDART_INF_F;
      if (tw + g + 16 >= valid_end) t[4] = t[5] = -CUDART_INF_F;
      if (tw + g + 24 >= valid_end) t[6] = t[7] = -CUDART_INF_F;
    }

    // V fragments first: their shared-memory latency hides behind the softmax
    const uint32_t vcodes = st + kDecCodeTile;
    const uint32_t vscales = st + 2 * kDecCodeTile + kDecScaleTile;
    VTile va, vb;
    v_tile_load(vcodes, vscales, vA, g, tail, t0 + vA, valid_end, va);
    v_tile_load(vcodes, vscales, vA + 16, g, tail, t0 + vA + 16, valid_end, vb);

    // ---------------- one online-softmax update for the 32 tokens
    float mx0 = fmaxf(fmaxf(t[0], t[2]), fmaxf(t[4], t[6]));
    float mx1 = fmaxf(fmaxf(t[1], t[3]), fmaxf(t[5], t[7]));
#pragma unroll
    for (int off = 4; off < 32; off <<= 1) {
      mx0 = fmaxf(mx0, shfl_xor(mx0, off));
      mx1 = fmaxf(mx1, shfl_xor(mx1, off));
    }
    if (__any_sync(0xffffffffu, (mx0 > m0 + kLazy) || (mx1 > m1 + kLazy))) {
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
#pragma unroll
    for (int i = 0; i < 8; i += 2) {
      t[i] = exp2_approx(t[i] - mu0);
      t[i + 1] = exp2_approx(t[i + 1] - mu1);
    }
    l0 += (t[0] + t[2]) + (t[4] + t[6]);
    l1 += (t[1] + t[3]) + (t[5] + t[7]);
    const PFrag pA = p_fragments(t[0], t[1], t[2], t[3]);
    const PFrag pB = p_fragments(t[4], t[5], t[6], t[7]);

    // ---------------- O^T += V^T P^T for both tiles
#pragma unroll
    for (int w4 = 0; w4 < 4; ++w4) {
      pv_tile_word(va, w4, pA, o);
      pv_tile_word(vb, w4, pB, o);
    }

    // release the slot; the last warp out issues the page three ahead into it
    __syncwarp();
    if (lane == 0) {
      __threadfence_block();
      if (atomicAdd(&meta->released[slot], 1) == kDecWarps - 1) {
        meta->released[slot] = 0;
        if (k + kDecStages < rg.n_st) {
          fence_proxy_async_smem();
          issue_page(p, pid, meta, rg, k + kDecStages, slot, sbase, bar_full, kvh);
        }
      }
    }
    if (++slot == kDecStages) {
      slot = 0;
      phase ^= 1u;
    }
  }

  __syncthreads();
  if (tid == 0) {  // never leave with copies in flight (only reachable after a timeout)
#pragma unroll
    for (int s = 0; s < kDecStages; ++s) {
      const int k = meta->last_issued[s];
      if (k >= 0 && !mbar_wait(bar_full + 8 * s, (k / kDecStages) & 1)) flag_error(kErrTimeout);
    }
  }
  __syncthreads();
  griddep_launch_dependents();
  decode_epilogue<kDecWarps>(p, smem, split, kvh, m0, m1, l0, l1, o, [](int d, int& gg, int& j) {
    gg = d >> 5;
    j = (d & 31) >> 1;
  });
}

template <typename T>
cudaError_t launch_nvfp4_decode(const SplitParams& p, cudaStream_t stream) {
  static_assert(epilogue_smem_bytes(kDecWarps) <= kDecStages * kDecStageBytes, "epilogue reuses the ring");
  auto kernel = nvfp4_decode_kernel<T>;
  cudaError_t e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, kDecSmemBytes);
  if (e != cudaSuccess) return e;
  return launch_pdl(kernel, dim3(p.num_splits, kKvHeads), dim3(kDecWarps * 32), kDecSmemBytes, stream, p);
}

}  // namespace qwz
