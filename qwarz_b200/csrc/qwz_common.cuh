// Device helpers shared by the NVFP4 / FP8 paged-attention kernels (sm_100a).
//
// Geometry is the one the reference attention boundary pins
// (src/qwasar_runtime/xqa.py:307-354 `_validate_nvfp4`): 24 query heads,
// 4 KV heads (GQA group 6), head_dim 256, 256-token pages.  Cache layout
// (engine/forward/attention.py:159-167 `empty_cache`): codes uint8
// [P, 256, 4, 128] with even d in the low nibble (xqa.py:103-109), scales
// E4M3 [P, 256, 4, 16], one per 16 head-dim elements (xqa.py:137-141).
#pragma once

#include <cuda_runtime.h>
#include <cuda_fp16.h>
#include <cuda_bf16.h>
#include <stdint.h>

#define QWZ_DEVINL __device__ __forceinline__

namespace qwz {

constexpr int kHeadDim = 256;
constexpr int kKvHeads = 4;
constexpr int kGroup = 6;
constexpr int kQHeads = kKvHeads * kGroup;
constexpr int kPage = 256;
constexpr int kCodeBytes = kHeadDim / 2;    // E2M1 codes per (token, head)
constexpr int kScaleBytes = kHeadDim / 16;  // E4M3 scales per (token, head)
constexpr int kRowBytesCodes = kKvHeads * kCodeBytes;   // 512 B per token
constexpr int kRowBytesScales = kKvHeads * kScaleBytes; // 64 B per token

// Bits OR-ed into the device error word by kernels that meet bad metadata.
enum DeviceError : int {
  kErrTableRange = 1,  // logical page beyond the block-table width
  kErrPageRange = 2,   // physical page id outside the cache pool
  kErrSlotRange = 4,   // FP8 draft slot beyond the store capacity
  kErrTimeout = 8,     // a bounded mbarrier wait gave up
};

// Device-wide error word.  The library is one translation unit
// (qwz_b200.cu), so the definition lives in this header.
__device__ int g_qwz_device_error = 0;

QWZ_DEVINL void flag_error(int bits) { atomicOr(&g_qwz_device_error, bits); }

// ---------------------------------------------------------------- converts
// Four packed E2M1 pairs (one 32-bit word, byte i holds two codes, low nibble
// first) -> four f16x2 (low nibble -> low half).  Hardware cvt, exact.
QWZ_DEVINL void e2m1x8_to_f16x2x4(uint32_t w, uint32_t (&h)[4]) {
  asm("{\n"
      " .reg .b8 b0, b1, b2, b3;\n"
      " mov.b32 {b0, b1, b2, b3}, %4;\n"
      " cvt.rn.f16x2.e2m1x2 %0, b0;\n"
      " cvt.rn.f16x2.e2m1x2 %1, b1;\n"
      " cvt.rn.f16x2.e2m1x2 %2, b2;\n"
      " cvt.rn.f16x2.e2m1x2 %3, b3;\n"
      "}\n"
      : "=r"(h[0]), "=r"(h[1]), "=r"(h[2]), "=r"(h[3])
      : "r"(w));
}

// Two packed E4M3 pairs -> two f16x2 (bytes 0,1 -> h0; bytes 2,3 -> h1).
// Every E4M3 value is exactly representable in FP16.
QWZ_DEVINL void e4m3x4_to_f16x2x2(uint32_t w, uint32_t& h0, uint32_t& h1) {
  asm("{\n"
      " .reg .b16 lo, hi;\n"
      " mov.b32 {lo, hi}, %2;\n"
      " cvt.rn.f16x2.e4m3x2 %0, lo;\n"
      " cvt.rn.f16x2.e4m3x2 %1, hi;\n"
      "}\n"
      : "=r"(h0), "=r"(h1)
      : "r"(w));
}

QWZ_DEVINL uint32_t hmul2_u32(uint32_t a, uint32_t b) {
  uint32_t d;
  asm("mul.rn.f16x2 %0, %1, %2;\n" : "=r"(d) : "r"(a), "r"(b));
  return d;
}

QWZ_DEVINL uint32_t pack_half2(float lo, float hi) {
  uint32_t d;
  asm("cvt.rn.f16x2.f32 %0, %2, %1;\n" : "=r"(d) : "f"(lo), "f"(hi));
  return d;
}

QWZ_DEVINL float exp2_approx(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;\n" : "=f"(y) : "f"(x));
  return y;
}

// ------------------------------------------------------------ tensor cores
// D += A(16x16, row) * B(16x8, col); f16 inputs, f32 accumulate.
QWZ_DEVINL void mma_16816(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2,
                          uint32_t a3, uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 "
      "{%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};\n"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

// Warp-wide transpose of one 8x8 b16 fragment.
QWZ_DEVINL uint32_t movmatrix_trans(uint32_t x) {
  uint32_t y;
  asm volatile("movmatrix.sync.aligned.m8n8.trans.b16 %0, %1;\n" : "=r"(y) : "r"(x));
  return y;
}

QWZ_DEVINL void ldmatrix_x4(uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3,
                            uint32_t addr) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];\n"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}

QWZ_DEVINL void ldmatrix_x2(uint32_t& r0, uint32_t& r1, uint32_t addr) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x2.shared.b16 {%0,%1}, [%2];\n"
               : "=r"(r0), "=r"(r1)
               : "r"(addr));
}

// ----------------------------------------------------------- shared memory
QWZ_DEVINL uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

QWZ_DEVINL uint4 lds128(uint32_t addr) {
  uint4 v;
  asm volatile("ld.shared.v4.u32 {%0,%1,%2,%3}, [%4];\n"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
               : "r"(addr));
  return v;
}
QWZ_DEVINL uint32_t lds32(uint32_t addr) {
  uint32_t v;
  asm volatile("ld.shared.u32 %0, [%1];\n" : "=r"(v) : "r"(addr));
  return v;
}
QWZ_DEVINL uint32_t lds16(uint32_t addr) {
  unsigned short v;
  asm volatile("ld.shared.u16 %0, [%1];\n" : "=h"(v) : "r"(addr));
  return v;
}
QWZ_DEVINL uint32_t lds8(uint32_t addr) {
  unsigned short v;
  asm volatile("ld.shared.u8 %0, [%1];\n" : "=h"(v) : "r"(addr));
  return v;
}
QWZ_DEVINL void sts128(uint32_t addr, uint32_t a, uint32_t b, uint32_t c, uint32_t d) {
  asm volatile("st.shared.v4.u32 [%0], {%1,%2,%3,%4};\n" ::"r"(addr), "r"(a), "r"(b), "r"(c), "r"(d));
}
QWZ_DEVINL void sts32(uint32_t addr, uint32_t v) {
  asm volatile("st.shared.u32 [%0], %1;\n" ::"r"(addr), "r"(v));
}

// 16-byte async global->shared copy; src_bytes == 0 zero-fills without a read.
QWZ_DEVINL void cp_async16(uint32_t dst, const void* src, uint32_t src_bytes) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;\n" ::"r"(dst), "l"(src),
               "r"(src_bytes));
}
QWZ_DEVINL void cp_async_commit() { asm volatile("cp.async.commit_group;\n"); }
template <int N>
QWZ_DEVINL void cp_async_wait() {
  asm volatile("cp.async.wait_group %0;\n" ::"n"(N));
}

// ------------------------------------------------------- mbarrier and TMA
// Spin budget of a bounded mbarrier wait: iterations of try_wait, each of
// which suspends for at most kWaitHintNs.  ~1 s in total; on expiry the
// waiter sets kErrTimeout and gives up instead of hanging the GPU.
constexpr int kWaitSpins = 1 << 17;
constexpr uint32_t kWaitHintNs = 8000;

QWZ_DEVINL void mbar_init(uint32_t bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;\n" ::"r"(bar), "r"(count) : "memory");
}
QWZ_DEVINL void mbar_fence_init() {
  asm volatile("fence.mbarrier_init.release.cluster;\n" ::: "memory");
}
QWZ_DEVINL void mbar_arrive(uint32_t bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];\n" ::"r"(bar) : "memory");
}
QWZ_DEVINL void mbar_arrive_expect_tx(uint32_t bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;\n" ::"r"(bar), "r"(bytes)
               : "memory");
}
// Waits for the phase with the given parity; false (and kErrTimeout) if the
// spin budget runs out.
QWZ_DEVINL bool mbar_wait(uint32_t bar, uint32_t parity) {
  for (int i = 0; i < kWaitSpins; ++i) {
    uint32_t done;
    asm volatile(
        "{\n .reg .pred p;\n"
        " mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n"
        " selp.u32 %0, 1, 0, p;\n}\n"
        : "=r"(done)
        : "r"(bar), "r"(parity), "r"(kWaitHintNs)
        : "memory");
    if (done) return true;
  }
  return false;
}

// 2-D tiled TMA load of one box into shared memory, completing on `bar`.
QWZ_DEVINL void tma_load_2d(uint32_t dst, const void* tmap, int x, int y, uint32_t bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%2, %3}], [%4];\n" ::"r"(dst),
      "l"(reinterpret_cast<uint64_t>(tmap)), "r"(x), "r"(y), "r"(bar)
      : "memory");
}
// Orders this thread's earlier shared-memory accesses (generic proxy) before
// its later TMA writes into the same bytes (async proxy).
QWZ_DEVINL void fence_proxy_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;\n" ::: "memory");
}
// Orders this thread's generic-proxy global writes before later async-proxy
// (TMA) reads of the same bytes.
QWZ_DEVINL void fence_proxy_async_global() {
  asm volatile("fence.proxy.async.global;\n" ::: "memory");
}
QWZ_DEVINL void tma_prefetch_desc(const void* tmap) {
  asm volatile("prefetch.tensormap [%0];\n" ::"l"(reinterpret_cast<uint64_t>(tmap)) : "memory");
}

// ------------------------------------------- programmatic dependent launch
// A kernel launched with the programmatic-stream-serialization attribute may
// start while its predecessor in the stream is still running: it must not
// read memory the predecessor writes (or write memory it reads) before
// griddep_wait(), which returns once the predecessor grid has completed and
// its writes are visible.  Without the attribute both are no-ops.
// griddep_launch_dependents() lets the next kernel in the stream begin its
// launch (its own griddep_wait() still waits for this grid to finish).
QWZ_DEVINL void griddep_wait() { asm volatile("griddepcontrol.wait;\n" ::: "memory"); }
QWZ_DEVINL void griddep_launch_dependents() { asm volatile("griddepcontrol.launch_dependents;\n" ::: "memory"); }

// Host: launch with programmatic stream serialisation (the kernel calls
// griddep_wait() before touching memory its predecessor may write).
template <typename... KArgs, typename... Args>
inline cudaError_t launch_pdl(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem,
                              cudaStream_t stream, Args... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, kernel, args...);
}

// 128-byte-row XOR swizzle of 16-byte chunks (rows of 128 B, chunk 0..7);
// the layout a TMA tiled load with CU_TENSOR_MAP_SWIZZLE_128B produces in a
// 1024-byte aligned destination.
QWZ_DEVINL uint32_t swz128(int row, int chunk) {
  return static_cast<uint32_t>(row * 128 + ((chunk ^ (row & 7)) << 4));
}

// ------------------------------------------------------------ input dtypes
template <typename T>
struct InTraits;
template <>
struct InTraits<__half> {
  static QWZ_DEVINL float2 to_float2(uint32_t w) {
    __half2 h = *reinterpret_cast<__half2*>(&w);
    return __half22float2(h);
  }
  static QWZ_DEVINL __half from_float(float x) { return __float2half_rn(x); }
};
template <>
struct InTraits<__nv_bfloat16> {
  static QWZ_DEVINL float2 to_float2(uint32_t w) {
    __nv_bfloat162 h = *reinterpret_cast<__nv_bfloat162*>(&w);
    return __bfloat1622float2(h);
  }
  static QWZ_DEVINL __nv_bfloat16 from_float(float x) { return __float2bfloat16_rn(x); }
};

}  // namespace qwz
