// qwz_nvfp4_attend_noalloc: the decode/verify route of qwz_nvfp4_attend for
// callers that cannot allocate device memory.
//
// Some hosts embed this library where no device allocator is reachable: a
// plugin loaded into an engine that owns every device allocation, a process
// whose memory pool is fixed at start-up, or code that only receives raw
// pointers through an FFI.  They can still hand over their inputs and
// outputs, but not the split-K workspace (partial_o / partial_ml).  This
// entry point keeps that workspace in a file-scope device array instead:
//   - the array is kNoAllocMaxRecords (query row x split) records of
//     (256 + 2) floats, 4 MiB + 32 KiB, and every GPU that loads the library
//     holds it until the process exits;
//   - requests with q_len * 24 * num_splits > kNoAllocMaxRecords are refused
//     with QWZ_EINVAL before anything is launched;
//   - host code cannot pass the array's name to a kernel (on the host it is a
//     stand-in, not a device address): the first call on each device resolves
//     the device address with cudaGetSymbolAddress, with that device current,
//     and caches it with the device's context, so that first call should be
//     made before any stream capture (after a cudaDeviceReset the next call
//     resolves it again, and that call too belongs outside a capture);
//   - all calls share the array and it keeps the last call's contents; the
//     split kernel rewrites every record it owns (empty splits write
//     m = -inf), so nothing needs clearing, but calls that overlap on the GPU
//     (issued on concurrent streams, or from several host threads without
//     ordering) race on it and must be serialised by the caller.
// Nothing here calls cudaMalloc, cudaFree or an allocating library routine.

#include "qwz_common.cuh"
#include "qwz_kernels.h"
#include "../../include/qwz_b200.h"

#include <mutex>

namespace qwz {

constexpr int kNoAllocMaxRecords = 4096;

static __device__ __align__(256) float g_noalloc_scratch[kNoAllocMaxRecords * (kHeadDim + 2)];

namespace {

constexpr int kMaxDevices = 64;

// The CUDA context current on this thread (through the runtime's driver
// entry point; the library links only the static runtime), or nullptr.
CUcontext current_context() {
  using Fn = CUresult (*)(CUcontext*);
  static Fn fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* f = nullptr;
    cudaDriverEntryPointQueryResult q{};
    if (cudaGetDriverEntryPoint("cuCtxGetCurrent", &f, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<Fn>(f);
  });
  CUcontext ctx = nullptr;
  if (fn == nullptr || fn(&ctx) != CUDA_SUCCESS) return nullptr;
  return ctx;
}

// Device address of g_noalloc_scratch on the current device, or nullptr
// with *err set.  Resolved once per device and context: the first call on a
// device looks it up with that device current, and a later call does so
// again only if the device's context has changed since (after
// cudaDeviceReset the module is loaded anew and the array may move).
float* noalloc_scratch(cudaError_t* err) {
  static std::mutex mu;
  static float* addr[kMaxDevices] = {};
  static CUcontext owner[kMaxDevices] = {};
  int dev = -1;
  *err = cudaGetDevice(&dev);
  if (*err != cudaSuccess) return nullptr;
  if (dev < 0 || dev >= kMaxDevices) {
    *err = cudaErrorInvalidDevice;
    return nullptr;
  }
  std::lock_guard<std::mutex> lock(mu);
  const CUcontext ctx = current_context();
  if (addr[dev] == nullptr || ctx != owner[dev]) {
    void* p = nullptr;
    *err = cudaGetSymbolAddress(&p, g_noalloc_scratch);
    if (*err != cudaSuccess) return nullptr;
    addr[dev] = static_cast<float*>(p);
    // the symbol lookup makes the runtime's context current if none was
    owner[dev] = ctx != nullptr ? ctx : current_context();
  }
  return addr[dev];
}

}  // namespace
}  // namespace qwz

extern "C" int qwz_nvfp4_attend_noalloc(const void* q, const void* k, const void* v,
                                        void* k_cache, void* v_cache, void* k_scales,
                                        void* v_scales, const int32_t* block_table,
                                        const int32_t* cache_seqlens, void* out,
                                        int32_t table_width, int32_t num_pages, int32_t q_len,
                                        int32_t num_splits, float sm_scale, int32_t dtype,
                                        void* stream) {
  if (q_len < 1 || q_len > 8) return fail(QWZ_EINVAL, "q_len must be in 1..8");
  if (num_splits < 1) return fail(QWZ_EINVAL, "num_splits must be positive");
  const long long records = (long long)q_len * qwz::kQHeads * num_splits;
  if (records > qwz::kNoAllocMaxRecords)
    return fail(QWZ_EINVAL,
                "qwz_nvfp4_attend_noalloc: q_len * 24 * num_splits exceeds the static workspace "
                "(4096 records); lower num_splits or use qwz_nvfp4_attend with your own workspace");
  cudaError_t err = cudaSuccess;
  float* base = qwz::noalloc_scratch(&err);
  if (base == nullptr) return launched(err, "qwz_nvfp4_attend_noalloc (workspace address)");
  float* partial_o = base;
  float* partial_ml = base + (size_t)qwz::kNoAllocMaxRecords * qwz::kHeadDim;
  return qwz_nvfp4_attend(q, k, v, k_cache, v_cache, k_scales, v_scales, block_table,
                          cache_seqlens, out, partial_o, partial_ml, table_width, num_pages, q_len,
                          num_splits, sm_scale, dtype, stream);
}
