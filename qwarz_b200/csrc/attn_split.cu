// Split-K paged attention over the NVFP4 one-level KV cache, for sm_100a:
// the dispatcher behind the reference's split/combine ABI
// (tests/test_attention_kernel_abi.py:13-55), which replaces the FlashInfer
// XQA launch of src/qwasar_runtime/xqa.py:484-554 (q_len <= 8 over NVFP4
// pages).
//
//   q_len 1     nvfp4_decode_kernel (attn_decode.cu): page-streamed by TMA,
//               dequantised in registers into mma.sync fragments (tokens on
//               M, the 6 GQA heads on N);
//   q_len 2..8  verify_tc_kernel<VtNvfp4> (attn_verify_tc.cu): 128-token
//               tiles by TMA, K dequantised into tensor memory and V into
//               shared memory, QK and PV on tcgen05 with accumulators in
//               tensor memory.
//
// Both write partials (m, l, O) with O unnormalised and m in log2 units of
// sm_scale * q.k, merged by lse_combine_kernel (attn_combine.cu); the online
// softmax is base-2 with lazy rescaling (the reference maximum of a column
// only moves when a tile exceeds it by more than 2^8).

#include "attn_common.cuh"

namespace qwz {

cudaError_t launch_nvfp4_split(const SplitParams& p, int dtype, cudaStream_t stream) {
  if (p.q_len == 1) {
    return dtype == kDtypeBF16 ? launch_nvfp4_decode<__nv_bfloat16>(p, stream)
                               : launch_nvfp4_decode<__half>(p, stream);
  }
  return dtype == kDtypeBF16 ? launch_verify_tc<__nv_bfloat16>(p, stream)
                             : launch_verify_tc<__half>(p, stream);
}

}  // namespace qwz
