// Graph patching of captured split and combine launches.
//
// The reference's decode graphs patch split arguments 3, 4, 11, 12 and 13
// (block_table, cache_seqlens, split_len, num_pages_per_seq, num_splits)
// and combine argument 4 (num_splits) between replays
// (docs/superpowers/specs/2026-09-11-qwasar-attention-kernel.md:66-74,
// asserted by tests/test_attention_kernel_abi.py:25-31).  A split or combine
// launch of this library is one kernel node whose single parameter is a
// packed struct (SplitParams / CombineParams); these entry points find such
// nodes in a captured graph and rewrite the same arguments inside that
// struct, in the graph and, when given, in its instantiated executable, so
// the next replay runs with them.  The grid of a split node follows
// num_splits (num_splits x 4 KV heads).

#include "qwz_common.cuh"
#include "qwz_kernels.h"
#include "../../include/qwz_b200.h"

#include <vector>

namespace {

bool is_split_kernel(const void* f) {
  using namespace qwz;
  const void* known[] = {
      reinterpret_cast<const void*>(nvfp4_decode_kernel<__half>),
      reinterpret_cast<const void*>(nvfp4_decode_kernel<__nv_bfloat16>),
      reinterpret_cast<const void*>(verify_tc_kernel<__half, 16, VtNvfp4>),
      reinterpret_cast<const void*>(verify_tc_kernel<__half, 32, VtNvfp4>),
      reinterpret_cast<const void*>(verify_tc_kernel<__half, 48, VtNvfp4>),
      reinterpret_cast<const void*>(verify_tc_kernel<__nv_bfloat16, 16, VtNvfp4>),
      reinterpret_cast<const void*>(verify_tc_kernel<__nv_bfloat16, 32, VtNvfp4>),
      reinterpret_cast<const void*>(verify_tc_kernel<__nv_bfloat16, 48, VtNvfp4>),
      reinterpret_cast<const void*>(verify_tc_kernel<__half, 16, VtK8v4>),
      reinterpret_cast<const void*>(verify_tc_kernel<__half, 32, VtK8v4>),
      reinterpret_cast<const void*>(verify_tc_kernel<__half, 48, VtK8v4>),
      reinterpret_cast<const void*>(verify_tc_kernel<__nv_bfloat16, 16, VtK8v4>),
      reinterpret_cast<const void*>(verify_tc_kernel<__nv_bfloat16, 32, VtK8v4>),
      reinterpret_cast<const void*>(verify_tc_kernel<__nv_bfloat16, 48, VtK8v4>),
  };
  for (const void* k : known)
    if (k == f) return true;
  return false;
}

bool is_combine_kernel(const void* f) {
  using namespace qwz;
  const void* known[] = {
      reinterpret_cast<const void*>(lse_combine_kernel<__half, kCombineFinal>),
      reinterpret_cast<const void*>(lse_combine_kernel<__nv_bfloat16, kCombineFinal>),
      reinterpret_cast<const void*>(lse_combine_kernel<float, kCombinePartial>),
      reinterpret_cast<const void*>(lse_combine_kernel<__half, kCombineRotate>),
      reinterpret_cast<const void*>(lse_combine_kernel<__nv_bfloat16, kCombineRotate>),
  };
  for (const void* k : known)
    if (k == f) return true;
  return false;
}

// The node's launch parameters when it is one of this library's kernel
// nodes of the given kind.
int node_params(cudaGraphNode_t node, int32_t kind, cudaKernelNodeParams* kp, const char* what) {
  cudaGraphNodeType type;
  cudaError_t e = cudaGraphNodeGetType(node, &type);
  if (e != cudaSuccess) return launched(e, what);
  if (type != cudaGraphNodeTypeKernel) return fail(QWZ_EINVAL, "%s: not a kernel node", what);
  e = cudaGraphKernelNodeGetParams(node, kp);
  if (e != cudaSuccess) return launched(e, what);
  const bool ok = kind == QWZ_NODE_SPLIT ? is_split_kernel(kp->func) : is_combine_kernel(kp->func);
  if (!ok) return fail(QWZ_EINVAL, "%s: the node is not a launch of this library's kernel of that kind", what);
  if (kp->kernelParams == nullptr || kp->kernelParams[0] == nullptr)
    return fail(QWZ_EINVAL, "%s: the node carries no parameter array", what);
  return QWZ_OK;
}

int apply(cudaGraphNode_t node, cudaGraphExec_t exec, cudaKernelNodeParams& np, const char* what) {
  cudaError_t e = cudaGraphKernelNodeSetParams(node, &np);
  if (e == cudaSuccess && exec != nullptr) e = cudaGraphExecKernelNodeSetParams(exec, node, &np);
  return launched(e, what);
}

}  // namespace

extern "C" {

int qwz_graph_kernel_nodes(void* graph, int32_t kind, void** nodes, int32_t max_nodes, int32_t* count) {
  if (!graph || !count) return fail(QWZ_EINVAL, "qwz_graph_kernel_nodes: graph and count are required");
  if (kind != QWZ_NODE_SPLIT && kind != QWZ_NODE_COMBINE)
    return fail(QWZ_EINVAL, "qwz_graph_kernel_nodes: kind must be QWZ_NODE_SPLIT or QWZ_NODE_COMBINE");
  if (max_nodes < 0 || (max_nodes > 0 && !nodes))
    return fail(QWZ_EINVAL, "qwz_graph_kernel_nodes: nodes is required when max_nodes > 0");
  cudaGraph_t g = static_cast<cudaGraph_t>(graph);
  size_t n = 0;
  cudaError_t e = cudaGraphGetNodes(g, nullptr, &n);
  if (e != cudaSuccess) return launched(e, "qwz_graph_kernel_nodes");
  std::vector<cudaGraphNode_t> all(n);
  if (n) e = cudaGraphGetNodes(g, all.data(), &n);
  if (e != cudaSuccess) return launched(e, "qwz_graph_kernel_nodes");
  int32_t found = 0;
  for (cudaGraphNode_t node : all) {
    cudaGraphNodeType type;
    if (cudaGraphNodeGetType(node, &type) != cudaSuccess || type != cudaGraphNodeTypeKernel) continue;
    cudaKernelNodeParams kp{};
    if (cudaGraphKernelNodeGetParams(node, &kp) != cudaSuccess) continue;
    const bool ok = kind == QWZ_NODE_SPLIT ? is_split_kernel(kp.func) : is_combine_kernel(kp.func);
    if (!ok) continue;
    if (found < max_nodes) nodes[found] = node;
    ++found;
  }
  *count = found;
  return QWZ_OK;
}

int qwz_graph_patch_split(void* graph, void* graph_exec, void* node, const int32_t* block_table,
                          const int32_t* cache_seqlens, int32_t split_len, int32_t num_pages_per_seq,
                          int32_t num_splits) {
  (void)graph;
  const char* what = "qwz_graph_patch_split";
  if (!node) return fail(QWZ_EINVAL, "%s: node is required", what);
  if (!block_table || !cache_seqlens) return fail(QWZ_EINVAL, "%s: block_table and cache_seqlens are required", what);
  if (num_pages_per_seq <= 0) return fail(QWZ_EINVAL, "%s: num_pages_per_seq must be positive", what);
  if (num_splits < 1 || num_splits > 65535) return fail(QWZ_EINVAL, "%s: num_splits must be in 1..65535", what);
  if (split_len < 0 || split_len % qwz::kPage != 0)
    return fail(QWZ_EINVAL, "%s: split_len must be 0 or a positive multiple of 256", what);
  cudaGraphNode_t n = static_cast<cudaGraphNode_t>(node);
  cudaKernelNodeParams kp{};
  int rc = node_params(n, QWZ_NODE_SPLIT, &kp, what);
  if (rc) return rc;
  qwz::SplitParams p = *static_cast<const qwz::SplitParams*>(kp.kernelParams[0]);
  p.block_table = block_table;
  p.seqlens = cache_seqlens;
  p.split_len = split_len;
  p.table_width = num_pages_per_seq;
  p.num_splits = num_splits;
  void* args[1] = {&p};
  cudaKernelNodeParams np = kp;
  np.kernelParams = args;
  np.extra = nullptr;
  np.gridDim = dim3(num_splits, qwz::kKvHeads, 1);
  return apply(n, static_cast<cudaGraphExec_t>(graph_exec), np, what);
}

int qwz_graph_patch_combine(void* graph, void* graph_exec, void* node, int32_t num_splits) {
  (void)graph;
  const char* what = "qwz_graph_patch_combine";
  if (!node) return fail(QWZ_EINVAL, "%s: node is required", what);
  if (num_splits < 1 || num_splits > 65535) return fail(QWZ_EINVAL, "%s: num_splits must be in 1..65535", what);
  cudaGraphNode_t n = static_cast<cudaGraphNode_t>(node);
  cudaKernelNodeParams kp{};
  int rc = node_params(n, QWZ_NODE_COMBINE, &kp, what);
  if (rc) return rc;
  qwz::CombineParams c = *static_cast<const qwz::CombineParams*>(kp.kernelParams[0]);
  if (c.o_split != qwz::kHeadDim || c.ml_split != 2)
    return fail(QWZ_EINVAL, "%s: the node combines records of another layout (the sharded merge)", what);
  c.num_splits = num_splits;
  c.o_row = (long long)num_splits * qwz::kHeadDim;
  c.ml_row = (long long)num_splits * 2;
  void* args[1] = {&c};
  cudaKernelNodeParams np = kp;
  np.kernelParams = args;
  np.extra = nullptr;
  return apply(n, static_cast<cudaGraphExec_t>(graph_exec), np, what);
}

}  // extern "C"
