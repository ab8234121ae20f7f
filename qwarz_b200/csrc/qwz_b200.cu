// Single translation unit of libqwz_b200.so: the kernels share one device
// error word (qwz::g_qwz_device_error) without relocatable device code.
#include "attn_decode.cu"
#include "attn_verify_tc.cu"
#include "attn_prefill.cu"
#include "attn_split.cu"
#include "attn_draft.cu"
#include "attn_combine.cu"
#include "shard_exchange.cu"
#include "kv_write.cu"
#include "capi.cu"
#include "noalloc.cu"
#include "graph_patch.cu"
