// nvllm_paged_attention_static: paged attention for callers that cannot
// allocate device memory.
//
// nvllm_paged_attention needs a device workspace from its caller. Some callers
// cannot provide one: a host that reaches the GPU only through this C ABI and
// has no device allocator of its own, or a serving loop whose device memory is
// owned by a pool that forbids further cudaMalloc / cudaFree (both synchronize
// the whole device, which would stall the other streams in the middle of a
// step). For them this entry point runs the same kernels on a workspace that
// the library itself owns: a file-scope __device__ array of
// kStaticWorkspaceBytes. Every GPU that loads the library holds one copy of it
// until the process exits.
#include <cstddef>

#include <cuda_runtime.h>

#include "../../include/nvllm.h"

namespace {

// Largest workspace a batch may need here (nvllm_paged_attention_workspace_size).
constexpr size_t kStaticWorkspaceBytes = size_t(64) << 20;  // 64 MiB

static __device__ __align__(256) unsigned char g_static_workspace[kStaticWorkspaceBytes];

// Host code must not use g_static_workspace's name as a pointer: on the host it
// is only a stand-in for the symbol. Its device address is looked up on every
// call, with the caller's device current. The lookup allocates nothing and is
// cheap, and it stays right if the device's context was torn down and the
// module reloaded at another address (after a cudaDeviceReset, for instance).
int static_workspace_address(void** addr) {
    void* p = nullptr;
    if (cudaGetSymbolAddress(&p, g_static_workspace) != cudaSuccess || p == nullptr) {
        return NVLLM_ERR_CUDA;
    }
    *addr = p;
    return NVLLM_OK;
}

}  // namespace

extern "C" int nvllm_paged_attention_static(
    float* out, const float* query, const float* k_arena, const float* v_arena,
    const int32_t* block_tables, int32_t max_blocks_per_seq, const int32_t* cu_seqlens_q,
    const int32_t* context_lens, int32_t num_seqs, int32_t max_query_len,
    int32_t max_context_len, int32_t layer, float scale, int32_t precision,
    const nvllm_kv_layout* layout, void* stream) {
    // A batch whose workspace would not fit is refused before anything runs.
    const size_t need =
        nvllm_paged_attention_workspace_size(num_seqs, max_query_len, max_context_len, layout);
    if (need > kStaticWorkspaceBytes) return NVLLM_ERR_WORKSPACE;
    void* ws = nullptr;
    const int rc = static_workspace_address(&ws);
    if (rc != NVLLM_OK) return rc;
    // The kernels reset the work-list counters themselves on every call and
    // write every partial before reading it, so the previous call's contents
    // need no clearing.
    return nvllm_paged_attention(out, query, k_arena, v_arena, block_tables, max_blocks_per_seq,
                                 cu_seqlens_q, context_lens, num_seqs, max_query_len,
                                 max_context_len, layer, scale, precision, ws,
                                 kStaticWorkspaceBytes, layout, stream);
}
