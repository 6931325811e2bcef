// noalloc.cu -- lca_swa_forward_noalloc: the attention forward for callers that must
// not allocate device memory.
//
// Some callers cannot call cudaMalloc: a serving loop whose device memory is entirely
// owned by its own pool allocator (an extra cudaMalloc can fail or fragment that pool),
// a plugin running inside another runtime that forbids allocation after start-up, or a
// latency-critical loop that must not risk the implicit device-wide synchronisation a
// cudaFree can cause.  For them this entry point takes no workspace argument: the
// scratch the forward needs (compact copies of the global-token rows and the
// global-row partial results) lives in a fixed array in this file, sized
// LCA_NOALLOC_SCRATCH_BYTES.  The caller still owns Q, K, V, the output and the LSE.
//
// Properties a caller must know:
//  * The array is a file-scope __device__ variable, part of the library's device code:
//    a GPU holds its LCA_NOALLOC_SCRATCH_BYTES from the moment that code is loaded there
//    until the process exits.  With lazy module loading (the CUDA default) that is the
//    first launch of any of the library's kernels on the GPU; with
//    CUDA_MODULE_LOADING=EAGER it is context creation, whether or not this entry point is
//    ever called.
//  * In host code the array's name only stands for it; the device address is obtained
//    with cudaGetSymbolAddress, once per device, on the first call made with that device
//    current.  That first call on a device should therefore come before any stream
//    capture on it.
//  * Every call on a device shares the one array, and it keeps whatever the last call
//    left in it.  Nothing in it needs to start at zero: every byte the kernels read is
//    written earlier in the same call.  Two calls whose work can overlap on the GPU
//    (different streams without ordering between them) race on the array; order them.
//  * Problems whose scratch requirement exceeds the array are rejected before any work
//    is enqueued (LCA_ERR_UNSUPPORTED, with the required size in lca_last_error()).
#include <cuda_runtime.h>

#include <mutex>
#include <vector>

#include "lca.h"
#include "swa_kernels.h"

namespace {

static __device__ __align__(256) unsigned char g_noalloc_scratch[LCA_NOALLOC_SCRATCH_BYTES];

constexpr int kMaxDevices = 64;
std::mutex g_mu;
void* g_scratch_ptr[kMaxDevices];

}  // namespace

extern "C" int lca_swa_forward_noalloc(const void* q, const void* k, const void* v, float* out, float* lse,
                                       int dtype, int64_t batch, int64_t heads, int64_t seq_len,
                                       int64_t head_dim, int64_t window_size, float scale,
                                       const int64_t* global_tokens, int64_t num_global_tokens, void* stream) {
    // Scratch this problem needs (host arithmetic only; argument errors are reported by
    // the same checks the allocating entry point uses).
    if (num_global_tokens < 0) return lca::report_error(LCA_ERR_INVALID_ARGUMENT, "negative global token count");
    std::vector<int32_t> norm((size_t)num_global_tokens + 1);
    int64_t G = 0;
    int st = lca_normalize_global_tokens(global_tokens, num_global_tokens, seq_len, norm.data(), &G);
    if (st != LCA_OK) return st;
    size_t need = 0;  // the forward's minimum; it also uses the optional part when the array holds that too
    st = lca::workspace_bytes(batch, heads, seq_len, head_dim, window_size, G, dtype, false, &need);
    if (st != LCA_OK) return st;
    if (need > (size_t)LCA_NOALLOC_SCRATCH_BYTES)
        return lca::report_error(LCA_ERR_UNSUPPORTED,
                                 "problem needs %zu bytes of scratch; the built-in scratch holds %zu "
                                 "(use lca_swa_forward with a caller-provided workspace)",
                                 need, (size_t)LCA_NOALLOC_SCRATCH_BYTES);
    void* scratch = nullptr;
    if (batch * heads > 0 && seq_len > 0) {
        int dev = 0;
        cudaError_t e = cudaGetDevice(&dev);
        if (e != cudaSuccess) return lca::report_error(LCA_ERR_CUDA, "cudaGetDevice: %s", cudaGetErrorString(e));
        if (dev < 0 || dev >= kMaxDevices) return lca::report_error(LCA_ERR_UNSUPPORTED, "device %d out of range", dev);
        std::lock_guard<std::mutex> lk(g_mu);
        if (g_scratch_ptr[dev] == nullptr) {
            void* p = nullptr;
            e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
            if (e != cudaSuccess || p == nullptr)
                return lca::report_error(LCA_ERR_CUDA, "cudaGetSymbolAddress(scratch): %s", cudaGetErrorString(e));
            g_scratch_ptr[dev] = p;
        }
        scratch = g_scratch_ptr[dev];
    }
    // The whole array goes to the forward, which uses the optional part (the fp16 copy of V,
    // the work-unit counter) whenever the array holds it as well.
    return lca_swa_forward(q, k, v, out, lse, dtype, batch, heads, seq_len, head_dim, window_size, scale,
                           global_tokens, num_global_tokens, scratch,
                           scratch != nullptr ? (size_t)LCA_NOALLOC_SCRATCH_BYTES : 0, stream);
}
