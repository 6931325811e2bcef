/*
 * lca.h -- C ABI of the B200 (sm_100a) sliding-window + global-token attention forward.
 *
 * Plain C: pointers, sizes and int status codes only.  Device pointers are CUDA device
 * memory on the current device; `stream` is a cudaStream_t passed as void* (NULL = the
 * legacy default stream).  Nothing here allocates device memory: outputs and the
 * workspace are owned by the caller.  Every entry point is thread-safe; work is enqueued
 * asynchronously on `stream` and no call synchronises unless its comment says so.
 *
 * Semantics follow the reference's dense Longformer-mask definition
 * (python/long_context_attention/__init__.py:24-53): key j is visible to query i iff
 * |i - j| <= window_size, or j is a global token, or i is a global token; the output is
 * fp32 softmax(scale * q k^T over the visible keys) v, per (batch, head).
 */
#ifndef LCA_H_
#define LCA_H_

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define LCA_ABI_VERSION 1

#if defined(LCA_BUILDING_LIBRARY) && defined(__GNUC__)
#define LCA_API __attribute__((visibility("default")))
#else
#define LCA_API
#endif

/* Status codes returned by every entry point. */
enum {
    LCA_OK = 0,
    LCA_ERR_INVALID_ARGUMENT = 1, /* null/misaligned pointer, bad size, window < 0, ... */
    LCA_ERR_INDEX = 2,            /* a global token outside [-seq_len, seq_len) */
    LCA_ERR_UNSUPPORTED = 3,      /* dtype / head_dim / device not supported by this build */
    LCA_ERR_WORKSPACE = 4,        /* workspace too small or misaligned */
    LCA_ERR_CUDA = 5,             /* a CUDA runtime/driver call or launch failed */
    LCA_ERR_DEVICE = 6            /* a kernel reported a device-side error (bounded wait gave up) */
};

/* Input element types (Q, K, V share one type; the output is always fp32). */
enum { LCA_DTYPE_F16 = 0, LCA_DTYPE_BF16 = 1 };

/* ABI version of the loaded library (== LCA_ABI_VERSION it was built with). */
LCA_API int lca_abi_version(void);

/* Short static description of a status code. */
LCA_API const char* lca_status_string(int status);

/* Detail message of the last failing call made on this thread ("" if none). */
LCA_API const char* lca_last_error(void);

/*
 * Normalise a global-token list the way the reference builds its mask
 * (python/long_context_attention/__init__.py:42-44, `global_mask[list(global_tokens)] = True`):
 * negative indices count from the end, duplicates collapse, any index outside
 * [-seq_len, seq_len) is an error (LCA_ERR_INDEX).  Writes the sorted unique indices to
 * `out` (capacity >= count) and their number to *out_count.  Host-only.
 */
LCA_API int lca_normalize_global_tokens(const int64_t* tokens, int64_t count, int64_t seq_len, int32_t* out,
                                int64_t* out_count);

/*
 * Bytes of device workspace lca_swa_forward needs for this problem (0 when there are no
 * global tokens).  `num_unique_global` is the count after normalisation.  Host-only.
 */
LCA_API int lca_swa_workspace_size(int64_t batch, int64_t heads, int64_t seq_len, int64_t head_dim,
                                   int64_t window_size, int64_t num_unique_global, int dtype, size_t* out_bytes);

/*
 * Sliding-window + global-token attention forward.
 * Replaces the reference's extension entry point
 *   sliding_window_attention_forward(Q, K, V, window_size, global_tokens, scale)
 *   (csrc/bindings.cpp:31-73) and the kernels it launches
 *   (csrc/sliding_window_attention.cu:48-174, csrc/global_attention.cu:29-176,
 *    csrc/combine.cu:18-70).
 *
 *   q, k, v      [batch, heads, seq_len, head_dim] contiguous, `dtype`, 16-byte aligned
 *   out          [batch, heads, seq_len, head_dim] contiguous fp32, 16-byte aligned
 *   lse          [batch, heads, seq_len] fp32 natural-log log-sum-exp of the scaled
 *                visible scores, or NULL
 *   head_dim     64 or 128
 *   window_size  band radius w >= 0 (keys with |i - j| <= w are visible)
 *   scale        score scale (the reference defaults it to 1/sqrt(head_dim) in Python)
 *   global_tokens / num_global_tokens: HOST array of token indices (any order,
 *                duplicates and negative indices allowed, as in the reference)
 *   workspace    device buffer of >= lca_swa_workspace_size(...) bytes, 256-byte aligned
 *                (may be NULL when that size is 0); must not be shared by calls that
 *                can run concurrently
 */
LCA_API int lca_swa_forward(const void* q, const void* k, const void* v, float* out, float* lse, int dtype,
                    int64_t batch, int64_t heads, int64_t seq_len, int64_t head_dim, int64_t window_size,
                    float scale, const int64_t* global_tokens, int64_t num_global_tokens, void* workspace,
                    size_t workspace_bytes, void* stream);

/*
 * Bytes of the fixed device scratch array used by lca_swa_forward_noalloc.
 */
#define LCA_NOALLOC_SCRATCH_BYTES (32u << 20)

/*
 * Same computation and arguments as lca_swa_forward, minus the workspace: for callers
 * that cannot allocate device memory (a serving loop whose memory belongs to its own pool
 * allocator, a plugin inside a runtime that forbids allocation after start-up, a loop
 * that must not risk the synchronisation a cudaFree can cause).  No counterpart in the
 * reference.  The scratch is a fixed LCA_NOALLOC_SCRATCH_BYTES device array inside the
 * library: each GPU that uses this entry point holds it from the first call until the
 * process exits; the first call on a device looks up the array's device address and
 * should come before any stream capture on that device.  All calls on a device share the
 * array, so calls that can overlap on the GPU race: order them.  Problems needing more
 * scratch than the array holds return LCA_ERR_UNSUPPORTED before any work is enqueued.
 */
LCA_API int lca_swa_forward_noalloc(const void* q, const void* k, const void* v, float* out, float* lse, int dtype,
                                    int64_t batch, int64_t heads, int64_t seq_len, int64_t head_dim,
                                    int64_t window_size, float scale, const int64_t* global_tokens,
                                    int64_t num_global_tokens, void* stream);

/*
 * Measurement hook (no counterpart in the reference): when both events are non-NULL,
 * subsequent lca_swa_forward calls made on THIS thread record `before_main` immediately
 * before and `after_main` immediately after the launch of the main attention kernel, on
 * the call's stream, so a caller can time that kernel alone with cudaEventElapsedTime.
 * Events are cudaEvent_t passed as void*; pass NULLs to switch the hook off.
 */
LCA_API int lca_set_timing_events(void* before_main, void* after_main);

/*
 * Read and clear the device-side error word of the current device (0 = no error; other
 * values identify which bounded wait of a kernel gave up).  Synchronises the device.
 * No counterpart in the reference, which never checks its launches
 * (csrc/bindings.cpp:49-70).
 */
LCA_API int lca_device_error(int* code);

#ifdef __cplusplus
}
#endif

#endif /* LCA_H_ */
