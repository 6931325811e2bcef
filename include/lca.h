/*
 * lca.h -- C ABI of the B200 (sm_100a) sliding-window + global-token attention forward.
 *
 * Plain C: pointers, sizes and int status codes only.  Device pointers are CUDA device
 * memory on the current device; `stream` is a cudaStream_t passed as void* (NULL = the
 * legacy default stream).  The compute entry points allocate no device memory: outputs
 * and the workspace are owned by the caller (lca_peer_alloc is the one call that
 * allocates, on request, for the peer-memory exchange).  Every entry point is
 * thread-safe; work is enqueued asynchronously on `stream` and no call synchronises
 * unless its comment says so.
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

#define LCA_ABI_VERSION 2

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

/* Values of the device-side error word (lca_device_error): which bounded wait of a
 * kernel gave up first.  A kernel whose wait gives up stops its own work and returns, so
 * the results of that call (and, for the peer exchange, of that step) are invalid. */
enum {
    LCA_DEVERR_NONE = 0,
    LCA_DEVERR_TIMEOUT_PRODUCER = 1, /* main kernel: the TMA producer waited for a free slot */
    LCA_DEVERR_TIMEOUT_MMA = 2,      /* main kernel: an MMA issuer waited for data or P */
    LCA_DEVERR_TIMEOUT_SOFTMAX = 3,  /* main kernel: a softmax warp waited for S or O */
    LCA_DEVERR_TIMEOUT_DRAIN = 4,    /* main kernel: waiting for its own copies at exit */
    LCA_DEVERR_TIMEOUT_PEER = 5,     /* peer exchange: another rank's data did not arrive */
    LCA_DEVERR_TIMEOUT_BACKWARD = 6  /* backward kernel: waited for a tile or an MMA */
};

/* Element types: Q, K, V share LCA_DTYPE_F16 or LCA_DTYPE_BF16; the output is fp32
 * (LCA_DTYPE_F32) except through lca_swa_forward_ex, which also writes fp16 or bf16. */
enum { LCA_DTYPE_F16 = 0, LCA_DTYPE_BF16 = 1, LCA_DTYPE_F32 = 2 };

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
 * Bytes of device workspace recommended for lca_swa_forward on this problem.
 * `num_unique_global` is the count after normalisation.  Host-only.
 * The workspace holds the compact global rows and the global-row partials (the required
 * part: nothing for fp16 inputs without global tokens), then an optional part: for bf16
 * inputs an fp16 copy of V, and for every dtype one word from which the main kernel's CTAs
 * take work units dynamically.  When the workspace passed to lca_swa_forward is at least
 * this size, units are handed out dynamically (else round-robin), and if every value of V
 * fits fp16 (exactly, or within 2^-25 for magnitudes below 2^-14 in a 128-row block whose
 * largest magnitude is at least 2^-4), P*V runs once per key tile in fp16 instead of twice
 * with bf16 P split into hi + lo.  A smaller workspace that still holds the required part is
 * accepted and runs without the optional part.
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
 *   workspace    device buffer of lca_swa_workspace_size(...) bytes, 256-byte aligned
 *                (a smaller buffer that still holds the required part runs without the
 *                optional part, and may be NULL when that part is empty; one below it
 *                returns LCA_ERR_WORKSPACE); must not be shared by calls that can run
 *                concurrently
 */
LCA_API int lca_swa_forward(const void* q, const void* k, const void* v, float* out, float* lse, int dtype,
                    int64_t batch, int64_t heads, int64_t seq_len, int64_t head_dim, int64_t window_size,
                    float scale, const int64_t* global_tokens, int64_t num_global_tokens, void* workspace,
                    size_t workspace_bytes, void* stream);

/* Flags of lca_swa_forward_ex. */
enum {
    /* Causal (one-sided) variant: the mask above intersected with j <= i -- the band
     * becomes [i - window_size, i], a global key is visible to the rows at or after it,
     * and a global row sees the keys up to itself. */
    LCA_FLAG_CAUSAL = 1,
    /* q, k, v and out are token-major, [batch, seq_len, heads, head_dim] (the layout of a
     * fused QKV projection's output), read and written in place without a transpose; lse
     * stays [batch, heads, seq_len].  Not with dilation. */
    LCA_FLAG_TOKEN_MAJOR = 2
};

/* Most heads that lca_swa_forward_ex accepts radii of their own for. */
#define LCA_MAX_HEAD_WINDOWS 256

/*
 * lca_swa_forward with options, none of which the reference has (its extension always
 * returns fp32, has no causal mode and one window for every head, csrc/bindings.cpp:31-73):
 *   out_dtype    type of `out` ([batch, heads, seq_len, head_dim], 16-byte aligned):
 *                LCA_DTYPE_F32, or LCA_DTYPE_F16 / LCA_DTYPE_BF16 -- the same fp32-accumulated
 *                result rounded to nearest, with half the output bytes.  `lse` stays fp32.
 *   head_window_sizes  NULL, or a HOST array of `heads` band radii (each >= 0): head h of
 *                every batch uses head_window_sizes[h] in place of window_size (which is then
 *                ignored).  At most LCA_MAX_HEAD_WINDOWS heads.
 *   flags        LCA_FLAG_CAUSAL and / or LCA_FLAG_TOKEN_MAJOR, or 0.
 * The other arguments are lca_swa_forward's; lca_swa_forward(...) is
 * lca_swa_forward_ex(..., LCA_DTYPE_F32, ..., NULL, ..., 0, ...).
 */
LCA_API int lca_swa_forward_ex(const void* q, const void* k, const void* v, void* out, int out_dtype, float* lse,
                               int dtype, int64_t batch, int64_t heads, int64_t seq_len, int64_t head_dim,
                               int64_t window_size, const int64_t* head_window_sizes, float scale, int flags,
                               const int64_t* global_tokens, int64_t num_global_tokens, void* workspace,
                               size_t workspace_bytes, void* stream);

/* Most sequences one lca_swa_forward_varlen call takes. */
#define LCA_MAX_SEQUENCES 512

/*
 * Packed variable-length sequences (no counterpart in the reference, which takes one
 * length per call).  q, k, v, out: [1, heads, total_len, head_dim] with sequence s in
 * rows [cu_seqlens[s], cu_seqlens[s + 1]) (num_seqs + 1 host offsets from 0 to total_len,
 * non-decreasing, at most LCA_MAX_SEQUENCES sequences); lse: [1, heads, total_len] or NULL.
 * Every sequence is its own problem: its bands, global keys and global rows stay inside
 * it.  The global-token list applies to every non-empty sequence, indexed within it as the
 * reference indexes one sequence (negative from its end; an index outside it returns
 * LCA_ERR_INDEX).  Workspace: lca_swa_workspace_size(1, heads, total_len, head_dim,
 * window, num_seqs * num_global_tokens, dtype) bytes (an upper bound).  The other arguments
 * are lca_swa_forward_ex's.
 */
LCA_API int lca_swa_forward_varlen(const void* q, const void* k, const void* v, void* out, int out_dtype, float* lse,
                                   int dtype, int64_t heads, int64_t total_len, int64_t head_dim, int64_t window_size,
                                   const int64_t* head_window_sizes, float scale, int flags,
                                   const int64_t* cu_seqlens, int64_t num_seqs, const int64_t* global_tokens,
                                   int64_t num_global_tokens, void* workspace, size_t workspace_bytes, void* stream);

/*
 * Dilated sliding window (no counterpart in the reference; its README lists dilated windows
 * as future work): key j is visible to query i iff |i - j| <= window_size * dilation and
 * (i - j) is a multiple of dilation, or j or i is a global token.  seq_len must be a
 * multiple of dilation; the causal flag is not supported with dilation > 1.  The forward
 * reorders Q, K, V into residue order (row r + dilation * t to r * (seq_len / dilation) + t)
 * inside the workspace, runs the banded kernels with each residue class as its own segment,
 * and writes out / lse back in sequence order.  Workspace: lca_swa_dilated_workspace_size
 * bytes, 256-byte aligned.  dilation == 1 is lca_swa_forward_ex.
 */
LCA_API int lca_swa_dilated_workspace_size(int64_t batch, int64_t heads, int64_t seq_len, int64_t head_dim,
                                           int64_t window_size, int64_t dilation, int64_t num_unique_global,
                                           int dtype, int out_dtype, size_t* out_bytes);
LCA_API int lca_swa_forward_dilated(const void* q, const void* k, const void* v, void* out, int out_dtype, float* lse,
                                    int dtype, int64_t batch, int64_t heads, int64_t seq_len, int64_t head_dim,
                                    int64_t window_size, const int64_t* head_window_sizes, int64_t dilation,
                                    float scale, int flags, const int64_t* global_tokens, int64_t num_global_tokens,
                                    void* workspace, size_t workspace_bytes, void* stream);

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
 * library, reserved on a GPU when the library's device code is loaded there and held until
 * the process exits: with lazy module loading (the CUDA default) that is the first launch
 * of one of the library's kernels on that GPU, with CUDA_MODULE_LOADING=EAGER it is
 * context creation, whether or not this entry point is ever called.  The first call on a
 * device looks up the array's device address and should come before any stream capture
 * on that device.  All calls on a device share the
 * array, so calls that can overlap on the GPU race: order them.  Problems needing more
 * scratch than the array holds return LCA_ERR_UNSUPPORTED before any work is enqueued.
 */
LCA_API int lca_swa_forward_noalloc(const void* q, const void* k, const void* v, float* out, float* lse, int dtype,
                                    int64_t batch, int64_t heads, int64_t seq_len, int64_t head_dim,
                                    int64_t window_size, float scale, const int64_t* global_tokens,
                                    int64_t num_global_tokens, void* stream);

/* ------------------------------------------------------------------------------------
 * Sequence shards.  A sequence too long for one GPU is cut into contiguous token shards,
 * one per rank: rank r holds rows [shard_offset, shard_offset + shard_len) of Q, K and V
 * for every (batch, head), and produces the same rows of the output.  The reference runs
 * one sequence on one device only; these calls split its forward
 * (csrc/bindings.cpp:31-73) into the compute steps around three exchanges that the
 * caller performs with its own collectives library (NCCL):
 *
 *   1. lca_swa_shard_prepare   -- on every rank
 *   2. exchange A+B (point-to-point, one group):
 *      A: the global rows.  The `globals` region holds one globals_row_bytes row per
 *         unique global token, in sorted token order; the rows of the tokens inside
 *         rank r's shard form one contiguous run, which rank r has filled.  Rank r sends
 *         its run to every other rank, and receives every other rank's run into the same
 *         offsets of its own region (ranks whose shard holds no global token send nothing).
 *      B: the halos.  Send side 0 of `halo_send` to rank r-1 and side 1 to rank r+1;
 *         receive from rank r-1 into side 0 of `halo_recv` and from rank r+1 into side 1
 *         (ranks without that neighbour skip the transfer)
 *   3. lca_swa_shard_forward   -- on every rank
 *   4. exchange C (all-gather): every rank's `rowpart` region into `rowpart_all`, rank
 *      order, rowpart_bytes per rank
 *   5. lca_swa_shard_finish    -- on every rank; writes the global rows this shard owns
 *
 * Exchanges A and C are skipped when there are no global tokens, B when halo_rows is 0.
 * Every step takes the same descriptor and global-token list; the workspace carries
 * state from one step to the next and must not be reused until step 5 has run.
 * Limits: every shard but the last holds a multiple of 128 tokens, and
 * min(window_size, seq_len) <= shard_len when world_size > 1 (halos come from the
 * adjacent shards only).
 */
typedef struct lca_shard_desc {
    int64_t batch, heads, seq_len, head_dim, window_size;
    int64_t shard_offset; /* absolute index of this shard's first token */
    int64_t shard_len;    /* tokens in this shard (rows of q / k / v / out / lse) */
    int64_t world_size;   /* number of shards */
    int64_t rank;         /* this shard's index; shard r-1 holds the tokens just before */
    int dtype;            /* LCA_DTYPE_* */
    float scale;
} lca_shard_desc;

/* Byte offsets of the exchanged regions inside the workspace, and sizes. */
typedef struct lca_shard_layout {
    size_t total_bytes;        /* workspace size */
    int64_t halo_rows;         /* K / V rows per halo side (0: no halo exchange) */
    size_t globals_offset;     /* exchange A region: [G][3 (q, k, v)][batch*heads][head_dim], input dtype */
    size_t globals_bytes;
    size_t globals_row_bytes;  /* one global row of that region */
    size_t halo_send_offset;   /* [2 sides][2 (k, v)][batch*heads][halo_rows][head_dim], input dtype */
    size_t halo_recv_offset;   /* same layout */
    size_t halo_side_bytes;    /* bytes of one side of halo_send / halo_recv */
    size_t rowpart_offset;     /* exchange C source: fp32 O [batch*heads][G][head_dim], then fp32 LSE
                                  [batch*heads][G], padded to a multiple of 16 bytes */
    size_t rowpart_bytes;
    size_t rowpart_all_offset; /* exchange C target: world_size * rowpart_bytes */
} lca_shard_layout;

/* Workspace layout of one shard's problem (`num_unique_global` after normalisation).
 * Host-only. */
LCA_API int lca_swa_shard_layout(const lca_shard_desc* desc, int64_t num_unique_global, lca_shard_layout* out);

/* Step 1: compact global rows owned by this shard, the sorted global index list and the
 * halo blocks for the neighbours.  q, k, v: [batch, heads, shard_len, head_dim]. */
LCA_API int lca_swa_shard_prepare(const lca_shard_desc* desc, const void* q, const void* k, const void* v,
                                  const int64_t* global_tokens, int64_t num_global_tokens, void* workspace,
                                  size_t workspace_bytes, void* stream);

/* Step 3: every row of this shard (global rows are finished in step 5) and this shard's
 * partial result for the global rows over its own keys.  out: [batch, heads, shard_len,
 * head_dim] fp32; lse: [batch, heads, shard_len] fp32 or NULL. */
LCA_API int lca_swa_shard_forward(const lca_shard_desc* desc, const void* q, const void* k, const void* v,
                                  float* out, float* lse, const int64_t* global_tokens, int64_t num_global_tokens,
                                  void* workspace, size_t workspace_bytes, void* stream);

/* Step 5: log-sum-exp merge of the shards' global-row partials; writes the global rows
 * that fall in this shard to out / lse. */
LCA_API int lca_swa_shard_finish(const lca_shard_desc* desc, float* out, float* lse, const int64_t* global_tokens,
                                 int64_t num_global_tokens, void* workspace, size_t workspace_bytes, void* stream);

/* ------------------------------------------------------------------------------------
 * Peer-memory exchange for sequence shards: one process per GPU, all GPUs in one NVLink
 * domain.  Instead of the caller's collectives, the library writes the halos, the global
 * rows and the row partials straight into the other ranks' workspaces over NVLink and
 * waits on counters there (bounded: a rank that stops leaves LCA_ERR_DEVICE to
 * lca_device_error on the others).  Each rank allocates its workspace with
 * lca_peer_alloc, sends the 64-byte handle to the others, and maps theirs with
 * lca_peer_open; `peer_workspaces[r]` is rank r's workspace (this rank's own at
 * [rank]).  A step is then: lca_swa_shard_prepare, lca_swa_shard_exchange_peer,
 * lca_swa_shard_forward, lca_swa_shard_finish_peer -- no other exchange.  Every rank must
 * run the same steps; never run two ranks on one GPU (their waits need both to run at
 * once).  Ranks hold consecutive shards in rank order.
 */

/* cudaMalloc `bytes` (zero-filled) and its CUDA IPC handle (64 bytes) for other processes. */
LCA_API int lca_peer_alloc(size_t bytes, void** dev_ptr, void* ipc_handle);
/* Map another process's lca_peer_alloc buffer from its IPC handle. */
LCA_API int lca_peer_open(const void* ipc_handle, void** dev_ptr);
/* Unmap a buffer mapped by lca_peer_open. */
LCA_API int lca_peer_close(void* dev_ptr);
/* Free a buffer from lca_peer_alloc. */
LCA_API int lca_peer_free(void* dev_ptr);

/* Exchange A+B by peer stores: this rank's global rows to every rank, its halo blocks to
 * its neighbours, then wait for every other rank's. */
LCA_API int lca_swa_shard_exchange_peer(const lca_shard_desc* desc, const int64_t* global_tokens,
                                        int64_t num_global_tokens, void* const* peer_workspaces,
                                        size_t workspace_bytes, void* stream);

/* Exchange C by peer stores, then step 5: this rank's global-row partial into every
 * rank's gathered region, wait for all, merge into the global rows this shard owns. */
LCA_API int lca_swa_shard_finish_peer(const lca_shard_desc* desc, float* out, float* lse,
                                      const int64_t* global_tokens, int64_t num_global_tokens,
                                      void* const* peer_workspaces, size_t workspace_bytes, void* stream);

/*
 * Backward pass (no counterpart in the reference, whose roadmap lists it first:
 * README.md:113).  Gradients of the attention of lca_swa_forward with respect to Q, K and
 * V, for the same q, k, v, dtype, shape, window_size, scale and global tokens:
 *   o    : the forward's fp32 output  [batch][heads][seq_len][head_dim]
 *   lse  : the forward's natural-log LSE  [batch][heads][seq_len]
 *   dout : the gradient of the loss with respect to o (fp32, o's shape)
 *   dq, dk, dv : fp32 outputs, q's shape (every element is written)
 * P is recomputed from lse; dO, P and the score gradient enter the tensor-core products in
 * the inputs' 16-bit type (fp32 accumulation).  Head-major layout, no causal / per-head
 * radius / packed-sequence options.  The workspace (lca_swa_backward_workspace_size bytes,
 * 256-byte aligned) is scratch: the call may overwrite all of it.
 */
LCA_API int lca_swa_backward_workspace_size(int64_t batch, int64_t heads, int64_t seq_len, int64_t head_dim,
                                            int64_t window_size, int64_t num_unique_global, int dtype,
                                            size_t* out_bytes);
LCA_API int lca_swa_backward(const void* q, const void* k, const void* v, const float* o, const float* lse,
                             const float* dout, float* dq, float* dk, float* dv, int dtype, int64_t batch,
                             int64_t heads, int64_t seq_len, int64_t head_dim, int64_t window_size, float scale,
                             const int64_t* global_tokens, int64_t num_global_tokens, void* workspace,
                             size_t workspace_bytes, void* stream);

/*
 * Measurement hook (no counterpart in the reference): when both events are non-NULL,
 * subsequent lca_swa_forward calls made on THIS thread record `before_main` immediately
 * before and `after_main` immediately after the launch of the main attention kernel, on
 * the call's stream, so a caller can time that kernel alone with cudaEventElapsedTime.
 * Events are cudaEvent_t passed as void*; pass NULLs to switch the hook off.
 */
LCA_API int lca_set_timing_events(void* before_main, void* after_main);

/*
 * Read and clear the device-side error word of the current device (LCA_DEVERR_NONE, or
 * the LCA_DEVERR_* code of the first bounded wait that gave up).  Synchronises the device.
 * No counterpart in the reference, which never checks its launches
 * (csrc/bindings.cpp:49-70).
 */
LCA_API int lca_device_error(int* code);

#ifdef __cplusplus
}
#endif

#endif /* LCA_H_ */
