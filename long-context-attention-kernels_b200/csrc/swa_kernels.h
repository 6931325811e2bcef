// swa_kernels.h -- internal interface between the C-ABI layer (capi.cpp) and the
// sm_100a kernels (swa_kernels.cu).  Not part of the public ABI (see include/lca.h).
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>
#include <cstddef>
#include <cstdint>

namespace lca {

// Device-side error codes written to the error word when a bounded wait gives up.
enum : int {
    LCA_DEVERR_NONE = 0,
    LCA_DEVERR_TIMEOUT_PRODUCER = 1,
    LCA_DEVERR_TIMEOUT_MMA = 2,
    LCA_DEVERR_TIMEOUT_SOFTMAX = 3,
    LCA_DEVERR_TIMEOUT_DRAIN = 4,
};

constexpr int kTileRows = 128;        // query rows / keys per tile
constexpr int kGatherChunk = 1024;    // global indices passed per gather launch

struct TensorMaps {
    CUtensorMap q, k, v;     // inputs [bh][n][d] (bf16 / f16), box 64 x 128 rows, 128B swizzle
    CUtensorMap qg, kg, vg;  // compact global rows [bh][gpad][d]
    CUtensorMap o;           // output [bh][n][d] fp32, box 32 x 128 rows, 128B swizzle
    CUtensorMap po;          // global-row partial outputs [2*splits*bh][gpad][d] fp32
};

struct MainParams {
    int n;            // sequence length
    int bh;           // batch * heads
    int window;       // band radius, clamped to n
    int q_tiles;      // ceil(n / 128)
    int num_global;   // G: unique global tokens
    int g_tiles;      // ceil(G / 128)
    int gpad;         // g_tiles * 128
    int n_splits;     // key splits per (bh, global tile)
    int split_tiles;  // key tiles per split
    int n_grow_units; // bh * g_tiles * n_splits global-row units (scheduled first)
    int n_band_units; // bh * q_pairs band units
    int q_pairs;      // ceil(q_tiles / 2): band units per (batch, head)
    float scale_log2; // scale * log2(e)
    const int* gidx;  // [gpad] sorted global indices (padding = INT_MAX)
    float* lse;       // [bh][n] natural-log LSE, or nullptr
    float* part_lse;  // [2 * n_splits][bh][gpad]
    int* err;         // device error word (first error wins)
    unsigned long long timeout_ns;  // per-wait budget
};

struct GatherParams {
    int n, gpad, num_global, bh;
    int first, count;  // compact rows [first, first + count) handled by this launch
    int* gidx_out;
    uint16_t *qg, *kg, *vg;
    int idx[kGatherChunk];
};

struct CombineParams {
    int n, bh, gpad, num_global, n_splits, split_tiles;
    const int* gidx;
    const float* part_o;
    const float* part_lse;
    float* o;
    float* lse;
};

cudaError_t launch_main(int head_dim, bool bf16, const TensorMaps& tm, const MainParams& p, int grid,
                        cudaStream_t stream);
cudaError_t launch_gather(int head_dim, const void* q, const void* k, const void* v, const GatherParams& gp,
                          int bh, cudaStream_t stream);
cudaError_t launch_combine(int head_dim, const CombineParams& cp, cudaStream_t stream);
int main_smem_bytes(int head_dim, bool bf16);
// Record `status` and a printf-style detail message as this thread's last C-ABI error
// (what lca_last_error() returns); returns `status`.
int report_error(int status, const char* fmt, ...);

// Device address (on the current device) of the device-side error word.
cudaError_t error_word_address(int** out);

}  // namespace lca
