// swa_backward.h -- internal interface between the C-ABI layer (capi.cpp) and the sm_100a
// backward kernels (swa_backward.cu).  Not part of the public ABI (see include/lca.h).
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>
#include <cstddef>
#include <cstdint>

namespace lca {

// Gradient of the sliding-window + global-token attention with respect to Q, K and V,
// from the forward's fp32 output O and its natural-log LSE.  Every visible (query i,
// key j) pair is counted once, by exactly one of four kinds of work:
//
//   band rows     (dQ kernel)   : rows i, keys j in the band with j not global, plus the
//                                 compact global keys; writes dQ of the non-global rows
//   global rows   (dQ kernel)   : the compact global rows against a split of all n keys;
//                                 partial dQ per split
//   band keys     (dK/dV kernel): keys j, rows i in the band with i not global, plus the
//                                 compact global rows; writes dK, dV of non-global keys
//   global keys   (dK/dV kernel): the compact global keys against a split of all n rows;
//                                 partial dK, dV per split
//
// and lca_bwd_reduce sums the split partials into the rows of the global tokens.
struct BwdParams {
    int n;             // sequence length
    int bh;            // batch * heads
    int window;        // band radius, clamped to n
    int num_global;    // G: unique global tokens
    int g_tiles;       // ceil(G / 128): compact outer tiles
    int gi_tiles;      // ceil(G / 64): compact inner tiles
    int n_tiles;       // ceil(n / 128): band units per (batch, head)
    int split_tiles;   // 64-row inner tiles of one split of the global-row / global-key units
    int n_splits;      // splits per (bh, global tile)
    int n_band_units;  // bh * n_tiles
    int n_units;       // n_band_units + bh * g_tiles * n_splits
    int grid;          // CTAs of the persistent grid (the SM count), at most n_units
    float scale;       // softmax scale (dQ and dK carry it)
    float scale_log2;  // scale * log2(e)
    const int* gidx;   // [G] sorted absolute global indices
    const uint32_t* gbitmap;  // bit i of word i / 32: row i is a global token (ceil(n / 32) + 3 words)
    const float* lse2;  // [bh][n] LSE * log2(e)
    const float* dvec;  // [bh][n] D_i = sum_c dO[i][c] * O[i][c]
    const float* lse2g; // [bh][G] the same for the global rows
    const float* dg;    // [bh][G]
    float* out_a;       // dQ kernel: dQ [bh][n][d]; dK/dV kernel: dV
    float* out_b;       // dK/dV kernel: dK
    float* part_a;      // [n_splits][bh][G][d]: dQ (dQ kernel) or dV (dK/dV kernel) partials
    float* part_b;      // [n_splits][bh][G][d]: dK partials (dK/dV kernel)
    int* err;           // device error word
    unsigned long long timeout_ns;
};

// Tensor maps of one backward kernel, 128-byte swizzle, box 64 columns x 128 rows (outer
// tiles) or x 64 rows (inner tiles):
//   x1, x2: the outer tile's two operands over [bh][n][d] (dQ kernel: Q, dO16; dK/dV: K, V)
//   y1, y2: the inner tiles' two operands (dQ kernel: K, V; dK/dV: Q, dO16)
//   x1g, x2g, y1g, y2g: the same tensors' compact global rows, maps {d, bh, G}
struct BwdMaps {
    CUtensorMap x1, x2, y1, y2;
    CUtensorMap x1g, x2g, y1g, y2g;
};

// Per-row preparation: D_i, the 16-bit copy of dO in the inputs' type, LSE * log2(e), and
// the compact copies of the global rows ([G][4 (q, k, v, dO16)][bh][d], stats [bh][G]).
struct BwdPrepParams {
    const void* q;
    const void* k;
    const void* v;
    const float* o;
    const float* dout;
    const float* lse;
    void* dout16;       // [bh][n][d] 16-bit
    float* lse2;        // [bh][n]
    float* dvec;        // [bh][n]
    void* compact;      // [G][4][bh][d] 16-bit
    float* lse2g;       // [bh][G]
    float* dg;          // [bh][G]
    const int* gidx;    // [G] sorted
    const uint32_t* gbitmap;  // global rows (lca_bwd_indices writes it first)
    int num_global;
    int n;
    int bh;
    int bf16;           // 16-bit type of q, k, v and dout16
};

// Sum of the split partials into the global tokens' rows of dQ, dK and dV.
struct BwdReduceParams {
    const float* part_q;  // [splits_q][bh][G][d]
    const float* part_k;  // [splits_k][bh][G][d]
    const float* part_v;
    float* dq;
    float* dk;
    float* dv;
    const int* gidx;
    int splits_q, splits_k;
    int num_global;
    int n;
    int bh;
};

// Up to kBwdIndexChunk sorted global indices written to dst[0, count) and set in the
// global-row bitmap (cleared first when clear_bitmap); the host passes the list in chunks
// through kernel parameters, so the copy is an ordinary capturable launch.
constexpr int kBwdIndexChunk = 1024;
struct BwdIndexParams {
    int* dst;
    uint32_t* bitmap;
    int bitmap_words;
    int clear_bitmap;
    int count;
    int idx[kBwdIndexChunk];
};

cudaError_t launch_bwd_indices(const BwdIndexParams& ip, cudaStream_t stream);
cudaError_t launch_bwd_prep(int head_dim, const BwdPrepParams& pp, cudaStream_t stream);
// key_major: the dK/dV kernel, else the dQ kernel
cudaError_t launch_bwd_main(int head_dim, bool bf16, bool key_major, const BwdMaps& maps, const BwdParams& p,
                            cudaStream_t stream);
cudaError_t launch_bwd_reduce(int head_dim, const BwdReduceParams& rp, cudaStream_t stream);

}  // namespace lca
