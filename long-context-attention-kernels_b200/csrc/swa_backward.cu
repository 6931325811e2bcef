// swa_backward.cu -- sm_100a backward of the sliding-window + global-token attention.
//
// The reference's roadmap lists the backward pass as its first open item (README.md:113);
// the reference itself is forward only.  The gradient follows from its mask definition
// (python/long_context_attention/__init__.py:24-53): with P = softmax(scale * Q K^T) over
// the visible keys of each row,
//
//   D_i  = sum_c dO[i][c] * O[i][c]
//   dP   = dO V^T,   dS = P * (dP - D)            (elementwise, visible pairs only)
//   dQ   = scale * dS K,   dK = scale * dS^T Q,   dV = P^T dO
//
// P is recomputed from the forward's LSE: P[i][j] = 2^(s * scale * log2 e - LSE_i * log2 e).
//
// Kernels (one stream, in this order):
//   lca_bwd_prep     : per row D_i, the 16-bit copy of dO (inputs' type), LSE * log2 e, and the
//                      compact copies of the global rows of Q, K, V and dO16 with their stats.
//   lca_bwd_main<D, BF16, KM = false> (dQ): one CTA per outer query tile.  Band units take
//                      the band's key tiles (global keys masked) and the compact global-key
//                      tiles, and write dQ of the non-global rows; global-row units take the
//                      compact global rows against a split of all n keys (partial dQ).
//   lca_bwd_main<D, BF16, KM = true> (dK, dV): one CTA per outer key tile, the same with the
//                      roles of rows and keys exchanged.
//   lca_bwd_reduce   : sums the split partials into the global tokens' rows.
//
// One CTA = one warpgroup (128 threads; thread r <-> TMEM lane r <-> outer row r).  Per inner
// tile: thread 0 issues S = X1 Y1^T and dP = X2 Y2^T (tcgen05.mma, SS, both operands K-major
// from shared memory, 128 x 128 fp32 in TMEM); every thread turns its row of S and dP into P
// and dS, packs them to 16-bit pairs and stores them back over S and dP (tcgen05.st); thread
// 0 then issues the TS MMAs that accumulate in TMEM (dQ += dS Y1; or dV += P^T Y2 and
// dK += dS^T Y1), with Y1 / Y2 read as MN-major B operands from the same shared tiles.  The
// inner tiles are double-buffered and loaded by TMA.  TMEM columns: S [0, 128), dP [128, 256),
// accumulators [256, 256 + D) and [256 + D, 256 + 2D).
#include <cuda.h>
#include <cuda_runtime.h>
#include <cuda_fp16.h>
#include <cuda_bf16.h>
#include <cstdint>
#include <climits>

#include "sm100_ptx.cuh"
#include "swa_backward.h"
#include "lca.h"

namespace lca {
namespace {

constexpr int kBM = 128;                 // rows of a tile (outer and inner)
constexpr int kBwdThreads = 128;         // one warpgroup
constexpr int kBwdPanel = 128 * 128;     // one 128-row x 128-byte swizzle panel
constexpr uint32_t kBwdTmemCols = 512;
constexpr float kLog2e = 1.4426950408889634f;

template <int D>
struct BwdCfg {
    static constexpr int kTileBytes = kBM * D * 2;  // one 16-bit tile: D / 64 panels
    static constexpr int kOffX = 0;                 // X1, X2
    static constexpr int kOffY = 2 * kTileBytes;    // [2 stages][Y1, Y2]
    static constexpr int kOffStat = kOffY + 4 * kTileBytes;  // [2 (lse2, D)][128] floats
    static constexpr int kOffMask = kOffStat + 2 * kBM * 4;  // 4 words: inner rows that are global
    static constexpr int kOffBar = kOffMask + 16;            // barriers
    static constexpr int kOffMisc = kOffBar + 8 * 8;         // TMEM base, abort flag
    static constexpr int kUsed = kOffMisc + 16;
    // one CTA per SM: the CTA holds 512 TMEM columns
    static constexpr int kSmemBytes = (kUsed + 1024 > 120 * 1024) ? kUsed + 1024 : 120 * 1024;
};

struct BwdUnit {
    bool all;    // global-row (dQ) / global-key (dK/dV) unit
    int bh;
    int outer0;  // band: first outer row; all: first compact row
    int split;
    int inner0;  // first inner row of the contiguous tiles
    int n_cont;  // contiguous inner tiles
    int n_comp;  // compact inner tiles after them
};

__device__ __forceinline__ BwdUnit bwd_decode(const BwdParams& p, int u) {
    BwdUnit un;
    if (u < p.n_band_units) {
        un.all = false;
        un.bh = u / p.n_tiles;
        un.outer0 = (u % p.n_tiles) * kBM;
        un.split = 0;
        // inner rows that can see / be seen by the outer tile: [o0 - w, o0 + 127 + w] within [0, n)
        int lo = un.outer0 - p.window;
        if (lo < 0) lo = 0;
        int hi = un.outer0 + kBM - 1 + p.window;
        if (hi > p.n - 1) hi = p.n - 1;
        un.inner0 = lo;
        un.n_cont = (hi - lo + kBM) / kBM;
        un.n_comp = p.g_tiles;
    } else {
        const int t = u - p.n_band_units;
        un.all = true;
        un.split = t % p.n_splits;
        const int rest = t / p.n_splits;
        un.outer0 = (rest % p.g_tiles) * kBM;
        un.bh = rest / p.g_tiles;
        un.inner0 = un.split * p.split_tiles * kBM;
        int tiles = (p.n - un.inner0 + kBM - 1) / kBM;
        if (tiles > p.split_tiles) tiles = p.split_tiles;
        un.n_cont = tiles;
        un.n_comp = 0;
    }
    return un;
}

// First index of the sorted list gl[0, count) whose value is >= key (count if none).
__device__ __forceinline__ int bwd_lower(const int* __restrict__ gl, int count, int key) {
    int a = 0, b = count;
    while (a < b) {
        const int mid = (a + b) >> 1;
        if (__ldg(gl + mid) < key) a = mid + 1; else b = mid;
    }
    return a;
}

__device__ __forceinline__ bool bwd_is_global(const BwdParams& p, int row) {
    if (p.num_global == 0) return false;
    const int a = bwd_lower(p.gidx, p.num_global, row);
    return a < p.num_global && __ldg(p.gidx + a) == row;
}

// 32-bit mask of the columns [c0, c0 + 32) that lie in [lo, hi].
__device__ __forceinline__ uint32_t range_bits(int c0, int lo, int hi) {
    const int a = lo - c0 > 0 ? lo - c0 : 0;
    const int b = hi - c0 < 31 ? hi - c0 : 31;
    if (a > b) return 0u;
    const uint32_t upto_b = (b == 31) ? 0xFFFFFFFFu : ((1u << (b + 1)) - 1u);
    return upto_b & ~((1u << a) - 1u);
}

template <int D>
__device__ __forceinline__ void bwd_load_tile(uint8_t* dst, const CUtensorMap* map, uint64_t* bar, bool compact,
                                              int row0, int bh) {
#pragma unroll
    for (int pn = 0; pn < D / 64; ++pn) {
        if (compact)
            ptx::tma_load_3d(dst + pn * kBwdPanel, map, bar, pn * 64, bh, row0);
        else
            ptx::tma_load_3d(dst + pn * kBwdPanel, map, bar, pn * 64, row0, bh);
    }
}

template <int D, bool BF16, bool KM>
__global__ void __launch_bounds__(kBwdThreads, 1)
    lca_bwd_main(const __grid_constant__ CUtensorMap tm_x1, const __grid_constant__ CUtensorMap tm_x2,
                 const __grid_constant__ CUtensorMap tm_y1, const __grid_constant__ CUtensorMap tm_y2,
                 const __grid_constant__ CUtensorMap tm_x1g, const __grid_constant__ CUtensorMap tm_x2g,
                 const __grid_constant__ CUtensorMap tm_y1g, const __grid_constant__ CUtensorMap tm_y2g,
                 const BwdParams p) {
    using C = BwdCfg<D>;
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint8_t* sX = smem + C::kOffX;
    uint8_t* sY = smem + C::kOffY;
    float* sStat = reinterpret_cast<float*>(smem + C::kOffStat);
    uint32_t* sMask = reinterpret_cast<uint32_t*>(smem + C::kOffMask);
    uint64_t* bars = reinterpret_cast<uint64_t*>(smem + C::kOffBar);
    uint64_t* bar_x = bars + 0;
    uint64_t* bar_y = bars + 1;  // [2]
    uint64_t* bar_s = bars + 3;
    uint64_t* bar_o = bars + 4;
    uint32_t* sTmem = reinterpret_cast<uint32_t*>(smem + C::kOffMisc);
    volatile int* abort_flag = reinterpret_cast<volatile int*>(smem + C::kOffMisc + 4);

    const int tid = threadIdx.x;
    const int warp = tid >> 5;
    const BwdUnit un = bwd_decode(p, blockIdx.x);
    const int T = un.n_cont + un.n_comp;

    if (tid == 0) {
        ptx::mbar_init(bar_x, 1);
        ptx::mbar_init(&bar_y[0], 1);
        ptx::mbar_init(&bar_y[1], 1);
        ptx::mbar_init(bar_s, 1);
        ptx::mbar_init(bar_o, 1);
        *abort_flag = 0;
        ptx::fence_mbar_init();
    }
    if (warp == 0) {
        ptx::tmem_alloc(sTmem, kBwdTmemCols);
        ptx::tmem_relinquish();
    }
    ptx::tc_fence_before();
    __syncthreads();
    ptx::tc_fence_after();
    const uint32_t tmem = *sTmem;
    const uint32_t t_lane = tmem + ((uint32_t)(warp * 32) << 16);
    constexpr uint32_t kColS = 0, kColDP = 128, kColA = 256, kColB = 256 + D;

    // inner tile t: contiguous rows inner0 + 128 t, or compact tile t - n_cont
    auto load_inner = [&](int t) {
        const int st = t & 1;
        uint8_t* y = sY + st * 2 * C::kTileBytes;
        ptx::mbar_arrive_expect_tx(&bar_y[st], 2 * C::kTileBytes);
        if (t < un.n_cont) {
            const int r0 = un.inner0 + t * kBM;
            bwd_load_tile<D>(y, &tm_y1, &bar_y[st], false, r0, un.bh);
            bwd_load_tile<D>(y + C::kTileBytes, &tm_y2, &bar_y[st], false, r0, un.bh);
        } else {
            const int r0 = (t - un.n_cont) * kBM;
            bwd_load_tile<D>(y, &tm_y1g, &bar_y[st], true, r0, un.bh);
            bwd_load_tile<D>(y + C::kTileBytes, &tm_y2g, &bar_y[st], true, r0, un.bh);
        }
    };
    bool ok = true;
    auto wait = [&](uint64_t* bar, int parity) {
        if (!ok) return;
        ok = ptx::mbar_wait(bar, (uint32_t)parity & 1u, abort_flag, p.err, LCA_DEVERR_TIMEOUT_BACKWARD,
                            p.timeout_ns);
    };

    if (tid == 0) {
        ptx::prefetch_tmap(&tm_x1);
        ptx::prefetch_tmap(&tm_y1);
        ptx::mbar_arrive_expect_tx(bar_x, 2 * C::kTileBytes);
        if (un.all) {
            bwd_load_tile<D>(sX, &tm_x1g, bar_x, true, un.outer0, un.bh);
            bwd_load_tile<D>(sX + C::kTileBytes, &tm_x2g, bar_x, true, un.outer0, un.bh);
        } else {
            bwd_load_tile<D>(sX, &tm_x1, bar_x, false, un.outer0, un.bh);
            bwd_load_tile<D>(sX + C::kTileBytes, &tm_x2, bar_x, false, un.outer0, un.bh);
        }
        for (int t = 0; t < 2 && t < T; ++t) load_inner(t);
    }

    // the outer row of this thread: valid, and (dQ kernel) its LSE and D
    const int orow = un.outer0 + tid;  // band: absolute row / key; all: compact index
    const bool row_ok = un.all ? (orow < p.num_global) : (orow < p.n);
    float row_lse2 = 0.f, row_d = 0.f;
    if constexpr (!KM) {
        if (row_ok) {
            const size_t idx = un.all ? (size_t)un.bh * p.num_global + orow : (size_t)un.bh * p.n + orow;
            row_lse2 = un.all ? __ldg(p.lse2g + idx) : __ldg(p.lse2 + idx);
            row_d = un.all ? __ldg(p.dg + idx) : __ldg(p.dvec + idx);
        }
    }

    const uint32_t dhi = ptx::smem_desc_sw128_hi(1024);
    const uint32_t idesc_s = ptx::idesc_f16(BF16, kBM, kBM, false);
    const uint32_t idesc_acc = ptx::idesc_f16(BF16, kBM, D, true);

    // Every exit from this loop is block-uniform (__syncthreads_or on the threads' `ok`):
    // a bounded wait that gives up in one thread ends the loop for all of them.
    for (int t = 0; t < T; ++t) {
        const int st = t & 1;
        const bool cont = t < un.n_cont;
        const int tile0 = cont ? un.inner0 + t * kBM : (t - un.n_cont) * kBM;
        // inner rows of a contiguous band tile that are global tokens (excluded: they are
        // counted by the global-row / global-key units or the compact tiles)
        if (tid == 0) {
            uint32_t m[4] = {0u, 0u, 0u, 0u};
            if (cont && !un.all && p.num_global > 0) {
                int a = bwd_lower(p.gidx, p.num_global, tile0);
                for (; a < p.num_global; ++a) {
                    const int c = __ldg(p.gidx + a) - tile0;
                    if (c >= kBM) break;
                    m[c >> 5] |= 1u << (c & 31);
                }
            }
            sMask[0] = m[0];
            sMask[1] = m[1];
            sMask[2] = m[2];
            sMask[3] = m[3];
        }
        if constexpr (KM) {
            // LSE and D of the inner (query) rows
            float l2 = 0.f, dd = 0.f;
            if (cont) {
                const int i = tile0 + tid;
                if (i >= 0 && i < p.n) {
                    l2 = __ldg(p.lse2 + (size_t)un.bh * p.n + i);
                    dd = __ldg(p.dvec + (size_t)un.bh * p.n + i);
                }
            } else {
                const int g = tile0 + tid;
                if (g < p.num_global) {
                    l2 = __ldg(p.lse2g + (size_t)un.bh * p.num_global + g);
                    dd = __ldg(p.dg + (size_t)un.bh * p.num_global + g);
                }
            }
            sStat[tid] = l2;
            sStat[kBM + tid] = dd;
        }
        if (__syncthreads_or(!ok)) {
            ok = false;
            break;
        }

        // S = X1 Y1^T, dP = X2 Y2^T
        if (tid == 0) {
            if (t == 0) wait(bar_x, 0);
            wait(&bar_y[st], t >> 1);
            if (ok) {
                ptx::tc_fence_after();
                const uint32_t xs = ptx::smem_u32(sX);
                const uint32_t ys = ptx::smem_u32(sY + st * 2 * C::kTileBytes);
#pragma unroll
                for (int ks = 0; ks < D / 16; ++ks) {
                    const uint32_t off = ((ks >> 2) * kBwdPanel + (ks & 3) * 32) >> 4;
                    ptx::mma_f16_ss(tmem + kColS, ptx::desc_join(ptx::smem_desc_sw128_lo(xs, 0) + off, dhi),
                                    ptx::desc_join(ptx::smem_desc_sw128_lo(ys, 0) + off, dhi), idesc_s,
                                    ks > 0 ? 1u : 0u);
                }
#pragma unroll
                for (int ks = 0; ks < D / 16; ++ks) {
                    const uint32_t off = ((ks >> 2) * kBwdPanel + (ks & 3) * 32) >> 4;
                    ptx::mma_f16_ss(tmem + kColDP,
                                    ptx::desc_join(ptx::smem_desc_sw128_lo(xs + C::kTileBytes, 0) + off, dhi),
                                    ptx::desc_join(ptx::smem_desc_sw128_lo(ys + C::kTileBytes, 0) + off, dhi),
                                    idesc_s, ks > 0 ? 1u : 0u);
                }
                ptx::mma_commit(bar_s);
            }
        }
        wait(bar_s, t);
        if (__syncthreads_or(!ok)) {
            ok = false;
            break;
        }
        ptx::tc_fence_after();

        // this thread's visible columns of the tile: [lo, hi], minus the mask's
        int lo, hi;
        if (un.all) {
            lo = 0;
            hi = row_ok ? p.n - 1 - tile0 : -1;
        } else if (cont) {
            lo = orow - tile0 - p.window;
            if (lo < -tile0) lo = -tile0;
            hi = orow - tile0 + p.window;
            if (hi > p.n - 1 - tile0) hi = p.n - 1 - tile0;
            if (!row_ok) hi = -1;
        } else {
            lo = 0;
            hi = row_ok ? p.num_global - 1 - tile0 : -1;
        }
#pragma unroll
        for (int ch = 0; ch < 4; ++ch) {
            const uint32_t bits = range_bits(ch * 32, lo, hi) & ~sMask[ch];
            float s[32], dp[32];
            ptx::tmem_ld32(t_lane + kColS + ch * 32, s);
            ptx::tmem_ld32(t_lane + kColDP + ch * 32, dp);
            ptx::tmem_wait_ld();
            uint32_t pk[16], dk[16];
#pragma unroll
            for (int e = 0; e < 32; e += 2) {
                float pv[2], dv[2];
#pragma unroll
                for (int h = 0; h < 2; ++h) {
                    const int c = e + h;
                    float l2, dd;
                    if constexpr (KM) {
                        l2 = sStat[ch * 32 + c];
                        dd = sStat[kBM + ch * 32 + c];
                    } else {
                        l2 = row_lse2;
                        dd = row_d;
                    }
                    const float pr = ptx::ex2(fmaf(s[c], p.scale_log2, -l2));
                    const float pm = ((bits >> c) & 1u) ? pr : 0.f;
                    pv[h] = pm;
                    dv[h] = pm * (dp[c] - dd);
                }
                if constexpr (BF16) {
                    pk[e >> 1] = ptx::pack_bf16x2(pv[0], pv[1]);
                    dk[e >> 1] = ptx::pack_bf16x2(dv[0], dv[1]);
                } else {
                    pk[e >> 1] = ptx::pack_f16x2(pv[0], pv[1]);
                    dk[e >> 1] = ptx::pack_f16x2(dv[0], dv[1]);
                }
            }
            // packed pairs of keys [32 ch, 32 ch + 32) in the first 16 columns of the chunk
            if constexpr (KM) ptx::tmem_st16u(t_lane + kColS + ch * 32, pk);
            ptx::tmem_st16u(t_lane + kColDP + ch * 32, dk);
        }
        ptx::tmem_wait_st();
        ptx::tc_fence_before();
        __syncthreads();

        // accumulate: dQ += dS Y1 (dQ kernel); dV += P^T Y2, dK += dS^T Y1 (dK/dV kernel)
        if (tid == 0) {
            ptx::tc_fence_after();
            const uint32_t ys = ptx::smem_u32(sY + st * 2 * C::kTileBytes);
            const uint32_t y1lo = ptx::smem_desc_sw128_lo(ys, kBwdPanel);
            const uint32_t y2lo = ptx::smem_desc_sw128_lo(ys + C::kTileBytes, kBwdPanel);
#pragma unroll
            for (int kk = 0; kk < kBM / 16; ++kk) {
                const int key = 16 * kk;
                const uint32_t acol = (key >> 5) * 32 + ((key >> 4) & 1) * 8;
                const uint32_t acc = (t > 0 || kk > 0) ? 1u : 0u;
                const uint32_t boff = (uint32_t)(key * 128) >> 4;
                if constexpr (KM) {
                    ptx::mma_f16_ts(tmem + kColA, tmem + kColS + acol, ptx::desc_join(y2lo + boff, dhi), idesc_acc,
                                    acc);
                    ptx::mma_f16_ts(tmem + kColB, tmem + kColDP + acol, ptx::desc_join(y1lo + boff, dhi),
                                    idesc_acc, acc);
                } else {
                    ptx::mma_f16_ts(tmem + kColA, tmem + kColDP + acol, ptx::desc_join(y1lo + boff, dhi),
                                    idesc_acc, acc);
                }
            }
            ptx::mma_commit(bar_o);
            // S / dP are overwritten by the next tile's MMAs and stage st by tile t + 2:
            // both wait for these MMAs to finish
            wait(bar_o, t);
            if (ok && t + 2 < T) load_inner(t + 2);
        }
    }
    if (__syncthreads_or(!ok) || *abort_flag) ok = false;

    if (ok && T > 0) {
        ptx::tc_fence_after();
        // epilogue: this thread's outer row of the accumulators
        bool write = row_ok;
        float* dst_a = nullptr;
        float* dst_b = nullptr;
        if (un.all) {
            const size_t r = ((size_t)un.split * p.bh + un.bh) * p.num_global + orow;
            dst_a = p.part_a + r * D;
            if constexpr (KM) dst_b = p.part_b + r * D;
        } else {
            write = write && !bwd_is_global(p, orow);
            const size_t r = (size_t)un.bh * p.n + orow;
            dst_a = p.out_a + r * D;
            if constexpr (KM) dst_b = p.out_b + r * D;
        }
#pragma unroll
        for (int ch = 0; ch < D / 32; ++ch) {
            float a[32];
            ptx::tmem_ld32(t_lane + kColA + ch * 32, a);
            ptx::tmem_wait_ld();
            if (write) {
                // dQ and dK carry the scale, dV does not
                const float f = KM ? 1.f : p.scale;
#pragma unroll
                for (int e = 0; e < 32; e += 4)
                    *reinterpret_cast<float4*>(dst_a + ch * 32 + e) =
                        make_float4(a[e] * f, a[e + 1] * f, a[e + 2] * f, a[e + 3] * f);
            }
            if constexpr (KM) {
                float b[32];
                ptx::tmem_ld32(t_lane + kColB + ch * 32, b);
                ptx::tmem_wait_ld();
                if (write) {
#pragma unroll
                    for (int e = 0; e < 32; e += 4)
                        *reinterpret_cast<float4*>(dst_b + ch * 32 + e) =
                            make_float4(b[e] * p.scale, b[e + 1] * p.scale, b[e + 2] * p.scale, b[e + 3] * p.scale);
                }
            }
        }
    }
    ptx::tc_fence_before();
    __syncthreads();
    if (warp == 0) ptx::tmem_dealloc(tmem, kBwdTmemCols);
}

__global__ void __launch_bounds__(256) lca_bwd_indices(BwdIndexParams ip) {
    for (int i = threadIdx.x; i < ip.count; i += blockDim.x) ip.dst[i] = ip.idx[i];
}

// One warp per row (bh, i): D_i in fp32, the 16-bit dO row, LSE * log2 e; a global row also
// goes to the compact buffers.
template <int D>
__global__ void __launch_bounds__(256) lca_bwd_prep(BwdPrepParams pp) {
    constexpr int kPer = D / 32;
    const long long w = (long long)blockIdx.x * 8 + (threadIdx.x >> 5);
    const int lane = threadIdx.x & 31;
    if (w >= (long long)pp.bh * pp.n) return;
    const int bh = (int)(w / pp.n);
    const int i = (int)(w % pp.n);
    const size_t off = (size_t)w * D + lane * kPer;
    float dov[kPer], ov[kPer];
#pragma unroll
    for (int e = 0; e < kPer; ++e) {
        dov[e] = __ldg(pp.dout + off + e);
        ov[e] = __ldg(pp.o + off + e);
    }
    float dot = 0.f;
#pragma unroll
    for (int e = 0; e < kPer; ++e) dot = fmaf(dov[e], ov[e], dot);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) dot += __shfl_xor_sync(0xffffffffu, dot, o);
    uint32_t packed[kPer / 2];
#pragma unroll
    for (int e = 0; e < kPer; e += 2)
        packed[e / 2] = pp.bf16 ? ptx::pack_bf16x2(dov[e], dov[e + 1]) : ptx::pack_f16x2(dov[e], dov[e + 1]);
    uint16_t* d16 = static_cast<uint16_t*>(pp.dout16) + off;
    if constexpr (kPer == 2)
        *reinterpret_cast<uint32_t*>(d16) = packed[0];
    else
        *reinterpret_cast<uint2*>(d16) = make_uint2(packed[0], packed[1]);
    const float l2 = __ldg(pp.lse + w) * kLog2e;
    if (lane == 0) {
        pp.lse2[w] = l2;
        pp.dvec[w] = dot;
    }
    if (pp.num_global > 0) {
        int g = -1;
        if (lane == 0) {
            const int a = bwd_lower(pp.gidx, pp.num_global, i);
            if (a < pp.num_global && __ldg(pp.gidx + a) == i) g = a;
        }
        g = __shfl_sync(0xffffffffu, g, 0);
        if (g >= 0) {
            // compact [G][4][bh][d]: planes q, k, v, dO16
            uint16_t* cbase = static_cast<uint16_t*>(pp.compact);
            const uint16_t* src[3] = {static_cast<const uint16_t*>(pp.q), static_cast<const uint16_t*>(pp.k),
                                      static_cast<const uint16_t*>(pp.v)};
#pragma unroll
            for (int pl = 0; pl < 4; ++pl) {
                uint16_t* dst = cbase + (((size_t)g * 4 + pl) * pp.bh + bh) * D + lane * kPer;
                const uint16_t* s = pl < 3 ? src[pl] + off : d16;
#pragma unroll
                for (int e = 0; e < kPer; ++e) dst[e] = s[e];
            }
            if (lane == 0) {
                pp.lse2g[(size_t)bh * pp.num_global + g] = l2;
                pp.dg[(size_t)bh * pp.num_global + g] = dot;
            }
        }
    }
}

// One warp per (bh, compact row g): the sums of the split partials, written to row gidx[g].
template <int D>
__global__ void __launch_bounds__(256) lca_bwd_reduce(BwdReduceParams rp) {
    constexpr int kPer = D / 32;
    const long long w = (long long)blockIdx.x * 8 + (threadIdx.x >> 5);
    const int lane = threadIdx.x & 31;
    if (w >= (long long)rp.bh * rp.num_global) return;
    const int bh = (int)(w / rp.num_global);
    const int g = (int)(w % rp.num_global);
    const size_t stride = (size_t)rp.bh * rp.num_global * D;
    const size_t src = (size_t)w * D + lane * kPer;
    const size_t dst = ((size_t)bh * rp.n + __ldg(rp.gidx + g)) * D + lane * kPer;
    float q[kPer], k[kPer], v[kPer];
#pragma unroll
    for (int e = 0; e < kPer; ++e) q[e] = k[e] = v[e] = 0.f;
    for (int s = 0; s < rp.splits_q; ++s)
#pragma unroll
        for (int e = 0; e < kPer; ++e) q[e] += __ldg(rp.part_q + s * stride + src + e);
    for (int s = 0; s < rp.splits_k; ++s)
#pragma unroll
        for (int e = 0; e < kPer; ++e) {
            k[e] += __ldg(rp.part_k + s * stride + src + e);
            v[e] += __ldg(rp.part_v + s * stride + src + e);
        }
#pragma unroll
    for (int e = 0; e < kPer; ++e) {
        rp.dq[dst + e] = q[e];
        rp.dk[dst + e] = k[e];
        rp.dv[dst + e] = v[e];
    }
}

template <int D, bool BF16, bool KM>
cudaError_t launch_bwd_t(const BwdMaps& m, const BwdParams& p, cudaStream_t stream) {
    auto kern = lca_bwd_main<D, BF16, KM>;
    constexpr int smem = BwdCfg<D>::kSmemBytes;
    constexpr int kDevices = 64;
    static bool attr_set[kDevices];
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return e;
    if (dev < 0 || dev >= kDevices || !attr_set[dev]) {
        e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
        if (e != cudaSuccess) return e;
        if (dev >= 0 && dev < kDevices) attr_set[dev] = true;
    }
    kern<<<(unsigned)p.n_units, kBwdThreads, smem, stream>>>(m.x1, m.x2, m.y1, m.y2, m.x1g, m.x2g, m.y1g, m.y2g, p);
    return cudaGetLastError();
}

}  // namespace

cudaError_t launch_bwd_indices(const BwdIndexParams& ip, cudaStream_t stream) {
    if (ip.count <= 0) return cudaSuccess;
    if (ip.count > kBwdIndexChunk) return cudaErrorInvalidValue;
    lca_bwd_indices<<<1, 256, 0, stream>>>(ip);
    return cudaGetLastError();
}

cudaError_t launch_bwd_prep(int head_dim, const BwdPrepParams& pp, cudaStream_t stream) {
    const long long rows = (long long)pp.bh * pp.n;
    if (rows <= 0) return cudaSuccess;
    if ((rows + 7) / 8 > INT_MAX) return cudaErrorInvalidValue;
    const unsigned grid = (unsigned)((rows + 7) / 8);
    if (head_dim == 64)
        lca_bwd_prep<64><<<grid, 256, 0, stream>>>(pp);
    else if (head_dim == 128)
        lca_bwd_prep<128><<<grid, 256, 0, stream>>>(pp);
    else
        return cudaErrorInvalidValue;
    return cudaGetLastError();
}

cudaError_t launch_bwd_main(int head_dim, bool bf16, bool key_major, const BwdMaps& maps, const BwdParams& p,
                            cudaStream_t stream) {
    if (p.n_units <= 0) return cudaSuccess;
    if (head_dim == 64) {
        if (bf16) return key_major ? launch_bwd_t<64, true, true>(maps, p, stream) : launch_bwd_t<64, true, false>(maps, p, stream);
        return key_major ? launch_bwd_t<64, false, true>(maps, p, stream) : launch_bwd_t<64, false, false>(maps, p, stream);
    }
    if (head_dim == 128) {
        if (bf16) return key_major ? launch_bwd_t<128, true, true>(maps, p, stream) : launch_bwd_t<128, true, false>(maps, p, stream);
        return key_major ? launch_bwd_t<128, false, true>(maps, p, stream) : launch_bwd_t<128, false, false>(maps, p, stream);
    }
    return cudaErrorInvalidValue;
}

cudaError_t launch_bwd_reduce(int head_dim, const BwdReduceParams& rp, cudaStream_t stream) {
    const long long rows = (long long)rp.bh * rp.num_global;
    if (rows <= 0) return cudaSuccess;
    const unsigned grid = (unsigned)((rows + 7) / 8);
    if (head_dim == 64)
        lca_bwd_reduce<64><<<grid, 256, 0, stream>>>(rp);
    else if (head_dim == 128)
        lca_bwd_reduce<128><<<grid, 256, 0, stream>>>(rp);
    else
        return cudaErrorInvalidValue;
    return cudaGetLastError();
}

}  // namespace lca
