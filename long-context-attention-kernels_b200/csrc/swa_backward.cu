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
// The main kernels run a persistent grid (one CTA per SM, units taken round-robin).  Per
// 64-row inner tile, S = X1 Y1^T and dP = X2 Y2^T (tcgen05.mma, SS, both operands K-major from
// shared memory, 128 x 64 fp32 in TMEM) are turned by 16 warps into P and dS, packed to 16-bit
// pairs and stored back over S and dP (tcgen05.st); the TS MMAs then accumulate in TMEM
// (dQ += dS Y1; or dV += P^T Y2 and dK += dS^T Y1), reading Y1 / Y2 as MN-major B operands from
// the same shared tiles.  Three control warps issue the S/dP MMAs, issue the accumulating MMAs
// and load (TMA), each on its own SM sub-partition: a tcgen05.mma of M = 128, K = 16 takes ~96
// cycles of issue at N = 64, so one thread issuing both kinds set the pace.
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

constexpr int kBM = 128;                 // rows of an outer tile
constexpr int kBN = 64;                  // rows of an inner tile
constexpr int kCalcThreads = 512;        // four warpgroups, two per group of alternate inner tiles
constexpr int kBwdThreads = kCalcThreads + 96;  // plus three control warps (S/dP issue, accumulate issue, loads)
constexpr uint32_t kBwdTmemCols = 512;
constexpr float kLog2e = 1.4426950408889634f;

template <int D>
struct BwdCfg {
    static constexpr int kYStages = D == 64 ? 8 : 4;  // inner tiles in flight (TMA ring)
    static constexpr int kXBufs = D == 64 ? 2 : 1;    // outer tiles in flight (the next unit's)
    static constexpr int kXPanel = kBM * 128;       // 128 rows x 128 bytes
    static constexpr int kYPanel = kBN * 128;       // 64 rows x 128 bytes
    static constexpr int kXBytes = kBM * D * 2;     // one outer tile: D / 64 panels
    static constexpr int kYBytes = kBN * D * 2;     // one inner tile
    static constexpr int kOffX = 0;                              // [kXBufs][X1, X2]
    static constexpr int kOffY = kXBufs * 2 * kXBytes;           // [kYStages][Y1, Y2]
    static constexpr int kOffStat = kOffY + kYStages * 2 * kYBytes;  // [kYStages][2 (lse2, D)][kBN] floats
    static constexpr int kNumBars = 2 * kXBufs + 11 + 3 * kYStages;
    static constexpr int kOffBar = kOffStat + kYStages * 2 * kBN * 4;  // kNumBars barriers
    static constexpr int kOffMisc = kOffBar + kNumBars * 8;            // TMEM base, abort flag
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
    int n_cont;  // contiguous inner tiles (kBN rows each)
    int n_comp;  // compact inner tiles after them
};

// Units [0, n_units - n_band_units) are the global-row / global-key units (the longer kind,
// scheduled first so the short band units fill the tail), then the band units.
__device__ __forceinline__ BwdUnit bwd_decode(const BwdParams& p, int u) {
    BwdUnit un;
    const int n_all = p.n_units - p.n_band_units;
    u = u < n_all ? p.n_band_units + u : u - n_all;
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
        un.n_cont = (hi - lo + kBN) / kBN;
        un.n_comp = p.gi_tiles;
    } else {
        const int t = u - p.n_band_units;
        un.all = true;
        un.split = t % p.n_splits;
        const int rest = t / p.n_splits;
        un.outer0 = (rest % p.g_tiles) * kBM;
        un.bh = rest / p.g_tiles;
        un.inner0 = un.split * p.split_tiles * kBN;
        int tiles = (p.n - un.inner0 + kBN - 1) / kBN;
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

// 32-bit mask of the columns [c0, c0 + 32) that lie in [lo, hi].
__device__ __forceinline__ uint32_t range_bits(int c0, int lo, int hi) {
    const int a = lo - c0 > 0 ? lo - c0 : 0;
    const int b = hi - c0 < 31 ? hi - c0 : 31;
    if (a > b) return 0u;
    const uint32_t upto_b = (b == 31) ? 0xFFFFFFFFu : ((1u << (b + 1)) - 1u);
    return upto_b & ~((1u << a) - 1u);
}

// Bits of the rows [r0, r0 + 32) that are global tokens (r0 >= 0; the bitmap has a zero
// word past the last row).
__device__ __forceinline__ uint32_t global_bits(const uint32_t* __restrict__ bm, int r0) {
    const uint32_t w0 = __ldg(bm + (r0 >> 5)), w1 = __ldg(bm + (r0 >> 5) + 1);
    return __funnelshift_r(w0, w1, r0 & 31);
}

// One tile of `rows` rows (128-byte swizzled panels of `panel` bytes, D / 64 of them).
template <int D>
__device__ __forceinline__ void bwd_load_tile(uint8_t* dst, int panel, const CUtensorMap* map, uint64_t* bar,
                                              bool compact, int row0, int bh) {
#pragma unroll
    for (int pn = 0; pn < D / 64; ++pn) {
        if (compact)
            ptx::tma_load_3d(dst + pn * panel, map, bar, pn * 64, bh, row0);
        else
            ptx::tma_load_3d(dst + pn * panel, map, bar, pn * 64, row0, bh);
    }
}

// A persistent grid: CTA c takes units c, c + gridDim.x, ... (the longer global units come
// first, so the short band units fill the tail).  Warps 0-15 turn S and dP into P and dS and
// write each unit's result; three control warps, each on its own SM sub-partition, drive the
// rest (one lane each, except where noted):
//   warp 16 (S issuer): S = X1 Y1^T and dP = X2 Y2^T of every inner tile into TMEM buffer
//           g % NB (g counts the CTA's inner tiles across its units) once that buffer's
//           previous accumulating MMAs have finished (buf_free), so S/dP run up to NB - 1
//           tiles ahead of warps 0-15, into the next unit too;
//   warp 17 (accumulate issuer): once P/dS of a tile are written (p_full), dQ += dS Y1 (dQ
//           kernel) or dV += P^T Y2 and dK += dS^T Y1 (dK/dV kernel), then commits that free
//           the tile's buffer (buf_free) and ring stage (stage_free); a unit's first MMAs wait
//           until the previous unit's accumulators have been read out (acc_free), and its
//           last commit tells warps 0-15 that the accumulators are complete (acc_full);
//   warp 18 (producer): the outer tiles (kXBufs buffers, so the next unit's loads early at
//           d = 64) and the inner tiles through a TMA ring of kYStages stages (8 at d = 64, 4
//           at d = 128), stage g % kYStages refilled with tile g + kYStages once tile g's
//           accumulating MMAs are done; for the dK/dV kernel its 32 lanes also stage the inner
//           rows' LSE and D.
// S / dP sit in one of NB TMEM buffers (NB = 3, or 2 for the d = 128 dK/dV kernel, whose
// accumulators take 256 columns; S in columns [128 b, 128 b + 64), dP in
// [128 b + 64, 128 b + 128)).  Every barrier is waited once per phase, in order, and none can
// complete its next phase before its waiter has passed the current one.
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
    uint64_t* bars = reinterpret_cast<uint64_t*>(smem + C::kOffBar);
    constexpr int kYStages = C::kYStages;
    constexpr int NX = C::kXBufs;
    constexpr int NB = (KM && D == 128) ? 2 : 3;  // S/dP buffers in TMEM
    uint64_t* bar_x = bars;                 // [NX] the buffer's outer tiles loaded
    uint64_t* x_free = bars + NX;           // [NX] every S/dP MMA reading the buffer finished
    uint64_t* s_full = bars + 2 * NX;       // [NB] S/dP of the buffer computed
    uint64_t* p_full = s_full + 3;          // [NB] P/dS of the buffer written
    uint64_t* buf_free = p_full + 3;        // [NB] the buffer's accumulating MMAs finished
    uint64_t* acc_full = buf_free + 3;      // the unit's accumulating MMAs finished
    uint64_t* acc_free = acc_full + 1;      // the unit's accumulators read out
    uint64_t* bar_y = acc_free + 1;         // [kYStages] the stage's inner tiles loaded
    uint64_t* st_full = bar_y + kYStages;   // [kYStages] dK/dV kernel: the stage's LSE and D staged
    uint64_t* stage_free = st_full + kYStages;  // [kYStages] the stage's accumulating MMAs finished
    uint32_t* sTmem = reinterpret_cast<uint32_t*>(smem + C::kOffMisc);
    volatile int* abort_flag = reinterpret_cast<volatile int*>(smem + C::kOffMisc + 4);

    const int tid = threadIdx.x;
    const int warp = tid >> 5;
    const int lane = tid & 31;
    const int u_first = blockIdx.x, u_step = gridDim.x;

    if (tid == 0) {
        for (int i = 0; i < NX; ++i) {
            ptx::mbar_init(&bar_x[i], 1);
            ptx::mbar_init(&x_free[i], 1);
        }
        for (int i = 0; i < NB; ++i) {
            ptx::mbar_init(&s_full[i], 1);
            ptx::mbar_init(&p_full[i], kCalcThreads / 64);  // the warps of the tile's group
            ptx::mbar_init(&buf_free[i], 1);
        }
        ptx::mbar_init(acc_full, 1);
        ptx::mbar_init(acc_free, kCalcThreads / 32);
        for (int i = 0; i < kYStages; ++i) {
            ptx::mbar_init(&bar_y[i], 1);
            ptx::mbar_init(&st_full[i], 32);  // the producer warp's lanes
            ptx::mbar_init(&stage_free[i], 1);
        }
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
    constexpr uint32_t kColA = 128 * NB, kColB = 128 * NB + D;
    static_assert(128 * NB + (KM ? 2 * D : D) <= (int)kBwdTmemCols, "TMEM columns");

    bool ok = true;
    auto wait = [&](uint64_t* bar, int parity) {
        if (!ok) return;
        ok = ptx::mbar_wait(bar, (uint32_t)parity & 1u, abort_flag, p.err, LCA_DEVERR_TIMEOUT_BACKWARD,
                            p.timeout_ns);
    };
    // inner tile t of unit un: contiguous rows inner0 + kBN t, or compact tile t - n_cont
    auto tile_row0 = [&](const BwdUnit& un, int t) {
        return t < un.n_cont ? un.inner0 + t * kBN : (t - un.n_cont) * kBN;
    };

    const uint32_t dhi = ptx::smem_desc_sw128_hi(1024);
    if (warp == kCalcThreads / 32) {
        // ============================================================ S issuer
        const uint32_t idesc_s = ptx::idesc_f16(BF16, kBM, kBN, false);
        if (lane == 0) {
            int g = 0;
            for (int k = 0, u = u_first; u < p.n_units && ok; ++k, u += u_step) {
                const BwdUnit un = bwd_decode(p, u);
                const int T = un.n_cont + un.n_comp;
                const int xb = k % NX;
                wait(&bar_x[xb], (k / NX) & 1);
                const uint32_t xs = ptx::smem_u32(sX + xb * 2 * C::kXBytes);
                for (int t = 0; t < T; ++t, ++g) {
                    if (g >= NB) wait(&buf_free[g % NB], ((g - NB) / NB) & 1);
                    wait(&bar_y[g % kYStages], (g / kYStages) & 1);
                    if (!ok) break;
                    ptx::tc_fence_after();
                    const uint32_t col = (uint32_t)(g % NB) * 128;
                    const uint32_t ys = ptx::smem_u32(sY + (g % kYStages) * 2 * C::kYBytes);
#pragma unroll
                    for (int m = 0; m < 2; ++m) {
                        const uint32_t alo = ptx::smem_desc_sw128_lo(xs + m * C::kXBytes, 0);
                        const uint32_t blo = ptx::smem_desc_sw128_lo(ys + m * C::kYBytes, 0);
#pragma unroll
                        for (int ks = 0; ks < D / 16; ++ks) {
                            const uint32_t aoff = ((ks >> 2) * C::kXPanel + (ks & 3) * 32) >> 4;
                            const uint32_t boff = ((ks >> 2) * C::kYPanel + (ks & 3) * 32) >> 4;
                            ptx::mma_f16_ss(tmem + col + m * kBN, ptx::desc_join(alo + aoff, dhi),
                                            ptx::desc_join(blo + boff, dhi), idesc_s, ks > 0 ? 1u : 0u);
                        }
                    }
                    ptx::mma_commit(&s_full[g % NB]);
                }
                if (!ok) break;
                ptx::mma_commit(&x_free[xb]);  // the unit's outer tile is no longer read
            }
        }
    } else if (warp == kCalcThreads / 32 + 1) {
        // ============================================================ accumulate issuer
        const uint32_t idesc_acc = ptx::idesc_f16(BF16, kBM, D, true);
        if (lane == 0) {
            int g = 0;
            for (int k = 0, u = u_first; u < p.n_units && ok; ++k, u += u_step) {
                const BwdUnit un = bwd_decode(p, u);
                const int T = un.n_cont + un.n_comp;
                if (k >= 1) wait(acc_free, (k - 1) & 1);  // the previous unit's accumulators read out
                for (int t = 0; t < T; ++t, ++g) {
                    wait(&p_full[g % NB], (g / NB) & 1);
                    // the stage's loads (already complete: S/dP of the tile read them)
                    wait(&bar_y[g % kYStages], (g / kYStages) & 1);
                    if (!ok) break;
                    ptx::tc_fence_after();
                    // dQ += dS Y1 (dQ kernel); dV += P^T Y2, dK += dS^T Y1 (dK/dV kernel)
                    const uint32_t ys = ptx::smem_u32(sY + (g % kYStages) * 2 * C::kYBytes);
                    const uint32_t y1lo = ptx::smem_desc_sw128_lo(ys, C::kYPanel);
                    const uint32_t y2lo = ptx::smem_desc_sw128_lo(ys + C::kYBytes, C::kYPanel);
                    const uint32_t col_s = (uint32_t)(g % NB) * 128, col_dp = col_s + kBN;
#pragma unroll
                    for (int kk = 0; kk < kBN / 16; ++kk) {
                        const int key = 16 * kk;
                        const uint32_t acol = key;  // keys [key, key + 16): 8 packed columns from column key
                        const uint32_t acc = (t > 0 || kk > 0) ? 1u : 0u;
                        const uint32_t boff = (uint32_t)(key * 128) >> 4;
                        if constexpr (KM) {
                            ptx::mma_f16_ts(tmem + kColA, tmem + col_s + acol, ptx::desc_join(y2lo + boff, dhi),
                                            idesc_acc, acc);
                            ptx::mma_f16_ts(tmem + kColB, tmem + col_dp + acol, ptx::desc_join(y1lo + boff, dhi),
                                            idesc_acc, acc);
                        } else {
                            ptx::mma_f16_ts(tmem + kColA, tmem + col_dp + acol, ptx::desc_join(y1lo + boff, dhi),
                                            idesc_acc, acc);
                        }
                    }
                    ptx::mma_commit(&buf_free[g % NB]);
                    ptx::mma_commit(&stage_free[g % kYStages]);
                }
                if (!ok) break;
                ptx::mma_commit(acc_full);  // every accumulating MMA of the unit (and before it)
            }
        }
    } else if (warp == kCalcThreads / 32 + 2) {
        // ============================================================ producer
        // dK/dV kernel: LSE and D of inner tile t of unit un into stage g % kYStages (all lanes;
        // asynchronous copies, each lane's arrival on st_full fires when its copies have landed,
        // so the producer does not wait for the loads)
        auto stage_stats = [&](const BwdUnit& un, int t, int g) {
            if constexpr (KM) {
                float* st = sStat + (g % kYStages) * 2 * kBN;
                const bool cont = t < un.n_cont;
                const int tile0 = tile_row0(un, t);
                const float* l2src = cont ? p.lse2 + (size_t)un.bh * p.n : p.lse2g + (size_t)un.bh * p.num_global;
                const float* ddsrc = cont ? p.dvec + (size_t)un.bh * p.n : p.dg + (size_t)un.bh * p.num_global;
                const int rows = cont ? p.n : p.num_global;
#pragma unroll
                for (int h = 0; h < kBN / 32; ++h) {
                    const int c = h * 32 + lane;
                    const bool valid = tile0 + c < rows;
                    const int i = valid ? tile0 + c : 0;  // (rows past the end are zero-filled)
                    ptx::cp_async_4(st + c, l2src + i, valid);
                    ptx::cp_async_4(st + kBN + c, ddsrc + i, valid);
                }
                ptx::cp_async_mbar_arrive(&st_full[g % kYStages]);
            }
        };
        if (lane == 0) {
            ptx::prefetch_tmap(&tm_x1);
            ptx::prefetch_tmap(&tm_y1);
        }
        int g = 0;
        for (int k = 0, u = u_first; u < p.n_units; ++k, u += u_step) {
            const BwdUnit un = bwd_decode(p, u);
            const int T = un.n_cont + un.n_comp;
            const int xb = k % NX;
            if (lane == 0) {
                if (k >= NX) wait(&x_free[xb], ((k - NX) / NX) & 1);
                if (ok) {
                    uint8_t* x = sX + xb * 2 * C::kXBytes;
                    ptx::mbar_arrive_expect_tx(&bar_x[xb], 2 * C::kXBytes);
                    bwd_load_tile<D>(x, C::kXPanel, un.all ? &tm_x1g : &tm_x1, &bar_x[xb], un.all, un.outer0, un.bh);
                    bwd_load_tile<D>(x + C::kXBytes, C::kXPanel, un.all ? &tm_x2g : &tm_x2, &bar_x[xb], un.all,
                                     un.outer0, un.bh);
                }
            }
            for (int t = 0; t < T; ++t, ++g) {
                // stage g % kYStages is free once tile g - kYStages's accumulating MMAs are done
                // (the P / dS warps read its stats before that tile's p_full, so before those MMAs)
                if (lane == 0 && g >= kYStages) wait(&stage_free[g % kYStages], ((g - kYStages) / kYStages) & 1);
                __syncwarp();
                ok = __shfl_sync(0xffffffffu, ok ? 1 : 0, 0) != 0;
                if (!ok) break;
                if (lane == 0) {
                    const int st = g % kYStages;
                    uint8_t* y = sY + st * 2 * C::kYBytes;
                    ptx::mbar_arrive_expect_tx(&bar_y[st], 2 * C::kYBytes);
                    const bool cont = t < un.n_cont;
                    const int r0 = tile_row0(un, t);
                    bwd_load_tile<D>(y, C::kYPanel, cont ? &tm_y1 : &tm_y1g, &bar_y[st], !cont, r0, un.bh);
                    bwd_load_tile<D>(y + C::kYBytes, C::kYPanel, cont ? &tm_y2 : &tm_y2g, &bar_y[st], !cont, r0,
                                     un.bh);
                }
                stage_stats(un, t, g);
            }
            if (!ok) break;
        }
    } else {
        // ============================================================ P / dS warps
        // Two groups of eight warps take alternate inner tiles (tile g goes to group g % 2), so
        // one group's TMEM loads and stores and barrier waits overlap the other group's
        // arithmetic, and each thread's per-tile bookkeeping covers 32 columns.  Warpgroups
        // 2 grp and 2 grp + 1 form group grp; both span the 128 TMEM lanes, one per column half.
        const int r = tid & (kBM - 1);  // outer row <-> TMEM lane
        const int q = tid >> 7;         // warpgroup; the epilogue's column quarter
        const int grp = q >> 1;
        const int c0 = (q & 1) * 32;    // this thread's columns of its group's tiles
        const uint32_t t_lane = tmem + ((uint32_t)((warp & 3) * 32) << 16);
        int g = 0;
        for (int k = 0, u = u_first; u < p.n_units && ok; ++k, u += u_step) {
            const BwdUnit un = bwd_decode(p, u);
            const int T = un.n_cont + un.n_comp;
            const int orow = un.outer0 + r;  // band: absolute row / key; all: compact index
            const bool row_ok = un.all ? (orow < p.num_global) : (orow < p.n);
            float row_lse2 = 0.f, row_d = 0.f;
            if constexpr (!KM) {
                if (row_ok) {
                    const size_t idx = un.all ? (size_t)un.bh * p.num_global + orow : (size_t)un.bh * p.n + orow;
                    row_lse2 = un.all ? __ldg(p.lse2g + idx) : __ldg(p.lse2 + idx);
                    row_d = un.all ? __ldg(p.dg + idx) : __ldg(p.dvec + idx);
                }
            }
            const bool use_bitmap = !un.all && p.num_global > 0;
            for (int t = 0; t < T; ++t, ++g) {
                if ((g & 1) != grp) continue;
                const int b = g % NB;
                const bool cont = t < un.n_cont;
                const int tile0 = tile_row0(un, t);
                // global rows / keys among a contiguous band tile's 32 columns of this thread
                // (counted by the global units or the compact tiles)
                const uint32_t gbits = (use_bitmap && cont) ? global_bits(p.gbitmap, tile0 + c0) : 0u;
                // the outer row's visible columns of the tile (this thread's are [c0, c0 + 32)): [lo, hi]
                int lo, hi;
                if (un.all) {
                    lo = 0;
                    hi = row_ok ? p.n - 1 - tile0 : -1;
                } else if (cont) {
                    lo = orow - tile0 - p.window;
                    hi = orow - tile0 + p.window;
                    if (hi > p.n - 1 - tile0) hi = p.n - 1 - tile0;
                    if (!row_ok) hi = -1;
                } else {
                    lo = 0;
                    hi = row_ok ? p.num_global - 1 - tile0 : -1;
                }
                const uint32_t bits = range_bits(c0, lo, hi) & ~gbits;
                wait(&s_full[b], (g / NB) & 1);
                if constexpr (KM) wait(&st_full[g % kYStages], (g / kYStages) & 1);
                ok = __all_sync(0xffffffffu, ok);  // warp-uniform, so the __syncwarp below is reached by all
                if (!ok) break;
                ptx::tc_fence_after();
                // the packed 16-bit pairs of each 16 columns go to the first 8 of them (the other
                // column half may still be reading its own)
                const uint32_t col_s = (uint32_t)b * 128 + c0;
                const uint32_t col_dp = col_s + kBN;
                const float* st = sStat + (g % kYStages) * 2 * kBN;
                uint32_t pk[2][8], dk[2][8];
#pragma unroll
                for (int j = 0; j < 2; ++j) {
                    float s[16], dp[16];
                    ptx::tmem_ld16(t_lane + col_s + 16 * j, s);
                    ptx::tmem_ld16(t_lane + col_dp + 16 * j, dp);
                    ptx::tmem_wait_ld();
#pragma unroll
                    for (int e = 0; e < 16; e += 2) {
                        float pv[2], dv[2];
#pragma unroll
                        for (int h = 0; h < 2; ++h) {
                            const int c = 16 * j + e + h;
                            float l2, dd;
                            if constexpr (KM) {
                                l2 = st[c0 + c];
                                dd = st[kBN + c0 + c];
                            } else {
                                l2 = row_lse2;
                                dd = row_d;
                            }
                            const float pr = ptx::ex2(fmaf(s[e + h], p.scale_log2, -l2));
                            const float pm = ((bits >> c) & 1u) ? pr : 0.f;
                            pv[h] = pm;
                            dv[h] = pm * (dp[e + h] - dd);
                        }
                        if constexpr (BF16) {
                            pk[j][e >> 1] = ptx::pack_bf16x2(pv[0], pv[1]);
                            dk[j][e >> 1] = ptx::pack_bf16x2(dv[0], dv[1]);
                        } else {
                            pk[j][e >> 1] = ptx::pack_f16x2(pv[0], pv[1]);
                            dk[j][e >> 1] = ptx::pack_f16x2(dv[0], dv[1]);
                        }
                    }
                }
                // keys [c0 + 16 j, c0 + 16 j + 16) as 8 packed columns from column c0 + 16 j: the
                // A operand of one 16-key step of the accumulating MMAs
#pragma unroll
                for (int j = 0; j < 2; ++j) {
                    if constexpr (KM) ptx::tmem_st8u(t_lane + col_s + 16 * j, pk[j]);
                    ptx::tmem_st8u(t_lane + col_dp + 16 * j, dk[j]);
                }
                ptx::tmem_wait_st();
                ptx::tc_fence_before();
                __syncwarp();
                if (lane == 0) ptx::mbar_arrive(&p_full[b]);
            }
            if (!ok) break;
            // the unit's result: this thread's outer row, columns [D/4 q, D/4 (q + 1)) of the
            // accumulators, once every accumulating MMA of the unit has finished
            wait(acc_full, k & 1);
            ok = __all_sync(0xffffffffu, ok);
            if (!ok) break;
            ptx::tc_fence_after();
            bool write = row_ok;
            float* dst_a = nullptr;
            float* dst_b = nullptr;
            if (un.all) {
                const size_t rr = ((size_t)un.split * p.bh + un.bh) * p.num_global + orow;
                dst_a = p.part_a + rr * D;
                if constexpr (KM) dst_b = p.part_b + rr * D;
            } else {
                if (write && p.num_global > 0 && ((__ldg(p.gbitmap + (orow >> 5)) >> (orow & 31)) & 1u))
                    write = false;
                const size_t rr = (size_t)un.bh * p.n + orow;
                dst_a = p.out_a + rr * D;
                if constexpr (KM) dst_b = p.out_b + rr * D;
            }
#pragma unroll
            for (int ch = 0; ch < D / 64; ++ch) {
                const int cc = (q * (D / 64) + ch) * 16;
                float a[16];
                ptx::tmem_ld16(t_lane + kColA + cc, a);
                float bb[16];
                if constexpr (KM) ptx::tmem_ld16(t_lane + kColB + cc, bb);
                ptx::tmem_wait_ld();
                if (write) {
                    // dQ and dK carry the scale, dV does not
                    const float f = KM ? 1.f : p.scale;
#pragma unroll
                    for (int e = 0; e < 16; e += 4)
                        *reinterpret_cast<float4*>(dst_a + cc + e) =
                            make_float4(a[e] * f, a[e + 1] * f, a[e + 2] * f, a[e + 3] * f);
                    if constexpr (KM) {
#pragma unroll
                        for (int e = 0; e < 16; e += 4)
                            *reinterpret_cast<float4*>(dst_b + cc + e) = make_float4(
                                bb[e] * p.scale, bb[e + 1] * p.scale, bb[e + 2] * p.scale, bb[e + 3] * p.scale);
                    }
                }
            }
            // the accumulators may be overwritten by the next unit
            ptx::tc_fence_before();
            __syncwarp();
            if (lane == 0) ptx::mbar_arrive(acc_free);
        }
    }
    if (__syncthreads_or(!ok) || *abort_flag) ok = false;
    ptx::tc_fence_before();
    __syncthreads();
    if (warp == 0) ptx::tmem_dealloc(tmem, kBwdTmemCols);
}

__global__ void __launch_bounds__(256) lca_bwd_indices(BwdIndexParams ip) {
    if (ip.clear_bitmap) {
        for (int i = threadIdx.x; i < ip.bitmap_words; i += blockDim.x) ip.bitmap[i] = 0u;
        __syncthreads();
    }
    for (int i = threadIdx.x; i < ip.count; i += blockDim.x) {
        const int g = ip.idx[i];
        ip.dst[i] = g;
        atomicOr(ip.bitmap + (g >> 5), 1u << (g & 31));
    }
}

// D / 4 threads per row (bh, i), four columns each (16-byte loads): D_i in fp32, the 16-bit
// dO row, LSE * log2 e; a global row also goes to the compact buffers.
template <int D>
__global__ void __launch_bounds__(256) lca_bwd_prep(BwdPrepParams pp) {
    constexpr int kLanes = D / 4;             // threads of one row
    constexpr int kRows = 256 / kLanes;       // rows of one block
    const int sub = threadIdx.x % kLanes;
    const long long w = (long long)blockIdx.x * kRows + threadIdx.x / kLanes;
    const bool live = w < (long long)pp.bh * pp.n;
    const long long wr = live ? w : 0;
    const int bh = (int)(wr / pp.n);
    const int i = (int)(wr % pp.n);
    const size_t off = (size_t)wr * D + sub * 4;
    float4 dov = make_float4(0.f, 0.f, 0.f, 0.f), ov = dov;
    if (live) {
        dov = __ldg(reinterpret_cast<const float4*>(pp.dout + off));
        ov = __ldg(reinterpret_cast<const float4*>(pp.o + off));
    }
    float dot = dov.x * ov.x + dov.y * ov.y + dov.z * ov.z + dov.w * ov.w;
#pragma unroll
    for (int o = kLanes / 2; o > 0; o >>= 1) dot += __shfl_xor_sync(0xffffffffu, dot, o, kLanes);
    if (!live) return;
    const uint2 packed = pp.bf16 ? make_uint2(ptx::pack_bf16x2(dov.x, dov.y), ptx::pack_bf16x2(dov.z, dov.w))
                                 : make_uint2(ptx::pack_f16x2(dov.x, dov.y), ptx::pack_f16x2(dov.z, dov.w));
    uint16_t* d16 = static_cast<uint16_t*>(pp.dout16) + off;
    *reinterpret_cast<uint2*>(d16) = packed;
    const float l2 = __ldg(pp.lse + w) * kLog2e;
    if (sub == 0) {
        pp.lse2[w] = l2;
        pp.dvec[w] = dot;
    }
    if (pp.num_global > 0) {
        // (rows of one block share a bitmap word or two; the bitmap is written before this launch)
        if (((__ldg(pp.gbitmap + (i >> 5)) >> (i & 31)) & 1u) == 0u) return;
        const int g = bwd_lower(pp.gidx, pp.num_global, i);
        // compact [G][4][bh][d]: planes q, k, v, dO16
        uint16_t* cbase = static_cast<uint16_t*>(pp.compact);
        const uint16_t* src[3] = {static_cast<const uint16_t*>(pp.q), static_cast<const uint16_t*>(pp.k),
                                  static_cast<const uint16_t*>(pp.v)};
#pragma unroll
        for (int pl = 0; pl < 4; ++pl) {
            uint2* dst = reinterpret_cast<uint2*>(cbase + (((size_t)g * 4 + pl) * pp.bh + bh) * D + sub * 4);
            *dst = pl < 3 ? *reinterpret_cast<const uint2*>(src[pl] + off) : packed;
        }
        if (sub == 0) {
            pp.lse2g[(size_t)bh * pp.num_global + g] = l2;
            pp.dg[(size_t)bh * pp.num_global + g] = dot;
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
    const unsigned grid = (unsigned)(p.n_units < p.grid ? p.n_units : p.grid);
    kern<<<grid, kBwdThreads, smem, stream>>>(m.x1, m.x2, m.y1, m.y2, m.x1g, m.x2g, m.y1g, m.y2g, p);
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
    if (head_dim != 64 && head_dim != 128) return cudaErrorInvalidValue;
    const long long per_block = 256 / (head_dim / 4);
    if ((rows + per_block - 1) / per_block > INT_MAX) return cudaErrorInvalidValue;
    const unsigned grid = (unsigned)((rows + per_block - 1) / per_block);
    if (head_dim == 64)
        lca_bwd_prep<64><<<grid, 256, 0, stream>>>(pp);
    else
        lca_bwd_prep<128><<<grid, 256, 0, stream>>>(pp);
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
