// swa_kernels.cu -- sm_100a kernels for sliding-window + global-token attention forward.
//
// Semantics (the contract of python/long_context_attention/__init__.py:24-53 in the
// reference): key j is visible to query i iff |i - j| <= w, or j is a global token, or
// i is a global token.  Output is fp32 softmax(scale * Q K^T restricted to that mask) V.
//
// Three launches per forward:
//   1. lca_gather_globals   : copies the G global rows of Q, K, V into compact,
//                             zero-padded [bh][gpad][d] buffers (gpad = 128 * ceil(G/128))
//                             and writes the sorted index list.
//   2. lca_swa_main         : one warp-specialised CTA per work unit.  Two unit kinds:
//        band unit   : 128 query rows of one (batch, head).  Key tiles: the band
//                      [q0 - w, q0 + 127 + w] in 128-key tiles (out-of-band tiles are
//                      never issued), then the compact global-key tiles, masked so a
//                      global key inside a row's band is counted only once (by the band).
//                      Replaces csrc/sliding_window_attention.cu:48-160 and the
//                      query-to-global-keys + combine kernels (csrc/global_attention.cu:
//                      104-152, csrc/combine.cu:18-56) with their merge done in-register.
//        global-row unit : 128 compact global queries against one contiguous split of
//                      all n keys, producing a normalised partial O and its log-sum-exp.
//                      Replaces csrc/global_attention.cu:29-96.
//   3. lca_combine_global_rows : log-sum-exp merge of the splits, written over the
//                      global rows of O (and LSE).
//
// Main-kernel CTA layout (192 threads):
//   warps 0-3  softmax / epilogue: thread r owns query row r of the tile, which is TMEM
//              lane r; S rows are read with tcgen05.ld, P is written to shared memory
//              (bf16/f16, 128-byte swizzled K-major), O stays in TMEM.
//   warp 4     TMA producer: Q tile once, then K_j / V_j tiles into a ring of slots.
//   warp 5     TMEM allocator + single-thread tcgen05.mma issuer:
//              S = Q K_j^T (M=128, N<=128, K=d) and O += P_j V_j (M=128, N=d, K<=128).
#include <cuda.h>
#include <cuda_runtime.h>
#include <cuda_fp16.h>
#include <cuda_bf16.h>
#include <cstdint>
#include <climits>

#include "sm100_ptx.cuh"
#include "swa_kernels.h"

namespace lca {

// Device-side error word: the first bounded wait that gives up records its code here.
__device__ int g_error_word = 0;

namespace {

constexpr int BM = 128;            // query rows per tile == TMEM lanes
constexpr int BN = 128;            // keys per tile
constexpr int kThreads = 192;
constexpr int kSoftmaxThreads = 128;
constexpr int kTmemCols = 256;     // S: columns [0,128), O: columns [128, 128 + d)
constexpr int kSCol = 0;
constexpr int kOCol = 128;
constexpr int kPanelBytes = 128 * 128;  // 128 rows x 128 bytes: one swizzle panel
constexpr float kLn2 = 0.6931471805599453f;
// The running max used for exponentiation is only raised when a new score exceeds it by
// more than this many powers of two; results are exact either way because l and O are
// accumulated against the same reference max.
constexpr float kRescaleThreshold = 8.0f;

// Shared-memory plan per CTA (all regions 1024-byte aligned):
//   Q tile | K/V ring of kSlots tiles | P (one 128x128 16-bit tile, or two for split P) | control
// For bf16 inputs P is kept as P_hi + P_lo (two bf16 tiles, P_hi = rn(p), P_lo = rn(p - P_hi))
// and P*V is issued twice into the same accumulator: a single bf16 P would carry ~1.5e-3
// relative L2 error into O, the split carries ~2^-16.  fp16 P is already accurate enough.
template <int D, bool BF16>
struct Cfg {
    static constexpr bool kSplitP = BF16;
    static constexpr int kPanels = D / 64;
    static constexpr int kTileBytes = BM * D * 2;
    static constexpr int kSlots = 3;
    static constexpr int kPTileBytes = BM * BN * 2;
    static constexpr int kPBytes = kPTileBytes * (kSplitP ? 2 : 1);
    static constexpr int kOffQ = 0;
    static constexpr int kOffSlots = kOffQ + kTileBytes;
    static constexpr int kOffP = kOffSlots + kSlots * kTileBytes;
    static constexpr int kOffCtl = kOffP + kPBytes;
    static constexpr int kCtlBytes = 1024;
    static constexpr int kSmemBytes = kOffCtl + kCtlBytes + 1024;  // +1024 for base alignment
    static constexpr int kMinBlocks = (2 * (kSmemBytes + 1024) <= 228 * 1024) ? 2 : 1;
};

struct Ctl {
    uint64_t q_full;
    uint64_t full[4];
    uint64_t empty[4];
    uint64_t s_full;
    uint64_t s_free;
    uint64_t p_full;
    uint64_t pv_done;
    uint64_t mma_drained;
    uint32_t tmem_base;
    int abort_flag;
    int epi_go;
};

// Description of one key tile of a work unit.
struct TileInfo {
    int row0;        // first key row (band/grow: absolute key index; global: compact row)
    int ncols;       // columns handed to the MMA (multiple of 16)
    bool global_key; // compact global-key tile
};

struct Unit {
    bool grow;       // global-row unit
    int bh;          // (batch * heads) index
    int qrow0;       // first query row (band: absolute; grow: compact global row)
    int split;       // grow: split index
    int num_band;    // band tiles (or split tiles for grow)
    int first_k0;    // key index of the first band/split tile
    int num_gtiles;  // global-key tiles (band units only)
    int ntiles;
};

__device__ __forceinline__ Unit decode_unit(const MainParams& p) {
    Unit u;
    int cta = blockIdx.x;
    if (cta < p.n_grow_ctas) {
        u.grow = true;
        u.split = cta % p.n_splits;
        int rest = cta / p.n_splits;
        int gt = rest % p.g_tiles;
        u.bh = rest / p.g_tiles;
        u.qrow0 = gt * BM;
        u.first_k0 = u.split * p.split_tiles * BN;
        int remaining = (p.n - u.first_k0 + BN - 1) / BN;
        u.num_band = remaining < p.split_tiles ? remaining : p.split_tiles;
        u.num_gtiles = 0;
    } else {
        u.grow = false;
        u.split = 0;
        int t = cta - p.n_grow_ctas;
        int qt = t % p.q_tiles;
        u.bh = t / p.q_tiles;
        u.qrow0 = qt * BM;
        // Band span for rows [q0, q0+127] is keys [q0 - w, q0 + 127 + w]: (2w + 128) keys
        // cut into 128-key tiles starting exactly at q0 - w, so the first and last tiles
        // carry the triangular band edges.  Tiles wholly outside [0, n) are never issued.
        long long kstart = (long long)u.qrow0 - p.window;
        long long span_tiles = ((long long)2 * p.window + BM + BN - 1) / BN;
        long long t_first = 0;
        if (kstart < 0) t_first = (-kstart) / BN;  // first tile whose end is > 0
        long long t_last = span_tiles - 1;
        long long last_ok = ((long long)p.n - 1 - kstart);
        if (last_ok / BN < t_last) t_last = last_ok / BN;
        u.first_k0 = (int)(kstart + t_first * BN);
        u.num_band = (int)(t_last - t_first + 1);
        u.num_gtiles = p.g_tiles;
    }
    u.ntiles = u.num_band + u.num_gtiles;
    return u;
}

__device__ __forceinline__ TileInfo tile_info(const MainParams& p, const Unit& u, int j) {
    TileInfo ti;
    if (j < u.num_band) {
        ti.row0 = u.first_k0 + j * BN;
        ti.ncols = BN;
        ti.global_key = false;
    } else {
        int gt = j - u.num_band;
        ti.row0 = gt * BN;
        int cnt = p.num_global - gt * BN;
        if (cnt > BN) cnt = BN;
        ti.ncols = (cnt + 15) & ~15;
        ti.global_key = true;
    }
    return ti;
}

// All 32 lanes wait; the warp proceeds only if every lane saw the phase complete, so
// warp-collective tcgen05 instructions that follow are never reached divergently.
__device__ __forceinline__ bool warp_wait(uint64_t* bar, uint32_t parity, volatile int* abort_flag, int* err,
                                          int code, uint64_t tmo) {
    const bool r = ptx::mbar_wait(bar, parity, abort_flag, err, code, tmo);
    return __all_sync(0xffffffffu, r);
}

__device__ __forceinline__ uint32_t swz128(int row, int chunk16) {
    // byte offset of 16-byte chunk `chunk16` (0..7) of row `row` in a 128-byte-swizzled panel
    return (uint32_t)(row * 128 + ((chunk16 ^ (row & 7)) << 4));
}

template <int D, bool BF16>
__global__ void __launch_bounds__(kThreads, Cfg<D, BF16>::kMinBlocks)
    lca_swa_main(const __grid_constant__ CUtensorMap tm_q, const __grid_constant__ CUtensorMap tm_k,
                 const __grid_constant__ CUtensorMap tm_v, const __grid_constant__ CUtensorMap tm_qg,
                 const __grid_constant__ CUtensorMap tm_kg, const __grid_constant__ CUtensorMap tm_vg,
                 const __grid_constant__ CUtensorMap tm_o, const __grid_constant__ CUtensorMap tm_po,
                 const MainParams p) {
    using C = Cfg<D, BF16>;
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint8_t* sQ = smem + C::kOffQ;
    uint8_t* sSlots = smem + C::kOffSlots;
    uint8_t* sP = smem + C::kOffP;
    Ctl* ctl = reinterpret_cast<Ctl*>(smem + C::kOffCtl);

    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;
    const Unit u = decode_unit(p);
    volatile int* abort_flag = &ctl->abort_flag;

    if (threadIdx.x == 0) {
        ptx::mbar_init(&ctl->q_full, 1);
        for (int s = 0; s < C::kSlots; ++s) {
            ptx::mbar_init(&ctl->full[s], 1);
            ptx::mbar_init(&ctl->empty[s], 1);
        }
        ptx::mbar_init(&ctl->s_full, 1);
        ptx::mbar_init(&ctl->s_free, 4);
        ptx::mbar_init(&ctl->p_full, 4);
        ptx::mbar_init(&ctl->pv_done, 1);
        ptx::mbar_init(&ctl->mma_drained, 1);
        ctl->abort_flag = 0;
        ptx::fence_mbar_init();
    }
    if (warp == 5) {
        ptx::tmem_alloc(&ctl->tmem_base, kTmemCols);
        ptx::tmem_relinquish();
    }
    ptx::tc_fence_before();
    __syncthreads();
    ptx::tc_fence_after();
    const uint32_t tmem = ctl->tmem_base;
    const uint64_t tmo = p.timeout_ns;

    if (warp == 4) {
        // ------------------------------------------------------------ TMA producer
        if (ptx::elect_one()) {
            const CUtensorMap* mq = u.grow ? &tm_qg : &tm_q;
            ptx::prefetch_tmap(mq);
            ptx::prefetch_tmap(&tm_k);
            ptx::prefetch_tmap(&tm_v);
            ptx::mbar_arrive_expect_tx(&ctl->q_full, C::kTileBytes);
#pragma unroll
            for (int pn = 0; pn < C::kPanels; ++pn)
                ptx::tma_load_3d(sQ + pn * kPanelBytes, mq, &ctl->q_full, pn * 64, u.qrow0, u.bh);
            int issued = 0;
            bool ok = true;
            for (int j = 0; j < u.ntiles && ok; ++j) {
                const TileInfo ti = tile_info(p, u, j);
                for (int kv = 0; kv < 2; ++kv) {
                    const int idx = 2 * j + kv;
                    const int slot = idx % C::kSlots;
                    if (idx >= C::kSlots) {
                        if (!ptx::mbar_wait(&ctl->empty[slot], ((idx / C::kSlots) + 1) & 1, abort_flag, p.err,
                                            LCA_DEVERR_TIMEOUT_PRODUCER, tmo)) {
                            ok = false;
                            break;
                        }
                    }
                    const CUtensorMap* m = ti.global_key ? (kv ? &tm_vg : &tm_kg) : (kv ? &tm_v : &tm_k);
                    uint8_t* dst = sSlots + slot * C::kTileBytes;
                    ptx::mbar_arrive_expect_tx(&ctl->full[slot], C::kTileBytes);
#pragma unroll
                    for (int pn = 0; pn < C::kPanels; ++pn)
                        ptx::tma_load_3d(dst + pn * kPanelBytes, m, &ctl->full[slot], pn * 64, ti.row0, u.bh);
                    ++issued;
                }
            }
            // Drain: every issued copy must land before the CTA may exit.
            ptx::mbar_wait(&ctl->q_full, 0, nullptr, p.err, LCA_DEVERR_TIMEOUT_DRAIN, tmo);
            int first = issued - C::kSlots;
            if (first < 0) first = 0;
            for (int idx = first; idx < issued; ++idx)
                ptx::mbar_wait(&ctl->full[idx % C::kSlots], (idx / C::kSlots) & 1, nullptr, p.err,
                               LCA_DEVERR_TIMEOUT_DRAIN, tmo);
        }
    } else if (warp == 5) {
        // ------------------------------------------------------------ MMA issuer
        if (ptx::elect_one()) {
            const uint32_t idesc_s_full = ptx::idesc_f16(BF16, BM, BN, false);
            const uint32_t sq = ptx::smem_u32(sQ);
            const uint32_t sp = ptx::smem_u32(sP);
            const uint32_t sslots = ptx::smem_u32(sSlots);
            bool ok = ptx::mbar_wait(&ctl->q_full, 0, abort_flag, p.err, LCA_DEVERR_TIMEOUT_MMA, tmo);

            auto issue_pv = [&](int j) -> bool {
                const TileInfo ti = tile_info(p, u, j);
                const int idx = 2 * j + 1;
                const int slot = idx % C::kSlots;
                if (!ptx::mbar_wait(&ctl->full[slot], (idx / C::kSlots) & 1, abort_flag, p.err,
                                    LCA_DEVERR_TIMEOUT_MMA, tmo))
                    return false;
                if (!ptx::mbar_wait(&ctl->p_full, j & 1, abort_flag, p.err, LCA_DEVERR_TIMEOUT_MMA, tmo))
                    return false;
                ptx::tc_fence_after();
                const uint32_t idesc_pv = ptx::idesc_f16(BF16, BM, D, true);
                const uint32_t vbase = sslots + slot * C::kTileBytes;
                const int ksteps = ti.ncols / 16;
#pragma unroll 1
                for (int part = 0; part < (C::kSplitP ? 2 : 1); ++part) {
                    const uint32_t pbase = sp + part * C::kPTileBytes;
                    for (int kk = 0; kk < ksteps; ++kk) {
                        const uint64_t adesc =
                            ptx::smem_desc_sw128(pbase + (kk >> 2) * kPanelBytes + (kk & 3) * 32, 0, 1024);
                        const uint64_t bdesc = ptx::smem_desc_sw128(vbase + kk * 16 * 128, kPanelBytes, 1024);
                        ptx::mma_f16_ss(tmem + kOCol, adesc, bdesc, idesc_pv,
                                        (j > 0 || part > 0 || kk > 0) ? 1u : 0u);
                    }
                }
                ptx::mma_commit(&ctl->pv_done);
                ptx::mma_commit(&ctl->empty[slot]);
                return true;
            };

            for (int j = 0; j < u.ntiles && ok; ++j) {
                const TileInfo ti = tile_info(p, u, j);
                const int idx = 2 * j;
                const int slot = idx % C::kSlots;
                if (!ptx::mbar_wait(&ctl->full[slot], (idx / C::kSlots) & 1, abort_flag, p.err,
                                    LCA_DEVERR_TIMEOUT_MMA, tmo)) {
                    ok = false;
                    break;
                }
                if (j > 0 &&
                    !ptx::mbar_wait(&ctl->s_free, (j - 1) & 1, abort_flag, p.err, LCA_DEVERR_TIMEOUT_MMA, tmo)) {
                    ok = false;
                    break;
                }
                ptx::tc_fence_after();
                const uint32_t idesc_s = (ti.ncols == BN) ? idesc_s_full : ptx::idesc_f16(BF16, BM, ti.ncols, false);
                const uint32_t kbase = sslots + slot * C::kTileBytes;
#pragma unroll
                for (int ks = 0; ks < D / 16; ++ks) {
                    const uint32_t off = (ks >> 2) * kPanelBytes + (ks & 3) * 32;
                    const uint64_t adesc = ptx::smem_desc_sw128(sq + off, 0, 1024);
                    const uint64_t bdesc = ptx::smem_desc_sw128(kbase + off, 0, 1024);
                    ptx::mma_f16_ss(tmem + kSCol, adesc, bdesc, idesc_s, ks > 0 ? 1u : 0u);
                }
                ptx::mma_commit(&ctl->s_full);
                ptx::mma_commit(&ctl->empty[slot]);
                if (j > 0 && !issue_pv(j - 1)) {
                    ok = false;
                    break;
                }
            }
            if (ok && u.ntiles > 0) issue_pv(u.ntiles - 1);
            // Drain: all tcgen05 ops issued by this thread complete before TMEM is freed.
            ptx::mma_commit(&ctl->mma_drained);
            ptx::mbar_wait(&ctl->mma_drained, 0, nullptr, p.err, LCA_DEVERR_TIMEOUT_DRAIN, tmo);
        }
    } else {
        // ------------------------------------------------------------ softmax warps
        const int r = threadIdx.x;  // row within the tile == TMEM lane
        const uint32_t t_lane = tmem + ((uint32_t)(warp * 32) << 16);
        const int qi = u.qrow0 + r;  // band: absolute query row
        const float sl2 = p.scale_log2;
        const uint32_t sp = ptx::smem_u32(sP);
        float m = -INFINITY;  // reference max (log2 units)
        float l = 0.f;
        bool ok = true;
        int j = 0;
        for (; j < u.ntiles; ++j) {
            const TileInfo ti = tile_info(p, u, j);
            if (!warp_wait(&ctl->s_full, j & 1, abort_flag, p.err, LCA_DEVERR_TIMEOUT_SOFTMAX, tmo)) {
                ok = false;
                break;
            }
            ptx::tc_fence_after();
            float s[BN];
#pragma unroll
            for (int c = 0; c < 4; ++c) {
                if (c * 32 < ti.ncols) {
                    float tmp[32];
                    ptx::tmem_ld32(t_lane + kSCol + c * 32, tmp);
#pragma unroll
                    for (int e = 0; e < 32; ++e) s[c * 32 + e] = tmp[e];
                } else {
#pragma unroll
                    for (int e = 0; e < 32; ++e) s[c * 32 + e] = 0.f;
                }
            }
            ptx::tmem_wait_ld();
            ptx::tc_fence_before();
            __syncwarp();
            if (lane == 0) ptx::mbar_arrive(&ctl->s_free);

            // ---- mask + scale into log2 units
            float mt = -INFINITY;
            if (!ti.global_key) {
                // visible columns kk in [lo, hi]
                int lo, hi;
                if (u.grow) {
                    lo = 0;
                    hi = p.n - 1 - ti.row0;
                } else {
                    int jlo = qi - p.window;
                    if (jlo < 0) jlo = 0;
                    long long jhi = (long long)qi + p.window;
                    if (jhi > p.n - 1) jhi = p.n - 1;
                    lo = jlo - ti.row0;
                    hi = (int)(jhi - ti.row0);
                }
                if (lo <= 0 && hi >= BN - 1) {
#pragma unroll
                    for (int c = 0; c < BN; ++c) {
                        s[c] *= sl2;
                        mt = fmaxf(mt, s[c]);
                    }
                } else {
#pragma unroll
                    for (int c = 0; c < BN; ++c) {
                        const bool vis = (c >= lo) && (c <= hi);
                        s[c] = vis ? s[c] * sl2 : -INFINITY;
                        mt = fmaxf(mt, s[c]);
                    }
                }
            } else {
                const int gbase = ti.row0;
                const int gcnt = p.num_global - gbase;
#pragma unroll
                for (int c = 0; c < BN; ++c) {
                    bool vis = false;
                    if (c < gcnt) {
                        const int g = __ldg(p.gidx + gbase + c);
                        const int dlt = qi - g;
                        vis = (dlt > p.window) || (dlt < -p.window);
                    }
                    s[c] = vis ? s[c] * sl2 : -INFINITY;
                    mt = fmaxf(mt, s[c]);
                }
            }

            // ---- online softmax with lazy rescale
            float alpha = 1.f;
            bool rescale = false;
            if (mt > m + kRescaleThreshold || (m == -INFINITY && mt > -INFINITY)) {
                const float m_new = mt;
                alpha = (m == -INFINITY) ? 0.f : ptx::ex2(m - m_new);
                rescale = (m != -INFINITY);
                m = m_new;
                l *= alpha;
            }
            const float m_use = (m == -INFINITY) ? 0.f : m;
            float lsum = 0.f;
#pragma unroll
            for (int c = 0; c < BN; ++c) {
                s[c] = ptx::ex2(s[c] - m_use);
                lsum += s[c];
            }
            l += lsum;

            // ---- P buffer and O are in use by PV_{j-1} until it completes
            if (j > 0) {
                if (!warp_wait(&ctl->pv_done, (j - 1) & 1, abort_flag, p.err, LCA_DEVERR_TIMEOUT_SOFTMAX, tmo)) {
                    ok = false;
                    break;
                }
                ptx::tc_fence_after();
                if (__any_sync(0xffffffffu, rescale)) {
                    const float a = rescale ? alpha : 1.f;
#pragma unroll
                    for (int c = 0; c < D / 32; ++c) {
                        float o[32];
                        ptx::tmem_ld32(t_lane + kOCol + c * 32, o);
                        ptx::tmem_wait_ld();
#pragma unroll
                        for (int e = 0; e < 32; ++e) o[e] *= a;
                        ptx::tmem_st32(t_lane + kOCol + c * 32, o);
                    }
                    ptx::tmem_wait_st();
                }
            }
            // ---- write P (row r, keys 0..127) into the swizzled K-major P buffer(s)
#pragma unroll
            for (int cc = 0; cc < BN / 8; ++cc) {
                const uint32_t off = (cc >> 3) * kPanelBytes + swz128(r, cc & 7);
                uint32_t w[4];
                if (BF16) {
                    uint32_t lo[4];
#pragma unroll
                    for (int e = 0; e < 4; ++e) {
                        const float a = s[cc * 8 + 2 * e], b = s[cc * 8 + 2 * e + 1];
                        w[e] = ptx::pack_bf16x2(a, b);
                        const float ha = __uint_as_float(w[e] << 16);
                        const float hb = __uint_as_float(w[e] & 0xFFFF0000u);
                        lo[e] = ptx::pack_bf16x2(a - ha, b - hb);
                    }
                    ptx::st_shared_v4(sp + C::kPTileBytes + off, lo[0], lo[1], lo[2], lo[3]);
                } else {
#pragma unroll
                    for (int e = 0; e < 4; ++e) w[e] = ptx::pack_f16x2(s[cc * 8 + 2 * e], s[cc * 8 + 2 * e + 1]);
                }
                ptx::st_shared_v4(sp + off, w[0], w[1], w[2], w[3]);
            }
            ptx::fence_proxy_async_smem();
            ptx::tc_fence_before();
            __syncwarp();
            if (lane == 0) ptx::mbar_arrive(&ctl->p_full);
        }

        // ---- wait for the last PV, then decide CTA-uniformly (among the softmax warps)
        // whether to run the epilogue: it contains named barriers, so either all four
        // warps enter it or none does.
        if (ok && u.ntiles > 0)
            warp_wait(&ctl->pv_done, (u.ntiles - 1) & 1, abort_flag, p.err, LCA_DEVERR_TIMEOUT_SOFTMAX, tmo);
        ptx::named_bar_sync(1, kSoftmaxThreads);
        if (threadIdx.x == 0) ctl->epi_go = (*abort_flag == 0) ? 1 : 0;
        ptx::named_bar_sync(1, kSoftmaxThreads);

        // ---- epilogue: O / l -> fp32 via swizzled staging panels + TMA store
        if (ctl->epi_go && u.ntiles > 0) {
            ptx::tc_fence_after();
            const float inv_l = 1.f / l;
            const CUtensorMap* mo = u.grow ? &tm_po : &tm_o;
            const int oz = u.grow ? (u.split * p.bh + u.bh) : u.bh;
#pragma unroll
            for (int c = 0; c < D / 32; ++c) {
                uint8_t* stage = sP + (c & 1) * kPanelBytes;
                if (c >= 2) {
                    if (threadIdx.x == 0) ptx::tma_store_wait_read<1>();
                    ptx::named_bar_sync(1, kSoftmaxThreads);
                }
                float o[32];
                ptx::tmem_ld32(t_lane + kOCol + c * 32, o);
                ptx::tmem_wait_ld();
                const uint32_t sbase = ptx::smem_u32(stage);
#pragma unroll
                for (int q = 0; q < 8; ++q) {
                    ptx::st_shared_v4(sbase + swz128(r, q), __float_as_uint(o[q * 4 + 0] * inv_l),
                                      __float_as_uint(o[q * 4 + 1] * inv_l), __float_as_uint(o[q * 4 + 2] * inv_l),
                                      __float_as_uint(o[q * 4 + 3] * inv_l));
                }
                ptx::fence_proxy_async_smem();
                ptx::named_bar_sync(1, kSoftmaxThreads);
                if (threadIdx.x == 0) {
                    ptx::tma_store_3d(mo, stage, c * 32, u.qrow0, oz);
                    ptx::tma_store_commit();
                }
            }
            const float lse = (((m == -INFINITY) ? 0.f : m) + __log2f(l)) * kLn2;
            if (u.grow) {
                p.part_lse[((size_t)u.split * p.bh + u.bh) * p.gpad + u.qrow0 + r] = lse;
            } else if (p.lse != nullptr && qi < p.n) {
                p.lse[(size_t)u.bh * p.n + qi] = lse;
            }
            if (threadIdx.x == 0) ptx::tma_store_wait_all();
        }
    }

    ptx::tc_fence_before();
    __syncthreads();
    ptx::tc_fence_after();
    if (warp == 5) ptx::tmem_dealloc(tmem, kTmemCols);
}

// ------------------------------------------------------------------------ gather

template <int D>
__global__ void __launch_bounds__(256) lca_gather_globals(const uint16_t* __restrict__ q,
                                                          const uint16_t* __restrict__ k,
                                                          const uint16_t* __restrict__ v, GatherParams gp) {
    // one warp per (bh, compact row); 16-byte chunks
    constexpr int kChunks = D * 2 / 16;
    const long long w = (long long)blockIdx.x * 8 + (threadIdx.x >> 5);
    const int lane = threadIdx.x & 31;
    if (w >= (long long)gp.count * gp.bh) return;
    const int row = (int)(w % gp.count);
    const int bh = (int)(w / gp.count);
    const int g = gp.first + row;  // compact row index
    const bool live = g < gp.num_global;
    const int src_row = live ? gp.idx[row] : 0;
    if (bh == 0 && lane == 0) gp.gidx_out[g] = live ? src_row : INT_MAX;
    const size_t src_off = ((size_t)bh * gp.n + src_row) * D;
    const size_t dst_off = ((size_t)bh * gp.gpad + g) * D;
    for (int c = lane; c < 3 * kChunks; c += 32) {
        const int which = c / kChunks;
        const int cc = c % kChunks;
        const uint16_t* src = which == 0 ? q : (which == 1 ? k : v);
        uint16_t* dst = which == 0 ? gp.qg : (which == 1 ? gp.kg : gp.vg);
        uint4 val = make_uint4(0, 0, 0, 0);
        if (live) val = *reinterpret_cast<const uint4*>(src + src_off + cc * 8);
        *reinterpret_cast<uint4*>(dst + dst_off + cc * 8) = val;
    }
}

// ------------------------------------------------------------------------ combine

template <int D>
__global__ void __launch_bounds__(128) lca_combine_global_rows(CombineParams cp) {
    // one warp per (bh, global row)
    const long long w = (long long)blockIdx.x * 4 + (threadIdx.x >> 5);
    const int lane = threadIdx.x & 31;
    if (w >= (long long)cp.num_global * cp.bh) return;
    const int g = (int)(w % cp.num_global);
    const int bh = (int)(w / cp.num_global);
    constexpr int kPer = D / 32;
    float mx = -INFINITY;
    for (int s = 0; s < cp.n_splits; ++s)
        mx = fmaxf(mx, cp.part_lse[((size_t)s * cp.bh + bh) * cp.gpad + g]);
    float acc[kPer];
#pragma unroll
    for (int e = 0; e < kPer; ++e) acc[e] = 0.f;
    float wsum = 0.f;
    for (int s = 0; s < cp.n_splits; ++s) {
        const size_t prow = (size_t)s * cp.bh + bh;
        const float w = __expf(cp.part_lse[prow * cp.gpad + g] - mx);
        wsum += w;
        const float* po = cp.part_o + (prow * cp.gpad + g) * D;
#pragma unroll
        for (int e = 0; e < kPer; ++e) acc[e] += w * po[lane + 32 * e];
    }
    const int row = cp.gidx[g];
    float* out = cp.o + ((size_t)bh * cp.n + row) * D;
    const float inv = 1.f / wsum;
#pragma unroll
    for (int e = 0; e < kPer; ++e) out[lane + 32 * e] = acc[e] * inv;
    if (cp.lse != nullptr && lane == 0) cp.lse[(size_t)bh * cp.n + row] = mx + __logf(wsum);
}

}  // namespace

// ------------------------------------------------------------------------ launchers

template <int D, bool BF16>
static cudaError_t launch_main_t(const TensorMaps& tm, const MainParams& p, int grid, cudaStream_t stream) {
    auto kern = lca_swa_main<D, BF16>;
    const int smem = Cfg<D, BF16>::kSmemBytes;
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
    if (e != cudaSuccess) return e;
    kern<<<grid, kThreads, smem, stream>>>(tm.q, tm.k, tm.v, tm.qg, tm.kg, tm.vg, tm.o, tm.po, p);
    return cudaGetLastError();
}

cudaError_t launch_main(int head_dim, bool bf16, const TensorMaps& tm, const MainParams& p, int grid,
                        cudaStream_t stream) {
    if (head_dim == 64) return bf16 ? launch_main_t<64, true>(tm, p, grid, stream) : launch_main_t<64, false>(tm, p, grid, stream);
    if (head_dim == 128) return bf16 ? launch_main_t<128, true>(tm, p, grid, stream) : launch_main_t<128, false>(tm, p, grid, stream);
    return cudaErrorInvalidValue;
}

cudaError_t launch_gather(int head_dim, const void* q, const void* k, const void* v, const GatherParams& gp,
                          int bh, cudaStream_t stream) {
    (void)bh;
    const long long rows = (long long)gp.count * gp.bh;
    if (rows <= 0) return cudaSuccess;
    const unsigned grid = (unsigned)((rows + 7) / 8);
    if (head_dim == 64)
        lca_gather_globals<64><<<grid, 256, 0, stream>>>(static_cast<const uint16_t*>(q), static_cast<const uint16_t*>(k),
                                                         static_cast<const uint16_t*>(v), gp);
    else if (head_dim == 128)
        lca_gather_globals<128><<<grid, 256, 0, stream>>>(static_cast<const uint16_t*>(q), static_cast<const uint16_t*>(k),
                                                          static_cast<const uint16_t*>(v), gp);
    else
        return cudaErrorInvalidValue;
    return cudaGetLastError();
}

cudaError_t launch_combine(int head_dim, const CombineParams& cp, cudaStream_t stream) {
    const long long rows = (long long)cp.num_global * cp.bh;
    if (rows <= 0) return cudaSuccess;
    const unsigned grid = (unsigned)((rows + 3) / 4);
    if (head_dim == 64)
        lca_combine_global_rows<64><<<grid, 128, 0, stream>>>(cp);
    else if (head_dim == 128)
        lca_combine_global_rows<128><<<grid, 128, 0, stream>>>(cp);
    else
        return cudaErrorInvalidValue;
    return cudaGetLastError();
}

int main_smem_bytes(int head_dim, bool bf16) {
    if (head_dim == 64) return bf16 ? Cfg<64, true>::kSmemBytes : Cfg<64, false>::kSmemBytes;
    return bf16 ? Cfg<128, true>::kSmemBytes : Cfg<128, false>::kSmemBytes;
}

cudaError_t error_word_address(int** out) {
    void* p = nullptr;
    cudaError_t e = cudaGetSymbolAddress(&p, g_error_word);
    *out = static_cast<int*>(p);
    return e;
}

}  // namespace lca
