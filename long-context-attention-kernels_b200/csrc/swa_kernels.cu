// swa_kernels.cu -- sm_100a kernels for sliding-window + global-token attention forward.
//
// Semantics (the contract of python/long_context_attention/__init__.py:24-53 in the
// reference): key j is visible to query i iff |i - j| <= w, or j is a global token, or
// i is a global token.  Output is fp32 softmax(scale * Q K^T restricted to that mask) V.
//
// Three launches per forward:
//   1. lca_gather_globals : copies the G global rows of Q, K, V into one compact
//                           [G][3][bh][d] buffer (TMA reads rows >= G as zeros) and
//                           writes the sorted index list.
//   2. lca_swa_main       : persistent, one CTA per SM, looping over work units (after its
//                           first, each CTA takes the next index from a launch-wide counter
//                           when the workspace has one, else round-robin; the TMA warp
//                           publishes it to the other roles through a shared-memory ring):
//        band unit      : two adjacent 128-row query tiles A, B of one (batch, head).
//                         Key tiles: the band [q0 - w, q0 + 255 + w] in 128-key tiles
//                         starting at q0 - lead (lead = w, or w rounded up to 128 for a
//                         sequence shard; A uses the first ceil((lead+w+128)/128) of
//                         them, B the same count shifted by one; each tile is loaded
//                         once for both), out-of-band and out-of-range tiles are never
//                         issued; then the compact global-key tiles, masked so a global
//                         key inside a row's band is counted once (by the band).
//                         Replaces csrc/sliding_window_attention.cu:48-160 and the
//                         query-to-global-keys + combine kernels (csrc/global_attention.cu:
//                         104-152, csrc/combine.cu:18-56), merged in the online softmax.
//        global-row unit: the compact global queries (one 128-row tile, loaded as both A
//                         and B) against one contiguous split of the keys (all n, or the
//                         shard's own), A taking the even key tiles and B the odd ones;
//                         each writes a normalised partial O and its log-sum-exp.
//                         Replaces csrc/global_attention.cu:29-96.
//   3. lca_combine_global_rows : log-sum-exp merge of the partials, written over the
//                           global rows of O (and LSE), or, for a sequence shard, into a
//                           per-shard partial that a second merge across shards finishes.
// Sequence shards add lca_pack_halo (the K / V rows the neighbours need as their halo).
//
// Main-kernel CTA layout.  Each query tile X (A or B) is served by H softmax warpgroups
// (H = 2 for d = 64, 1 for d = 128); warpgroup (X, h) owns key columns
// [128h/H, 128(h+1)/H) of every S tile of X and runs an independent online softmax over
// them into its own accumulator O_{X,h}; the H partial results of a row are merged by
// log-sum-exp in the epilogue.  Thread r of a warpgroup <-> query row r <-> TMEM lane r.
//   d = 64 : warps 0-15 softmax (A0, A1, B0, B1), warp 16 TMA producer, warps 17/18 MMA
//            issuers for A/B, warp 19 idle (640 threads; setmaxnreg: warpgroup 4 drops
//            to 64 registers, warpgroups 0-3 rise to 104; 128*64 + 512*104 = 640*96, the
//            launch allocation)
//   d = 128: warps 0-7 softmax (A, B), warp 8 TMA, warps 9/10 MMA issuers for A/B, warp 11
//            idle
//            (384 threads; setmaxnreg: warpgroup 2 drops to 72 registers, warpgroups 0-1
//            rise to 216; 128*72 + 256*216 = 384*168, the launch allocation)
// TMEM (512 columns): S_A [0,128), S_B [128,256), then O_{A,0..H-1}, O_{B,0..H-1}, d each.
// P overwrites S in place: warpgroup (X, h) writes its 16-bit P (hi pairs, then lo pairs
// for bf16) into its own S columns, and P*V reads it as the TMEM A operand.
// Each query tile has its own MMA-issuing thread, which issues PV_X(j) then S_X(j+1):
// while one tile's softmax runs, the tensor cores work for the other.  tcgen05 ops
// issued by one thread execute in order, so S_X(j+1) never overwrites P_X(j) before
// PV_X(j) read it, and the commit that signals S_X(j+1) also covers PV_X(j), so O_X is
// stable whenever its softmax warps see a new S.
#include <cuda.h>
#include <cuda_runtime.h>
#include <cuda_fp16.h>
#include <cuda_bf16.h>
#include <cstdint>
#include <algorithm>
#include <climits>
#include <cstdlib>
#include <utility>

#include "sm100_ptx.cuh"
#include "swa_kernels.h"
#include "trace.cuh"

namespace lca {

// Device-side error word: the first bounded wait that gives up records its code here.
__device__ int g_error_word = 0;

// trace events from lane 0 of a warp (no code unless built with LCA_TRACE)
#define LCA_TRACE_LANE0(code)                  \
    do {                                       \
        if (lane == 0) LCA_TRACE_EVENT(code); \
    } while (0)

namespace {

constexpr int BM = 128;            // query rows per tile == TMEM lanes
constexpr int BN = 128;            // keys per tile
constexpr int kWgThreads = 128;
constexpr int kTmemCols = 512;
constexpr int kPanelBytes = 128 * 128;  // 128 rows x 128 bytes: one swizzle panel
constexpr int kMaxSlots = 8;            // K / V ring slots (barrier pairs in Ctl)
constexpr int kUnitRing = 4;            // work-unit indices the producer publishes ahead
constexpr float kLn2 = 0.6931471805599453f;
// The running max used for exponentiation is only raised when a new score exceeds it by
// more than this many powers of two; results are exact either way because l and O are
// accumulated against the same reference max.
constexpr float kRescaleThreshold = 8.0f;
// Build options for measured alternatives (the defaults are the fastest measured):
//   LCA_D64_HALVES     softmax warpgroups per query tile at d = 64 (2, or 1 as at d = 128)
//   LCA_FAST_EXP_D64   the exponent pass before the max pass at d = 64 (spills at 104 registers)
//   LCA_POLY_MASK_D64 / LCA_POLY_MASK_D128   pairs of each 8-pair group exponentiated on the
//                      FMA pipe (Cfg::kPolyMask)
#ifndef LCA_D64_HALVES
#define LCA_D64_HALVES 2
#endif
#ifndef LCA_FAST_EXP_D64
#define LCA_FAST_EXP_D64 0
#endif
#ifndef LCA_POLY_MASK_D64
#define LCA_POLY_MASK_D64 0u
#endif
#ifndef LCA_POLY_MASK_D128
#define LCA_POLY_MASK_D128 0u
#endif

// For bf16 inputs P is split as P_hi + P_lo (P_hi = rn_bf16(p), P_lo = rn_bf16(p - P_hi))
// and P*V is issued twice into the same accumulator: a single bf16 P carries ~1.5e-3
// relative L2 error into O, the split ~2^-16.  fp16 P is accurate enough on its own, so the
// V16 variant (bf16 inputs whose V has an fp16 copy in the workspace that holds every value
// without loss that matters) writes fp16 P and runs P*V once, from the copy.
template <int D, bool BF16, bool V16 = false>
struct Cfg {
    static constexpr bool kSplitP = BF16 && !V16;
    // Pairs of each 8-pair (16-key) group whose exponentials run as a polynomial on the FMA
    // pipe instead of the MUFU unit (bit e: pair e), so the two pipes share the exponent
    // pass.  fp16 P only: the polynomial's relative error (8.6e-5) is below half an fp16
    // ulp but above the 16-bit precision of the split bf16 P.
    static constexpr unsigned kPolyMask = kSplitP ? 0u : (D == 64 ? LCA_POLY_MASK_D64 : LCA_POLY_MASK_D128);
    static constexpr int kHalves = (D == 64) ? LCA_D64_HALVES : 1;  // softmax warpgroups per query tile
    // Each S tile is two 64-key chains (S -> P -> P*V per chain).  At d = 64 each chain has
    // its own warpgroup and accumulator; at d = 128 one warpgroup runs both chains in turn
    // into one accumulator, so the second chain's S is ready while the first one's P*V and
    // next S run.
    static constexpr int kChains = 2;
    static constexpr int kCols = BN / kChains;             // S columns per chain
    static constexpr int kSoftmaxWarps = 8 * kHalves;
    // Exponentiate against the current reference max before knowing the row max (the max
    // pass then runs only when an argument exceeds the rescale threshold).  The scores stay
    // live through the pass, which the 104-register softmax warps of d = 64 cannot afford.
    static constexpr bool kFastExp = (kHalves == 1) || LCA_FAST_EXP_D64;
    static constexpr int kTmaWarp = kSoftmaxWarps;
    static constexpr int kMmaWarp = kSoftmaxWarps + 1;
    // softmax warpgroups, then one control warpgroup (TMA warp, two MMA warps, one idle)
    static constexpr int kThreads = (kSoftmaxWarps + 4) * 32;
    // registers per thread: at launch, after setmaxnreg in the softmax / control warpgroups
    static constexpr int kRegsLaunch = (kHalves == 2) ? 96 : 168;
    static constexpr int kRegsSoftmax = (kHalves == 2) ? 104 : 216;
    static constexpr int kRegsControl = (kHalves == 2) ? 64 : 72;
    static constexpr int kEpiCols = D / kHalves;           // output columns per warpgroup
    static constexpr int kPanels = D / 64;
    static constexpr int kTileBytes = BM * D * 2;
    static constexpr int kSlots = (D == 64) ? 7 : 3;  // K / V ring: one K or V tile per slot
    static constexpr int kStagePanels = (kHalves == 2) ? 1 : 2;  // epilogue staging panels per softmax warpgroup
    static constexpr int kStageBytes = kStagePanels * kPanelBytes;
    static constexpr int kOffQ = 0;
    static constexpr int kOffSlots = kOffQ + 2 * kTileBytes;
    static constexpr int kOffStage = kOffSlots + kSlots * kTileBytes;
    static constexpr int kOffCtl = kOffStage + 2 * kHalves * kStageBytes;
    static constexpr int kCtlBytes = 1024;
    static constexpr int kOffXchg = kOffCtl + kCtlBytes;    // (m, l) rows exchanged by the halves
    static constexpr int kXchgBytes = (kHalves == 2) ? 2 * 2 * 2 * 128 * 2 * 4 : 0;
    // sorted global indices for the per-row searches, when at most kSmemGlobals (d = 64 has
    // the shared memory to spare)
    static constexpr int kSmemGlobals = (D == 64) ? 2048 : 0;
    static constexpr int kOffGidx = kOffXchg + kXchgBytes;
    static constexpr int kSmemBytes = kOffGidx + kSmemGlobals * 4 + 1024;  // +1024 for base alignment
    static constexpr int kOCol = 256;
    static_assert(128 * kRegsControl + kSoftmaxWarps * 32 * kRegsSoftmax == kThreads * kRegsLaunch,
                  "register split must match the launch allocation");
    static_assert(kThreads * kRegsLaunch <= 65536, "launch allocation exceeds the register file");
    static_assert(kOCol + 2 * kHalves * D <= kTmemCols, "TMEM columns");
    static_assert(kSmemBytes <= 227 * 1024, "shared memory per CTA");
    static_assert(kSlots <= kMaxSlots, "ring barriers");
};

struct Ctl {
    uint64_t q_full[2];
    uint64_t q_empty[2];
    uint64_t kv_full[kMaxSlots];
    uint64_t kv_empty[kMaxSlots];
    uint64_t s_full[2][2];   // [query tile][chain]: S columns of the chain ready
    uint64_t p_full[2][2];   // [query tile][chain]: P of the chain written
    uint64_t pv_done[2][2];  // [query tile][chain]: P*V of the chain completed (one phase per member tile)
    uint64_t o_full[2];
    uint64_t o_free[2];
    uint64_t mma_drained[2];
    uint64_t unit_full[kUnitRing];   // the producer published the slot's unit index
    uint64_t unit_empty[kUnitRing];  // every other role has read it
    int unit_ring[kUnitRing];
    uint32_t tmem_base;
    int abort_flag;
};

static_assert(sizeof(Ctl) <= 1024, "control block");

struct Unit {
    bool grow;        // global-row unit
    bool active[2];   // query tile A / B has work
    int bh;           // (batch * heads) index
    int qrow[2];      // first query row of A / B (band: local; grow: compact)
    int ntiles;       // issued key tiles
    int kstart;       // band: absolute key index of pair tile 0 (= q_off + q0 - lead)
    int p_lo;         // band: first issued pair tile
    int nA;           // band: pair tiles used by each query tile
    int num_band;     // band: issued band tiles
    int split;        // grow: split index
    int k0;           // grow: first key of the split
    int w;            // band: the head's radius
};

struct Tile {
    int row0;         // first key row (band/grow: absolute key; global: compact row)
    int ncols;        // columns of S (multiple of 16)
    bool global_key;  // compact global-key tile
    bool mem[2];      // query tile A / B uses this key tile
};

// Units [0, n_grow_units) are global-row units and the rest band units when grow_first,
// else band units come first: the longer kind goes first, so the short ones fill the tail.
// EXT: the extended masks (causal, radius per head, segments) are compiled in; the plain
// build leaves them out, so the common case carries none of their state.
template <bool EXT>
__device__ __forceinline__ Unit decode_unit(const MainParams& p, int u) {
    const int n_hw = EXT ? p.n_head_windows : 0;
    Unit un;
    const bool grow = p.grow_first ? (u < p.n_grow_units) : (u >= p.n_band_units);
    const int t = grow ? (p.grow_first ? u : u - p.n_band_units) : (p.grow_first ? u - p.n_grow_units : u);
    if (grow) {
        un.grow = true;
        un.split = t % p.n_splits;
        const int rest = t / p.n_splits;
        const int gt = rest % p.g_tiles;
        un.bh = rest / p.g_tiles;
        un.qrow[0] = un.qrow[1] = gt * BM;
        un.k0 = p.gk_lo + un.split * p.split_tiles * BN;
        const int rem = (p.gk_lo + p.gk_n - un.k0 + BN - 1) / BN;
        un.ntiles = rem < p.split_tiles ? rem : p.split_tiles;
        un.active[0] = true;
        un.active[1] = un.ntiles >= 2;
        un.kstart = un.p_lo = un.nA = un.num_band = 0;
        un.w = 0;
    } else {
        un.grow = false;
        un.split = un.k0 = 0;
        const int pair = t % p.q_pairs;
        un.bh = t / p.q_pairs;
        const int q0 = pair * 2 * BM;
        un.qrow[0] = q0;
        un.qrow[1] = q0 + BM;
        un.active[0] = true;
        un.active[1] = q0 + BM < p.n;
        // the head's own radius, which is also its lead, when heads have radii of their own
        un.w = n_hw > 0 ? p.head_window[un.bh % n_hw] : p.window;
        const int lead = n_hw > 0 ? un.w : p.lead;
        un.kstart = p.q_off + q0 - lead;
        // causal: A's rows [q0, q0 + 127] need keys up to q0 + 127 only
        un.nA = (EXT && p.causal) ? (lead + BM - 1) / BN + 1 : (lead + un.w + BM + BN - 1) / BN;
        const int p_first = un.kstart < p.key_lo ? (p.key_lo - un.kstart) / BN : 0;
        int p_last = un.active[1] ? un.nA : un.nA - 1;
        const int p_overlap_last = (p.key_hi - 1 - un.kstart) / BN;
        if (p_overlap_last < p_last) p_last = p_overlap_last;
        un.p_lo = p_first;
        un.num_band = p_last - p_first + 1;
        un.ntiles = un.num_band + p.g_tiles;
    }
    return un;
}

__device__ __forceinline__ Tile tile_of(const MainParams& p, const Unit& un, int j) {
    Tile t;
    if (un.grow) {
        t.row0 = un.k0 + j * BN;
        t.ncols = BN;
        t.global_key = false;
        t.mem[0] = (j & 1) == 0;
        t.mem[1] = (j & 1) == 1;
    } else if (j < un.num_band) {
        const int pp = un.p_lo + j;
        t.row0 = un.kstart + pp * BN;
        t.ncols = BN;
        t.global_key = false;
        t.mem[0] = pp <= un.nA - 1;
        t.mem[1] = un.active[1] && pp >= 1;
    } else {
        const int gt = j - un.num_band;
        t.row0 = gt * BN;
        int cnt = p.num_global - gt * BN;
        if (cnt > BN) cnt = BN;
        t.ncols = (cnt + 15) & ~15;
        t.global_key = true;
        t.mem[0] = true;
        t.mem[1] = un.active[1];
    }
    return t;
}

// First index of the sorted list gl[0, count) whose value is >= key (count if none).
__device__ __forceinline__ int lower_index(const int* gl, int count, int key) {
    int a = 0, b = count;
    while (a < b) {
        const int mid = (a + b) >> 1;
        if (gl[mid] < key) a = mid + 1; else b = mid;
    }
    return a;
}

// The segment [s_lo, s_hi) holding absolute token `x`: equal segments of seg_len tokens, or
// the packed sequences of seg_start.
__device__ __forceinline__ void segment_of(const MainParams& p, int x, int& s_lo, int& s_hi) {
    if (p.seg_mode == kSegEqual) {
        s_lo = (x / p.seg_len) * p.seg_len;
        s_hi = s_lo + p.seg_len;
        return;
    }
    int a = 0, b = p.n_segs;  // last segment whose start is <= x
    while (b - a > 1) {
        const int mid = (a + b) >> 1;
        if (p.seg_start[mid] <= x) a = mid; else b = mid;
    }
    s_lo = p.seg_start[a];
    s_hi = p.seg_start[a + 1];
}

// All 32 lanes wait; the warp proceeds only if every lane saw the phase complete, so
// warp-collective tcgen05 instructions that follow are never reached divergently.
__device__ __forceinline__ bool warp_wait(uint64_t* bar, uint32_t parity, volatile int* abort_flag, int* err,
                                          int code, uint64_t tmo) {
    const bool r = ptx::mbar_wait(bar, parity, abort_flag, err, code, tmo);
    return __all_sync(0xffffffffu, r);
}

// Bit e set iff column c0 + e lies in [a, b) (e = 0..31; empty when b <= a).
__device__ __forceinline__ uint32_t span_bits(int a, int b, int c0) {
    const int x = min(max(a - c0, 0), 32);
    const int y = min(max(b - c0, 0), 32);
    return (uint32_t)((1ull << y) - 1ull) & ~(uint32_t)((1ull << x) - 1ull);
}

__device__ __forceinline__ uint32_t swz128(int row, int chunk16) {
    // byte offset of 16-byte chunk `chunk16` (0..7) of row `row` in a 128-byte-swizzled panel
    return (uint32_t)(row * 128 + ((chunk16 ^ (row & 7)) << 4));
}

// The main kernel's body: tensor maps by reference to the kernel's __grid_constant__
// parameters (TMA reads them where they lie).
template <int D, bool BF16, bool V16, bool EXT>
__device__ __forceinline__ void swa_main_body(const CUtensorMap& tm_q, const CUtensorMap& tm_k, const CUtensorMap& tm_v,
                                              const CUtensorMap& tm_kh, const CUtensorMap& tm_vh,
                                              const CUtensorMap& tm_qg, const CUtensorMap& tm_kg,
                                              const CUtensorMap& tm_vg, const CUtensorMap& tm_o,
                                              const CUtensorMap& tm_po, const CUtensorMap& tm_v16,
                                              const CUtensorMap& tm_vg16, const CUtensorMap& tm_vh16,
                                              const MainParams& p) {
    using C = Cfg<D, BF16, V16>;
    constexpr int H = C::kHalves;
    constexpr int NC = C::kChains;
    constexpr int KC = C::kCols;
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint8_t* sQ = smem + C::kOffQ;
    uint8_t* sSlots = smem + C::kOffSlots;
    Ctl* ctl = reinterpret_cast<Ctl*>(smem + C::kOffCtl);

    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;
#ifdef LCA_TRACE
    unsigned int trace_i = 0;  // events recorded by this thread
#endif
    volatile int* abort_flag = &ctl->abort_flag;
    const int n_units = p.n_grow_units + p.n_band_units;
    const uint64_t tmo = p.timeout_ns;
    const bool causal = EXT && p.causal;
    const int seg_mode = EXT ? p.seg_mode : kSegNone;

    if (threadIdx.x == 0) {
        for (int x = 0; x < 2; ++x) {
            ptx::mbar_init(&ctl->q_full[x], 1);
            ptx::mbar_init(&ctl->q_empty[x], 1);
            for (int h = 0; h < 2; ++h) {
                ptx::mbar_init(&ctl->s_full[x][h], 1);
                ptx::mbar_init(&ctl->p_full[x][h], 4);
                ptx::mbar_init(&ctl->pv_done[x][h], 1);
            }
            ptx::mbar_init(&ctl->o_full[x], 1);
            ptx::mbar_init(&ctl->o_free[x], 4 * H);
        }
        for (int s = 0; s < C::kSlots; ++s) {
            ptx::mbar_init(&ctl->kv_full[s], 1);
            ptx::mbar_init(&ctl->kv_empty[s], 2);  // one release per MMA issuer
        }
        ptx::mbar_init(&ctl->mma_drained[0], 1);
        ptx::mbar_init(&ctl->mma_drained[1], 1);
        for (int i = 0; i < kUnitRing; ++i) {
            ptx::mbar_init(&ctl->unit_full[i], 1);
            ptx::mbar_init(&ctl->unit_empty[i], 2 + C::kSoftmaxWarps);  // MMA issuers, softmax warps
        }
        ctl->abort_flag = 0;
        ptx::fence_mbar_init();
    }
    if (warp == C::kMmaWarp) {
        ptx::tmem_alloc(&ctl->tmem_base, kTmemCols);
        ptx::tmem_relinquish();
    }
    int* sGidx = reinterpret_cast<int*>(smem + C::kOffGidx);
    const bool gidx_in_smem = p.g_tiles > 0 && p.num_global <= C::kSmemGlobals;
    if (gidx_in_smem)
        for (int i = threadIdx.x; i < p.num_global; i += blockDim.x) sGidx[i] = __ldg(p.gidx + i);
    ptx::tc_fence_before();
    __syncthreads();
    ptx::tc_fence_after();
    const uint32_t tmem = ctl->tmem_base;

    if (warp >= C::kSoftmaxWarps) {
        ptx::setmaxnreg_dec<C::kRegsControl>();
        if (warp == C::kTmaWarp) {
            // ======================================================== TMA producer
            if (ptx::elect_one()) {
                ptx::prefetch_tmap(&tm_q);
                ptx::prefetch_tmap(&tm_k);
                ptx::prefetch_tmap(&tm_v);
                if (p.sharded) {
                    ptx::prefetch_tmap(&tm_kh);
                    ptx::prefetch_tmap(&tm_vh);
                }
                int L = 0;   // K/V loads issued
                int qn = 0;  // Q loads issued per tile buffer
                bool ok = true;
                for (int k = 0; ok; ++k) {
                    // Next unit: the CTA's own first one, then one from the launch-wide counter
                    // (dynamic: the CTAs that finish first take more), or round-robin without it.
                    // Published through the unit ring; an index >= n_units ends every role.
                    int u = blockIdx.x + k * gridDim.x;
                    if (k > 0 && p.unit_counter != nullptr) u = (int)gridDim.x + (int)atomicAdd(p.unit_counter, 1u);
                    if (u > n_units) u = n_units;
                    const int us = k % kUnitRing;
                    if (k >= kUnitRing && !ptx::mbar_wait(&ctl->unit_empty[us], ((k / kUnitRing) - 1) & 1, abort_flag,
                                                           p.err, LCA_DEVERR_TIMEOUT_PRODUCER, tmo)) {
                        ok = false;
                        break;
                    }
                    ctl->unit_ring[us] = u;
                    ptx::mbar_arrive(&ctl->unit_full[us]);
                    if (u >= n_units) break;
                    const Unit un = decode_unit<EXT>(p, u);
                    const CUtensorMap* mq = un.grow ? &tm_qg : &tm_q;
                    for (int x = 0; x < 2 && ok; ++x) {
                        // the compact global rows are [G][3][bh][d]: their maps index (col, bh, row)
                        const int qy = un.grow ? un.bh : (x ? un.qrow[1] : un.qrow[0]);
                        const int qz = un.grow ? un.qrow[x] : un.bh;
                        if (qn > 0 && !ptx::mbar_wait(&ctl->q_empty[x], (qn - 1) & 1, abort_flag, p.err,
                                                      LCA_DEVERR_TIMEOUT_PRODUCER, tmo)) {
                            ok = false;
                            break;
                        }
                        ptx::mbar_arrive_expect_tx(&ctl->q_full[x], C::kTileBytes);
#pragma unroll
                        for (int pn = 0; pn < C::kPanels; ++pn) {
                            if (p.heads4d > 0 && !un.grow)  // token-major: (column, head, row, batch)
                                ptx::tma_load_4d(sQ + x * C::kTileBytes + pn * kPanelBytes, mq, &ctl->q_full[x],
                                                 pn * 64, qz % p.heads4d, qy, qz / p.heads4d);
                            else
                                ptx::tma_load_3d(sQ + x * C::kTileBytes + pn * kPanelBytes, mq, &ctl->q_full[x],
                                                 pn * 64, qy, qz);
                        }
                    }
                    if (!ok) break;
                    ++qn;
                    for (int j = 0; j < un.ntiles && ok; ++j) {
                        const Tile t = tile_of(p, un, j);
                        for (int kv = 0; kv < 2; ++kv) {
                            const int slot = L % C::kSlots;
                            LCA_TRACE_EVENT(trace::EV_TMA_SLOT_WAIT);
                            if (L >= C::kSlots &&
                                !ptx::mbar_wait(&ctl->kv_empty[slot], ((L / C::kSlots) + 1) & 1, abort_flag, p.err,
                                                LCA_DEVERR_TIMEOUT_PRODUCER, tmo)) {
                                ok = false;
                                break;
                            }
                            LCA_TRACE_EVENT(trace::EV_TMA_SLOT_FREE);
                            const CUtensorMap* m = t.global_key ? (kv ? (V16 ? &tm_vg16 : &tm_vg) : &tm_kg)
                                                                : (kv ? (V16 ? &tm_v16 : &tm_v) : &tm_k);
                            int y = t.row0, z = un.bh;
                            if (t.global_key) {
                                y = un.bh;
                                z = t.row0;
                            } else if (p.sharded) {
                                // the tile lies wholly in the left halo, the shard or the right halo
                                if (y < p.q_off) {
                                    m = kv ? (V16 ? &tm_vh16 : &tm_vh) : &tm_kh;
                                    y -= p.q_off - p.halo;
                                } else if (y >= p.q_off + p.n) {
                                    m = kv ? (V16 ? &tm_vh16 : &tm_vh) : &tm_kh;
                                    y -= p.q_off + p.n;
                                    z += 2 * p.bh;
                                } else {
                                    y -= p.q_off;
                                }
                            }
                            uint8_t* dst = sSlots + slot * C::kTileBytes;
                            ptx::mbar_arrive_expect_tx(&ctl->kv_full[slot], C::kTileBytes);
                            // token-major K / V (not the fp16 copy of V, which is head-major)
                            const bool four = p.heads4d > 0 && (m == &tm_k || m == &tm_v);
#pragma unroll
                            for (int pn = 0; pn < C::kPanels; ++pn) {
                                if (four)
                                    ptx::tma_load_4d(dst + pn * kPanelBytes, m, &ctl->kv_full[slot], pn * 64,
                                                     z % p.heads4d, y, z / p.heads4d);
                                else
                                    ptx::tma_load_3d(dst + pn * kPanelBytes, m, &ctl->kv_full[slot], pn * 64, y, z);
                            }
                            ++L;
                        }
                    }
                }
                // Drain: every issued copy lands before the CTA may exit.
                if (qn > 0)
                    for (int x = 0; x < 2; ++x)
                        ptx::mbar_wait(&ctl->q_full[x], (qn - 1) & 1, nullptr, p.err, LCA_DEVERR_TIMEOUT_DRAIN, tmo);
                for (int idx = (L > C::kSlots ? L - C::kSlots : 0); idx < L; ++idx)
                    ptx::mbar_wait(&ctl->kv_full[idx % C::kSlots], (idx / C::kSlots) & 1, nullptr, p.err,
                                   LCA_DEVERR_TIMEOUT_DRAIN, tmo);
            }
        } else if (warp == C::kMmaWarp || warp == C::kMmaWarp + 1) {
            // ======================================================== MMA issuers
            // One issuing thread per query tile X, so the two tiles' MMA streams progress
            // independently.  Every K/V slot use is released once by each issuer (the
            // kv_empty barriers count 2): by a commit after the issuer's last MMA reading
            // it, or by a plain arrive if the tile is not one of its members.  An issuer
            // always waits for a slot's data to land before releasing it, so its releases
            // can never run ahead into the slot's next phase.
            const int X = warp - C::kMmaWarp;
            if (ptx::elect_one()) {
                const uint32_t sslots = ptx::smem_u32(sSlots);
                // descriptor high words are loop-invariant (128-byte swizzle, 1024-byte 8-row
                // groups); a k-step only advances the low word's start address
                const uint32_t dhi = ptx::smem_desc_sw128_hi(1024);
                const uint32_t qlo = ptx::smem_desc_sw128_lo(ptx::smem_u32(sQ) + X * C::kTileBytes, 0);
                const uint32_t idesc_s_full = ptx::idesc_f16(BF16, BM, KC, false);
                const uint32_t idesc_pv = ptx::idesc_f16(BF16 && !V16, BM, D, true);  // P and V types
                const uint32_t sx = tmem + X * 128;
                int L = 0, qn = 0, pc = 0, oc = 0;
                bool ok = true;

                auto W = [&](uint64_t* bar, int parity) -> bool {
                    if (!ok) return false;
                    ok = ptx::mbar_wait(bar, (uint32_t)parity & 1u, abort_flag, p.err, LCA_DEVERR_TIMEOUT_MMA, tmo);
                    if (ok) ptx::tc_fence_after();
                    return ok;
                };
                // S_X[:, half h] = Q_X K[keys of half h]^T: keys [KC*h, KC*h + n) of the tile
                // (n = ncols - KC*h, at most KC) into TMEM columns [KC*h, KC*h + n).  The K
                // rows of half h start KC*h rows (KC*h*128 bytes, whole 8-row swizzle atoms)
                // into each panel.
                auto issue_s = [&](int slot, int ncols, int h) {
                    int n = ncols - KC * h;
                    if (n <= 0) return;
                    if (n > KC) n = KC;
                    const uint32_t idesc = (n == KC) ? idesc_s_full : ptx::idesc_f16(BF16, BM, n, false);
                    const uint32_t klo =
                        ptx::smem_desc_sw128_lo(sslots + slot * C::kTileBytes + KC * h * 128, 0);
#pragma unroll
                    for (int ks = 0; ks < D / 16; ++ks) {
                        const uint32_t off = ((ks >> 2) * kPanelBytes + (ks & 3) * 32) >> 4;
                        ptx::mma_f16_ss(sx + KC * h, ptx::desc_join(qlo + off, dhi), ptx::desc_join(klo + off, dhi),
                                        idesc, ks > 0 ? 1u : 0u);
                    }
                };
                // O_{X,h} += P_{X,h} V[keys of half h].  P lives in S_X's TMEM columns: keys
                // [32c, 32c + 32) of the tile occupy columns [32c, 32c + 32), hi pairs in the
                // first 16 and, for bf16, lo pairs in the next 16 (two 16-bit elements per
                // 32-bit column).  Half h owns keys [KC*h, KC*(h+1)) and accumulates into O_{X,h}.
                auto issue_pv = [&](int slot, int ncols, bool first, int h) {
                    const uint32_t vlo = ptx::smem_desc_sw128_lo(sslots + slot * C::kTileBytes, kPanelBytes);
                    {
                        // d = 64: chain h's own accumulator; d = 128: one accumulator, which
                        // chain 1 adds to from its first MMA on
                        const uint32_t dcol = tmem + C::kOCol + (X * H + (H == 2 ? h : 0)) * D;
                        const bool fresh = first && (H == 2 || h == 0);
#pragma unroll
                        for (int part = 0; part < (C::kSplitP ? 2 : 1); ++part) {
#pragma unroll
                            for (int kk = 0; kk < KC / 16; ++kk) {
                                const int key = KC * h + 16 * kk;  // first key of this k-step
                                if (key < ncols) {
                                    const uint32_t acol = sx + (key >> 5) * 32 + part * 16 + ((key >> 4) & 1) * 8;
                                    ptx::mma_f16_ts(dcol, acol, ptx::desc_join(vlo + ((key * 128) >> 4), dhi),
                                                    idesc_pv, (!fresh || part > 0 || kk > 0) ? 1u : 0u);
                                }
                            }
                        }
                    }
                };

                for (int k = 0; ok; ++k) {
                    const int us = k % kUnitRing;
                    if (!W(&ctl->unit_full[us], k / kUnitRing)) break;
                    const int u = *reinterpret_cast<volatile int*>(&ctl->unit_ring[us]);
                    ptx::mbar_arrive(&ctl->unit_empty[us]);
                    if (u >= n_units) break;
                    const Unit un = decode_unit<EXT>(p, u);
                    const bool act = X ? un.active[1] : un.active[0];
                    if (!W(&ctl->q_full[X], qn)) break;
                    ++qn;
                    bool first = true;       // next P*V starts the accumulators
                    int pend_lv = -1;        // slot use of V for the member tile whose P*V is pending
                    int pend_cols = 0;
                    // P*V of the pending member tile for half h, after that half's P is written;
                    // it precedes the half's next S MMA, which overwrites the TMEM columns
                    // holding that P.  The first half also waits for the accumulators to be free
                    // and for the V tile.
                    auto pv_half = [&](int h) -> bool {
                        // (the accumulators and the V tile are usually ready long before P:
                        // check them first, off the P -> P*V -> S chain)
                        if (h == 0) {
                            if (first && oc > 0 && !W(&ctl->o_free[X], oc - 1)) return false;
                            if (!W(&ctl->kv_full[pend_lv % C::kSlots], pend_lv / C::kSlots)) return false;
                        }
                        LCA_TRACE_EVENT(trace::EV_MMA_P_WAIT);
                        if (!W(&ctl->p_full[X][h], pc)) return false;
                        LCA_TRACE_EVENT(trace::EV_MMA_P_READY);
                        issue_pv(pend_lv % C::kSlots, pend_cols, first, h);
                        ptx::mma_commit(&ctl->pv_done[X][h]);
                        LCA_TRACE_EVENT(trace::EV_MMA_PV_ISSUED);
                        return true;
                    };
                    auto pv_done = [&]() {
                        ++pc;
                        first = false;
                        ptx::mma_commit(&ctl->kv_empty[pend_lv % C::kSlots]);
                        pend_lv = -1;
                    };
                    for (int j = 0; j < un.ntiles && ok; ++j) {
                        const Tile t = tile_of(p, un, j);
                        const bool mem = act && (X ? t.mem[1] : t.mem[0]);
                        const int lk = L + 2 * j, lv = lk + 1;
                        if (!mem) {
                            // Not a member tile: the pending P*V goes first (it releases its V
                            // slot, which the producer may need before it can load this tile),
                            // then this tile's K and V slots are released once landed.
                            if (pend_lv >= 0) {
                                bool pv_ok = true;
#pragma unroll
                                for (int h = 0; h < NC; ++h) pv_ok = pv_ok && pv_half(h);
                                if (!pv_ok) break;
                                pv_done();
                            }
                            LCA_TRACE_EVENT(trace::EV_MMA_K_WAIT);
                            if (!W(&ctl->kv_full[lk % C::kSlots], lk / C::kSlots)) break;
                            LCA_TRACE_EVENT(trace::EV_MMA_K_READY);
                        } else {
                            // Member tile: each chain runs P*V of the pending tile, then S of
                            // this one, as soon as that chain's P is written.  Chain 0's P*V
                            // goes before the wait for this tile's K (it does not need it).
                            bool s_ok = true;
#pragma unroll
                            for (int h = 0; h < NC; ++h) {
                                if (pend_lv >= 0 && !pv_half(h)) {
                                    s_ok = false;
                                    break;
                                }
                                if (h == 0) {
                                    LCA_TRACE_EVENT(trace::EV_MMA_K_WAIT);
                                    if (!W(&ctl->kv_full[lk % C::kSlots], lk / C::kSlots)) {
                                        s_ok = false;
                                        break;
                                    }
                                    LCA_TRACE_EVENT(trace::EV_MMA_K_READY);
                                }
                                issue_s(lk % C::kSlots, t.ncols, h);
                                ptx::mma_commit(&ctl->s_full[X][h]);
                                LCA_TRACE_EVENT(trace::EV_MMA_S_ISSUED);
                            }
                            if (!s_ok) break;
                            if (pend_lv >= 0) pv_done();
                        }
                        if (mem) {
                            ptx::mma_commit(&ctl->kv_empty[lk % C::kSlots]);
                            pend_lv = lv;
                            pend_cols = t.ncols;
                        } else {
                            ptx::mbar_arrive(&ctl->kv_empty[lk % C::kSlots]);
                            if (!W(&ctl->kv_full[lv % C::kSlots], lv / C::kSlots)) break;
                            ptx::mbar_arrive(&ctl->kv_empty[lv % C::kSlots]);
                        }
                    }
                    if (!ok) break;
                    // every S MMA of this unit has been issued: Q_X may be refilled once they complete
                    ptx::mma_commit(&ctl->q_empty[X]);
                    if (pend_lv >= 0) {
                        bool pv_ok = true;
#pragma unroll
                        for (int h = 0; h < NC; ++h) pv_ok = pv_ok && pv_half(h);
                        if (!pv_ok) break;
                        pv_done();
                    }
                    if (!first) {
                        ptx::mma_commit(&ctl->o_full[X]);
                        ++oc;
                    }
                    L += 2 * un.ntiles;
                }
                // Drain: all tcgen05 ops issued by this thread complete before TMEM is freed.
                ptx::mma_commit(&ctl->mma_drained[X]);
                ptx::mbar_wait(&ctl->mma_drained[X], 0, nullptr, p.err, LCA_DEVERR_TIMEOUT_DRAIN, tmo);
            }
        }
    } else {
        ptx::setmaxnreg_inc<C::kRegsSoftmax>();
        // ============================================================ softmax warpgroups
        const int sw = warp >> 2;         // softmax warpgroup
        const int X = sw / H;             // query tile of this warpgroup
        const int hh = sw % H;            // key-column half of this warpgroup
        const int wq = warp & 3;          // TMEM lane quarter
        const int r = wq * 32 + lane;     // row within the tile == TMEM lane
        const int tile_bar = 1 + X;       // named barrier: all warpgroups of tile X
        const int wg_bar = 3 + sw;        // named barrier: this warpgroup
        const uint32_t t_lane = tmem + ((uint32_t)(wq * 32) << 16);
        const uint32_t o_col = C::kOCol + (X * H + hh) * D;  // this warpgroup's accumulator
        const uint32_t o_col0 = C::kOCol + (X * H) * D;      // accumulator of half 0 of tile X
        uint8_t* stage = smem + C::kOffStage + sw * C::kStageBytes;
        float* xchg = reinterpret_cast<float*>(smem + C::kOffXchg);
        // scale * log2(e) (the host passes a tiny positive value for scale == 0 so that
        // visible scores stay finite and masked ones still map to -inf)
        const float sl2 = p.scale_log2;
        const bool neg_scale = sl2 < 0.f;
        const float sent = neg_scale ? INFINITY : -INFINITY;
        int sc = 0, oc = 0;
        bool ok = true;  // warp-uniform; after a failed wait the warp skips work and leaves at the next unit

        for (int k = 0;; ++k) {
            const int us = k % kUnitRing;
            if (ok) ok = warp_wait(&ctl->unit_full[us], (k / kUnitRing) & 1, abort_flag, p.err,
                                   LCA_DEVERR_TIMEOUT_SOFTMAX, tmo);
            if (!ok) break;
            const int u = *reinterpret_cast<volatile int*>(&ctl->unit_ring[us]);
            __syncwarp();
            if (lane == 0) ptx::mbar_arrive(&ctl->unit_empty[us]);
            if (u >= n_units) break;
            const Unit un = decode_unit<EXT>(p, u);
            LCA_TRACE_LANE0(trace::EV_UNIT_DECODED);
            const bool active_x = X ? un.active[1] : un.active[0];
            if (!active_x) continue;
            const int qrow_x = X ? un.qrow[1] : un.qrow[0];
            const int qi = qrow_x + r;         // local (band) or compact (global-row unit) row
            const int qa = p.q_off + qi;       // band: absolute query index
            const bool live = un.grow ? (qi < p.num_global) : (qi < p.n);
            const bool warp_live = __any_sync(0xffffffffu, live);
            // row's visible keys in band / split tiles: [jlo, jhi] (absolute key index)
            int jlo = p.gk_lo, jhi = p.gk_lo + p.gk_n - 1;
            // band units: run [g_lo, g_hi) of sorted global indices inside the row's band, and
            // the compact columns [gv_lo, gv_hi) of the global keys the row may see at all
            int g_lo = 0, g_hi = 0, gv_lo = 0, gv_hi = p.num_global;
            const int* gl = gidx_in_smem ? sGidx : p.gidx;
            if (un.grow) {
                if (qi < p.num_global && (causal || seg_mode == kSegVarlen)) {
                    const int g_tok = gl[qi];
                    if (causal && g_tok < jhi) jhi = g_tok;  // causal: keys up to the row's own token
                    if (seg_mode == kSegVarlen) {           // packed sequences: keys of its own sequence
                        int s_lo, s_hi;
                        segment_of(p, g_tok, s_lo, s_hi);
                        if (s_lo > jlo) jlo = s_lo;
                        if (s_hi - 1 < jhi) jhi = s_hi - 1;
                    }
                }
            } else {
                const int w = un.w;
                jlo = qa - w > 0 ? qa - w : 0;
                jhi = (qa + w < p.n_total - 1) ? qa + w : p.n_total - 1;
                int s_lo = 0, s_hi = p.n_total;
                if (seg_mode != kSegNone) {  // the band stops at the row's segment
                    segment_of(p, qa, s_lo, s_hi);
                    if (s_lo > jlo) jlo = s_lo;
                    if (s_hi - 1 < jhi) jhi = s_hi - 1;
                }
                if (causal && qa < jhi) jhi = qa;  // causal band [i - w, i]
                if (p.g_tiles > 0) {
                    // first global at or after the band's start, then the run inside the band
                    // (a few entries at most unless globals are dense: then a second search)
                    g_lo = lower_index(gl, p.num_global, jlo);
                    int a = g_lo, scan = 0;
                    while (a < p.num_global && scan < 4 && gl[a] <= jhi) {
                        ++a;
                        ++scan;
                    }
                    g_hi = scan == 4 ? lower_index(gl, p.num_global, jhi + 1) : a;
                    if (seg_mode == kSegVarlen) {  // packed sequences: the globals of the row's own
                        gv_lo = lower_index(gl, p.num_global, s_lo);
                        gv_hi = lower_index(gl, p.num_global, s_hi);
                    }
                    if (causal) {  // only the globals before the band: the rest are in it or after i
                        gv_hi = g_lo;
                        g_hi = g_lo;
                    }
                }
            }
            LCA_TRACE_LANE0(trace::EV_UNIT_READY);
            float m = -INFINITY;  // reference max (log2 units)
            float l = 0.f;
            bool seen = false;    // a previous member tile of this unit was processed
            for (int j = 0; j < un.ntiles; ++j) {
                const Tile t = tile_of(p, un, j);
                if (!(X ? t.mem[1] : t.mem[0])) continue;
                // the chains of this tile this warpgroup runs: its own (d = 64) or both (d = 128)
                for (int ch = (H == 2 ? hh : 0); ch < (H == 2 ? hh + 1 : NC); ++ch) {
                    LCA_TRACE_LANE0(trace::EV_S_WAIT);
                    if (ok) ok = warp_wait(&ctl->s_full[X][ch], sc & 1, abort_flag, p.err,
                                           LCA_DEVERR_TIMEOUT_SOFTMAX, tmo);
                    LCA_TRACE_LANE0(trace::EV_S_READY);
                    const uint32_t s_col = X * 128 + KC * ch;  // this chain's S / P columns
                    const int col0 = t.row0 + KC * ch;  // key (band) or compact global row of column 0
                    const int ncols_h = t.ncols - KC * ch;
                    if (ok && warp_live && ncols_h > 0) {
                        ptx::tc_fence_after();
                        // visible columns of this row in this tile: [lo, hi] minus the hole [h_lo, h_hi)
                        int lo, hi, h_lo = 0, h_hi = 0;
                        if (t.global_key) {
                            lo = gv_lo - col0;
                            hi = gv_hi - 1 - col0;
                            h_lo = g_lo - col0;
                            h_hi = g_hi - col0;
                        } else {
                            lo = jlo - col0;
                            hi = jhi - col0;
                        }
                        if (hi > ncols_h - 1) hi = ncols_h - 1;
                        const int nchunks = ((ncols_h < KC ? ncols_h : KC) + 31) >> 5;
                        // ---- pass 1: S row into registers, masked row max
                        float s[KC];
    #pragma unroll
                        for (int c = 0; c < KC / 32; ++c) {
                            if (c < nchunks) {
                                float tmp[32];
                                ptx::tmem_ld32(t_lane + s_col + c * 32, tmp);
    #pragma unroll
                                for (int e = 0; e < 32; ++e) s[c * 32 + e] = tmp[e];
                            } else {
    #pragma unroll
                                for (int e = 0; e < 32; ++e) s[c * 32 + e] = sent;
                            }
                        }
                        const bool need = lo > 0 || hi < KC - 1 || (h_lo < h_hi && h_hi > 0 && h_lo < KC);
                        const bool any_mask = __any_sync(0xffffffffu, need);
                        // visible columns of each 32-column chunk as a bit mask: [lo, hi] minus
                        // [h_lo, h_hi) (all ones when the warp needs no mask)
                        uint32_t vis[KC / 32];
    #pragma unroll
                        for (int c = 0; c < KC / 32; ++c)
                            vis[c] = any_mask ? (span_bits(lo, hi + 1, c * 32) & ~span_bits(h_lo, h_hi, c * 32)) : ~0u;
                        ptx::tmem_wait_ld();
                        if (any_mask) {
    #pragma unroll
                            for (int c = 0; c < KC; ++c) s[c] = ((vis[c >> 5] >> (c & 31)) & 1u) ? s[c] : sent;
                        }
                        LCA_TRACE_LANE0(trace::EV_S_LOADED);
                        // ---- exponent pass, one 32-key chunk at a time, from the registers:
                        // p = 2^(s * scale * log2(e) - mref) (masked scores are already `sent`,
                        // which maps to 0), row sums into acc, 16-bit pairs written over the
                        // chunk's own S columns (hi pairs, then lo pairs for bf16).  Chunks masked
                        // for the whole warp skip the exponentials.  Pairs of columns go through
                        // the packed fp32x2 pipe: one FMA for the exponent arguments, one add for
                        // the row sums and, for bf16, one subtract for the low parts.  Returns the
                        // largest exponent argument of the row.
                        auto exp_pass = [&](float mref, uint64_t& acc0, uint64_t& acc1) -> float {
                            const float neg_m = (mref == -INFINITY) ? 0.f : -mref;
                            const uint64_t sl2x2 = ptx::f2_pack(sl2, sl2);
                            const uint64_t negm2 = ptx::f2_pack(neg_m, neg_m);
                            float xm = -INFINITY;
    #pragma unroll
                            for (int c = 0; c < KC / 32; ++c) {
                                if (c >= nchunks) break;
                                const int c0 = c * 32;
                                if (__all_sync(0xffffffffu, vis[c] == 0u)) {
                                    uint32_t z[16];
    #pragma unroll
                                    for (int e = 0; e < 16; ++e) z[e] = 0u;
                                    ptx::tmem_st16u(t_lane + s_col + c0, z);
                                    if (C::kSplitP) ptx::tmem_st16u(t_lane + s_col + c0 + 16, z);
                                } else {
                                    const float* v = s + c0;
    #pragma unroll
                                    for (int g8 = 0; g8 < 2; ++g8) {  // 8 pairs (16 keys) per store
                                        uint32_t w[8];
                                        uint32_t wl[8];
    #pragma unroll
                                        for (int e = 0; e < 8; ++e) {
                                            const uint64_t x = ptx::f2_fma(
                                                ptx::f2_pack(v[g8 * 16 + 2 * e], v[g8 * 16 + 2 * e + 1]), sl2x2, negm2);
                                            xm = ptx::fmax3(xm, ptx::f2_lo(x), ptx::f2_hi(x));
                                            float p0, p1;
                                            uint64_t pp;
                                            if (((C::kPolyMask >> e) & 1u) != 0u) {
                                                pp = ptx::f2_exp2_poly(x);
                                                p0 = ptx::f2_lo(pp);
                                                p1 = ptx::f2_hi(pp);
                                            } else {
                                                p0 = ptx::ex2(ptx::f2_lo(x));
                                                p1 = ptx::ex2(ptx::f2_hi(x));
                                                pp = ptx::f2_pack(p0, p1);
                                            }
                                            if (e & 1) acc1 = ptx::f2_add(acc1, pp); else acc0 = ptx::f2_add(acc0, pp);
                                            if (C::kSplitP) {
                                                w[e] = ptx::pack_bf16x2(p0, p1);
                                                const uint64_t rest = ptx::f2_sub(
                                                    pp, ptx::f2_pack(__uint_as_float(w[e] << 16),
                                                                     __uint_as_float(w[e] & 0xFFFF0000u)));
                                                wl[e] = ptx::pack_bf16x2(ptx::f2_lo(rest), ptx::f2_hi(rest));
                                            } else {
                                                w[e] = ptx::pack_f16x2(p0, p1);
                                            }
                                        }
                                        ptx::tmem_st8u(t_lane + s_col + c0 + g8 * 8, w);
                                        if (C::kSplitP) ptx::tmem_st8u(t_lane + s_col + c0 + 16 + g8 * 8, wl);
                                    }
                                }
                            }
                            return xm;
                        };
                        uint64_t acc0 = 0ull, acc1 = 0ull;  // {+0.f, +0.f}
                        // Fast path: once every row of the warp has a reference max, exponentiate
                        // against it straight away; the row max is only needed if some argument
                        // exceeds the rescale threshold (rare), and then the chunk is redone below.
                        bool done = false;
                        if (C::kFastExp && !__any_sync(0xffffffffu, m == -INFINITY)) {
                            const float xm = exp_pass(m, acc0, acc1);
                            done = !__any_sync(0xffffffffu, xm > kRescaleThreshold);
                            if (!done) {
                                ptx::tmem_wait_st();  // the redo rewrites the same P columns
                                acc0 = acc1 = 0ull;
                            }
                        }
                        if (!done) {
                            // ---- masked row max
                            float r0 = sent, r1 = sent, r2 = sent, r3 = sent;
                            if (!neg_scale) {
    #pragma unroll
                                for (int c = 0; c < KC; c += 8) {
                                    r0 = ptx::fmax3(r0, s[c + 0], s[c + 1]);
                                    r1 = ptx::fmax3(r1, s[c + 2], s[c + 3]);
                                    r2 = ptx::fmax3(r2, s[c + 4], s[c + 5]);
                                    r3 = ptx::fmax3(r3, s[c + 6], s[c + 7]);
                                }
                            } else {
    #pragma unroll
                                for (int c = 0; c < KC; c += 8) {
                                    r0 = ptx::fmin3(r0, s[c + 0], s[c + 1]);
                                    r1 = ptx::fmin3(r1, s[c + 2], s[c + 3]);
                                    r2 = ptx::fmin3(r2, s[c + 4], s[c + 5]);
                                    r3 = ptx::fmin3(r3, s[c + 6], s[c + 7]);
                                }
                            }
                            const float mr =
                                neg_scale ? fminf(fminf(r0, r1), fminf(r2, r3)) : fmaxf(fmaxf(r0, r1), fmaxf(r2, r3));
                            const float mt = (mr == sent) ? -INFINITY : mr * sl2;

                            // ---- online softmax with lazy rescale (O is stable: see header)
                            bool rescale = false;
                            float alpha = 1.f;
                            if (mt > m + kRescaleThreshold || (m == -INFINITY && mt > -INFINITY)) {
                                rescale = seen && (m != -INFINITY);
                                alpha = (m == -INFINITY) ? 0.f : ptx::ex2(m - mt);
                                m = mt;
                                l *= alpha;
                            }
                            if (__any_sync(0xffffffffu, rescale)) {
                                // rare: rescale this row's accumulator, 8 columns at a time (few
                                // live registers).  At d = 64 the accumulator's last P*V is this
                                // chain's, covered by the commit of this S.  At d = 128 it is the
                                // other chain's (of the previous tile for chain 0, of this tile for
                                // chain 1): wait for it; its completion is the current or the
                                // preceding phase of that chain's barrier (this S's commit covers
                                // the one before).
                                if constexpr (H == 1) {
                                    const int pc_ch = ch == 0 ? 1 : 0;
                                    const int pc_tile = ch == 0 ? sc - 1 : sc;
                                    if (ok) ok = warp_wait(&ctl->pv_done[X][pc_ch], pc_tile & 1, abort_flag, p.err,
                                                           LCA_DEVERR_TIMEOUT_SOFTMAX, tmo);
                                    if (ok) ptx::tc_fence_after();
                                }
                                const float a = rescale ? alpha : 1.f;
    #pragma unroll 1
                                for (int c = 0; c < D / 8 && ok; ++c) {
                                    uint32_t o[8];
                                    ptx::tmem_ld8(t_lane + o_col + c * 8, o);
                                    ptx::tmem_wait_ld();
    #pragma unroll
                                    for (int e = 0; e < 8; ++e) o[e] = __float_as_uint(__uint_as_float(o[e]) * a);
                                    ptx::tmem_st8u(t_lane + o_col + c * 8, o);
                                }
                            }
                            LCA_TRACE_LANE0(trace::EV_MAX_DONE);
                            exp_pass(m, acc0, acc1);
                        }
                        {
                            const uint64_t a = ptx::f2_add(acc0, acc1);
                            l += ptx::f2_lo(a) + ptx::f2_hi(a);
                        }
                        LCA_TRACE_LANE0(trace::EV_EXP_DONE);
                        ptx::tmem_wait_st();
                    }
                    seen = true;
                    ptx::tc_fence_before();
                    __syncwarp();
                    if (lane == 0) ptx::mbar_arrive(&ctl->p_full[X][ch]);
                    LCA_TRACE_LANE0(trace::EV_P_ARRIVED);
                }
                ++sc;  // member tiles: one phase of each chain's s_full / pv_done
            }

            // ---- epilogue: merge the halves, O / l -> fp32 rows via staging + TMA store
            LCA_TRACE_LANE0(trace::EV_EPI_WAIT);
            if (ok) ok = warp_wait(&ctl->o_full[X], oc & 1, abort_flag, p.err, LCA_DEVERR_TIMEOUT_SOFTMAX, tmo);
            LCA_TRACE_LANE0(trace::EV_EPI_READY);
            if (ok) ptx::tc_fence_after();
            float M = m, Lsum = l, w_own = 1.f, w_oth = 0.f;
            if constexpr (H == 2) {
                float* xb = xchg + (((oc & 1) * 2 + X) * 2) * 256;  // [half][row][2]
                xb[(hh * 128 + r) * 2 + 0] = m;
                xb[(hh * 128 + r) * 2 + 1] = l;
                ptx::named_bar_sync(tile_bar, H * kWgThreads);
                const float mo = xb[((1 - hh) * 128 + r) * 2 + 0];
                const float lo2 = xb[((1 - hh) * 128 + r) * 2 + 1];
                M = fmaxf(m, mo);
                w_own = (m == -INFINITY) ? 0.f : ptx::ex2(m - M);
                w_oth = (mo == -INFINITY) ? 0.f : ptx::ex2(mo - M);
                Lsum = l * w_own + lo2 * w_oth;
            }
            LCA_TRACE_LANE0(trace::EV_EPI_MERGED);
            ++oc;
            // staging from this warpgroup's previous unit must have been read by its TMA stores
            if (r == 0) ptx::tma_store_wait_read<0>();
            ptx::named_bar_sync(wg_bar, kWgThreads);
            const float inv_l = 1.f / Lsum;
            // weights of the half-0 and half-1 accumulators for this row
            const float w0 = (hh == 0) ? w_own : w_oth;
            const float w1 = (hh == 0) ? w_oth : w_own;
            const CUtensorMap* mo = un.grow ? &tm_po : &tm_o;
            const int oz = un.grow ? ((2 * un.split + X) * p.bh + un.bh) : un.bh;
            const int out16 = un.grow ? 0 : p.out16;  // global-row partials stay fp32
#pragma unroll
            for (int c = 0; c < C::kEpiCols / 32; ++c) {
                const int ocol = hh * C::kEpiCols + c * 32;  // output column of this chunk
                uint8_t* panel = stage + (c % C::kStagePanels) * kPanelBytes;
                if (c >= C::kStagePanels) {  // the store issued kStagePanels chunks ago has read this panel
                    if (r == 0) ptx::tma_store_wait_read<C::kStagePanels - 1>();
                    ptx::named_bar_sync(wg_bar, kWgThreads);
                }
                if (ok) {
                    float o[32];
                    ptx::tmem_ld32(t_lane + o_col0 + ocol, o);
                    if constexpr (H == 2) {
                        float o1[32];
                        ptx::tmem_ld32(t_lane + o_col0 + D + ocol, o1);
                        ptx::tmem_wait_ld();
#pragma unroll
                        for (int e = 0; e < 32; ++e) o[e] = (o[e] * w0 + o1[e] * w1) * inv_l;
                    } else {
                        ptx::tmem_wait_ld();
#pragma unroll
                        for (int e = 0; e < 32; ++e) o[e] *= inv_l;
                    }
                    const uint32_t sbase = ptx::smem_u32(panel);
                    if (out16) {
                        // 16-bit rows of 64 bytes, unswizzled (the 16-bit output map's layout)
#pragma unroll
                        for (int q = 0; q < 4; ++q) {
                            uint32_t w[4];
#pragma unroll
                            for (int e = 0; e < 4; ++e) {
                                const float a = o[q * 8 + 2 * e], b = o[q * 8 + 2 * e + 1];
                                w[e] = out16 == kOut16BF16 ? ptx::pack_bf16x2(a, b) : ptx::pack_f16x2(a, b);
                            }
                            ptx::st_shared_v4(sbase + r * 64 + q * 16, w[0], w[1], w[2], w[3]);
                        }
                    } else {
#pragma unroll
                        for (int q = 0; q < 8; ++q)
                            ptx::st_shared_v4(sbase + swz128(r, q), __float_as_uint(o[q * 4 + 0]),
                                              __float_as_uint(o[q * 4 + 1]), __float_as_uint(o[q * 4 + 2]),
                                              __float_as_uint(o[q * 4 + 3]));
                    }
                }
                ptx::fence_proxy_async_smem();
                ptx::named_bar_sync(wg_bar, kWgThreads);
                if (r == 0 && ok) {
                    if (p.heads4d > 0 && !un.grow)
                        ptx::tma_store_4d(mo, panel, ocol, oz % p.heads4d, qrow_x, oz / p.heads4d);
                    else
                        ptx::tma_store_3d(mo, panel, ocol, qrow_x, oz);
                    ptx::tma_store_commit();
                }
            }
            ptx::tc_fence_before();
            __syncwarp();
            if (lane == 0) ptx::mbar_arrive(&ctl->o_free[X]);
            LCA_TRACE_LANE0(trace::EV_EPI_DONE);
            if (ok && hh == 0) {
                const float lse = (((M == -INFINITY) ? 0.f : M) + __log2f(Lsum)) * kLn2;
                if (un.grow) {
                    if (qi < p.num_global)
                        p.part_lse[((size_t)(2 * un.split + X) * p.bh + un.bh) * p.num_global + qi] = lse;
                } else if (p.lse != nullptr && qi < p.n) {
                    p.lse[(size_t)un.bh * p.n + qi] = lse;
                }
            }
        }
        if (r == 0) ptx::tma_store_wait_all();
    }

    LCA_TRACE_FLUSH();
    ptx::tc_fence_before();
    __syncthreads();
    ptx::tc_fence_after();
    if (warp == C::kMmaWarp) ptx::tmem_dealloc(tmem, kTmemCols);
}

#define LCA_MAIN_PARAMS                                                                                           \
    const __grid_constant__ CUtensorMap tm_q, const __grid_constant__ CUtensorMap tm_k,                           \
        const __grid_constant__ CUtensorMap tm_v, const __grid_constant__ CUtensorMap tm_kh,                      \
        const __grid_constant__ CUtensorMap tm_vh, const __grid_constant__ CUtensorMap tm_qg,                     \
        const __grid_constant__ CUtensorMap tm_kg, const __grid_constant__ CUtensorMap tm_vg,                     \
        const __grid_constant__ CUtensorMap tm_o, const __grid_constant__ CUtensorMap tm_po,                      \
        const __grid_constant__ CUtensorMap tm_v16, const __grid_constant__ CUtensorMap tm_vg16,                  \
        const __grid_constant__ CUtensorMap tm_vh16, const MainParams p
#define LCA_MAIN_ARGS tm_q, tm_k, tm_v, tm_kh, tm_vh, tm_qg, tm_kg, tm_vg, tm_o, tm_po, tm_v16, tm_vg16, tm_vh16, p

// fp16 inputs (fp16 P), or bf16 inputs without the fp16 copy of V (bf16 P split into hi + lo)
template <int D, bool BF16, bool EXT>
__global__ void __launch_bounds__(Cfg<D, BF16, false>::kThreads, 1) lca_swa_main(LCA_MAIN_PARAMS) {
    ptx::griddep_wait();  // the compact global rows and the unit counter are written before
    ptx::griddep_launch();
    swa_main_body<D, BF16, false, EXT>(LCA_MAIN_ARGS);
}

// bf16 inputs with the fp16 copy of V: one launch that reads the word lca_convert_v16 set and
// runs fp16 P with one P*V per tile from the copy when every value of V fitted fp16, else the
// split bf16 P (no host synchronisation, so the choice stays capturable in a graph)
template <int D, bool EXT>
__global__ void __launch_bounds__(Cfg<D, true, true>::kThreads, 1) lca_swa_main_v16(LCA_MAIN_PARAMS) {
    static_assert(Cfg<D, true, true>::kSmemBytes == Cfg<D, true, false>::kSmemBytes &&
                      Cfg<D, true, true>::kThreads == Cfg<D, true, false>::kThreads,
                  "both paths share one launch configuration");
    ptx::griddep_wait();  // the fp16 copy, its word, the compact rows and the counter
    ptx::griddep_launch();
    if (*reinterpret_cast<const volatile int*>(p.v16_bad) == 0)
        swa_main_body<D, true, true, EXT>(LCA_MAIN_ARGS);
    else
        swa_main_body<D, true, false, EXT>(LCA_MAIN_ARGS);
}

// ------------------------------------------------------------------------ gather

template <int D>
__global__ void __launch_bounds__(256) lca_gather_globals(const uint16_t* __restrict__ q,
                                                          const uint16_t* __restrict__ k,
                                                          const uint16_t* __restrict__ v, GatherParams gp) {
    // one warp per (bh, compact row); 16-byte chunks
    constexpr int kChunks = D * 2 / 16;
    ptx::griddep_launch();
    const long long w = (long long)blockIdx.x * 8 + (threadIdx.x >> 5);
    const int lane = threadIdx.x & 31;
    if (w >= (long long)gp.count * gp.bh) return;
    const int row = (int)(w % gp.count);
    const int bh = (int)(w / gp.count);
    const int g = gp.first + row;  // compact row index
    const int src_abs = gp.idx[row];
    const int src_row = src_abs - gp.q_off;
    if (bh == 0 && lane == 0) gp.gidx_out[g] = src_abs;
    if (src_row < 0 || src_row >= gp.n) return;  // owned by another shard
    const size_t src_off = (size_t)(bh / gp.heads) * gp.s_b + (size_t)(bh % gp.heads) * gp.s_h + (size_t)src_row * gp.s_n;
    for (int c = lane; c < 3 * kChunks; c += 32) {
        const int which = c / kChunks;
        const int cc = c % kChunks;
        const uint16_t* src = which == 0 ? q : (which == 1 ? k : v);
        const size_t dst_off = (((size_t)g * 3 + which) * gp.bh + bh) * D;
        *reinterpret_cast<uint4*>(gp.compact + dst_off + cc * 8) =
            *reinterpret_cast<const uint4*>(src + src_off + cc * 8);
    }
}

// ------------------------------------------------------------------------ fp16 copy of V

// One block per 128-row block of one plane of one segment (segments in order); each thread
// converts 16-byte chunks (8 values) of the block's rows.
template <int D>
__global__ void __launch_bounds__(256) lca_convert_v16(ConvertParams cp) {
    constexpr int kChunksPerRow = D / 8;
    long long blk = blockIdx.x;
    int si = 0;
    for (; si < cp.n_segments; ++si) {
        const long long nb = (long long)cp.seg[si].planes * ((cp.seg[si].rows + 127) / 128);
        if (blk < nb) break;
        blk -= nb;
    }
    ptx::griddep_launch();
    if (si >= cp.n_segments) return;
    // segment 0 is the caller's V, complete before this forward's first launch; the others
    // (compact global rows, received halos) are written by the launch before this one
    if (si > 0) ptx::griddep_wait();
    const ConvertSegment sg = cp.seg[si];
    const int per_plane = (sg.rows + 127) / 128;
    const int pl = (int)(blk / per_plane);
    const int r0 = (int)(blk % per_plane) * 128;
    const int rows = min(128, sg.rows - r0);
    bool bad = false, inexact = false;
    float amax = 0.f;
    // every chunk load of this thread first, then the conversions and stores (the loads
    // stay in flight together)
    constexpr int kPer = 128 * kChunksPerRow / 256;  // chunks per thread (blockDim.x == 256)
    const int total = rows * kChunksPerRow;
    uint4 in[kPer];
#pragma unroll
    for (int i = 0; i < kPer; ++i) {
        const int c = (int)threadIdx.x + i * 256;
        if (c < total) {
            const long long r = r0 + c / kChunksPerRow;
            in[i] = *reinterpret_cast<const uint4*>(sg.src + (long long)(pl / sg.heads) * sg.src_plane +
                                                    (long long)(pl % sg.heads) * sg.src_head + r * sg.src_row +
                                                    (c % kChunksPerRow) * 8);
        }
    }
#pragma unroll
    for (int i = 0; i < kPer; ++i) {
        const int c = (int)threadIdx.x + i * 256;
        if (c >= total) break;
        const long long r = r0 + c / kChunksPerRow;
        const uint32_t w[4] = {in[i].x, in[i].y, in[i].z, in[i].w};
        uint32_t o[4];
#pragma unroll
        for (int e = 0; e < 4; ++e) {
            const float f0 = __uint_as_float(w[e] << 16), f1 = __uint_as_float(w[e] & 0xFFFF0000u);
            const __half2 h = __floats2half2_rn(f0, f1);
            const float2 back = __half22float2(h);
            // bf16 values in the fp16 normal range convert exactly; below 2^-14 they round to
            // fp16 subnormals (error <= 2^-25); beyond 65504 (or NaN) they do not fit
            if (back.x != f0) (fabsf(f0) < 6.103515625e-05f ? inexact : bad) = true;
            if (back.y != f1) (fabsf(f1) < 6.103515625e-05f ? inexact : bad) = true;
            amax = fmaxf(amax, fmaxf(fabsf(f0), fabsf(f1)));
            o[e] = *reinterpret_cast<const uint32_t*>(&h);
        }
        *reinterpret_cast<uint4*>(sg.dst + pl * sg.dst_plane + r * sg.dst_row + (c % kChunksPerRow) * 8) =
            make_uint4(o[0], o[1], o[2], o[3]);
    }
    __shared__ float s_max[8];
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, off));
    if ((threadIdx.x & 31) == 0) s_max[threadIdx.x >> 5] = amax;
    const bool blk_bad = __syncthreads_or(bad);
    const bool blk_inexact = __syncthreads_or(inexact);
    if (threadIdx.x == 0) {
        float m = 0.f;
        for (int i = 0; i < (int)(blockDim.x >> 5); ++i) m = fmaxf(m, s_max[i]);
        ptx::griddep_wait();  // the word is cleared before
        if (blk_bad || (blk_inexact && m < 0.0625f)) *cp.any_bad = 1;
    }
}

// ------------------------------------------------------------------------ residue order

// Rows of [planes][n][row_bytes] between the sequence order and the residue order of `dil`
// (m = n / dil): residue-order row r * m + t is sequence row r + dil * t.  One thread per
// 16-byte chunk (4-byte word for rows of 4 bytes).
__global__ void __launch_bounds__(256) lca_permute_rows(PermuteParams pp) {
    const int unit = (pp.row_bytes % 16 == 0) ? 16 : 4;
    const long long per_row = pp.row_bytes / unit;
    const long long total = pp.planes * pp.n * per_row;
    const int m = pp.n / pp.dil;
    for (long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x; i < total;
         i += (long long)gridDim.x * blockDim.x) {
        const long long c = i % per_row;
        const long long rest = i / per_row;
        const int row = (int)(rest % pp.n);
        const long long plane = rest / pp.n;
        // the output row `row` reads input row `from`
        const int from = pp.to_residue ? (row / m) + pp.dil * (row % m) : (row % pp.dil) * m + row / pp.dil;
        const uint8_t* src = pp.src + (plane * pp.n + from) * pp.row_bytes + c * unit;
        uint8_t* dst = pp.dst + (plane * pp.n + row) * pp.row_bytes + c * unit;
        if (unit == 16)
            *reinterpret_cast<uint4*>(dst) = *reinterpret_cast<const uint4*>(src);
        else
            *reinterpret_cast<uint32_t*>(dst) = *reinterpret_cast<const uint32_t*>(src);
    }
}

// ------------------------------------------------------------------------ halo pack

__global__ void __launch_bounds__(256) lca_pack_halo(HaloPackParams hp) {
    // one thread per 16-byte chunk of send[2][2][bh][halo][d]
    const int per_row = hp.d * 2 / 16;
    const long long total = 4ll * hp.bh * hp.halo * per_row;
    for (long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x; i < total;
         i += (long long)gridDim.x * blockDim.x) {
        const int c = (int)(i % per_row);
        long long rest = i / per_row;
        const int r = (int)(rest % hp.halo);
        rest /= hp.halo;
        const int b = (int)(rest % hp.bh);
        rest /= hp.bh;
        const int kv = (int)(rest & 1);
        const int side = (int)(rest >> 1);
        const int row = side == 0 ? r : hp.n - hp.halo + r;
        const uint16_t* src = (kv ? hp.v : hp.k) + ((size_t)b * hp.n + row) * hp.d + c * 8;
        *reinterpret_cast<uint4*>(hp.send + (size_t)i * 8) = *reinterpret_cast<const uint4*>(src);
    }
}

// ------------------------------------------------------------------------ combine

template <int D>
__global__ void __launch_bounds__(kCombineThreads) lca_combine_global_rows(CombineParams cp) {
    // One block per (bh, global row).  The block's threads form groups of D / 4 lanes;
    // group g reads partials g, g + kGroups, ... (lane = 4 adjacent output columns, one
    // 16-byte load each), four of them in flight per thread, and folds them into its own
    // running (max, sum, acc) with an online log-sum-exp.  The groups' results meet in
    // shared memory.  The loads of a batch do not depend on one another, so a row's
    // partials arrive in a few round trips to L2 however many splits there are.
    constexpr int kLanes = D / 4;
    constexpr int kGroups = kCombineThreads / kLanes;
    constexpr int kBatch = 4;
    __shared__ float4 s_acc[kGroups][kLanes];
    __shared__ float s_m[kGroups], s_l[kGroups];
    ptx::griddep_wait();  // the partials are written by the launch before this one
    const long long row = blockIdx.x;  // b * G + g
    if (row >= (long long)cp.num_global * cp.bh) {  // no global rows: only the epoch step below
        if (cp.epoch != nullptr && threadIdx.x == 0) {
            __threadfence();
            if (atomicAdd(cp.ticket, 1u) == gridDim.x - 1) {
                *cp.ticket = 0u;
                atomicAdd(cp.epoch, 1u);
            }
        }
        return;
    }
    const int g = (int)(row % cp.num_global);
    const int bh = (int)(row / cp.num_global);
    const int grp = (int)threadIdx.x / kLanes;
    const int lane = (int)threadIdx.x % kLanes;
    if (cp.epoch != nullptr && ((*reinterpret_cast<volatile unsigned int*>(cp.epoch) + 1u) & 1u)) {
        cp.part_o += cp.parity_floats;
        cp.part_lse += cp.parity_floats;
    }
    // a split past the end of the keys, or the odd half of a one-tile split, wrote nothing
    auto valid = [&](int part) {
        if (part >= cp.n_parts) return false;
        if (cp.split_tiles == 0) return true;
        const int s = part >> 1;
        const int first_key = s * cp.split_tiles * 128;
        int tiles = (cp.split_keys - first_key + 127) / 128;
        if (tiles > cp.split_tiles) tiles = cp.split_tiles;
        return tiles > (part & 1);
    };
    float m = -INFINITY, l = 0.f;
    float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
    for (int base = grp; base < cp.n_parts; base += kBatch * kGroups) {
        float ls[kBatch];
        float4 v[kBatch];
#pragma unroll
        for (int j = 0; j < kBatch; ++j) {
            const int s = base + j * kGroups;
            ls[j] = -INFINITY;
            v[j] = make_float4(0.f, 0.f, 0.f, 0.f);
            if (valid(s)) {
                ls[j] = __ldg(cp.part_lse + (size_t)s * cp.part_stride_lse + row);
                v[j] = __ldg(reinterpret_cast<const float4*>(cp.part_o + (size_t)s * cp.part_stride_o + row * D) + lane);
            }
        }
#pragma unroll
        for (int j = 0; j < kBatch; ++j) {
            if (ls[j] == -INFINITY) continue;
            if (ls[j] > m) {
                const float c = __expf(m - ls[j]);  // 0 while m is -inf (l and acc are 0)
                l *= c;
                acc.x *= c;
                acc.y *= c;
                acc.z *= c;
                acc.w *= c;
                m = ls[j];
            }
            const float wt = __expf(ls[j] - m);
            l += wt;
            acc.x += wt * v[j].x;
            acc.y += wt * v[j].y;
            acc.z += wt * v[j].z;
            acc.w += wt * v[j].w;
        }
    }
    s_acc[grp][lane] = acc;
    if (lane == 0) {
        s_m[grp] = m;
        s_l[grp] = l;
    }
    __syncthreads();
    float mx = -INFINITY;
#pragma unroll
    for (int i = 0; i < kGroups; ++i) mx = fmaxf(mx, s_m[i]);
    float wtot = 0.f;
    float sc[kGroups];
#pragma unroll
    for (int i = 0; i < kGroups; ++i) {
        sc[i] = s_m[i] == -INFINITY ? 0.f : __expf(s_m[i] - mx);
        wtot += sc[i] * s_l[i];
    }
    const float inv = 1.f / wtot;
    const float lse = mx + __logf(wtot);
    float* out_row = nullptr;
    float* lse_out = nullptr;
    size_t out_idx = 0;  // 16-bit output: element index of the row
    int out16 = 0;
    if (cp.out_o != nullptr) {
        out_row = cp.out_o + row * D;
        lse_out = cp.out_lse + row;
    } else {
        const int orow = cp.gidx[g] - cp.row_off;
        if (orow >= 0 && orow < cp.n_rows) {  // else owned by another shard
            out_idx = (size_t)(bh / cp.heads) * cp.o_b + (size_t)(bh % cp.heads) * cp.o_h + (size_t)orow * cp.o_n;
            out16 = cp.out16;
            out_row = static_cast<float*>(cp.o) + (out16 ? 0 : out_idx);
            lse_out = cp.lse != nullptr ? cp.lse + (size_t)bh * cp.n_rows + orow : nullptr;
        }
    }
    if (out_row != nullptr) {
        for (int c = threadIdx.x; c < D; c += blockDim.x) {
            const float* col = reinterpret_cast<const float*>(&s_acc[0][0]) + c;
            float a = 0.f;
#pragma unroll
            for (int i = 0; i < kGroups; ++i) a += sc[i] * col[i * D];
            const float val = a * inv;
            if (out16 == kOut16BF16)
                static_cast<__nv_bfloat16*>(cp.o)[out_idx + c] = __float2bfloat16_rn(val);
            else if (out16 == kOut16F16)
                static_cast<__half*>(cp.o)[out_idx + c] = __float2half_rn(val);
            else
                out_row[c] = val;
        }
        if (threadIdx.x == 0 && lse_out != nullptr) *lse_out = lse;
    }
    if (cp.epoch != nullptr) {
        // the last block of the merge ends the peer step: every block has read the epoch
        __syncthreads();
        if (threadIdx.x == 0) {
            __threadfence();
            if (atomicAdd(cp.ticket, 1u) == gridDim.x - 1) {
                *cp.ticket = 0u;
                atomicAdd(cp.epoch, 1u);
            }
        }
    }
}

// ------------------------------------------------------------------------ peer put

__global__ void __launch_bounds__(256) lca_peer_put(PeerPutParams pp) {
    const unsigned int e = *reinterpret_cast<volatile const unsigned int*>(pp.epoch) + 1u;
    const unsigned long long tid = (unsigned long long)blockIdx.x * blockDim.x + threadIdx.x;
    const unsigned long long nthr = (unsigned long long)gridDim.x * blockDim.x;
    for (int j = 0; j < pp.n_jobs; ++j) {
        const uint4* src = static_cast<const uint4*>(pp.src[j]);
        uint4* dst = reinterpret_cast<uint4*>(static_cast<uint8_t*>(pp.dst[j]) + ((e & 1u) ? pp.parity_bytes[j] : 0ull));
        const unsigned long long n = pp.bytes[j] / 16;
        for (unsigned long long i = tid; i < n; i += nthr) dst[i] = src[i];
    }
    __threadfence_system();
    __syncthreads();
    if ((int)threadIdx.x < pp.world && pp.signal[threadIdx.x] != nullptr)
        atomicAdd_system(pp.signal[threadIdx.x], 1u);
    if (blockIdx.x == 0 && (int)threadIdx.x < pp.world && pp.wait[threadIdx.x] != nullptr) {
        // bounded wait for every other rank's blocks of this step
        const unsigned int target = e * gridDim.x;
        const unsigned int* c = pp.wait[threadIdx.x];
        const uint64_t t0 = ptx::global_timer_ns();
        while ((int)(ptx::ld_acquire_sys(c) - target) < 0) {
            if (ptx::global_timer_ns() - t0 > pp.timeout_ns) {
                atomicCAS(pp.err, 0, LCA_DEVERR_TIMEOUT_PEER);
                break;
            }
            __nanosleep(200);
        }
    }
}

}  // namespace

// ------------------------------------------------------------------------ launchers

// Launch with programmatic stream serialisation: the kernel may start while the previous
// kernel of the stream is still running, and waits for it on the device (griddep_wait)
// before it reads what that kernel writes.  The kernels launched this way are exactly the
// ones that call griddep_wait first.  LCA_PDL=0 in the environment launches them in plain
// stream order instead.
static bool pdl_enabled() {
    static const bool on = [] {
        const char* e = getenv("LCA_PDL");
        return !(e != nullptr && e[0] == '0');
    }();
    return on;
}

template <typename... KArgs, typename... Args>
static cudaError_t launch_after_prev(void (*kern)(KArgs...), unsigned grid, unsigned block, size_t smem,
                                     cudaStream_t stream, Args&&... args) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(grid);
    cfg.blockDim = dim3(block);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = pdl_enabled() ? 1 : 0;
    return cudaLaunchKernelEx(&cfg, kern, std::forward<Args>(args)...);
}

template <int D, bool BF16, bool V16, bool EXT>
static cudaError_t launch_main_t(const TensorMaps& tm, const MainParams& p, int grid, cudaStream_t stream) {
    auto kern = V16 ? lca_swa_main_v16<D, EXT> : lca_swa_main<D, BF16, EXT>;
    const int smem = Cfg<D, BF16, V16>::kSmemBytes;
    // the shared-memory attribute is set once per device (it persists in the context)
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
    return launch_after_prev(kern, (unsigned)grid, Cfg<D, BF16, V16>::kThreads, smem, stream, tm.q, tm.k, tm.v, tm.kh,
                             tm.vh, tm.qg, tm.kg, tm.vg, tm.o, tm.po, tm.v16, tm.vg16, tm.vh16, p);
}

template <bool EXT>
static cudaError_t launch_main_v(int head_dim, bool bf16, const TensorMaps& tm, const MainParams& p, int grid,
                                 cudaStream_t stream, bool v16) {
    if (bf16 && v16)  // one launch; it picks fp16 P or the split on the device (p.v16_bad)
        return head_dim == 64 ? launch_main_t<64, true, true, EXT>(tm, p, grid, stream)
                              : launch_main_t<128, true, true, EXT>(tm, p, grid, stream);
    if (head_dim == 64)
        return bf16 ? launch_main_t<64, true, false, EXT>(tm, p, grid, stream)
                    : launch_main_t<64, false, false, EXT>(tm, p, grid, stream);
    return bf16 ? launch_main_t<128, true, false, EXT>(tm, p, grid, stream)
                : launch_main_t<128, false, false, EXT>(tm, p, grid, stream);
}

cudaError_t launch_main(int head_dim, bool bf16, const TensorMaps& tm, const MainParams& p, int grid,
                        cudaStream_t stream, bool v16) {
    if (head_dim != 64 && head_dim != 128) return cudaErrorInvalidValue;
    // the extended masks only when a call uses them
    if (p.causal || p.seg_mode != kSegNone || p.n_head_windows > 0) return launch_main_v<true>(head_dim, bf16, tm, p, grid, stream, v16);
    return launch_main_v<false>(head_dim, bf16, tm, p, grid, stream, v16);
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
    if (rows <= 0 && cp.epoch == nullptr) return cudaSuccess;
    if (rows > INT_MAX) return cudaErrorInvalidValue;
    const unsigned grid = rows > 0 ? (unsigned)rows : 1u;  // one block for the epoch step alone
    if (head_dim == 64) return launch_after_prev(lca_combine_global_rows<64>, grid, kCombineThreads, 0, stream, cp);
    if (head_dim == 128) return launch_after_prev(lca_combine_global_rows<128>, grid, kCombineThreads, 0, stream, cp);
    return cudaErrorInvalidValue;
}

cudaError_t launch_convert_v16(int head_dim, const ConvertParams& cp, cudaStream_t stream) {
    long long blocks = 0;
    for (int i = 0; i < cp.n_segments; ++i) blocks += (long long)cp.seg[i].planes * ((cp.seg[i].rows + 127) / 128);
    if (blocks <= 0) return cudaSuccess;
    if (blocks > INT_MAX) return cudaErrorInvalidValue;
    if (head_dim == 64) return launch_after_prev(lca_convert_v16<64>, (unsigned)blocks, 256, 0, stream, cp);
    if (head_dim == 128) return launch_after_prev(lca_convert_v16<128>, (unsigned)blocks, 256, 0, stream, cp);
    return cudaErrorInvalidValue;
}

cudaError_t launch_halo_pack(const HaloPackParams& hp, cudaStream_t stream) {
    const long long chunks = 4ll * hp.bh * hp.halo * (hp.d * 2 / 16);
    if (chunks <= 0) return cudaSuccess;
    const long long blocks = std::min<long long>((chunks + 255) / 256, 148ll * 16);
    lca_pack_halo<<<(unsigned)blocks, 256, 0, stream>>>(hp);
    return cudaGetLastError();
}

cudaError_t launch_permute_rows(const PermuteParams& pp, cudaStream_t stream) {
    if (pp.row_bytes % 4 != 0 || pp.dil < 1 || pp.n % pp.dil != 0) return cudaErrorInvalidValue;
    const long long units = pp.planes * pp.n * (pp.row_bytes % 16 == 0 ? pp.row_bytes / 16 : pp.row_bytes / 4);
    if (units <= 0) return cudaSuccess;
    const long long blocks = std::min<long long>((units + 255) / 256, 148ll * 16);
    lca_permute_rows<<<(unsigned)blocks, 256, 0, stream>>>(pp);
    return cudaGetLastError();
}

cudaError_t launch_peer_put(const PeerPutParams& pp, int blocks, cudaStream_t stream) {
    lca_peer_put<<<blocks, 256, 0, stream>>>(pp);
    return cudaGetLastError();
}

int main_smem_bytes(int head_dim, bool bf16) {
    if (head_dim == 64) return bf16 ? Cfg<64, true>::kSmemBytes : Cfg<64, false>::kSmemBytes;
    return bf16 ? Cfg<128, true>::kSmemBytes : Cfg<128, false>::kSmemBytes;
}

#ifdef LCA_TRACE
cudaError_t trace_read(void* host, size_t bytes) {
    const size_t need = sizeof(trace::g_trace) + sizeof(trace::g_trace_count);
    if (bytes < need) return cudaErrorInvalidValue;
    cudaError_t e = cudaMemcpyFromSymbol(host, trace::g_trace, sizeof(trace::g_trace));
    if (e == cudaSuccess)
        e = cudaMemcpyFromSymbol(static_cast<uint8_t*>(host) + sizeof(trace::g_trace), trace::g_trace_count,
                                 sizeof(trace::g_trace_count));
    static const unsigned int zeros[trace::kTraceCtas][trace::kTraceWarps] = {};
    if (e == cudaSuccess) e = cudaMemcpyToSymbol(trace::g_trace_count, zeros, sizeof(zeros));
    return e;
}
#endif

cudaError_t error_word_address(int** out) {
    void* p = nullptr;
    cudaError_t e = cudaGetSymbolAddress(&p, g_error_word);
    *out = static_cast<int*>(p);
    return e;
}

}  // namespace lca
