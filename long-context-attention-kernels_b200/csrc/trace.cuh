// trace.cuh -- optional in-kernel event trace of the main attention kernel.
//
// Off by default: LCA_TRACE_EVENT expands to nothing.  A build with -DLCA_TRACE (see
// build_native.py --trace, which writes liblca_b200_trace.so) records, for the first
// kTraceCtas CTAs, one 64-bit entry per event and warp: the event code in the top 8 bits
// and the SM clock (clock64) in the low 56.  The trace build exports lca_trace_read
// (capi.cpp; not in the public header), which copies the buffer out and clears the
// counters.  Each event costs a clock read and one global store.
#pragma once

#include <cstdint>

namespace lca {
namespace trace {

constexpr int kTraceCtas = 4;
constexpr int kTraceWarps = 24;
constexpr int kTraceEvents = 8192;

enum : int {
    // softmax warps (lane 0)
    EV_S_WAIT = 1,      // before waiting for S
    EV_S_READY = 2,     // S ready
    EV_S_LOADED = 3,    // S in registers, masked
    EV_MAX_DONE = 4,    // row max and rescale decision done
    EV_EXP_DONE = 5,    // exponentials written to TMEM (before the store wait)
    EV_P_ARRIVED = 6,   // P signalled to the MMA issuer
    EV_EPI_WAIT = 7,    // before waiting for the final O
    EV_EPI_READY = 8,   // final O ready
    EV_EPI_DONE = 9,    // epilogue done
    EV_UNIT_DECODED = 10,  // next work unit decoded
    EV_UNIT_READY = 11,    // row bounds of the unit computed
    EV_EPI_MERGED = 12,    // halves' (m, l) exchanged
    // MMA issuers (elected thread)
    EV_MMA_P_WAIT = 20,  // before waiting for P
    EV_MMA_P_READY = 21, // P ready
    EV_MMA_PV_ISSUED = 22,
    EV_MMA_K_WAIT = 23,  // before waiting for a K tile
    EV_MMA_K_READY = 24,
    EV_MMA_S_ISSUED = 25,
    // TMA producer (elected thread)
    EV_TMA_SLOT_WAIT = 30,
    EV_TMA_SLOT_FREE = 31,
};

#ifdef LCA_TRACE
// Defined here: only swa_kernels.cu includes this header.
__device__ unsigned long long g_trace[kTraceCtas][kTraceWarps][kTraceEvents];
__device__ unsigned int g_trace_count[kTraceCtas][kTraceWarps];

// `idx` is the calling thread's event count (a register); flush() stores it at exit.
__device__ __forceinline__ void event(unsigned int& idx, int code) {
    const unsigned int cta = blockIdx.x;
    const unsigned int warp = threadIdx.x >> 5;
    if (cta < (unsigned)kTraceCtas && warp < (unsigned)kTraceWarps && idx < (unsigned)kTraceEvents) {
        g_trace[cta][warp][idx] = ((unsigned long long)code << 56) | ((unsigned long long)clock64() & ((1ull << 56) - 1));
        ++idx;
    }
}
__device__ __forceinline__ void flush(unsigned int idx) {
    const unsigned int cta = blockIdx.x;
    const unsigned int warp = threadIdx.x >> 5;
    if (idx > 0 && cta < (unsigned)kTraceCtas && warp < (unsigned)kTraceWarps) g_trace_count[cta][warp] = idx;
}
// Events go through a per-thread counter `trace_i` that must be in scope.
#define LCA_TRACE_EVENT(code) ::lca::trace::event(trace_i, code)
#define LCA_TRACE_FLUSH() ::lca::trace::flush(trace_i)
#else
#define LCA_TRACE_EVENT(code) ((void)0)
#define LCA_TRACE_FLUSH() ((void)0)
#endif

}  // namespace trace
}  // namespace lca
