// swa_kernels.h -- internal interface between the C-ABI layer (capi.cpp) and the
// sm_100a kernels (swa_kernels.cu).  Not part of the public ABI (see include/lca.h).
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>
#include <cstddef>
#include <cstdint>

#include "lca.h"

namespace lca {

// The device-side error codes written to the error word when a bounded wait gives up are
// the LCA_DEVERR_* values of lca.h.

constexpr int kTileRows = 128;        // query rows / keys per tile
constexpr int kMaxPeers = 16;         // ranks of a peer-memory shard exchange
constexpr int kPeerPrepBlocks = 64;   // blocks of the peer prepare kernel (each signals every peer)
constexpr int kPeerCopyBlocks = 8;    // blocks of the peer row-partial copy kernel

// Counters at the start of a shard workspace.  Other ranks add to them over NVLink
// (system-scope atomics); they only grow, so one step's target is epoch * blocks.
struct PeerSignals {
    unsigned int prep[kMaxPeers];   // prepare blocks of rank s that finished writing here
    unsigned int fin[kMaxPeers];    // copy blocks of rank s that finished writing here
    unsigned int epoch;             // completed peer steps of this rank
    unsigned int ticket;            // merge blocks done in the current step
};
constexpr int kGatherChunk = 1024;    // global indices passed per gather launch
constexpr int kCombineThreads = 256;  // threads of one global-row merge block
constexpr int kMaxHeadWindows = 256;  // heads with a radius of their own (kernel parameter space)
constexpr int kMaxSegments = 512;     // packed sequences of one varlen call (kernel parameter space)

struct TensorMaps {
    CUtensorMap q, k, v;     // inputs [bh][n][d] (bf16 / f16), box 64 x 128 rows, 128B swizzle
    CUtensorMap kh, vh;      // sequence shards: K / V halo blocks (z = bh + b left, 2*bh + b right)
    CUtensorMap qg, kg, vg;  // compact global rows [G][3 (q, k, v)][bh][d]; maps {d, bh, G}, box 64 x 1 x 128
                             // (rows >= G read as zeros)
    CUtensorMap o;           // output [bh][n][d]: fp32 with box 32 x 128 rows and 128B swizzle, or
                             // 16-bit (MainParams::out16) with box 32 x 128 rows and no swizzle
    CUtensorMap po;          // global-row partial outputs [2*splits*bh][G][d] fp32
    CUtensorMap v16, vg16;   // bf16 inputs: fp16 copies of V [bh][n][d] and of the compact global V
                             // rows [G][bh][d] (maps {d, bh, G}); the bf16 maps when unused
    CUtensorMap vh16;        // fp16 copy of the V halo blocks (encoded like vh); vh when unused
};

// Key and query indices below are absolute positions in the full sequence unless named
// local.  Without sequence sharding q_off = 0, n = n_total and the K / V maps cover all
// keys.  With it, the K / V maps cover the local shard [q_off, q_off + n) and the halo
// maps the `halo` keys on either side; band key tiles are then aligned to the shard
// start (lead is a multiple of 128 and n of the non-last shards too), so every key tile
// lies in exactly one of left halo, shard or right halo.
struct MainParams {
    int n;            // local query rows (rows of Q, O and LSE)
    int q_off;        // absolute index of local query row 0
    int n_total;      // sequence length
    int sharded;      // K / V maps cover the shard only; keys outside it come from the halo maps
    int halo;         // rows per halo block
    int bh;           // batch * heads
    int window;       // band radius, clamped to n_total
    int lead;         // band: pair tile 0 starts `lead` keys before the pair's first query
    int key_lo, key_hi;  // band keys that exist in the maps: [key_lo, key_hi)
    int gk_lo, gk_n;  // global-row units: keys [gk_lo, gk_lo + gk_n)
    int q_tiles;      // ceil(n / 128)
    int num_global;   // G: unique global tokens
    int g_tiles;      // ceil(G / 128)
    int n_splits;     // key splits per (bh, global tile)
    int split_tiles;  // key tiles per split
    int n_grow_units; // bh * g_tiles * n_splits global-row units
    int n_band_units; // bh * q_pairs band units
    int grow_first;   // global-row units take the low unit indices (they are the longer kind)
    unsigned int* unit_counter;  // zeroed word handing out units dynamically, or nullptr (round-robin)
    int q_pairs;      // ceil(q_tiles / 2): band units per (batch, head)
    float scale_log2; // scale * log2(e)
    const int* gidx;  // [G] sorted absolute global indices
    float* lse;       // [bh][n] natural-log LSE, or nullptr
    float* part_lse;  // [2 * n_splits][bh][G]
    // bf16 inputs with an fp16 copy of V (else nullptr): 0 when every value of V converted
    // to fp16 without loss that matters (lca_convert_v16), else nonzero.  Both main-kernel
    // variants are launched; the one that does not match returns at once.
    const int* v16_bad;
    int* err;         // device error word (first error wins)
    unsigned long long timeout_ns;  // per-wait budget
    int out16;        // band rows' output type: 0 fp32, kOut16F16 fp16, kOut16BF16 bf16
    int causal;       // only keys j <= i (whole-sequence problems): band [i - w, i], global keys
                      // before the band, global rows up to themselves
    // A band radius per head (whole-sequence problems): head h of every batch uses
    // head_window[h] (each <= window) in place of window, with lead = its own radius;
    // n_head_windows = 0 means one radius for all.
    int n_head_windows;  // = heads, or 0
    int head_window[kMaxHeadWindows];
    // Segments (whole-sequence problems): the band of a row stops at the row's segment.
    // kSegEqual: segments of seg_len tokens, every global key visible to every row and every
    // global row over all keys (the dilated window, run on a residue-permuted sequence).
    // kSegVarlen: n_segs packed sequences [seg_start[s], seg_start[s + 1]); global keys and
    // global rows stay inside their own sequence.
    int seg_mode;
    int seg_len;
    int n_segs;
    int seg_start[kMaxSegments + 1];
    // Token-major q, k, v and out ([batch][n][heads][d], whole-sequence problems): their maps
    // (tm.q, tm.k, tm.v, tm.o) are 4-D {d, heads, n, batch} and take (column, head, row,
    // batch); heads4d = heads, or 0 for the 3-D head-major maps.
    int heads4d;
};
constexpr int kSegNone = 0;
constexpr int kSegEqual = 1;
constexpr int kSegVarlen = 2;
constexpr int kOut16F16 = 1;
constexpr int kOut16BF16 = 2;

// Copies the global rows owned by this shard into the compact buffer [G][3][bh][d] and
// writes the sorted index list; rows owned by other shards are left untouched (their
// owners send them).
struct GatherParams {
    int n, q_off;      // local rows of q / k / v and the absolute index of row 0
    int num_global, bh;
    int heads;         // element offset of (bh, row): (bh / heads) * s_b + (bh % heads) * s_h + row * s_n
    long long s_b, s_h, s_n;
    int first, count;  // compact rows [first, first + count) handled by this launch
    int* gidx_out;
    uint16_t* compact;
    int idx[kGatherChunk];
};

// Halo blocks sent to the neighbours: send[s][kv][b][r][:] = (kv ? v : k)[b][row][:] with
// row = r (s = 0, towards the left neighbour) or n - halo + r (s = 1, towards the right).
struct HaloPackParams {
    int n, halo, bh, d;
    const uint16_t* k;
    const uint16_t* v;
    uint16_t* send;
};

// Log-sum-exp merge of `n_parts` normalised partial results per (bh, global row).
// Partial s of row (b, g): O at part_o + s * part_stride_o + (b * G + g) * d, LSE at
// part_lse + s * part_stride_lse + b * G + g.  With split_tiles > 0 the partials are the
// main kernel's (part 2s + x covers the x-parity key tiles of split s of `split_keys`
// keys and exists only if that split has more than x tiles); with split_tiles == 0 all
// are present.  The result goes to the rows gidx[g] - row_off of o / lse that fall in
// [0, n_rows), or, when out_o is set, to out_o [bh][G][d] and out_lse [bh][G].
struct CombineParams {
    int bh, num_global, n_parts;
    int split_tiles, split_keys;
    size_t part_stride_o, part_stride_lse;
    const float* part_o;
    const float* part_lse;
    const int* gidx;
    void* o;          // fp32, or 16-bit per out16
    float* lse;
    int out16;        // type of o: 0 fp32, kOut16F16, kOut16BF16
    int heads;        // element offset of row (bh, r) of o: (bh / heads) * o_b + (bh % heads) * o_h + r * o_n
    long long o_b, o_h, o_n;
    int n_rows, row_off;
    float* out_o;
    float* out_lse;
    // peer exchange: when `epoch` is set the partials are read from the buffer of parity
    // (epoch + 1) & 1 (parity_floats further on for odd), and the last block to finish
    // advances *epoch
    unsigned int* epoch;
    unsigned int* ticket;
    size_t parity_floats;
};

// fp16 copy of bf16 V rows.  A segment is `planes` arrays of `rows` rows of d values: row
// r of plane pl at src + pl * src_plane + r * src_row (elements), written to the same
// place of dst with dst_plane / dst_row.  Rows are converted in blocks of 128.  A block
// passes when every value converts without overflow and either exactly or, for magnitudes
// below 2^-14 (fp16 subnormals, absolute error at most 2^-25), in a block whose largest
// magnitude is at least 2^-4; a block that fails sets *any_bad (which the host zeroes
// beforehand).
constexpr int kMaxConvertSegments = 4;
struct ConvertSegment {
    const uint16_t* src;
    uint16_t* dst;
    int planes, rows;
    long long src_plane, src_row, dst_plane, dst_row;
    int heads;            // source plane pl at (pl / heads) * src_plane + (pl % heads) * src_head
    long long src_head;
};
struct ConvertParams {
    int n_segments;
    ConvertSegment seg[kMaxConvertSegments];
    int* any_bad;
};
cudaError_t launch_convert_v16(int head_dim, const ConvertParams& cp, cudaStream_t stream);

// Workspace bytes of lca_swa_forward: the minimum, or with the optional fp16 copy of V
// (what lca_swa_workspace_size reports).
int workspace_bytes(int64_t batch, int64_t heads, int64_t seq_len, int64_t head_dim, int64_t window_size,
                    int64_t num_unique_global, int dtype, bool with_fp16_v, size_t* out_bytes);

// Copies contiguous 16-byte-aligned ranges into other ranks' workspaces (or this rank's),
// then bumps one counter on every other rank and, in block 0, waits until this rank's
// counters from every other rank reach (epoch + 1) * gridDim.x.  The destination of job
// j moves by parity_bytes[j] when epoch + 1 is odd (double-buffered regions).
constexpr int kMaxPutJobs = kMaxPeers + 2;
struct PeerPutParams {
    int n_jobs;
    int world;
    const void* src[kMaxPutJobs];
    void* dst[kMaxPutJobs];
    unsigned long long bytes[kMaxPutJobs];
    unsigned long long parity_bytes[kMaxPutJobs];
    unsigned int* signal[kMaxPeers];   // counter on rank r to bump (nullptr: none, e.g. self)
    unsigned int* wait[kMaxPeers];     // this rank's counter for rank s (nullptr: none)
    const unsigned int* epoch;         // this rank's completed-step count
    int* err;
    unsigned long long timeout_ns;
};

// Rows of [planes][n][row_bytes] (row_bytes a multiple of 4, n a multiple of dil) moved
// into the residue order of `dil` (to_residue) or back: residue-order row r * (n / dil) + t
// is sequence row r + dil * t.
struct PermuteParams {
    const uint8_t* src;
    uint8_t* dst;
    long long planes;
    int n, dil, row_bytes, to_residue;
};
cudaError_t launch_permute_rows(const PermuteParams& pp, cudaStream_t stream);

cudaError_t launch_peer_put(const PeerPutParams& pp, int blocks, cudaStream_t stream);

// Main kernel.  `v16`: bf16 inputs with the fp16 copy of V in tm.v16 / tm.vg16 -- launches
// the variant that reads it (fp16 P, one P*V per tile) and the one that splits bf16 P;
// p.v16_bad selects which of the two runs.
cudaError_t launch_main(int head_dim, bool bf16, const TensorMaps& tm, const MainParams& p, int grid,
                        cudaStream_t stream, bool v16 = false);
cudaError_t launch_gather(int head_dim, const void* q, const void* k, const void* v, const GatherParams& gp,
                          int bh, cudaStream_t stream);
cudaError_t launch_combine(int head_dim, const CombineParams& cp, cudaStream_t stream);
cudaError_t launch_halo_pack(const HaloPackParams& hp, cudaStream_t stream);
int main_smem_bytes(int head_dim, bool bf16);
// Record `status` and a printf-style detail message as this thread's last C-ABI error
// (what lca_last_error() returns); returns `status`.
int report_error(int status, const char* fmt, ...);

// Device address (on the current device) of the device-side error word.
cudaError_t error_word_address(int** out);

#ifdef LCA_TRACE
// Copy the main kernel's event trace (trace.cuh) to `host` and clear its counters.
cudaError_t trace_read(void* host, size_t bytes);
#endif

}  // namespace lca
