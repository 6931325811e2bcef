// capi.cpp -- the C ABI (include/lca.h): argument validation with the reference's
// semantics, workspace layout, TMA tensor-map construction and the launch sequence
// gather -> main -> combine on the caller's stream.
#include "lca.h"

#include <cuda.h>
#include <cuda_runtime.h>

#include <algorithm>
#include <climits>
#include <cstdarg>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <mutex>
#include <string>
#include <vector>

#include "swa_kernels.h"

namespace {

thread_local std::string g_last_error;
thread_local cudaEvent_t g_ev_before_main = nullptr;
thread_local cudaEvent_t g_ev_after_main = nullptr;

int fail(int status, const char* fmt, ...) {
    char buf[512];
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(buf, sizeof(buf), fmt, ap);
    va_end(ap);
    g_last_error = buf;
    return status;
}

}  // namespace

int lca::report_error(int status, const char* fmt, ...) {
    char buf[512];
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(buf, sizeof(buf), fmt, ap);
    va_end(ap);
    g_last_error = buf;
    return status;
}

namespace {

int fail_cuda(cudaError_t e, const char* what) {
    return fail(LCA_ERR_CUDA, "%s: %s (%s)", what, cudaGetErrorName(e), cudaGetErrorString(e));
}

// ------------------------------------------------------------------ device checks

constexpr int kMaxDevices = 64;
std::mutex g_dev_mu;
int g_dev_state[kMaxDevices];          // 0 unknown, 1 ok, -1 unsupported
int* g_dev_err_word[kMaxDevices];      // device address of the error word
int g_dev_sms[kMaxDevices];            // multiprocessor count

typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                  const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                  CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn get_encode_fn() {
    static EncodeTiledFn fn = nullptr;
    static std::once_flag once;
    std::call_once(once, [] {
        void* p = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<EncodeTiledFn>(p);
    });
    return fn;
}

int check_device(int* dev_out, int** err_word) {
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return fail_cuda(e, "cudaGetDevice");
    if (dev < 0 || dev >= kMaxDevices) return fail(LCA_ERR_UNSUPPORTED, "device ordinal %d out of range", dev);
    std::lock_guard<std::mutex> lk(g_dev_mu);
    if (g_dev_state[dev] == 0) {
        int major = 0, minor = 0;
        cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, dev);
        cudaDeviceGetAttribute(&minor, cudaDevAttrComputeCapabilityMinor, dev);
        if (major != 10 || minor != 0) {
            g_dev_state[dev] = -1;
        } else {
            int* addr = nullptr;
            e = lca::error_word_address(&addr);
            if (e != cudaSuccess) return fail_cuda(e, "cudaGetSymbolAddress(error word)");
            g_dev_err_word[dev] = addr;
            cudaDeviceGetAttribute(&g_dev_sms[dev], cudaDevAttrMultiProcessorCount, dev);
            if (g_dev_sms[dev] <= 0) g_dev_sms[dev] = 148;
            g_dev_state[dev] = 1;
        }
    }
    if (g_dev_state[dev] < 0)
        return fail(LCA_ERR_UNSUPPORTED, "device %d is not an sm_100 (B200-class) GPU; this library is built for sm_100a",
                    dev);
    *dev_out = dev;
    *err_word = g_dev_err_word[dev];
    return LCA_OK;
}

// ------------------------------------------------------------------ problem layout

constexpr int kMinGrowUnits = 148;  // at least one global-row unit per SM when possible
constexpr size_t kAlign = 1024;

size_t align_up(size_t x, size_t a) { return (x + a - 1) / a * a; }

struct Layout {
    int64_t bh = 0, n = 0, d = 0, G = 0;
    int g_tiles = 0, gpad = 0, key_tiles = 0, n_splits = 0, split_tiles = 0;
    size_t off_gidx = 0, off_qg = 0, off_kg = 0, off_vg = 0, off_po = 0, off_plse = 0, total = 0;
};

// Split of the n keys for the global-row units.  A unit covers `split_tiles` key tiles
// (its two query-tile warpgroups take alternate tiles), sized at about twice a band
// unit's work so units stay similar in length, but shrunk until there are enough units
// to occupy every SM.  Each split yields two partial results (even / odd tiles).
Layout make_layout(int64_t bh, int64_t n, int64_t d, int64_t G, int64_t window) {
    Layout L;
    L.bh = bh;
    L.n = n;
    L.d = d;
    L.G = G;
    if (G <= 0 || bh <= 0 || n <= 0) return L;
    L.g_tiles = (int)((G + lca::kTileRows - 1) / lca::kTileRows);
    L.gpad = L.g_tiles * lca::kTileRows;
    L.key_tiles = (int)((n + lca::kTileRows - 1) / lca::kTileRows);
    const int64_t w = std::min(window, n);
    const int64_t band_tiles = (2 * w + 2 * lca::kTileRows - 1) / lca::kTileRows + L.g_tiles;
    int64_t split = std::max<int64_t>(4, std::min<int64_t>(64, 4 * band_tiles));
    const int64_t units_per_split_count = bh * L.g_tiles;
    while (split > 2 && units_per_split_count * ((L.key_tiles + split - 1) / split) < kMinGrowUnits) split -= 2;
    split += split & 1;
    L.split_tiles = (int)split;
    L.n_splits = (L.key_tiles + L.split_tiles - 1) / L.split_tiles;
    const int64_t parts = 2 * (int64_t)L.n_splits;
    size_t off = 0;
    L.off_gidx = off;
    off = align_up(off + sizeof(int) * L.gpad, kAlign);
    const size_t gbytes = (size_t)bh * L.gpad * d * 2;
    L.off_qg = off;
    off = align_up(off + gbytes, kAlign);
    L.off_kg = off;
    off = align_up(off + gbytes, kAlign);
    L.off_vg = off;
    off = align_up(off + gbytes, kAlign);
    L.off_po = off;
    off = align_up(off + (size_t)parts * bh * L.gpad * d * 4, kAlign);
    L.off_plse = off;
    off = align_up(off + (size_t)parts * bh * L.gpad * 4, kAlign);
    L.total = off;
    return L;
}

// ------------------------------------------------------------------ tensor maps

int encode_3d(CUtensorMap* m, CUtensorMapDataType dt, int esize, const void* base, uint64_t d, uint64_t rows,
              uint64_t planes, uint32_t box_x, const char* name) {
    EncodeTiledFn enc = get_encode_fn();
    if (enc == nullptr) return fail(LCA_ERR_CUDA, "cuTensorMapEncodeTiled is unavailable from the driver");
    cuuint64_t dims[3] = {d, rows, planes};
    cuuint64_t strides[2] = {d * (uint64_t)esize, d * rows * (uint64_t)esize};
    cuuint32_t box[3] = {box_x, (cuuint32_t)lca::kTileRows, 1};
    cuuint32_t estr[3] = {1, 1, 1};
    CUresult r = enc(m, dt, 3, const_cast<void*>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                     CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                     CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) return fail(LCA_ERR_CUDA, "cuTensorMapEncodeTiled(%s) failed with CUresult %d", name, (int)r);
    return LCA_OK;
}

unsigned long long wait_timeout_ns() {
    static unsigned long long v = [] {
        const char* s = getenv("LCA_WAIT_TIMEOUT_MS");
        long long ms = s ? atoll(s) : 2000;
        if (ms <= 0) ms = 2000;
        return (unsigned long long)ms * 1000000ull;
    }();
    return v;
}

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

}  // namespace

// ====================================================================== C ABI

extern "C" {

int lca_abi_version(void) { return LCA_ABI_VERSION; }

const char* lca_status_string(int status) {
    switch (status) {
        case LCA_OK: return "ok";
        case LCA_ERR_INVALID_ARGUMENT: return "invalid argument";
        case LCA_ERR_INDEX: return "global token index out of range";
        case LCA_ERR_UNSUPPORTED: return "unsupported configuration";
        case LCA_ERR_WORKSPACE: return "workspace too small or misaligned";
        case LCA_ERR_CUDA: return "CUDA error";
        case LCA_ERR_DEVICE: return "device-side error";
        default: return "unknown status";
    }
}

const char* lca_last_error(void) { return g_last_error.c_str(); }

int lca_normalize_global_tokens(const int64_t* tokens, int64_t count, int64_t seq_len, int32_t* out,
                                int64_t* out_count) {
    if (out_count == nullptr) return fail(LCA_ERR_INVALID_ARGUMENT, "out_count is NULL");
    if (count < 0) return fail(LCA_ERR_INVALID_ARGUMENT, "negative global token count %lld", (long long)count);
    if (count > 0 && (tokens == nullptr || out == nullptr))
        return fail(LCA_ERR_INVALID_ARGUMENT, "global token arrays are NULL");
    if (seq_len < 0 || seq_len > INT_MAX) return fail(LCA_ERR_INVALID_ARGUMENT, "seq_len %lld out of range", (long long)seq_len);
    std::vector<int32_t> v;
    v.reserve((size_t)count);
    for (int64_t i = 0; i < count; ++i) {
        int64_t t = tokens[i];
        if (t < -seq_len || t >= seq_len)
            return fail(LCA_ERR_INDEX, "index %lld is out of bounds for dimension 0 with size %lld", (long long)t,
                        (long long)seq_len);
        if (t < 0) t += seq_len;
        v.push_back((int32_t)t);
    }
    std::sort(v.begin(), v.end());
    v.erase(std::unique(v.begin(), v.end()), v.end());
    std::copy(v.begin(), v.end(), out);
    *out_count = (int64_t)v.size();
    return LCA_OK;
}

int lca_swa_workspace_size(int64_t batch, int64_t heads, int64_t seq_len, int64_t head_dim, int64_t window_size,
                           int64_t num_unique_global, int dtype, size_t* out_bytes) {
    if (out_bytes == nullptr) return fail(LCA_ERR_INVALID_ARGUMENT, "out_bytes is NULL");
    if (batch < 0 || heads < 0 || seq_len < 0 || num_unique_global < 0)
        return fail(LCA_ERR_INVALID_ARGUMENT, "negative size");
    if (dtype != LCA_DTYPE_F16 && dtype != LCA_DTYPE_BF16) return fail(LCA_ERR_UNSUPPORTED, "dtype %d", dtype);
    if (head_dim != 64 && head_dim != 128)
        return fail(LCA_ERR_UNSUPPORTED, "head_dim %lld (supported: 64, 128)", (long long)head_dim);
    if (window_size < 0) return fail(LCA_ERR_INVALID_ARGUMENT, "window_size must be >= 0");
    *out_bytes = make_layout(batch * heads, seq_len, head_dim, std::min(num_unique_global, seq_len), window_size).total;
    return LCA_OK;
}

int lca_swa_forward(const void* q, const void* k, const void* v, float* out, float* lse, int dtype,
                    int64_t batch, int64_t heads, int64_t seq_len, int64_t head_dim, int64_t window_size,
                    float scale, const int64_t* global_tokens, int64_t num_global_tokens, void* workspace,
                    size_t workspace_bytes, void* stream_ptr) {
    g_last_error.clear();
    // ---- argument checks (csrc/bindings.cpp:25-42 restated for a C caller)
    if (dtype != LCA_DTYPE_F16 && dtype != LCA_DTYPE_BF16)
        return fail(LCA_ERR_UNSUPPORTED, "dtype %d is not supported (fp16 or bf16 inputs)", dtype);
    if (head_dim != 64 && head_dim != 128)
        return fail(LCA_ERR_UNSUPPORTED, "head_dim %lld is not supported (64 or 128)", (long long)head_dim);
    if (batch < 0 || heads < 0 || seq_len < 0) return fail(LCA_ERR_INVALID_ARGUMENT, "negative shape");
    if (window_size < 0) return fail(LCA_ERR_INVALID_ARGUMENT, "window_size must be >= 0 (got %lld)", (long long)window_size);
    if (seq_len > ((int64_t)1 << 29))
        return fail(LCA_ERR_UNSUPPORTED, "seq_len %lld too large (max 2^29)", (long long)seq_len);
    const int64_t bh = batch * heads;
    if (bh > INT_MAX / 64) return fail(LCA_ERR_UNSUPPORTED, "batch*heads %lld too large", (long long)bh);
    if (num_global_tokens < 0) return fail(LCA_ERR_INVALID_ARGUMENT, "negative global token count");
    if (num_global_tokens > 0 && global_tokens == nullptr)
        return fail(LCA_ERR_INVALID_ARGUMENT, "global_tokens is NULL");

    // Global tokens are validated even for empty problems, as the reference's mask
    // construction would raise on them.
    std::vector<int32_t> gl((size_t)num_global_tokens + 1);
    int64_t G = 0;
    int st = lca_normalize_global_tokens(global_tokens, num_global_tokens, seq_len, gl.data(), &G);
    if (st != LCA_OK) return st;
    if (bh == 0 || seq_len == 0) return LCA_OK;  // nothing to compute

    if (q == nullptr || k == nullptr || v == nullptr || out == nullptr)
        return fail(LCA_ERR_INVALID_ARGUMENT, "q, k, v and out must be non-NULL");
    if (!aligned16(q) || !aligned16(k) || !aligned16(v) || !aligned16(out))
        return fail(LCA_ERR_INVALID_ARGUMENT, "q, k, v and out must be 16-byte aligned");
    if (lse != nullptr && (reinterpret_cast<uintptr_t>(lse) & 3u))
        return fail(LCA_ERR_INVALID_ARGUMENT, "lse must be 4-byte aligned");

    int dev = 0;
    int* err_word = nullptr;
    st = check_device(&dev, &err_word);
    if (st != LCA_OK) return st;

    const Layout L = make_layout(bh, seq_len, head_dim, G, window_size);
    if (workspace_bytes < L.total) return fail(LCA_ERR_WORKSPACE, "workspace needs %zu bytes, got %zu", L.total, workspace_bytes);
    if (L.total > 0 && (workspace == nullptr || (reinterpret_cast<uintptr_t>(workspace) % 256) != 0))
        return fail(LCA_ERR_WORKSPACE, "workspace must be non-NULL and 256-byte aligned");

    cudaStream_t stream = static_cast<cudaStream_t>(stream_ptr);
    const bool bf16 = dtype == LCA_DTYPE_BF16;
    const CUtensorMapDataType tdt = bf16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
    const int n = (int)seq_len;
    const int d = (int)head_dim;
    uint8_t* ws = static_cast<uint8_t*>(workspace);

    lca::TensorMaps tm;
    memset(&tm, 0, sizeof(tm));
    if ((st = encode_3d(&tm.q, tdt, 2, q, d, n, bh, 64, "q")) != LCA_OK) return st;
    if ((st = encode_3d(&tm.k, tdt, 2, k, d, n, bh, 64, "k")) != LCA_OK) return st;
    if ((st = encode_3d(&tm.v, tdt, 2, v, d, n, bh, 64, "v")) != LCA_OK) return st;
    if ((st = encode_3d(&tm.o, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 4, out, d, n, bh, 32, "out")) != LCA_OK) return st;

    lca::MainParams p;
    memset(&p, 0, sizeof(p));
    p.n = n;
    p.bh = (int)bh;
    p.window = (int)std::min<int64_t>(window_size, seq_len);
    p.q_tiles = (n + lca::kTileRows - 1) / lca::kTileRows;
    p.num_global = (int)G;
    p.scale_log2 = scale * 1.4426950408889634f;
    // scale == 0 gives every visible key the same weight; a tiny positive factor keeps
    // that (scores * 1e-30 round to 0 in the exponent) while masked scores stay -inf.
    if (p.scale_log2 == 0.f) p.scale_log2 = 1e-30f;
    p.lse = lse;
    p.err = err_word;
    p.timeout_ns = wait_timeout_ns();

    if (G > 0) {
        p.g_tiles = L.g_tiles;
        p.gpad = L.gpad;
        p.n_splits = L.n_splits;
        p.split_tiles = L.split_tiles;
        p.n_grow_units = (int)(bh * L.g_tiles * L.n_splits);
        p.gidx = reinterpret_cast<const int*>(ws + L.off_gidx);
        p.part_lse = reinterpret_cast<float*>(ws + L.off_plse);
        void* qg = ws + L.off_qg;
        void* kg = ws + L.off_kg;
        void* vg = ws + L.off_vg;
        if ((st = encode_3d(&tm.qg, tdt, 2, qg, d, L.gpad, bh, 64, "q_global")) != LCA_OK) return st;
        if ((st = encode_3d(&tm.kg, tdt, 2, kg, d, L.gpad, bh, 64, "k_global")) != LCA_OK) return st;
        if ((st = encode_3d(&tm.vg, tdt, 2, vg, d, L.gpad, bh, 64, "v_global")) != LCA_OK) return st;
        if ((st = encode_3d(&tm.po, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 4, ws + L.off_po, d, L.gpad,
                            (uint64_t)2 * L.n_splits * bh, 32, "partial_out")) != LCA_OK)
            return st;

        // 1. gather the global rows (chunks of kGatherChunk indices per launch)
        static thread_local lca::GatherParams gp;
        for (int first = 0; first < L.gpad; first += lca::kGatherChunk) {
            gp.n = n;
            gp.gpad = L.gpad;
            gp.num_global = (int)G;
            gp.bh = (int)bh;
            gp.first = first;
            gp.count = std::min(lca::kGatherChunk, L.gpad - first);
            gp.gidx_out = reinterpret_cast<int*>(ws + L.off_gidx);
            gp.qg = static_cast<uint16_t*>(qg);
            gp.kg = static_cast<uint16_t*>(kg);
            gp.vg = static_cast<uint16_t*>(vg);
            for (int i = 0; i < gp.count; ++i) gp.idx[i] = (first + i < G) ? gl[first + i] : 0;
            cudaError_t e = lca::launch_gather(d, q, k, v, gp, (int)bh, stream);
            if (e != cudaSuccess) return fail_cuda(e, "gather launch");
        }
    } else {
        // unused maps still need valid encodings for the kernel parameter block
        tm.qg = tm.q;
        tm.kg = tm.k;
        tm.vg = tm.v;
        tm.po = tm.o;
    }

    // 2. band + global-row units
    p.q_pairs = (p.q_tiles + 1) / 2;
    const long long units = (long long)p.n_grow_units + (long long)bh * p.q_pairs;
    if (units > INT_MAX) return fail(LCA_ERR_UNSUPPORTED, "problem too large (%lld work units)", units);
    p.n_band_units = (int)(bh * p.q_pairs);
    const int grid = (int)std::min<long long>(units, g_dev_sms[dev]);
    const bool timed = g_ev_before_main != nullptr && g_ev_after_main != nullptr;
    cudaError_t e;
    if (timed && (e = cudaEventRecord(g_ev_before_main, stream)) != cudaSuccess)
        return fail_cuda(e, "timing event record");
    e = lca::launch_main(d, bf16, tm, p, grid, stream);
    if (e != cudaSuccess) return fail_cuda(e, "main kernel launch");
    if (timed && (e = cudaEventRecord(g_ev_after_main, stream)) != cudaSuccess)
        return fail_cuda(e, "timing event record");

    // 3. merge the global-row splits over the global rows of out / lse
    if (G > 0) {
        lca::CombineParams cp;
        cp.n = n;
        cp.bh = (int)bh;
        cp.gpad = L.gpad;
        cp.num_global = (int)G;
        cp.n_splits = L.n_splits;
        cp.split_tiles = L.split_tiles;
        cp.gidx = p.gidx;
        cp.part_o = reinterpret_cast<const float*>(ws + L.off_po);
        cp.part_lse = p.part_lse;
        cp.o = out;
        cp.lse = lse;
        e = lca::launch_combine(d, cp, stream);
        if (e != cudaSuccess) return fail_cuda(e, "combine launch");
    }
    return LCA_OK;
}

int lca_set_timing_events(void* before_main, void* after_main) {
    g_ev_before_main = static_cast<cudaEvent_t>(before_main);
    g_ev_after_main = static_cast<cudaEvent_t>(after_main);
    return LCA_OK;
}

int lca_device_error(int* code) {
    if (code == nullptr) return fail(LCA_ERR_INVALID_ARGUMENT, "code is NULL");
    int dev = 0;
    int* err_word = nullptr;
    int st = check_device(&dev, &err_word);
    if (st != LCA_OK) return st;
    cudaError_t e = cudaDeviceSynchronize();
    if (e != cudaSuccess) return fail_cuda(e, "cudaDeviceSynchronize");
    int val = 0;
    e = cudaMemcpy(&val, err_word, sizeof(int), cudaMemcpyDeviceToHost);
    if (e != cudaSuccess) return fail_cuda(e, "read error word");
    const int zero = 0;
    e = cudaMemcpy(err_word, &zero, sizeof(int), cudaMemcpyHostToDevice);
    if (e != cudaSuccess) return fail_cuda(e, "clear error word");
    *code = val;
    return LCA_OK;
}

}  // extern "C"
