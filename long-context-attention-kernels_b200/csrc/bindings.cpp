// bindings.cpp -- the torch extension module `long_context_attention_kernels`, a thin
// pybind11 layer over the C ABI in include/lca.h.
//
// Mirrors the reference extension (csrc/bindings.cpp:31-80): same module name, same
// function `sliding_window_attention_forward(Q, K, V, window_size, global_tokens, scale)`
// returning a new fp32 tensor allocated through torch's caching allocator, launched on
// the current CUDA stream, errors raised as RuntimeError (IndexError for an out-of-range
// global token, as the reference's mask construction raises).  Differences: fp16 and
// bf16 inputs, head_dim 64 or 128, and launch/device errors are checked.
#include <torch/extension.h>
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>

#include <vector>

#include "lca.h"

namespace {

void check_input(const torch::Tensor& t, const char* name) {
    TORCH_CHECK(t.is_cuda(), name, " must be a CUDA tensor");
    TORCH_CHECK(t.scalar_type() == torch::kFloat16 || t.scalar_type() == torch::kBFloat16, name,
                " must be fp16 or bf16");
    TORCH_CHECK(t.is_contiguous(), name, " must be contiguous");
}

void raise_status(int st, const char* what) {
    if (st == LCA_OK) return;
    const char* detail = lca_last_error();
    if (st == LCA_ERR_INDEX) TORCH_CHECK_INDEX(false, what, ": ", detail);
    TORCH_CHECK(false, what, " failed (", lca_status_string(st), "): ", detail);
}

std::vector<torch::Tensor> forward_impl(const torch::Tensor& Q, const torch::Tensor& K, const torch::Tensor& V,
                                        int64_t window_size, const std::vector<int64_t>& globals, double scale,
                                        bool want_lse, c10::ScalarType out_type = torch::kFloat32,
                                        bool causal = false, const std::vector<int64_t>& head_windows = {},
                                        int64_t dilation = 1, const std::vector<int64_t>& cu_seqlens = {},
                                        bool token_major = false) {
    check_input(Q, "Q");
    check_input(K, "K");
    check_input(V, "V");
    TORCH_CHECK(Q.dim() == 4, token_major ? "Q must be [batch, seq_len, heads, head_dim]"
                                          : "Q must be [batch, heads, seq_len, head_dim]");
    TORCH_CHECK(K.sizes() == Q.sizes() && V.sizes() == Q.sizes(), "Q, K and V must have the same shape");
    TORCH_CHECK(K.scalar_type() == Q.scalar_type() && V.scalar_type() == Q.scalar_type(),
                "Q, K and V must have the same dtype");
    TORCH_CHECK(K.device() == Q.device() && V.device() == Q.device(), "Q, K and V must be on the same device");
    const int64_t batch = Q.size(0), heads = Q.size(token_major ? 2 : 1), seq_len = Q.size(token_major ? 1 : 2),
                  head_dim = Q.size(3);
    TORCH_CHECK(head_dim == 64 || head_dim == 128, "head_dim must be 64 or 128 (got ", head_dim, ")");
    TORCH_CHECK(window_size >= 0, "window_size must be >= 0 (got ", window_size, ")");
    TORCH_CHECK(head_windows.empty() || (int64_t)head_windows.size() == heads,
                "window_size per head needs one radius per head (got ", head_windows.size(), " for ", heads,
                " heads)");
    TORCH_CHECK(out_type == torch::kFloat32 || out_type == torch::kFloat16 || out_type == torch::kBFloat16,
                "out_dtype must be float32, float16 or bfloat16");

    c10::cuda::CUDAGuard guard(Q.device());
    auto O = torch::empty(Q.sizes(), Q.options().dtype(out_type));  // the input's layout
    torch::Tensor L;
    if (want_lse) L = torch::empty({batch, heads, seq_len}, Q.options().dtype(torch::kFloat32));

    const int dtype = Q.scalar_type() == torch::kBFloat16 ? LCA_DTYPE_BF16 : LCA_DTYPE_F16;
    std::vector<int32_t> norm(globals.size() + 1);
    int64_t G = 0;
    if (cu_seqlens.empty())
        raise_status(lca_normalize_global_tokens(globals.data(), (int64_t)globals.size(), seq_len, norm.data(), &G),
                     "global_tokens");
    size_t ws_bytes = 0;
    int64_t wmax = window_size;
    for (int64_t hw : head_windows) wmax = std::max(wmax, hw);
    TORCH_CHECK(dilation >= 1, "dilation must be >= 1");
    TORCH_CHECK(cu_seqlens.empty() || (batch == 1 && dilation == 1),
                "packed sequences take Q of shape [1, heads, total_len, head_dim] and no dilation");
    const int out_dtype = out_type == torch::kFloat32 ? LCA_DTYPE_F32
                          : (out_type == torch::kBFloat16 ? LCA_DTYPE_BF16 : LCA_DTYPE_F16);
    if (!cu_seqlens.empty()) {
        const int64_t nseq = (int64_t)cu_seqlens.size() - 1;
        G = nseq * (int64_t)globals.size();  // an upper bound on the unique global rows
        raise_status(lca_swa_workspace_size(1, heads, seq_len, head_dim, wmax, G, dtype, &ws_bytes),
                     "workspace size");
    } else if (dilation > 1) {
        raise_status(lca_swa_dilated_workspace_size(batch, heads, seq_len, head_dim, wmax, dilation, G, dtype,
                                                    out_dtype, &ws_bytes),
                     "workspace size");
    } else {
        raise_status(lca_swa_workspace_size(batch, heads, seq_len, head_dim, wmax, G, dtype, &ws_bytes),
                     "workspace size");
    }
    torch::Tensor ws;
    void* ws_ptr = nullptr;
    if (ws_bytes > 0) {
        ws = torch::empty({(int64_t)ws_bytes}, Q.options().dtype(torch::kUInt8));
        ws_ptr = ws.data_ptr();
    }
    cudaStream_t stream = at::cuda::getCurrentCUDAStream();
    const int64_t* hw = head_windows.empty() ? nullptr : head_windows.data();
    const int flags = (causal ? LCA_FLAG_CAUSAL : 0) | (token_major ? LCA_FLAG_TOKEN_MAJOR : 0);
    float* lse_ptr = want_lse ? L.data_ptr<float>() : nullptr;
    void* sp = static_cast<void*>(stream);
    int st;
    if (!cu_seqlens.empty())
        st = lca_swa_forward_varlen(Q.data_ptr(), K.data_ptr(), V.data_ptr(), O.data_ptr(), out_dtype, lse_ptr, dtype,
                                    heads, seq_len, head_dim, window_size, hw, static_cast<float>(scale), flags,
                                    cu_seqlens.data(), (int64_t)cu_seqlens.size() - 1, globals.data(),
                                    (int64_t)globals.size(), ws_ptr, ws_bytes, sp);
    else
        st = lca_swa_forward_dilated(Q.data_ptr(), K.data_ptr(), V.data_ptr(), O.data_ptr(), out_dtype, lse_ptr, dtype,
                                     batch, heads, seq_len, head_dim, window_size, hw, dilation,
                                     static_cast<float>(scale), flags, globals.data(), (int64_t)globals.size(), ws_ptr,
                                     ws_bytes, sp);
    raise_status(st, "sliding_window_attention_forward");
    if (want_lse) return {O, L};
    return {O};
}

std::vector<int64_t> tokens_from_tensor(const torch::Tensor& global_tokens) {
    // The reference accepts the index tensor on any device and converts it to int32
    // (csrc/bindings.cpp:47); here it is read on the host (a device tensor costs a copy).
    auto t = global_tokens.to(torch::kCPU, torch::kInt64).contiguous().view({-1});
    const int64_t* p = t.data_ptr<int64_t>();
    return std::vector<int64_t>(p, p + t.numel());
}

torch::Tensor sliding_window_attention_forward(torch::Tensor Q, torch::Tensor K, torch::Tensor V,
                                               int64_t window_size, torch::Tensor global_tokens, double scale) {
    return forward_impl(Q, K, V, window_size, tokens_from_tensor(global_tokens), scale, false)[0];
}

torch::Tensor sliding_window_attention_forward_list(torch::Tensor Q, torch::Tensor K, torch::Tensor V,
                                                    int64_t window_size, std::vector<int64_t> global_tokens,
                                                    double scale) {
    return forward_impl(Q, K, V, window_size, global_tokens, scale, false)[0];
}

std::vector<torch::Tensor> sliding_window_attention_forward_lse(torch::Tensor Q, torch::Tensor K, torch::Tensor V,
                                                                int64_t window_size,
                                                                std::vector<int64_t> global_tokens, double scale) {
    return forward_impl(Q, K, V, window_size, global_tokens, scale, true);
}

std::vector<torch::Tensor> sliding_window_attention_forward_ex(torch::Tensor Q, torch::Tensor K, torch::Tensor V,
                                                               int64_t window_size, std::vector<int64_t> global_tokens,
                                                               double scale, c10::ScalarType out_dtype, bool causal,
                                                               bool want_lse, std::vector<int64_t> head_windows,
                                                               int64_t dilation, std::vector<int64_t> cu_seqlens,
                                                               bool token_major) {
    return forward_impl(Q, K, V, window_size, global_tokens, scale, want_lse, out_dtype, causal, head_windows,
                        dilation, cu_seqlens, token_major);
}

// Gradients of the forward (include/lca.h lca_swa_backward): dQ, dK, dV in fp32, from the
// forward's fp32 O and LSE and the fp32 gradient dO of O.  No counterpart in the reference.
std::vector<torch::Tensor> sliding_window_attention_backward(torch::Tensor Q, torch::Tensor K, torch::Tensor V,
                                                             torch::Tensor O, torch::Tensor LSE, torch::Tensor dO,
                                                             int64_t window_size,
                                                             std::vector<int64_t> global_tokens, double scale) {
    check_input(Q, "Q");
    check_input(K, "K");
    check_input(V, "V");
    TORCH_CHECK(Q.dim() == 4, "Q must be [batch, heads, seq_len, head_dim]");
    TORCH_CHECK(K.sizes() == Q.sizes() && V.sizes() == Q.sizes(), "Q, K and V must have the same shape");
    TORCH_CHECK(K.scalar_type() == Q.scalar_type() && V.scalar_type() == Q.scalar_type(),
                "Q, K and V must have the same dtype");
    for (const torch::Tensor* t : {&O, &dO}) {
        TORCH_CHECK(t->is_cuda() && t->scalar_type() == torch::kFloat32 && t->is_contiguous() &&
                        t->sizes() == Q.sizes(),
                    "O and dO must be contiguous fp32 CUDA tensors of Q's shape");
    }
    const int64_t batch = Q.size(0), heads = Q.size(1), seq_len = Q.size(2), head_dim = Q.size(3);
    TORCH_CHECK(LSE.is_cuda() && LSE.scalar_type() == torch::kFloat32 && LSE.is_contiguous() &&
                    LSE.numel() == batch * heads * seq_len,
                "LSE must be a contiguous fp32 CUDA tensor [batch, heads, seq_len]");
    TORCH_CHECK(head_dim == 64 || head_dim == 128, "head_dim must be 64 or 128 (got ", head_dim, ")");
    TORCH_CHECK(window_size >= 0, "window_size must be >= 0 (got ", window_size, ")");
    c10::cuda::CUDAGuard guard(Q.device());
    const int dtype = Q.scalar_type() == torch::kBFloat16 ? LCA_DTYPE_BF16 : LCA_DTYPE_F16;
    std::vector<int32_t> norm(global_tokens.size() + 1);
    int64_t G = 0;
    raise_status(lca_normalize_global_tokens(global_tokens.data(), (int64_t)global_tokens.size(), seq_len, norm.data(),
                                             &G),
                 "global_tokens");
    size_t ws_bytes = 0;
    raise_status(lca_swa_backward_workspace_size(batch, heads, seq_len, head_dim, window_size, G, dtype, &ws_bytes),
                 "backward workspace size");
    torch::Tensor ws;
    void* ws_ptr = nullptr;
    if (ws_bytes > 0) {
        ws = torch::empty({(int64_t)ws_bytes}, Q.options().dtype(torch::kUInt8));
        ws_ptr = ws.data_ptr();
    }
    auto f32 = Q.options().dtype(torch::kFloat32);
    auto dQ = torch::empty(Q.sizes(), f32), dK = torch::empty(Q.sizes(), f32), dV = torch::empty(Q.sizes(), f32);
    cudaStream_t stream = at::cuda::getCurrentCUDAStream();
    const int st = lca_swa_backward(Q.data_ptr(), K.data_ptr(), V.data_ptr(), O.data_ptr<float>(),
                                    LSE.data_ptr<float>(), dO.data_ptr<float>(), dQ.data_ptr<float>(),
                                    dK.data_ptr<float>(), dV.data_ptr<float>(), dtype, batch, heads, seq_len, head_dim,
                                    window_size, static_cast<float>(scale), global_tokens.data(),
                                    (int64_t)global_tokens.size(), ws_ptr, ws_bytes, static_cast<void*>(stream));
    raise_status(st, "sliding_window_attention_backward");
    return {dQ, dK, dV};
}

int device_error() {
    int code = 0;
    raise_status(lca_device_error(&code), "device_error");
    return code;
}

}  // namespace

PYBIND11_MODULE(TORCH_EXTENSION_NAME, m) {
    m.def("sliding_window_attention_forward", &sliding_window_attention_forward,
          "Sliding window + global token attention forward (B200 sm_100a)", py::arg("Q"), py::arg("K"),
          py::arg("V"), py::arg("window_size"), py::arg("global_tokens"), py::arg("scale"));
    m.def("sliding_window_attention_forward_list", &sliding_window_attention_forward_list,
          "As sliding_window_attention_forward, with global tokens as a list of ints", py::arg("Q"), py::arg("K"),
          py::arg("V"), py::arg("window_size"), py::arg("global_tokens"), py::arg("scale"));
    m.def("sliding_window_attention_forward_lse", &sliding_window_attention_forward_lse,
          "Forward returning (O, LSE); LSE is the natural-log log-sum-exp per query row", py::arg("Q"),
          py::arg("K"), py::arg("V"), py::arg("window_size"), py::arg("global_tokens"), py::arg("scale"));
    m.def("sliding_window_attention_forward_ex", &sliding_window_attention_forward_ex,
          "Forward with the output in out_dtype (float32, float16 or bfloat16), optionally causal (keys j <= i); "
          "returns [O] or [O, LSE]",
          py::arg("Q"), py::arg("K"), py::arg("V"), py::arg("window_size"), py::arg("global_tokens"),
          py::arg("scale"), py::arg("out_dtype"), py::arg("causal"), py::arg("want_lse"),
          py::arg("head_windows") = std::vector<int64_t>{}, py::arg("dilation") = 1,
          py::arg("cu_seqlens") = std::vector<int64_t>{}, py::arg("token_major") = false);
    m.def("sliding_window_attention_backward", &sliding_window_attention_backward,
          "Gradients (dQ, dK, dV), fp32, of the forward from its O and LSE and the gradient dO of O",
          py::arg("Q"), py::arg("K"), py::arg("V"), py::arg("O"), py::arg("LSE"), py::arg("dO"),
          py::arg("window_size"), py::arg("global_tokens"), py::arg("scale"));
    m.def("device_error", &device_error, "Read and clear the device-side error word (synchronises)");
    m.attr("abi_version") = lca_abi_version();
}
