// The thin PyTorch extension over the C ABI: the per-step calls of the decode
// path (ingress, scan, and both in one call) registered as torch operators.
//
// Nothing here computes. Each operator checks its tensors, takes torch's
// current CUDA stream, calls the C ABI of libinsitu_b200.so and raises on a
// non-zero status; device memory comes from torch's allocator. The cache
// handle crosses as an int64 (the ins_cache pointer the Python mirror holds).
// The Python mirror (insitu_b200.engine.PagedCache) routes its ingress and
// scan through these operators, which keeps the per-call host work in C++.

#include <ATen/ATen.h>
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include <torch/library.h>

#include <cstdint>
#include <string>
#include <vector>

#include "../../include/insitu_b200.h"

namespace {

ins_cache *handle(int64_t h) {
    TORCH_CHECK(h != 0, "insitu: the cache handle is closed");
    return reinterpret_cast<ins_cache *>(static_cast<intptr_t>(h));
}

void check(int rc) {
    if (rc == INS_OK) return;
    const std::string msg = std::string("[status ") + std::to_string(rc) + "] " + ins_last_error();
    switch (rc) {
        case INS_EBADLEN:
        case INS_EINVAL:
            TORCH_CHECK_VALUE(false, msg);
        case INS_ERANGE:
        case INS_ETIMEOUT:
        default:
            TORCH_CHECK(false, msg);
    }
}

void check_i32(const at::Tensor &t, const char *name, int64_t tail0, int64_t tail1) {
    TORCH_CHECK(t.is_cuda() && t.scalar_type() == at::kInt && t.is_contiguous(), "insitu: ", name,
                " must be a contiguous int32 CUDA tensor");
    TORCH_CHECK(t.dim() == 3 && t.size(1) == tail0 && t.size(2) == tail1, "insitu: ", name, " must be (n, ",
                tail0, ", ", tail1, "), got ", t.sizes());
}

std::vector<int32_t> ids32(at::IntArrayRef ids) {
    std::vector<int32_t> v(ids.size());
    for (size_t i = 0; i < ids.size(); ++i) {
        TORCH_CHECK(ids[i] >= INT32_MIN && ids[i] <= INT32_MAX, "insitu: sequence id out of range");
        v[i] = static_cast<int32_t>(ids[i]);
    }
    return v;
}

// ins_ingress: rotate, quantise, pack and append one token per row of k, v
// ((n, n_kv, 64) int32); q ((n, n_kv*groups, 64) int32) is rotated into the
// returned tensor, or omitted.
c10::optional<at::Tensor> ingress(int64_t h, at::IntArrayRef seq_ids, const at::Tensor &k,
                                  const at::Tensor &v, const c10::optional<at::Tensor> &q,
                                  int64_t n_kv, int64_t q_heads, bool prerotated) {
    check_i32(k, "k", n_kv, 64);
    check_i32(v, "v", n_kv, 64);
    const int64_t n = k.size(0);
    TORCH_CHECK(v.size(0) == n && (int64_t)seq_ids.size() == n, "insitu: k, v and seq_ids disagree on n");
    c10::cuda::CUDAGuard guard(k.device());
    c10::optional<at::Tensor> q_rot;
    if (q.has_value()) {
        check_i32(*q, "q", q_heads, 64);
        TORCH_CHECK(q->size(0) == n, "insitu: q carries a different token count");
        q_rot = at::empty_like(*q);
    }
    const std::vector<int32_t> ids = ids32(seq_ids);
    check(ins_ingress(handle(h), (int32_t)n, ids.data(), q.has_value() ? q->data_ptr<int32_t>() : nullptr,
                      k.data_ptr<int32_t>(), v.data_ptr<int32_t>(),
                      q_rot.has_value() ? q_rot->data_ptr<int32_t>() : nullptr,
                      prerotated ? INS_INGRESS_PREROTATED : 0u, at::cuda::getCurrentCUDAStream().stream()));
    return q_rot;
}

// ins_scan: one decode step of attention for B sequences; returns out
// ((B, q_heads, 64) int64) and, when asked, stats ((B, n_kv, 6) int64).
std::tuple<at::Tensor, c10::optional<at::Tensor>> scan(int64_t h, at::IntArrayRef seq_ids,
                                                       c10::optional<at::IntArrayRef> lengths,
                                                       const at::Tensor &q_rot, int64_t n_kv, int64_t mode,
                                                       bool with_stats) {
    TORCH_CHECK(q_rot.dim() == 3, "insitu: q_rot must be (B, q_heads, 64)");
    check_i32(q_rot, "q_rot", q_rot.size(1), 64);
    const int64_t B = q_rot.size(0);
    TORCH_CHECK((int64_t)seq_ids.size() == B, "insitu: seq_ids and q_rot disagree on B");
    c10::cuda::CUDAGuard guard(q_rot.device());
    at::Tensor out = at::empty({B, q_rot.size(1), 64}, q_rot.options().dtype(at::kLong));
    c10::optional<at::Tensor> st;
    if (with_stats) st = at::empty({B, n_kv, 6}, q_rot.options().dtype(at::kLong));
    const std::vector<int32_t> ids = ids32(seq_ids);
    const int64_t *lens = nullptr;
    if (lengths.has_value()) {
        TORCH_CHECK((int64_t)lengths->size() == B, "insitu: lengths and q_rot disagree on B");
        lens = lengths->data();
    }
    check(ins_scan(handle(h), (int32_t)B, ids.data(), lens, q_rot.data_ptr<int32_t>(), out.data_ptr<int64_t>(),
                   st.has_value() ? reinterpret_cast<ins_stats *>(st->data_ptr<int64_t>()) : nullptr,
                   static_cast<ins_softmax>(mode), at::cuda::getCurrentCUDAStream().stream()));
    return {out, st};
}

// One decode token per sequence: the ingress of q, k, v, then the scan of
// every sequence with the new token included (kernel.py:253-355 below the
// seam), in one operator call.
std::tuple<at::Tensor, c10::optional<at::Tensor>> step(int64_t h, at::IntArrayRef seq_ids, const at::Tensor &q,
                                                       const at::Tensor &k, const at::Tensor &v, int64_t n_kv,
                                                       int64_t mode, bool with_stats) {
    TORCH_CHECK(q.dim() == 3, "insitu: q must be (B, q_heads, 64)");
    c10::optional<at::Tensor> q_rot = ingress(h, seq_ids, k, v, q, n_kv, q.size(1), false);
    return scan(h, seq_ids, c10::nullopt, *q_rot, n_kv, mode, with_stats);
}

// ins_project: y = fp16(x) @ w16^T (+ bias) with fp32 products and sums;
// w16 (out, in) fp16, x (n, in) fp32, bias (out) fp32 or none -> y (n, out) fp32.
at::Tensor project(const at::Tensor &w16, const at::Tensor &x, const c10::optional<at::Tensor> &bias) {
    TORCH_CHECK(w16.is_cuda() && w16.scalar_type() == at::kHalf && w16.dim() == 2 && w16.is_contiguous(),
                "insitu: w16 must be a contiguous (out, in) float16 CUDA tensor");
    TORCH_CHECK(x.is_cuda() && x.scalar_type() == at::kFloat && x.dim() == 2 && x.is_contiguous() &&
                    x.size(1) == w16.size(1),
                "insitu: x must be a contiguous (n, in) float32 CUDA tensor");
    c10::cuda::CUDAGuard guard(x.device());
    at::Tensor y = at::empty({x.size(0), w16.size(0)}, x.options());
    const float *b = nullptr;
    if (bias.has_value()) {
        TORCH_CHECK(bias->scalar_type() == at::kFloat && bias->is_contiguous() && bias->numel() == w16.size(0),
                    "insitu: bias must be a contiguous float32 tensor of out elements");
        b = bias->data_ptr<float>();
    }
    check(ins_project((int32_t)x.size(0), (int32_t)x.size(1), (int32_t)w16.size(0),
                      reinterpret_cast<const uint16_t *>(w16.data_ptr<at::Half>()), x.data_ptr<float>(), b,
                      y.data_ptr<float>(), at::cuda::getCurrentCUDAStream().stream()));
    return y;
}

}  // namespace

TORCH_LIBRARY(insitu, m) {
    m.def("ingress(int handle, int[] seq_ids, Tensor k, Tensor v, Tensor? q, int n_kv, int q_heads, "
          "bool prerotated) -> Tensor?");
    m.def("scan(int handle, int[] seq_ids, int[]? lengths, Tensor q_rot, int n_kv, int mode, "
          "bool with_stats) -> (Tensor, Tensor?)");
    m.def("step(int handle, int[] seq_ids, Tensor q, Tensor k, Tensor v, int n_kv, int mode, "
          "bool with_stats) -> (Tensor, Tensor?)");
    m.def("project(Tensor w16, Tensor x, Tensor? bias) -> Tensor");
}

TORCH_LIBRARY_IMPL(insitu, CUDA, m) {
    m.impl("ingress", ingress);
    m.impl("scan", scan);
    m.impl("step", step);
    m.impl("project", project);
}
