// torch_binding.cpp — thin TORCH_LIBRARY shim over the C ABI (include/w4a8_b200.h).
//
// Registers the reference's op namespace and schemas byte for byte
// (w4a8_fp8_wmma/bindings.cpp:388-413) with the same argument checks (bindings.cpp:98-379).
// Each op allocates its output and its scratch from torch's caching allocator on the current
// device, and launches on torch's current CUDA stream, so the ops stay graph-capturable.
// No compute happens here: every op forwards to an extern "C" launcher and raises on a
// non-zero status. There is no CPU kernel: a CPU tensor fails the is_cuda check.
#include <ATen/ATen.h>
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include <torch/library.h>

#include "w4a8_b200.h"

namespace {

constexpr int64_t kPackFactor = 8;

void check_status(int rc, const char* op) {
    if (rc == W4A8_OK) return;
    if (rc == W4A8_ERR_INVALID) TORCH_CHECK(false, op, ": ", w4a8_last_error());
    TORCH_CHECK(false, op, ": CUDA error ", rc, " (",
                cudaGetErrorString(static_cast<cudaError_t>(rc)), ")");
}

w4a8_stream_t cur_stream() {
    return reinterpret_cast<w4a8_stream_t>(at::cuda::getCurrentCUDAStream().stream());
}

at::Tensor workspace(const at::Tensor& like, size_t bytes) {
    return at::empty({(int64_t)std::max<size_t>(bytes, 1)}, like.options().dtype(at::kByte));
}

const int32_t* zeros_ptr(const at::Tensor& z) {
    return (z.defined() && z.numel() > 0) ? z.data_ptr<int32_t>() : nullptr;
}

at::Tensor mmq_fp8_gemm_forward(const at::Tensor& x, const at::Tensor& w_packed,
                                const at::Tensor& scales, const at::Tensor& w_zeros,
                                int64_t kernel, bool weight_is_e2m1) {
    TORCH_CHECK(x.is_cuda() && w_packed.is_cuda() && scales.is_cuda(),
                "x, w_packed, scales must be CUDA");
    TORCH_CHECK(x.scalar_type() == at::kHalf, "x must be fp16");
    TORCH_CHECK(w_packed.scalar_type() == at::kInt, "w_packed must be int32");
    TORCH_CHECK(scales.scalar_type() == at::kHalf, "scales must be fp16");
    TORCH_CHECK(x.dim() == 2 && w_packed.dim() == 2 && scales.dim() == 2, "all inputs must be 2D");
    TORCH_CHECK(x.is_contiguous() && w_packed.is_contiguous() && scales.is_contiguous(),
                "all inputs must be contiguous");
    const int64_t M = x.size(0), K = x.size(1), N = w_packed.size(0);
    TORCH_CHECK(w_packed.size(1) * kPackFactor == K, "w_packed last dim mismatch: expected K/8 = ",
                K / kPackFactor, " got ", w_packed.size(1));
    TORCH_CHECK(scales.size(0) == N, "scales.size(0) must equal N=", N);
    TORCH_CHECK(scales.size(1) > 0, "scales must have at least one group");
    const int64_t group_size = K / scales.size(1);
    TORCH_CHECK(scales.size(1) * group_size == K, "K not divisible by scales' K dim");
    if (w_zeros.defined() && w_zeros.numel() > 0) {
        TORCH_CHECK(!weight_is_e2m1, "mxfp4 (E2M1) weights are symmetric; w_zeros must be empty");
        TORCH_CHECK(w_zeros.is_cuda() && w_zeros.scalar_type() == at::kInt,
                    "w_zeros must be CUDA int32 (packed)");
        TORCH_CHECK(w_zeros.dim() == 2 && w_zeros.size(0) * 8 == N &&
                        w_zeros.size(1) == scales.size(1),
                    "w_zeros shape mismatch: expected (", N / 8, ", ", scales.size(1), ")");
        TORCH_CHECK(w_zeros.is_contiguous(), "w_zeros must be contiguous");
    }
    const c10::cuda::CUDAGuard guard(x.device());
    auto out = at::empty({M, N}, x.options());
    auto ws = workspace(x, w4a8_mmq_fp8_gemm_workspace_size(M, N, K));
    check_status(w4a8_mmq_fp8_gemm(x.data_ptr(), w_packed.data_ptr<int32_t>(), scales.data_ptr(),
                                   zeros_ptr(w_zeros), out.data_ptr(), M, N, K, group_size,
                                   (int32_t)kernel, weight_is_e2m1 ? 1 : 0, ws.data_ptr(),
                                   (size_t)ws.numel(), cur_stream()),
                 "mmq_fp8_gemm");
    return out;
}

at::Tensor regdirect_unsupported(const at::Tensor&, const at::Tensor&, const at::Tensor&,
                                 const at::Tensor&, int64_t) {
    TORCH_CHECK(false,
                "mmq_regdirect_* are parked gfx1201 research ops (register-direct WMMA "
                "weight layout); the B200 build does not provide them");
}

struct MoeDims {
    int64_t T, K, N, P, E, group_size;
};

MoeDims check_moe(const char* op, const at::Tensor& x, const at::Tensor& w_packed,
                  const at::Tensor& scales, const at::Tensor& w_zeros,
                  const at::Tensor& sorted_token_ids, const at::Tensor& expert_ids,
                  const at::Tensor& ntp, int64_t block_m, bool silu) {
    TORCH_CHECK(x.is_cuda() && w_packed.is_cuda() && scales.is_cuda(),
                "x, w_packed, scales must be CUDA");
    TORCH_CHECK(sorted_token_ids.is_cuda() && expert_ids.is_cuda() && ntp.is_cuda(),
                "routing tensors must be CUDA");
    TORCH_CHECK(x.scalar_type() == at::kHalf, "x must be fp16");
    TORCH_CHECK(w_packed.scalar_type() == at::kInt, "w_packed must be int32");
    TORCH_CHECK(scales.scalar_type() == at::kHalf, "scales must be fp16");
    TORCH_CHECK(x.dim() == 2, "x must be (T, K)");
    TORCH_CHECK(w_packed.dim() == 3 && scales.dim() == 3,
                silu ? "w_packed (E,2*inter,K/8) and scales (E,2*inter,K/group) must be 3D"
                     : "w_packed (E,N,K/8) and scales (E,N,K/group) must be 3D");
    TORCH_CHECK(sorted_token_ids.scalar_type() == at::kInt &&
                    expert_ids.scalar_type() == at::kInt && ntp.scalar_type() == at::kInt,
                "routing tensors must be int32");
    TORCH_CHECK(x.is_contiguous() && w_packed.is_contiguous() && scales.is_contiguous(),
                "x, w_packed, scales must be contiguous");
    TORCH_CHECK(sorted_token_ids.is_contiguous() && expert_ids.is_contiguous(),
                "routing tensors must be contiguous");
    TORCH_CHECK(ntp.numel() >= 1, "num_tokens_post_padded must hold one value");
    MoeDims d;
    d.T = x.size(0);
    d.K = x.size(1);
    d.E = w_packed.size(0);
    d.N = w_packed.size(1);
    d.P = sorted_token_ids.size(0);
    TORCH_CHECK(w_packed.size(2) * kPackFactor == d.K, "w_packed last dim must be K/8=",
                d.K / kPackFactor);
    TORCH_CHECK(scales.size(0) == d.E && scales.size(1) == d.N,
                "scales must be (E, N, K/group) matching w_packed");
    TORCH_CHECK(scales.size(2) > 0, "scales must have at least one group");
    d.group_size = d.K / scales.size(2);
    TORCH_CHECK(block_m > 0 && d.P % block_m == 0, "P=", d.P, " not divisible by block_m=",
                block_m);
    TORCH_CHECK(expert_ids.size(0) == d.P / block_m, "expert_ids must have P/block_m=",
                d.P / block_m, " entries");
    if (w_zeros.defined() && w_zeros.numel() > 0) {
        TORCH_CHECK(w_zeros.is_cuda() && w_zeros.scalar_type() == at::kInt && w_zeros.dim() == 3 &&
                        w_zeros.size(0) == d.E && w_zeros.size(1) * 8 == d.N &&
                        w_zeros.size(2) == scales.size(2),
                    silu ? "w_zeros must be (E, (2*inter)/8, K/group) int32"
                         : "w_zeros must be (E, N/8, K/group) int32");
        TORCH_CHECK(w_zeros.is_contiguous(), "w_zeros must be contiguous");
    }
    (void)op;
    return d;
}

at::Tensor mmq_fp8_moe_gemm_forward(const at::Tensor& x, const at::Tensor& w_packed,
                                    const at::Tensor& scales, const at::Tensor& w_zeros,
                                    const at::Tensor& sorted_token_ids,
                                    const at::Tensor& expert_ids, const at::Tensor& ntp,
                                    int64_t top_k, int64_t block_m, int64_t kernel,
                                    bool weight_is_e2m1) {
    const MoeDims d = check_moe("mmq_fp8_moe_gemm", x, w_packed, scales, w_zeros,
                                sorted_token_ids, expert_ids, ntp, block_m, false);
    const c10::cuda::CUDAGuard guard(x.device());
    auto out = at::empty({d.P, d.N}, x.options());
    auto ws = workspace(x, w4a8_moe_gemm_workspace_size(d.T, d.P, d.N, d.K));
    check_status(w4a8_mmq_fp8_moe_gemm(
                     x.data_ptr(), w_packed.data_ptr<int32_t>(), scales.data_ptr(),
                     zeros_ptr(w_zeros), sorted_token_ids.data_ptr<int32_t>(),
                     expert_ids.data_ptr<int32_t>(), ntp.data_ptr<int32_t>(), out.data_ptr(), d.T,
                     d.E, d.N, d.K, d.P, d.group_size, top_k, block_m, (int32_t)kernel,
                     weight_is_e2m1 ? 1 : 0, ws.data_ptr(), (size_t)ws.numel(), cur_stream()),
                 "mmq_fp8_moe_gemm");
    return out;
}

at::Tensor gemm1_silu_impl(const at::Tensor& x, const at::Tensor& w_packed,
                           const at::Tensor& scales, const at::Tensor& w_zeros,
                           const at::Tensor& sorted_token_ids, const at::Tensor& expert_ids,
                           const at::Tensor& ntp, int64_t top_k, int64_t block_m, int64_t kernel,
                           bool weight_is_e2m1) {
    const MoeDims d = check_moe("mmq_fp8_moe_gemm1_silu", x, w_packed, scales, w_zeros,
                                sorted_token_ids, expert_ids, ntp, block_m, true);
    TORCH_CHECK(d.N % 2 == 0, "w13 N must be 2*inter (even); got ", d.N);
    const c10::cuda::CUDAGuard guard(x.device());
    auto out = at::empty({d.P, d.N / 2}, x.options());
    auto ws = workspace(x, w4a8_moe_gemm_workspace_size(d.T, d.P, d.N, d.K));
    check_status(w4a8_mmq_fp8_moe_gemm1_silu(
                     x.data_ptr(), w_packed.data_ptr<int32_t>(), scales.data_ptr(),
                     zeros_ptr(w_zeros), sorted_token_ids.data_ptr<int32_t>(),
                     expert_ids.data_ptr<int32_t>(), ntp.data_ptr<int32_t>(), out.data_ptr(), d.T,
                     d.E, d.N, d.K, d.P, d.group_size, top_k, block_m, (int32_t)kernel,
                     weight_is_e2m1 ? 1 : 0, ws.data_ptr(), (size_t)ws.numel(), cur_stream()),
                 "mmq_fp8_moe_gemm1_silu");
    return out;
}

at::Tensor mmq_fp8_moe_gemm1_silu_forward(const at::Tensor& x, const at::Tensor& w_packed,
                                          const at::Tensor& scales, const at::Tensor& w_zeros,
                                          const at::Tensor& sorted_token_ids,
                                          const at::Tensor& expert_ids, const at::Tensor& ntp,
                                          int64_t top_k, int64_t block_m, int64_t kernel,
                                          bool weight_is_e2m1) {
    TORCH_CHECK(kernel == W4A8_MOE_WMMA, "fused gemm1+silu needs the 'wmma' kernel; got id ",
                kernel);
    return gemm1_silu_impl(x, w_packed, scales, w_zeros, sorted_token_ids, expert_ids, ntp, top_k,
                           block_m, kernel, weight_is_e2m1);
}

void mmq_fp8_moe_gemm_scatter_forward(const at::Tensor& x, const at::Tensor& w_packed,
                                      const at::Tensor& scales, const at::Tensor& w_zeros,
                                      const at::Tensor& sorted_token_ids,
                                      const at::Tensor& expert_ids, const at::Tensor& ntp,
                                      const at::Tensor& topk_weights, const at::Tensor& output,
                                      int64_t top_k, int64_t block_m, int64_t kernel,
                                      bool weight_is_e2m1) {
    const MoeDims d = check_moe("mmq_fp8_moe_gemm_scatter", x, w_packed, scales, w_zeros,
                                sorted_token_ids, expert_ids, ntp, block_m, false);
    TORCH_CHECK(topk_weights.is_cuda() && output.is_cuda(), "topk_weights, output must be CUDA");
    TORCH_CHECK(topk_weights.scalar_type() == at::kFloat && output.scalar_type() == at::kFloat,
                "topk_weights and output must be fp32");
    TORCH_CHECK(topk_weights.is_contiguous() && output.is_contiguous(),
                "x, w_packed, scales, topk_weights, output must be contiguous");
    TORCH_CHECK(output.dim() == 2 && output.size(1) == d.N, "output must be (M, N) with N=", d.N);
    const int64_t M = output.size(0);
    TORCH_CHECK(topk_weights.numel() == M * top_k, "topk_weights must have M*top_k=", M * top_k,
                " entries");
    const c10::cuda::CUDAGuard guard(x.device());
    auto ws = workspace(x, w4a8_moe_gemm_workspace_size(d.P, d.P, d.N, d.K));
    check_status(w4a8_mmq_fp8_moe_gemm_scatter(
                     x.data_ptr(), w_packed.data_ptr<int32_t>(), scales.data_ptr(),
                     zeros_ptr(w_zeros), sorted_token_ids.data_ptr<int32_t>(),
                     expert_ids.data_ptr<int32_t>(), ntp.data_ptr<int32_t>(),
                     topk_weights.data_ptr<float>(), output.data_ptr<float>(), M, d.E, d.N, d.K,
                     d.P, d.group_size, top_k, block_m, (int32_t)kernel, weight_is_e2m1 ? 1 : 0,
                     ws.data_ptr(), (size_t)ws.numel(), cur_stream()),
                 "mmq_fp8_moe_gemm_scatter");
}

at::Tensor mmq_fp8_moe_gather_reduce_forward(const at::Tensor& out2,
                                             const at::Tensor& sorted_token_ids,
                                             const at::Tensor& topk_weights,
                                             const at::Tensor& ntp, int64_t top_k) {
    TORCH_CHECK(out2.is_cuda() && out2.scalar_type() == at::kHalf && out2.dim() == 2,
                "out2 must be (P,N) fp16 CUDA");
    TORCH_CHECK(sorted_token_ids.scalar_type() == at::kInt && ntp.scalar_type() == at::kInt,
                "sorted_token_ids / num_tokens_post_padded must be int32");
    TORCH_CHECK(topk_weights.scalar_type() == at::kFloat, "topk_weights must be fp32");
    TORCH_CHECK(out2.is_contiguous() && topk_weights.is_contiguous(),
                "out2 and topk_weights must be contiguous");
    TORCH_CHECK(top_k > 0 && topk_weights.numel() % top_k == 0,
                "topk_weights.numel() must be M*top_k");
    TORCH_CHECK(sorted_token_ids.size(0) <= out2.size(0),
                "sorted_token_ids must not be longer than out2's rows");
    const int64_t N = out2.size(1);
    const int64_t M = topk_weights.numel() / top_k;
    const c10::cuda::CUDAGuard guard(out2.device());
    auto out = at::empty({M, N}, out2.options().dtype(at::kFloat));
    auto ws = workspace(out2, w4a8_moe_gather_reduce_workspace_size(M, top_k));
    check_status(w4a8_moe_gather_reduce(out2.data_ptr(), sorted_token_ids.data_ptr<int32_t>(),
                                        topk_weights.data_ptr<float>(), ntp.data_ptr<int32_t>(),
                                        out.data_ptr<float>(), M, N, sorted_token_ids.size(0),
                                        top_k, ws.data_ptr(), (size_t)ws.numel(), cur_stream()),
                 "mmq_fp8_moe_gather_reduce");
    return out;
}

// ---- Library extras of the B200 build (own namespace, not part of the reference surface) ----

std::vector<at::Tensor> act_quant_fp8_forward(const at::Tensor& x) {
    TORCH_CHECK(x.is_cuda() && x.scalar_type() == at::kHalf && x.dim() == 2 && x.is_contiguous(),
                "x must be a contiguous (M, K) fp16 CUDA tensor");
    const c10::cuda::CUDAGuard guard(x.device());
    auto q = at::empty({x.size(0), x.size(1)}, x.options().dtype(at::kByte));
    auto s = at::empty({x.size(0)}, x.options().dtype(at::kFloat));
    check_status(w4a8_act_quant_fp8(x.data_ptr(), q.data_ptr<uint8_t>(), s.data_ptr<float>(),
                                    x.size(0), x.size(1), cur_stream()),
                 "act_quant_fp8");
    return {q, s};
}

std::vector<at::Tensor> route_topk_forward(const at::Tensor& logits, int64_t top_k,
                                           bool renormalize) {
    TORCH_CHECK(logits.is_cuda() && logits.dim() == 2 && logits.is_contiguous(),
                "logits must be a contiguous (T, E) CUDA tensor");
    int32_t dt;
    if (logits.scalar_type() == at::kFloat) dt = 0;
    else if (logits.scalar_type() == at::kHalf) dt = 1;
    else if (logits.scalar_type() == at::kBFloat16) dt = 2;
    else TORCH_CHECK(false, "logits must be fp32, fp16 or bf16");
    const c10::cuda::CUDAGuard guard(logits.device());
    auto ids = at::empty({logits.size(0), top_k}, logits.options().dtype(at::kInt));
    auto w = at::empty({logits.size(0), top_k}, logits.options().dtype(at::kFloat));
    auto counts = at::empty({logits.size(1)}, logits.options().dtype(at::kInt));
    check_status(w4a8_route_topk(logits.data_ptr(), dt, logits.size(0), (int32_t)logits.size(1),
                                 (int32_t)top_k, renormalize ? 1 : 0, ids.data_ptr<int32_t>(),
                                 w.data_ptr<float>(), counts.data_ptr<int32_t>(), cur_stream()),
                 "route_topk");
    return {ids, w, counts};
}

std::vector<at::Tensor> moe_align_block_size_forward(const at::Tensor& topk_ids, int64_t block_m,
                                                     int64_t num_experts,
                                                     const c10::optional<at::Tensor>& expert_map,
                                                     int64_t num_local_experts) {
    TORCH_CHECK(topk_ids.is_cuda() && topk_ids.scalar_type() == at::kInt &&
                    topk_ids.is_contiguous(),
                "topk_ids must be a contiguous int32 CUDA tensor");
    const int64_t slots = topk_ids.numel();
    const int64_t n_local = num_local_experts > 0 ? num_local_experts : num_experts;
    const int32_t* map = nullptr;
    if (expert_map.has_value() && expert_map->defined()) {
        TORCH_CHECK(expert_map->is_cuda() && expert_map->scalar_type() == at::kInt &&
                        expert_map->numel() == num_experts && expert_map->is_contiguous(),
                    "expert_map must be a contiguous (num_experts,) int32 CUDA tensor");
        map = expert_map->data_ptr<int32_t>();
    }
    int64_t cap = slots + n_local * (block_m - 1);
    cap = (cap + block_m - 1) / block_m * block_m;
    const c10::cuda::CUDAGuard guard(topk_ids.device());
    auto opts = topk_ids.options();
    auto sorted = at::empty({cap}, opts);
    auto eids = at::empty({cap / block_m}, opts);
    auto ntp = at::empty({1}, opts);
    auto ws = workspace(topk_ids, w4a8_moe_align_workspace_size((int32_t)n_local));
    check_status(w4a8_moe_align_block_size(topk_ids.data_ptr<int32_t>(), slots,
                                           (int32_t)num_experts, (int32_t)n_local,
                                           (int32_t)block_m, map, sorted.data_ptr<int32_t>(), cap,
                                           eids.data_ptr<int32_t>(), ntp.data_ptr<int32_t>(),
                                           ws.data_ptr(), (size_t)ws.numel(), cur_stream()),
                 "moe_align_block_size");
    return {sorted, eids, ntp};
}

at::Tensor silu_and_mul_forward(const at::Tensor& x) {
    TORCH_CHECK(x.is_cuda() && x.scalar_type() == at::kHalf && x.dim() == 2 && x.is_contiguous() &&
                    x.size(1) % 2 == 0,
                "x must be a contiguous (M, 2*inter) fp16 CUDA tensor");
    const c10::cuda::CUDAGuard guard(x.device());
    auto out = at::empty({x.size(0), x.size(1) / 2}, x.options());
    check_status(w4a8_silu_and_mul(x.data_ptr(), out.data_ptr(), x.size(0), x.size(1) / 2,
                                   cur_stream()),
                 "silu_and_mul");
    return out;
}

std::vector<at::Tensor> ep_pack_forward(const at::Tensor& x, const at::Tensor& topk_ids,
                                        const at::Tensor& topk_weights, int64_t experts_per_rank,
                                        int64_t world, int64_t shared_local_id) {
    TORCH_CHECK(x.is_cuda() && x.scalar_type() == at::kHalf && x.dim() == 2 && x.is_contiguous(),
                "x must be a contiguous (T, H) fp16 CUDA tensor");
    TORCH_CHECK(topk_ids.scalar_type() == at::kInt && topk_ids.is_contiguous() &&
                    topk_ids.dim() == 2 && topk_ids.size(0) == x.size(0) &&
                    topk_weights.scalar_type() == at::kFloat && topk_weights.is_contiguous() &&
                    topk_weights.sizes() == topk_ids.sizes(),
                "topk_ids (T, k) int32 / topk_weights (T, k) fp32 must be contiguous");
    const c10::cuda::CUDAGuard guard(x.device());
    const int64_t T = x.size(0), H = x.size(1), k = topk_ids.size(1);
    const int64_t rb = (int64_t)w4a8_ep_row_bytes(H, k);
    // rows [0, world*T): the send chunks; [world*T, (world+1)*T): the own shared-expert rows
    auto rows = at::empty({(world + 1) * T, rb}, x.options().dtype(at::kByte));
    auto pos = at::empty({world, T}, topk_ids.options());
    uint8_t* base = rows.data_ptr<uint8_t>();
    check_status(w4a8_ep_pack(x.data_ptr(), topk_ids.data_ptr<int32_t>(),
                              topk_weights.data_ptr<float>(), T, k, H, (int32_t)experts_per_rank,
                              (int32_t)world, (int32_t)shared_local_id, base,
                              shared_local_id >= 0 ? base + world * T * rb : nullptr,
                              pos.data_ptr<int32_t>(), cur_stream()),
                 "ep_pack");
    return {rows, pos};
}

at::Tensor ep_moe_rows_forward(const at::Tensor& rows, const at::Tensor& p13, const at::Tensor& p2,
                               int64_t E, int64_t H, int64_t I, int64_t top_k) {
    TORCH_CHECK(rows.is_cuda() && rows.scalar_type() == at::kByte && rows.dim() == 2 &&
                    rows.is_contiguous() && (size_t)rows.size(1) == w4a8_ep_row_bytes(H, top_k),
                "rows must be contiguous (R, ep_row_bytes) uint8 payload rows");
    TORCH_CHECK(p13.scalar_type() == at::kByte && p2.scalar_type() == at::kByte &&
                    (size_t)p13.numel() == w4a8_stream_pack_size(E, 2 * I, H) &&
                    (size_t)p2.numel() == w4a8_stream_pack_size(E, H, I),
                "p13 / p2 must be stream_pack outputs for (E, 2*inter, hidden) / (E, hidden, inter)");
    const c10::cuda::CUDAGuard guard(rows.device());
    const int64_t R = rows.size(0);
    auto out = at::empty({R, H}, rows.options().dtype(at::kFloat));
    auto ws = workspace(rows, w4a8_ep_moe_rows_workspace_size(R, top_k, E, H, I));
    check_status(w4a8_ep_moe_rows(rows.data_ptr(), R, top_k, E, p13.data_ptr(), p2.data_ptr(), H,
                                  I, out.data_ptr<float>(), ws.data_ptr(), (size_t)ws.numel(),
                                  cur_stream()),
                 "ep_moe_rows");
    return out;
}

at::Tensor ep_gather_forward(const at::Tensor& back, const at::Tensor& pos,
                             const c10::optional<at::Tensor>& own_out) {
    TORCH_CHECK(back.is_cuda() && back.scalar_type() == at::kFloat && back.dim() == 2 &&
                    back.is_contiguous(),
                "back must be a contiguous (world*T, H) fp32 CUDA tensor");
    TORCH_CHECK(pos.scalar_type() == at::kInt && pos.is_contiguous() && pos.dim() == 2 &&
                    pos.size(0) * pos.size(1) == back.size(0),
                "pos must be a contiguous (world, T) int32 tensor");
    const c10::cuda::CUDAGuard guard(back.device());
    const int64_t W = pos.size(0), T = pos.size(1), H = back.size(1);
    const float* own = nullptr;
    if (own_out.has_value() && own_out->defined()) {
        TORCH_CHECK(own_out->scalar_type() == at::kFloat && own_out->is_contiguous() &&
                        own_out->size(0) == T && own_out->size(1) == H,
                    "own_out must be a contiguous (T, H) fp32 tensor");
        own = own_out->data_ptr<float>();
    }
    auto out = at::empty({T, H}, back.options());
    check_status(w4a8_ep_gather(back.data_ptr<float>(), pos.data_ptr<int32_t>(), own,
                                out.data_ptr<float>(), T, (int32_t)W, H, cur_stream()),
                 "ep_gather");
    return out;
}

at::Tensor stream_pack_forward(const at::Tensor& w, const at::Tensor& s, const at::Tensor& z,
                               bool gate_up) {
    TORCH_CHECK(w.is_cuda() && w.dim() == 3 && w.scalar_type() == at::kInt && w.is_contiguous(),
                "w must be a contiguous (E, N, K/8) int32 CUDA tensor");
    TORCH_CHECK(s.scalar_type() == at::kHalf && s.is_contiguous(), "scales must be contiguous fp16");
    const int64_t E = w.size(0), N = w.size(1), K = w.size(2) * 8;
    TORCH_CHECK(s.numel() == E * N * (K / 128), "scales must be (E, N, K/128)");
    const bool zz = z.defined() && z.numel() > 0;
    if (zz)
        TORCH_CHECK(z.scalar_type() == at::kInt && z.is_contiguous() && z.numel() == E * (N / 8) * (K / 128),
                    "zeros must be (E, N/8, K/128) int32");
    const c10::cuda::CUDAGuard guard(w.device());
    const size_t bytes = w4a8_stream_pack_size(E, N, K);
    TORCH_CHECK(bytes > 0, "stream_pack: needs K % 512 == 0 and N % 128 == 0");
    auto out = at::empty({(int64_t)bytes}, w.options().dtype(at::kByte));
    check_status(w4a8_stream_pack(w.data_ptr<int32_t>(), s.data_ptr(), zz ? z.data_ptr<int32_t>() : nullptr,
                                  E, N, K, gate_up ? 1 : 0, out.data_ptr(), bytes, cur_stream()),
                 "stream_pack");
    return out;
}

at::Tensor moe_decode_packed_forward(const at::Tensor& x, const at::Tensor& p13,
                                     const at::Tensor& p2, int64_t E, int64_t I,
                                     const at::Tensor& topk_weights, const at::Tensor& topk_ids) {
    TORCH_CHECK(x.is_cuda() && x.scalar_type() == at::kHalf && x.dim() == 2 && x.is_contiguous(),
                "x must be a contiguous (T, H) fp16 CUDA tensor");
    TORCH_CHECK(topk_ids.scalar_type() == at::kInt && topk_weights.scalar_type() == at::kFloat &&
                    topk_ids.is_contiguous() && topk_weights.is_contiguous() &&
                    topk_ids.dim() == 2 && topk_weights.sizes() == topk_ids.sizes() &&
                    topk_ids.size(0) == x.size(0),
                "topk_ids (T, k) int32 and topk_weights (T, k) fp32 must be contiguous");
    const int64_t T = x.size(0), H = x.size(1), k = topk_ids.size(1);
    TORCH_CHECK(p13.scalar_type() == at::kByte && p2.scalar_type() == at::kByte &&
                    (size_t)p13.numel() == w4a8_stream_pack_size(E, 2 * I, H) &&
                    (size_t)p2.numel() == w4a8_stream_pack_size(E, H, I),
                "p13 / p2 must be stream_pack outputs for (E, 2*inter, hidden) / (E, hidden, inter)");
    const c10::cuda::CUDAGuard guard(x.device());
    auto out = at::empty({T, H}, x.options());
    auto ws = workspace(x, w4a8_moe_decode_workspace_size(T, k, E, H, I));
    check_status(w4a8_moe_decode_packed(x.data_ptr(), topk_ids.data_ptr<int32_t>(),
                                        topk_weights.data_ptr<float>(), T, k, E, p13.data_ptr(),
                                        p2.data_ptr(), H, I, out.data_ptr(), ws.data_ptr(),
                                        (size_t)ws.numel(), cur_stream()),
                 "moe_decode_packed");
    return out;
}

at::Tensor moe_decode_forward(const at::Tensor& x, const at::Tensor& w13, const at::Tensor& s13,
                              const at::Tensor& z13, const at::Tensor& w2, const at::Tensor& s2,
                              const at::Tensor& z2, const at::Tensor& topk_weights,
                              const at::Tensor& topk_ids) {
    TORCH_CHECK(x.is_cuda() && x.scalar_type() == at::kHalf && x.dim() == 2 && x.is_contiguous(),
                "x must be a contiguous (T, H) fp16 CUDA tensor");
    TORCH_CHECK(w13.dim() == 3 && w2.dim() == 3 && w13.scalar_type() == at::kInt &&
                    w2.scalar_type() == at::kInt && w13.is_contiguous() && w2.is_contiguous(),
                "w13 (E, 2I, H/8) and w2 (E, H, I/8) must be contiguous int32");
    TORCH_CHECK(s13.scalar_type() == at::kHalf && s2.scalar_type() == at::kHalf &&
                    s13.is_contiguous() && s2.is_contiguous(),
                "scales must be contiguous fp16");
    TORCH_CHECK(topk_ids.scalar_type() == at::kInt && topk_weights.scalar_type() == at::kFloat &&
                    topk_ids.is_contiguous() && topk_weights.is_contiguous() &&
                    topk_ids.dim() == 2 && topk_weights.sizes() == topk_ids.sizes(),
                "topk_ids (T, k) int32 and topk_weights (T, k) fp32 must be contiguous");
    const int64_t T = x.size(0), H = x.size(1), E = w13.size(0), I = w13.size(1) / 2;
    const int64_t k = topk_ids.size(1);
    TORCH_CHECK(topk_ids.size(0) == T, "topk_ids must have T rows");
    TORCH_CHECK(w13.size(2) * 8 == H && w2.size(0) == E && w2.size(1) == H && w2.size(2) * 8 == I,
                "weight shapes do not match x");
    TORCH_CHECK(s13.numel() == E * 2 * I * (H / 128) && s2.numel() == E * H * (I / 128),
                "scales must be (E, N, K/128)");
    const bool zz = z13.defined() && z13.numel() > 0;
    TORCH_CHECK(zz == (z2.defined() && z2.numel() > 0), "give both zero tensors or neither");
    if (zz)
        TORCH_CHECK(z13.numel() == E * (2 * I / 8) * (H / 128) && z2.numel() == E * (H / 8) * (I / 128) &&
                        z13.is_contiguous() && z2.is_contiguous(),
                    "zeros must be (E, N/8, K/128) int32");
    const c10::cuda::CUDAGuard guard(x.device());
    auto out = at::empty({T, H}, x.options());
    auto ws = workspace(x, w4a8_moe_decode_workspace_size(T, k, E, H, I));
    check_status(w4a8_moe_decode(x.data_ptr(), topk_ids.data_ptr<int32_t>(),
                                 topk_weights.data_ptr<float>(), T, k, E,
                                 w13.data_ptr<int32_t>(), s13.data_ptr(), zz ? z13.data_ptr<int32_t>() : nullptr,
                                 w2.data_ptr<int32_t>(), s2.data_ptr(), zz ? z2.data_ptr<int32_t>() : nullptr,
                                 H, I, 128, out.data_ptr(), ws.data_ptr(), (size_t)ws.numel(),
                                 cur_stream()),
                 "moe_decode");
    return out;
}

}  // namespace

// pt2_compliant_tag on every op, as the reference registers them (bindings.cpp:388-413); the
// fake (meta) impls live in the Python package.
TORCH_LIBRARY(w4a8_fp8_wmma, m) {
    m.def("mmq_fp8_gemm(Tensor x, Tensor w_packed, Tensor scales, Tensor w_zeros, int kernel, bool weight_is_e2m1=False) -> Tensor",
          {at::Tag::pt2_compliant_tag});
    m.def("mmq_regdirect_fp8(Tensor x, Tensor w_rep, Tensor scales, Tensor w_zeros, int N) -> Tensor",
          {at::Tag::pt2_compliant_tag});
    m.def("mmq_regdirect_f16(Tensor x, Tensor w_rep, Tensor scales, Tensor w_zeros, int N) -> Tensor",
          {at::Tag::pt2_compliant_tag});
    m.def("mmq_regdirect_w4a16(Tensor x, Tensor w_rep, Tensor scales, Tensor w_zeros, int N) -> Tensor",
          {at::Tag::pt2_compliant_tag});
    m.def("mmq_fp8_moe_gemm(Tensor x, Tensor w_packed, Tensor scales, Tensor w_zeros, "
          "Tensor sorted_token_ids, Tensor expert_ids, Tensor num_tokens_post_padded, "
          "int top_k, int block_m, int kernel, bool weight_is_e2m1=False) -> Tensor",
          {at::Tag::pt2_compliant_tag});
    m.def("mmq_fp8_moe_gemm1_silu(Tensor x, Tensor w_packed, Tensor scales, Tensor w_zeros, "
          "Tensor sorted_token_ids, Tensor expert_ids, Tensor num_tokens_post_padded, "
          "int top_k, int block_m, int kernel, bool weight_is_e2m1=False) -> Tensor",
          {at::Tag::pt2_compliant_tag});
    m.def("mmq_fp8_moe_gemm_scatter(Tensor x, Tensor w_packed, Tensor scales, "
          "Tensor w_zeros, Tensor sorted_token_ids, Tensor expert_ids, "
          "Tensor num_tokens_post_padded, Tensor topk_weights, Tensor(a!) output, "
          "int top_k, int block_m, int kernel, bool weight_is_e2m1=False) -> ()",
          {at::Tag::pt2_compliant_tag});
    m.def("mmq_fp8_moe_gather_reduce(Tensor out2, Tensor sorted_token_ids, "
          "Tensor topk_weights, Tensor num_tokens_post_padded, int top_k) -> Tensor",
          {at::Tag::pt2_compliant_tag});
}

TORCH_LIBRARY_IMPL(w4a8_fp8_wmma, CUDA, m) {
    m.impl("mmq_fp8_gemm", &mmq_fp8_gemm_forward);
    m.impl("mmq_regdirect_fp8", &regdirect_unsupported);
    m.impl("mmq_regdirect_f16", &regdirect_unsupported);
    m.impl("mmq_regdirect_w4a16", &regdirect_unsupported);
    m.impl("mmq_fp8_moe_gemm", &mmq_fp8_moe_gemm_forward);
    m.impl("mmq_fp8_moe_gemm1_silu", &mmq_fp8_moe_gemm1_silu_forward);
    m.impl("mmq_fp8_moe_gemm_scatter", &mmq_fp8_moe_gemm_scatter_forward);
    m.impl("mmq_fp8_moe_gather_reduce", &mmq_fp8_moe_gather_reduce_forward);
}

TORCH_LIBRARY(w4a8_b200, m) {
    m.def("act_quant_fp8(Tensor x) -> Tensor[]");
    m.def("silu_and_mul(Tensor x) -> Tensor");
    m.def("route_topk(Tensor logits, int top_k, bool renormalize) -> Tensor[]");
    m.def("ep_pack(Tensor x, Tensor topk_ids, Tensor topk_weights, int experts_per_rank, int world, "
          "int shared_local_id) -> Tensor[]");
    m.def("ep_moe_rows(Tensor rows, Tensor p13, Tensor p2, int num_experts, int hidden, int inter, "
          "int top_k) -> Tensor");
    m.def("ep_gather(Tensor back, Tensor pos, Tensor? own_out) -> Tensor");
    // Whole gated MoE layer at decode sizes (align -> gate_up+SiLU -> down -> reduce).
    m.def("stream_pack(Tensor w, Tensor scales, Tensor zeros, bool gate_up) -> Tensor");
    m.def("moe_decode_packed(Tensor x, Tensor p13, Tensor p2, int num_experts, int inter, "
          "Tensor topk_weights, Tensor topk_ids) -> Tensor");
    m.def("moe_decode(Tensor x, Tensor w13, Tensor s13, Tensor z13, Tensor w2, Tensor s2, "
          "Tensor z2, Tensor topk_weights, Tensor topk_ids) -> Tensor");
    // Fused gate_up + SiLU with any MoE kernel id (0 scalar, 6 tile, 7 GEMV).
    m.def("moe_gemm1_silu(Tensor x, Tensor w_packed, Tensor scales, Tensor w_zeros, "
          "Tensor sorted_token_ids, Tensor expert_ids, Tensor num_tokens_post_padded, "
          "int top_k, int block_m, int kernel, bool weight_is_e2m1=False) -> Tensor");
    m.def("moe_align_block_size(Tensor topk_ids, int block_m, int num_experts, "
          "Tensor? expert_map=None, int num_local_experts=0) -> Tensor[]");
}

TORCH_LIBRARY_IMPL(w4a8_b200, CUDA, m) {
    m.impl("act_quant_fp8", &act_quant_fp8_forward);
    m.impl("silu_and_mul", &silu_and_mul_forward);
    m.impl("route_topk", &route_topk_forward);
    m.impl("ep_pack", &ep_pack_forward);
    m.impl("ep_moe_rows", &ep_moe_rows_forward);
    m.impl("ep_gather", &ep_gather_forward);
    m.impl("moe_decode", &moe_decode_forward);
    m.impl("stream_pack", &stream_pack_forward);
    m.impl("moe_decode_packed", &moe_decode_packed_forward);
    m.impl("moe_gemm1_silu", &gemm1_silu_impl);
    m.impl("moe_align_block_size", &moe_align_block_size_forward);
}
