// capi.cu — extern "C" entry points of libw4a8_b200.so: argument validation (mirroring the
// TORCH_CHECKs of w4a8_fp8_wmma/bindings.cpp), workspace carving and kernel dispatch.
#include <algorithm>
#include <string>

#include "common.cuh"
#include "gemm_common.h"
#include "internal.h"

namespace w4a8 {

static thread_local std::string g_last_error;

int set_error(const std::string& msg) {
    g_last_error = msg;
    return W4A8_ERR_INVALID;
}

namespace {

// Scratch layout of every GEMM entry point, in order (each 256-byte aligned):
//   x_fp8 (rows, K) e4m3 | act_scales (rows,) f32 | xh (rows, K) fp16 | xsum (rows, K/128+1)
//   float2 | counter | partials | tile scratch
// xh and partials are used by the streaming GEMV path only; the tile scratch (sorted-order
// operand rows, see tc_carve) by the tcgen05 tile path only.
struct Scratch {
    uint8_t* xq;
    float* scales;
    __half* xh;
    float2* xsum;
    int* counter;
    float* part;
    void* tc;
};

size_t scratch_bytes(int64_t rows, int64_t K, int64_t P, int64_t N) {
    return align_up((size_t)rows * (size_t)K, 256) + align_up((size_t)rows * 4, 256) +
           align_up((size_t)rows * (size_t)K * 2, 256) +
           align_up((size_t)rows * (size_t)(K / 128 + 1) * 8, 256) + 256 +
           stream_partials_bytes(P, N, K) + tc_scratch_bytes(P, K);
}

bool carve(void* ws, size_t ws_bytes, int64_t rows, int64_t K, int64_t P, int64_t N,
           Scratch& s) {
    if (!ws || ws_bytes < scratch_bytes(rows, K, P, N)) return false;
    uint8_t* p = static_cast<uint8_t*>(ws);
    s.xq = p;
    p += align_up((size_t)rows * (size_t)K, 256);
    s.scales = reinterpret_cast<float*>(p);
    p += align_up((size_t)rows * 4, 256);
    s.xh = reinterpret_cast<__half*>(p);
    p += align_up((size_t)rows * (size_t)K * 2, 256);
    s.xsum = reinterpret_cast<float2*>(p);
    p += align_up((size_t)rows * (size_t)(K / 128 + 1) * 8, 256);
    s.counter = reinterpret_cast<int*>(p);
    p += 256;
    s.part = reinterpret_cast<float*>(p);
    p += stream_partials_bytes(P, N, K);
    s.tc = p;
    return true;
}

int check_group(int64_t K, int64_t group_size) {
    if (group_size <= 0 || K % group_size != 0)
        return set_error("K not divisible by scales' K dim");
    if (group_size % 16 != 0 || group_size > 128)
        return set_error("group_size must be a multiple of 16 and <= 128; got " +
                         std::to_string(group_size));
    return W4A8_OK;
}

bool dense_kernel_valid(int v) { return v == 0 || v == 1 || v == 2 || (v >= 4 && v <= 14); }
bool moe_kernel_valid(int v) { return v == 0 || v == 6 || v == 7; }

}  // namespace

}  // namespace w4a8

using namespace w4a8;

extern "C" const char* w4a8_last_error(void) { return g_last_error.c_str(); }

extern "C" const char* w4a8_version(void) { return "w4a8_b200 0.1 sm_100a"; }

extern "C" size_t w4a8_mmq_fp8_gemm_workspace_size(int64_t M, int64_t N, int64_t K) {
    return scratch_bytes(M, K, M, N);
}

extern "C" size_t w4a8_moe_gemm_workspace_size(int64_t x_rows, int64_t P, int64_t N, int64_t K) {
    return scratch_bytes(x_rows, K, P, N);
}

extern "C" int w4a8_mmq_fp8_gemm(const void* x, const int32_t* w_packed, const void* scales,
                                 const int32_t* w_zeros, void* out, int64_t M, int64_t N,
                                 int64_t K, int64_t group_size, int32_t kernel,
                                 int32_t weight_is_e2m1, void* workspace, size_t workspace_bytes,
                                 w4a8_stream_t stream) {
    if (M < 0 || N <= 0 || K <= 0) return set_error("mmq_fp8_gemm: bad sizes");
    if (K % 8 != 0) return set_error("w_packed last dim mismatch: K must be a multiple of 8");
    if (N % 8 != 0) return set_error("mmq_fp8_gemm: N must be a multiple of 8");
    if (int st = check_group(K, group_size)) return st;
    if (!dense_kernel_valid(kernel))
        return set_error("dense kernel id invalid (got " + std::to_string(kernel) +
                         "); must be a DenseKernel value 0..14 (rejecting the retired v3 gap)");
    if (kernel != W4A8_DENSE_REFERENCE_SCALAR && kernel != W4A8_DENSE_PREFILL_WMMA &&
        kernel != W4A8_DENSE_PREFILL_WMMA_ASHUFFLE && kernel != W4A8_DENSE_DECODE_GEMV)
        return set_error("dense kernel id " + std::to_string(kernel) +
                         " is a retired gfx1201 research kernel; the B200 build serves "
                         "reference_scalar(0), prefill_wmma(5), prefill_wmma_ashuffle(10), "
                         "decode_gemv(11)");
    if (weight_is_e2m1 && w_zeros)
        return set_error("mxfp4 (E2M1) weights are symmetric; w_zeros must be empty");
    if (M > INT32_MAX / 2 || N > INT32_MAX / 2) return set_error("mmq_fp8_gemm: size overflow");
    if (M == 0) return W4A8_OK;
    if (!x || !w_packed || !scales || !out) return set_error("mmq_fp8_gemm: null pointer");
    Scratch s;
    if (!carve(workspace, workspace_bytes, M, K, M, N, s))
        return set_error("mmq_fp8_gemm: workspace too small");
    cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
    const int G = (int)(K / group_size);
    const bool stream_path = kernel != W4A8_DENSE_REFERENCE_SCALAR && M <= 32 &&
                             stream_path_ok(K, G, weight_is_e2m1, w_packed);
    if (stream_path) {
        if (int rc = launch_operand_quant(x, OperandOut{s.xq, s.scales, s.xh, s.xsum}, M, K,
                                          nullptr, st))
            return rc;
        StreamArgs sa{};
        sa.xh = s.xh;
        sa.xsum = s.xsum;
        sa.act_scales = s.scales;
        sa.w = w_packed;
        sa.scales = static_cast<const __half*>(scales);
        sa.zeros = w_zeros;
        sa.out16 = static_cast<__half*>(out);
        sa.part = s.part;
        sa.counter = s.counter;
        sa.K = K;
        sa.N = (int)N;
        sa.G = G;
        sa.E = 1;
        sa.P = (int)M;
        sa.num_valid = (int)M;
        sa.top_k = 1;
        sa.out_top_k = 1;
        sa.block_m = 1 << 20;
        sa.mode = kStreamStore;
        return launch_w4_stream(sa, st);
    }
    if (kernel != W4A8_DENSE_REFERENCE_SCALAR && kernel != W4A8_DENSE_DECODE_GEMV && M > 32 &&
        tc_path_ok(K, (int)group_size, weight_is_e2m1, w_packed, 1 << 20) &&
        (reinterpret_cast<uintptr_t>(x) & 15) == 0) {
        cudaError_t ce = cudaMemsetAsync(s.counter, 0, sizeof(int), st);
        if (ce != cudaSuccess) return (int)ce;
        TcArgs t{};
        t.x = static_cast<const __half*>(x);
        t.w = w_packed;
        t.scales = static_cast<const __half*>(scales);
        t.zeros = w_zeros;
        t.out16 = static_cast<__half*>(out);
        t.err = s.counter;
        t.K = K;
        t.N = (int)N;
        t.G = G;
        t.E = 1;
        t.P = (int)M;
        t.num_valid = (int)M;
        t.top_k = 1;
        t.block_m = 1 << 20;
        tc_carve(s.tc, M, K, t);
        return launch_w4_tc(t, st);
    }
    if (int rc = launch_act_quant(x, s.xq, s.scales, M, K, st)) return rc;
    GemmArgs a{};
    a.x_fp8 = s.xq;
    a.act_scales = s.scales;
    a.w = w_packed;
    a.scales = static_cast<const __half*>(scales);
    a.zeros = w_zeros;
    a.out16 = static_cast<__half*>(out);
    a.K = K;
    a.N = (int)N;
    a.G = G;
    a.E = 1;
    a.P = (int)M;
    a.num_valid = (int)M;
    a.top_k = 1;
    a.out_top_k = 1;
    a.block_m = 1 << 20;
    a.src_identity = 0;
    a.e2m1 = weight_is_e2m1;
    int row_tile = M <= 8 ? 8 : M <= 16 ? 16 : M <= 32 ? 32 : 64;
    if (kernel == W4A8_DENSE_DECODE_GEMV && row_tile > 16) row_tile = 16;
    return launch_w4_gemm(a, kEpiStore, row_tile, kernel == W4A8_DENSE_REFERENCE_SCALAR, M, st);
}

namespace {

int moe_launch(const char* op, int epi, const void* x, const int32_t* w_packed,
               const void* scales, const int32_t* w_zeros, const int32_t* sorted_ids,
               const int32_t* expert_ids, const int32_t* ntp, const float* topk_weights,
               void* out, int64_t x_rows, int64_t M_out, int64_t E, int64_t N, int64_t K,
               int64_t P, int64_t group_size, int64_t top_k, int64_t block_m, int32_t kernel,
               int32_t e2m1, void* ws, size_t ws_bytes, w4a8_stream_t stream) {
    const std::string o(op);
    if (int st0 = [&] {
            if (x_rows < 0 || E <= 0 || N <= 0 || K <= 0 || P < 0 || top_k <= 0 || block_m <= 0)
                return set_error(o + ": sizes must be positive");
            if (K % 8 != 0) return set_error(o + ": w_packed last dim must be K/8");
            if (N % 8 != 0) return set_error(o + ": N must be a multiple of 8");
            if (int st = check_group(K, group_size)) return st;
            if (P % block_m != 0)
                return set_error(o + ": P=" + std::to_string(P) + " not divisible by block_m=" +
                                 std::to_string(block_m));
            if (!moe_kernel_valid(kernel))
                return set_error(o + ": moe kernel id must be 0 (scalar) / 6 (wmma) / 7 (gemv); got " +
                                 std::to_string(kernel));
            if (kernel == W4A8_MOE_WMMA && (block_m % 16 != 0 || block_m > 128))
                return set_error(o + ": wmma block_m must be mult of 16 and <=128; got " +
                                 std::to_string(block_m));
            if (kernel == W4A8_MOE_GEMV &&
                (block_m % 8 != 0 || block_m > 64 || K % 32 != 0 || group_size % 32 != 0))
                return set_error(o + ": gemv needs block_m mult of 8 <=64, K%32==0, group_size%32==0");
            if (e2m1 && w_zeros)
                return set_error(o + ": mxfp4 (E2M1) weights are symmetric; w_zeros must be empty");
            if (P > INT32_MAX / 2 || N > INT32_MAX / 2 || E > INT32_MAX / 2 ||
                x_rows * top_k > INT32_MAX / 2)
                return set_error(o + ": size overflow");
            if (P > 0 && (!x || !w_packed || !scales || !sorted_ids || !expert_ids || !ntp || !out))
                return set_error(o + ": null pointer");
            return (int)W4A8_OK;
        }())
        return st0;
    if (P == 0) return W4A8_OK;
    Scratch s;
    if (!carve(ws, ws_bytes, x_rows, K, P, N, s)) return set_error(o + ": workspace too small");
    cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
    const int G = (int)(K / group_size);
    const bool stream_path = kernel == W4A8_MOE_GEMV && stream_path_ok(K, G, e2m1, w_packed);
    const int32_t* row_limit = (epi == kEpiScatter) ? ntp : nullptr;
    if (stream_path) {
        if (int rc = launch_operand_quant(x, OperandOut{s.xq, s.scales, s.xh, s.xsum}, x_rows, K,
                                          row_limit, st))
            return rc;
        StreamArgs sa{};
        sa.xh = s.xh;
        sa.xsum = s.xsum;
        sa.act_scales = s.scales;
        sa.w = w_packed;
        sa.scales = static_cast<const __half*>(scales);
        sa.zeros = w_zeros;
        sa.sorted_ids = sorted_ids;
        sa.expert_ids = expert_ids;
        sa.ntp = ntp;
        sa.topk_weights = topk_weights;
        sa.part = s.part;
        sa.counter = s.counter;
        sa.K = K;
        sa.N = (int)N;
        sa.G = G;
        sa.E = (int)E;
        sa.P = (int)P;
        sa.block_m = (int)block_m;
        if (epi == kEpiScatter) {
            sa.out32 = static_cast<float*>(out);
            sa.src_identity = 1;
            sa.num_valid = (int)(M_out * top_k);
            sa.top_k = 1;
            sa.out_top_k = (int)top_k;
            sa.mode = kStreamScatter;
        } else {
            sa.out16 = static_cast<__half*>(out);
            sa.num_valid = (int)(x_rows * top_k);
            sa.top_k = (int)top_k;
            sa.out_top_k = (int)top_k;
            sa.mode = epi == kEpiSilu ? kStreamSilu : kStreamStore;
        }
        return launch_w4_stream(sa, st);
    }
    if (kernel == W4A8_MOE_WMMA && epi != kEpiScatter &&
        tc_path_ok(K, (int)group_size, e2m1, w_packed, (int)block_m) &&
        (reinterpret_cast<uintptr_t>(x) & 15) == 0 &&
        (epi != kEpiSilu || (N / 2) % 64 == 0)) {
        cudaError_t ce = cudaMemsetAsync(s.counter, 0, sizeof(int), st);
        if (ce != cudaSuccess) return (int)ce;
        TcArgs t{};
        t.x = static_cast<const __half*>(x);
        t.w = w_packed;
        t.scales = static_cast<const __half*>(scales);
        t.zeros = w_zeros;
        t.sorted_ids = sorted_ids;
        t.expert_ids = expert_ids;
        t.ntp = ntp;
        t.out16 = static_cast<__half*>(out);
        t.err = s.counter;
        t.K = K;
        t.N = (int)N;
        t.G = G;
        t.E = (int)E;
        t.P = (int)P;
        t.num_valid = (int)(x_rows * top_k);
        t.top_k = (int)top_k;
        t.block_m = (int)block_m;
        t.silu = epi == kEpiSilu ? 1 : 0;
        tc_carve(s.tc, P, K, t);
        if (x_rows < P) {  // gather: quantise each token once (the stream path's scratch)
            t.tq = s.xq;
            t.tq_scale = s.scales;
            t.tq_sum = reinterpret_cast<float*>(s.xsum);
            t.x_rows = (int)x_rows;
        }
        return launch_w4_tc(t, st);
    }
    if (x_rows > 0)
        if (int rc = launch_act_quant(x, s.xq, s.scales, x_rows, K, st, row_limit)) return rc;
    GemmArgs a{};
    a.x_fp8 = s.xq;
    a.act_scales = s.scales;
    a.w = w_packed;
    a.scales = static_cast<const __half*>(scales);
    a.zeros = w_zeros;
    a.sorted_ids = sorted_ids;
    a.expert_ids = expert_ids;
    a.ntp = ntp;
    a.topk_weights = topk_weights;
    a.K = K;
    a.N = (int)N;
    a.G = G;
    a.E = (int)E;
    a.P = (int)P;
    a.block_m = (int)block_m;
    a.e2m1 = e2m1;
    if (epi == kEpiScatter) {
        a.out32 = static_cast<float*>(out);
        a.src_identity = 1;
        a.num_valid = (int)(M_out * top_k);
        a.top_k = 1;
        a.out_top_k = (int)top_k;
    } else {
        a.out16 = static_cast<__half*>(out);
        a.src_identity = 0;
        a.num_valid = (int)(x_rows * top_k);
        a.top_k = (int)top_k;
        a.out_top_k = (int)top_k;
    }
    const int row_tile = kernel == W4A8_MOE_GEMV ? 8 : (int)std::min<int64_t>(block_m, 64);
    const int64_t est_rows = std::min<int64_t>(P, (int64_t)a.num_valid + E);
    return launch_w4_gemm(a, epi, row_tile, kernel == W4A8_MOE_SCALAR, est_rows, st);
}

}  // namespace

extern "C" int w4a8_mmq_fp8_moe_gemm(const void* x, const int32_t* w_packed, const void* scales,
                                     const int32_t* w_zeros, const int32_t* sorted_token_ids,
                                     const int32_t* expert_ids,
                                     const int32_t* num_tokens_post_padded, void* out, int64_t T,
                                     int64_t E, int64_t N, int64_t K, int64_t P,
                                     int64_t group_size, int64_t top_k, int64_t block_m,
                                     int32_t kernel, int32_t weight_is_e2m1, void* workspace,
                                     size_t workspace_bytes, w4a8_stream_t stream) {
    return moe_launch("mmq_fp8_moe_gemm", kEpiStore, x, w_packed, scales, w_zeros,
                      sorted_token_ids, expert_ids, num_tokens_post_padded, nullptr, out, T, 0, E,
                      N, K, P, group_size, top_k, block_m, kernel, weight_is_e2m1, workspace,
                      workspace_bytes, stream);
}

extern "C" int w4a8_mmq_fp8_moe_gemm1_silu(const void* x, const int32_t* w_packed,
                                           const void* scales, const int32_t* w_zeros,
                                           const int32_t* sorted_token_ids,
                                           const int32_t* expert_ids,
                                           const int32_t* num_tokens_post_padded, void* out,
                                           int64_t T, int64_t E, int64_t N, int64_t K, int64_t P,
                                           int64_t group_size, int64_t top_k, int64_t block_m,
                                           int32_t kernel, int32_t weight_is_e2m1,
                                           void* workspace, size_t workspace_bytes,
                                           w4a8_stream_t stream) {
    if (N % 2 != 0) return set_error("w13 N must be 2*inter (even); got " + std::to_string(N));
    if ((N / 2) % 8 != 0) return set_error("mmq_fp8_moe_gemm1_silu: inter must be a multiple of 8");
    return moe_launch("mmq_fp8_moe_gemm1_silu", kEpiSilu, x, w_packed, scales, w_zeros,
                      sorted_token_ids, expert_ids, num_tokens_post_padded, nullptr, out, T, 0, E,
                      N, K, P, group_size, top_k, block_m, kernel, weight_is_e2m1, workspace,
                      workspace_bytes, stream);
}

extern "C" int w4a8_mmq_fp8_moe_gemm_scatter(const void* x, const int32_t* w_packed,
                                             const void* scales, const int32_t* w_zeros,
                                             const int32_t* sorted_token_ids,
                                             const int32_t* expert_ids,
                                             const int32_t* num_tokens_post_padded,
                                             const float* topk_weights, float* output,
                                             int64_t M_out, int64_t E, int64_t N, int64_t K,
                                             int64_t P, int64_t group_size, int64_t top_k,
                                             int64_t block_m, int32_t kernel,
                                             int32_t weight_is_e2m1, void* workspace,
                                             size_t workspace_bytes, w4a8_stream_t stream) {
    if (M_out < 0) return set_error("mmq_fp8_moe_gemm_scatter: M must be >= 0");
    if (P > 0 && M_out > 0 && !topk_weights)
        return set_error("mmq_fp8_moe_gemm_scatter: null topk_weights");
    return moe_launch("mmq_fp8_moe_gemm_scatter", kEpiScatter, x, w_packed, scales, w_zeros,
                      sorted_token_ids, expert_ids, num_tokens_post_padded, topk_weights, output,
                      P, M_out, E, N, K, P, group_size, top_k, block_m, kernel, weight_is_e2m1,
                      workspace, workspace_bytes, stream);
}
