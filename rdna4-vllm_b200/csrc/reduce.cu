// reduce.cu — topk-weighted gather-reduce of the down-projection rows back to tokens.
//
// Semantics of mmq_fp8_moe_gather_reduce (w4a8_fp8_wmma/moe_kernel.hip:1230-1262):
//   slot_to_row[slot] = r for every r < ntp with sorted_token_ids[r] = slot < M*top_k, else -1;
//   out[t, n] = sum_{j ascending} w[t*top_k + j] * out2[slot_to_row[t*top_k + j], n]   (fp32)
// The sum is a plain fp32 multiply then add in slot order, the order the reference oracle uses
// (w4a8_fp8_wmma/test_moe_experts.py:182-190).
#include <algorithm>

#include "common.cuh"
#include "internal.h"

namespace w4a8 {

namespace {

__global__ void build_inverse_map_kernel(const int32_t* __restrict__ sorted_ids,
                                         const int32_t* __restrict__ ntp, int32_t* slot_to_row,
                                         int64_t P, int64_t num_slots) {
    const int64_t r = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (r >= P || r >= ntp[0]) return;
    const int32_t slot = sorted_ids[r];
    if (slot >= 0 && slot < num_slots) slot_to_row[slot] = (int32_t)r;
}

// One CTA per (token, 512-channel chunk); each thread reduces 2 adjacent channels. Generic
// path for N % 8 != 0 or unaligned rows.
template <typename OutT>
__global__ void __launch_bounds__(256)
gather_reduce_kernel(const __half* __restrict__ out2, const int32_t* __restrict__ slot_to_row,
                     const float* __restrict__ topk_w, OutT* __restrict__ out, int64_t N,
                     int top_k) {
    const int64_t t = blockIdx.y;
    const int64_t n = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) * 2;
    if (n >= N) return;
    float a0 = 0.f, a1 = 0.f;
    const bool pair = (n + 1 < N);
    for (int j = 0; j < top_k; ++j) {
        const int32_t r = slot_to_row[t * top_k + j];
        if (r < 0) continue;
        const float w = topk_w[t * top_k + j];
        const __half* rowp = out2 + (int64_t)r * N + n;
        if (pair && (N % 2 == 0)) {
            const __half2 v = *reinterpret_cast<const __half2*>(rowp);
            a0 = __fadd_rn(a0, __fmul_rn(w, __low2float(v)));
            a1 = __fadd_rn(a1, __fmul_rn(w, __high2float(v)));
        } else {
            a0 = __fadd_rn(a0, __fmul_rn(w, __half2float(rowp[0])));
            if (pair) a1 = __fadd_rn(a1, __fmul_rn(w, __half2float(rowp[1])));
        }
    }
    out[t * N + n] = (OutT)a0;
    if (pair) out[t * N + n + 1] = (OutT)a1;
}

// Vector path (N % 8 == 0, 16-byte aligned rows): one warp-row of 8-channel chunks per thread;
// the top_k row indices and weights of the token are staged once per CTA, then every slot's
// 16-byte row chunk is requested before the in-order accumulation.
constexpr int kMaxTopK = 16;
template <typename OutT>
__global__ void __launch_bounds__(256)
gather_reduce_vec_kernel(const __half* __restrict__ out2, const int32_t* __restrict__ slot_to_row,
                         const float* __restrict__ topk_w, OutT* __restrict__ out, int64_t N,
                         int top_k) {
    __shared__ int32_t rows[kMaxTopK];
    __shared__ float wts[kMaxTopK];
    const int64_t t = blockIdx.y;
    if (threadIdx.x < top_k) {
        rows[threadIdx.x] = slot_to_row[t * top_k + threadIdx.x];
        wts[threadIdx.x] = topk_w[t * top_k + threadIdx.x];
    }
    __syncthreads();
    const int64_t n = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) * 8;
    if (n >= N) return;
    uint4 v[kMaxTopK];
#pragma unroll
    for (int j = 0; j < kMaxTopK; ++j)
        if (j < top_k && rows[j] >= 0)
            v[j] = __ldg(reinterpret_cast<const uint4*>(out2 + (int64_t)rows[j] * N + n));
    float acc[8];
#pragma unroll
    for (int c = 0; c < 8; ++c) acc[c] = 0.f;
#pragma unroll
    for (int j = 0; j < kMaxTopK; ++j) {
        if (j < top_k && rows[j] >= 0) {
            const float w = wts[j];
            const uint32_t h[4] = {v[j].x, v[j].y, v[j].z, v[j].w};
#pragma unroll
            for (int c = 0; c < 4; ++c) {
                const float2 f = __half22float2(*reinterpret_cast<const __half2*>(&h[c]));
                acc[2 * c] = __fadd_rn(acc[2 * c], __fmul_rn(w, f.x));
                acc[2 * c + 1] = __fadd_rn(acc[2 * c + 1], __fmul_rn(w, f.y));
            }
        }
    }
    if constexpr (sizeof(OutT) == 4) {
        float4* o = reinterpret_cast<float4*>(reinterpret_cast<float*>(out) + t * N + n);
        o[0] = make_float4(acc[0], acc[1], acc[2], acc[3]);
        o[1] = make_float4(acc[4], acc[5], acc[6], acc[7]);
    } else {
        uint4 o;
        uint32_t* ow = reinterpret_cast<uint32_t*>(&o);
#pragma unroll
        for (int c = 0; c < 4; ++c) {
            const __half2 h2 = __floats2half2_rn(acc[2 * c], acc[2 * c + 1]);
            ow[c] = *reinterpret_cast<const uint32_t*>(&h2);
        }
        *reinterpret_cast<uint4*>(reinterpret_cast<__half*>(out) + t * N + n) = o;
    }
}

}  // namespace

int launch_gather_reduce(const __half* out2, const int32_t* slot_to_row, const float* topk_w,
                         void* out, bool out_half, int64_t M, int64_t N, int top_k,
                         cudaStream_t stream) {
    if (M <= 0) return W4A8_OK;
    const bool vec = N % 8 == 0 && top_k <= kMaxTopK &&
                     (reinterpret_cast<uintptr_t>(out2) & 15) == 0 &&
                     (reinterpret_cast<uintptr_t>(out) & 15) == 0;
    if (vec) {
        const dim3 grid((unsigned)((N / 8 + 255) / 256), (unsigned)M);
        if (out_half)
            gather_reduce_vec_kernel<__half><<<grid, 256, 0, stream>>>(
                out2, slot_to_row, topk_w, static_cast<__half*>(out), N, top_k);
        else
            gather_reduce_vec_kernel<float><<<grid, 256, 0, stream>>>(
                out2, slot_to_row, topk_w, static_cast<float*>(out), N, top_k);
        return launch_status();
    }
    const dim3 grid((unsigned)((N + 511) / 512), (unsigned)M);    return launch_status();
}

}  // namespace w4a8

extern "C" size_t w4a8_moe_gather_reduce_workspace_size(int64_t M, int64_t top_k) {
    return w4a8::align_up((size_t)(M * top_k) * sizeof(int32_t), 256);
}

extern "C" int w4a8_moe_gather_reduce(const void* out2, const int32_t* sorted_token_ids,
                                      const float* topk_weights,
                                      const int32_t* num_tokens_post_padded, float* out,
                                      int64_t M, int64_t N, int64_t P, int64_t top_k,
                                      void* workspace, size_t workspace_bytes,
                                      w4a8_stream_t stream) {
    using namespace w4a8;
    if (M < 0 || N <= 0 || P < 0 || top_k <= 0) return set_error("gather_reduce: bad sizes");
    if (M * top_k > INT32_MAX) return set_error("gather_reduce: size overflow");
    if (M == 0) return W4A8_OK;
    if (!out || !topk_weights || (P > 0 && (!out2 || !sorted_token_ids || !num_tokens_post_padded)))
        return set_error("gather_reduce: null pointer");
    if (!workspace || workspace_bytes < w4a8_moe_gather_reduce_workspace_size(M, top_k))
        return set_error("gather_reduce: workspace too small");
    cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
    int32_t* map = static_cast<int32_t*>(workspace);
    cudaError_t e = cudaMemsetAsync(map, 0xFF, (size_t)(M * top_k) * sizeof(int32_t), st);
    if (e != cudaSuccess) return (int)e;
    if (P > 0) {
        build_inverse_map_kernel<<<(unsigned)((P + 255) / 256), 256, 0, st>>>(
            sorted_token_ids, num_tokens_post_padded, map, P, M * top_k);
        if (int rc = launch_status()) return rc;
    }
    return launch_gather_reduce(static_cast<const __half*>(out2), map, topk_weights, out, false, M,
                                N, (int)top_k, st);
}

namespace w4a8 {
namespace {

// out[r][i] = fp16(silu(fp16 gate)) * fp16 up with gate = x[r][i], up = x[r][I + i]: vLLM's
// silu_and_mul on fp16 tensors, the step between gate_up and down in the unfused composition.
__global__ void __launch_bounds__(256) silu_and_mul_kernel(const __half* __restrict__ x,
                                                           __half* __restrict__ out, int64_t M,
                                                           int64_t I) {
    const int64_t n = M * I;
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n;
         i += (int64_t)gridDim.x * blockDim.x) {
        const int64_t r = i / I, c = i - r * I;
        out[i] = silu_mul_h(x[r * 2 * I + c], x[r * 2 * I + I + c]);
    }
}

}  // namespace
}  // namespace w4a8

extern "C" int w4a8_silu_and_mul(const void* x, void* out, int64_t M, int64_t inter,
                                 w4a8_stream_t stream) {
    using namespace w4a8;
    if (M < 0 || inter < 0) return set_error("silu_and_mul: negative size");
    if (M == 0 || inter == 0) return W4A8_OK;
    if (!x || !out) return set_error("silu_and_mul: null pointer");
    const int64_t n = M * inter;
    const unsigned grid = (unsigned)std::min<int64_t>((n + 255) / 256, 148 * 16);
    silu_and_mul_kernel<<<grid, 256, 0, reinterpret_cast<cudaStream_t>(stream)>>>(
        static_cast<const __half*>(x), static_cast<__half*>(out), M, inter);
    return launch_status();
}
