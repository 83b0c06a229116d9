// router.cu — the MoE router in one launch: softmax over the expert logits, top-k, renormalise,
// and the per-expert slot counts that the expert grouping (moe_align_block_size) starts from.
//
// The reference takes topk_ids / topk_weights from vLLM's router (softmax -> top-k ->
// renormalise, the `renormalize=True` fused_topk path) and hands them to the align call at
// w4a8_fp8_wmma/w4a8_fp8_wmma/moe_experts.py:587-589; the restatement the results are checked
// against is oracle/w4a8_oracle.py:route_topk.
//
// One warp per token; each lane holds E/32 logits in registers (E <= 1024).
// - ids: k rounds of a warp arg-max over the logits still in play, ties to the lower expert
//   index. Softmax is monotonic, so this is the top-k of the probabilities in the oracle's
//   order (a stable descending sort) except where two different logits round to the same fp32
//   probability, which the oracle would then order by index.
// - weights: p_e = exp(l_e - max) / sum over all experts (fp32, expf), then the k chosen p's
//   divided by their sum in pick order — the reference's sequence of operations.
// - counts (optional): one atomic per valid slot into a caller buffer the entry point zeroes.
#include <cuda_bf16.h>

#include <string>

#include "common.cuh"
#include "internal.h"

namespace w4a8 {

namespace {

constexpr int kRouterWarps = 8;
constexpr int kRouterMaxE = 1024;
constexpr int kRouterMaxK = 16;

template <typename T>
__device__ __forceinline__ float to_f32(T v);
template <>
__device__ __forceinline__ float to_f32<float>(float v) { return v; }
template <>
__device__ __forceinline__ float to_f32<__half>(__half v) { return __half2float(v); }
template <>
__device__ __forceinline__ float to_f32<__nv_bfloat16>(__nv_bfloat16 v) { return __bfloat162float(v); }

template <typename T, int PER>
__global__ void __launch_bounds__(kRouterWarps * 32)
route_topk_kernel(const T* __restrict__ logits, int64_t T_rows, int E, int k, int renorm,
                  int32_t* __restrict__ ids, float* __restrict__ wts, int32_t* __restrict__ counts) {
    const int lane = threadIdx.x & 31;
    const int64_t t = (int64_t)blockIdx.x * kRouterWarps + (threadIdx.x >> 5);
    if (t >= T_rows) return;
    // lane holds experts lane, lane + 32, ... (PER of them; -inf past E)
    float l[PER];
#pragma unroll
    for (int i = 0; i < PER; ++i) {
        const int e = lane + 32 * i;
        l[i] = e < E ? to_f32(logits[t * E + e]) : -INFINITY;
    }
    float m = -INFINITY;
#pragma unroll
    for (int i = 0; i < PER; ++i) m = fmaxf(m, l[i]);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
    float sum = 0.f;
#pragma unroll
    for (int i = 0; i < PER; ++i)
        if (lane + 32 * i < E) sum += expf(l[i] - m);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, o);
    unsigned taken = 0;  // bit i: expert lane + 32 i already chosen
    float p_sel = 0.f, tot = 0.f;
    int my_id = -1;      // lane j < k ends with pick j
    for (int j = 0; j < k; ++j) {
        // lane-local best among the experts still in play (lowest index on ties)
        float bv = -INFINITY;
        int be = 0x7fffffff;
#pragma unroll
        for (int i = 0; i < PER; ++i) {
            const int e = lane + 32 * i;
            if (e < E && !((taken >> i) & 1u) && (l[i] > bv || (l[i] == bv && e < be))) {
                bv = l[i];
                be = e;
            }
        }
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) {
            const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
            const int oe = __shfl_xor_sync(0xffffffffu, be, o);
            if (ov > bv || (ov == bv && oe < be)) {
                bv = ov;
                be = oe;
            }
        }
        if ((be & 31) == lane) taken |= 1u << (be >> 5);
        const float p = expf(bv - m) / sum;
        tot += p;
        if (lane == j) {
            my_id = be;
            p_sel = p;
        }
    }
    if (lane < k) {
        ids[t * k + lane] = my_id;
        wts[t * k + lane] = renorm ? p_sel / tot : p_sel;
        if (counts) atomicAdd(counts + my_id, 1);
    }
}

template <typename T>
int launch_route(const void* logits, int64_t T_rows, int E, int k, int renorm, int32_t* ids,
                 float* wts, int32_t* counts, cudaStream_t st) {
    const unsigned grid = (unsigned)((T_rows + kRouterWarps - 1) / kRouterWarps);
    const T* lg = static_cast<const T*>(logits);
    const int per = (E + 31) / 32;
    if (per <= 8)
        route_topk_kernel<T, 8><<<grid, kRouterWarps * 32, 0, st>>>(lg, T_rows, E, k, renorm, ids, wts, counts);
    else
        route_topk_kernel<T, 32><<<grid, kRouterWarps * 32, 0, st>>>(lg, T_rows, E, k, renorm, ids, wts, counts);
    return launch_status();
}

}  // namespace

}  // namespace w4a8

using namespace w4a8;

extern "C" int w4a8_route_topk(const void* logits, int32_t logits_dtype, int64_t num_tokens,
                               int32_t num_experts, int32_t top_k, int32_t renormalize,
                               int32_t* topk_ids, float* topk_weights, int32_t* expert_counts,
                               w4a8_stream_t stream) {
    const std::string o = "route_topk";
    if (num_tokens < 0 || num_experts <= 0 || num_experts > kRouterMaxE || top_k <= 0 ||
        top_k > kRouterMaxK || top_k > num_experts)
        return set_error(o + ": bad sizes (1 <= top_k <= min(16, num_experts), num_experts <= 1024)");
    if (logits_dtype < 0 || logits_dtype > 2)
        return set_error(o + ": logits_dtype must be 0 (fp32), 1 (fp16) or 2 (bf16)");
    cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
    if (expert_counts) {
        const cudaError_t e = cudaMemsetAsync(expert_counts, 0, (size_t)num_experts * 4, st);
        if (e != cudaSuccess) return (int)e;
    }
    if (num_tokens == 0) return W4A8_OK;
    if (!logits || !topk_ids || !topk_weights) return set_error(o + ": null pointer");
    switch (logits_dtype) {
        case 0:
            return launch_route<float>(logits, num_tokens, num_experts, top_k, renormalize != 0,
                                       topk_ids, topk_weights, expert_counts, st);
        case 1:
            return launch_route<__half>(logits, num_tokens, num_experts, top_k, renormalize != 0,
                                        topk_ids, topk_weights, expert_counts, st);
        default:
            return launch_route<__nv_bfloat16>(logits, num_tokens, num_experts, top_k,
                                               renormalize != 0, topk_ids, topk_weights,
                                               expert_counts, st);
    }
}
