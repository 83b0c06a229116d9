// act_quant.cu — per-token e4m3 activation quantisation (one warp per row).
//
// Arithmetic follows the reference oracle (w4a8_fp8_wmma/test_correctness.py:74-76):
//   a_scale = max(amax, 4.48e-6f) / 448      (IEEE divide)
//   q       = e4m3_rn_satfinite(x / a_scale) (IEEE divide, not a reciprocal multiply)
// The reference HIP kernel (moe_kernel.hip:87-130) multiplies by 1/scale instead, which can
// flip a byte at a rounding boundary; this kernel matches the oracle bit for bit.
#include "internal.h"
#include "common.cuh"

namespace w4a8 {

namespace {

constexpr int kWarpsPerCta = 8;

__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
    return v;
}

// Vector path: K % 8 == 0 and 16-byte aligned rows.
__global__ void __launch_bounds__(kWarpsPerCta * 32)
act_quant_vec_kernel(const __half* __restrict__ x, uint8_t* __restrict__ xq,
                     float* __restrict__ scales, int64_t M, int64_t K,
                     const int32_t* __restrict__ row_limit) {
    const int lane = threadIdx.x & 31;
    const int64_t row = (int64_t)blockIdx.x * kWarpsPerCta + (threadIdx.x >> 5);
    if (row >= M || (row_limit && row >= row_limit[0])) return;
    const uint4* xr = reinterpret_cast<const uint4*>(x + row * K);
    const int64_t nvec = K / 8;
    float amax = 0.f;
    for (int64_t i = lane; i < nvec; i += 32) {
        uint4 v = __ldg(xr + i);
        const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            __half2 h = __habs2(*reinterpret_cast<const __half2*>(&w[j]));
            amax = fmaxf(amax, fmaxf(__low2float(h), __high2float(h)));
        }
    }
    amax = warp_max(amax);
    const float s = __fdiv_rn(fmaxf(amax, kAmaxFloor), kE4m3Max);
    if (lane == 0) scales[row] = s;
    uint2* qr = reinterpret_cast<uint2*>(xq + row * K);
    for (int64_t i = lane; i < nvec; i += 32) {
        uint4 v = __ldg(xr + i);
        const uint32_t w[4] = {v.x, v.y, v.z, v.w};
        uint32_t out[2];
#pragma unroll
        for (int j = 0; j < 4; j += 2) {
            const __half2 h0 = *reinterpret_cast<const __half2*>(&w[j]);
            const __half2 h1 = *reinterpret_cast<const __half2*>(&w[j + 1]);
            const uint16_t p0 = f32x2_to_e4m3x2(__fdiv_rn(__low2float(h0), s),
                                                __fdiv_rn(__high2float(h0), s));
            const uint16_t p1 = f32x2_to_e4m3x2(__fdiv_rn(__low2float(h1), s),
                                                __fdiv_rn(__high2float(h1), s));
            out[j / 2] = (uint32_t)p0 | ((uint32_t)p1 << 16);
        }
        qr[i] = make_uint2(out[0], out[1]);
    }
}

// Scalar path for unaligned rows or K % 8 != 0.
__global__ void __launch_bounds__(kWarpsPerCta * 32)
act_quant_scalar_kernel(const __half* __restrict__ x, uint8_t* __restrict__ xq,
                        float* __restrict__ scales, int64_t M, int64_t K,
                        const int32_t* __restrict__ row_limit) {
    const int lane = threadIdx.x & 31;
    const int64_t row = (int64_t)blockIdx.x * kWarpsPerCta + (threadIdx.x >> 5);
    if (row >= M || (row_limit && row >= row_limit[0])) return;
    const __half* xr = x + row * K;
    float amax = 0.f;
    for (int64_t k = lane; k < K; k += 32) amax = fmaxf(amax, fabsf(__half2float(xr[k])));
    amax = warp_max(amax);
    const float s = __fdiv_rn(fmaxf(amax, kAmaxFloor), kE4m3Max);
    if (lane == 0) scales[row] = s;
    for (int64_t k = lane; k < K; k += 32)
        xq[row * K + k] = (uint8_t)(f32x2_to_e4m3x2(__fdiv_rn(__half2float(xr[k]), s), 0.f));
}

}  // namespace

int launch_act_quant(const void* x, uint8_t* xq, float* scales, int64_t M, int64_t K,
                     cudaStream_t stream, const int32_t* row_limit) {
    if (M <= 0 || K <= 0) return W4A8_OK;
    const dim3 grid((unsigned)((M + kWarpsPerCta - 1) / kWarpsPerCta));
    const bool vec = (K % 8 == 0) && ((reinterpret_cast<uintptr_t>(x) & 15) == 0) &&
                     ((reinterpret_cast<uintptr_t>(xq) & 7) == 0);
    if (vec)
        act_quant_vec_kernel<<<grid, kWarpsPerCta * 32, 0, stream>>>(
            static_cast<const __half*>(x), xq, scales, M, K, row_limit);
    else
        act_quant_scalar_kernel<<<grid, kWarpsPerCta * 32, 0, stream>>>(
            static_cast<const __half*>(x), xq, scales, M, K, row_limit);
    return launch_status();
}

}  // namespace w4a8

extern "C" int w4a8_act_quant_fp8(const void* x, uint8_t* x_fp8, float* act_scales, int64_t M,
                                  int64_t K, w4a8_stream_t stream) {
    if (M < 0 || K < 0) return w4a8::set_error("act_quant: negative size");
    if (M > 0 && (!x || !x_fp8 || !act_scales))
        return w4a8::set_error("act_quant: null pointer");
    return w4a8::launch_act_quant(x, x_fp8, act_scales, M, K, stream);
}
