// e4_operand.cuh — the e4m3 activation operand of the mma.sync e4m3 GEMV (moe_decode.cu) and
// of the expert-parallel payload rows (ep_dispatch.cu).
#pragma once

#include "common.cuh"

namespace w4a8 {

// e4m3 operand of one row: the oracle's rounding (scale = max(amax, 4.48e-6) / 448 and
// q = e4m3_rn(x / scale), IEEE divides; w4a8_fp8_wmma/test_correctness.py:74-76), bytes stored
// in the GEMV's order (per 8-element unit: elements 0,2,4,6 then 1,3,5,7), the per 128-group
// sums S of the e4m3 values, and the scale. WARP: one warp per row reading memory written by
// other CTAs of the same launch (L2 loads); else the whole block. K % 256 == 0.
template <bool WARP>
static __device__ void quant_row_e4(const __half* src, int K, int64_t row, uint8_t* xe, float* xs,
                             float* scale, float* red) {
    const int n_thr = WARP ? 32 : (int)blockDim.x;
    const int tid = WARP ? (int)(threadIdx.x & 31) : (int)threadIdx.x;
    const int nch = K / 8;
    auto ld = [&](int i) {
        return WARP ? __ldcg(reinterpret_cast<const uint4*>(src) + i)
                    : *reinterpret_cast<const uint4*>(src + (int64_t)i * 8);
    };
    float amax = 0.f;
    for (int i = tid; i < nch; i += n_thr) {
        const uint4 v = ld(i);
        const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            const __half2 h = __habs2(*reinterpret_cast<const __half2*>(&w[j]));
            amax = fmaxf(amax, fmaxf(__low2float(h), __high2float(h)));
        }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
    if (!WARP) {
        const int w = threadIdx.x >> 5, l = threadIdx.x & 31;
        if (l == 0) red[w] = amax;
        __syncthreads();
        if (w == 0) {
            float v = l < (int)(blockDim.x >> 5) ? red[l] : 0.f;
#pragma unroll
            for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
            if (l == 0) red[0] = v;
        }
        __syncthreads();
        amax = red[0];
    }
    const float s = __fdiv_rn(fmaxf(amax, kAmaxFloor), kE4m3Max);
    const float rcp = __frcp_rn(s);
    if (tid == 0) scale[row] = s;
    const int G = K / 128;
    for (int i0 = 0; i0 < nch; i0 += n_thr) {  // lanes 0-15 / 16-31 of a warp: one group each
        const int i = i0 + tid;
        float sum = 0.f;
        if (i < nch) {
            const uint4 v = ld(i);
            const uint32_t w[4] = {v.x, v.y, v.z, v.w};
            uint32_t q[2];
#pragma unroll
            for (int j = 0; j < 4; j += 2) {
                const __half2 h0 = *reinterpret_cast<const __half2*>(&w[j]);
                const __half2 h1 = *reinterpret_cast<const __half2*>(&w[j + 1]);
                const uint16_t p0 = quant_pair(__low2float(h0), __high2float(h0), s, rcp);
                const uint16_t p1 = quant_pair(__low2float(h1), __high2float(h1), s, rcp);
                q[j / 2] = (uint32_t)p0 | ((uint32_t)p1 << 16);
                const uint32_t e0 = e4m3x2_to_f16x2(p0), e1 = e4m3x2_to_f16x2(p1);
                const float2 d0 = __half22float2(*reinterpret_cast<const __half2*>(&e0));
                const float2 d1 = __half22float2(*reinterpret_cast<const __half2*>(&e1));
                sum += (d0.x + d0.y) + (d1.x + d1.y);
            }
            // natural bytes q0..q7 -> GEMV order q0 q2 q4 q6 | q1 q3 q5 q7
            reinterpret_cast<uint2*>(xe + row * K)[i] =
                make_uint2(prmt(q[0], q[1], 0x6420u), prmt(q[0], q[1], 0x7531u));
        }
#pragma unroll
        for (int o = 8; o > 0; o >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, o);
        if ((tid & 15) == 0 && i < nch) xs[row * G + i / 16] = sum;
    }
}

// The block version for one row written at the given pointers (row 0).
static __device__ __forceinline__ void quant_row_e4_block(const __half* src, int K, uint8_t* xe,
                                                          float* xs, float* scale, float* red) {
    quant_row_e4<false>(src, K, 0, xe, xs, scale, red);
}

}  // namespace w4a8
