// common.cuh — shared device helpers for the sm_100a W4A8 kernels.
#pragma once

#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <string>

#include "w4a8_b200.h"

namespace w4a8 {

constexpr float kE4m3Max = 448.0f;
// The oracle clamps amax at 1e-8 * 448 before dividing by 448 (test_correctness.py:74-75).
constexpr float kAmaxFloor = 4.48e-6f;

// Host-side error channel (thread-local message + W4A8_ERR_INVALID).
int set_error(const std::string& msg);
inline int launch_status() {
    cudaError_t e = cudaGetLastError();
    return e == cudaSuccess ? W4A8_OK : static_cast<int>(e);
}

inline size_t align_up(size_t v, size_t a) { return (v + a - 1) / a * a; }

// ---- e4m3 conversions (hardware cvt, round-to-nearest-even, saturating) ----
// Packs two fp32 into two e4m3 bytes: lo byte from `lo`, hi byte from `hi`.
__device__ __forceinline__ uint16_t f32x2_to_e4m3x2(float lo, float hi) {
    uint16_t r;
    asm("cvt.rn.satfinite.e4m3x2.f32 %0, %1, %2;" : "=h"(r) : "f"(hi), "f"(lo));
    return r;
}
// e4m3 bytes of x0 / s and x1 / s (IEEE quotients, RNE, satfinite), from the product with the
// reciprocal r = 1 / s: the product is within 2^-23 (relative) of the quotient, so when both
// ends of [y (1 - 2^-21), y (1 + 2^-21)] round to the same byte, that byte is the quotient's
// (the rounding is monotonic); otherwise the IEEE divide decides.
__device__ __forceinline__ uint16_t quant_pair(float x0, float x1, float s, float r) {
    const float y0 = x0 * r, y1 = x1 * r;
    const uint16_t lo = f32x2_to_e4m3x2(y0 * (1.f - 0x1p-21f), y1 * (1.f - 0x1p-21f));
    const uint16_t hi = f32x2_to_e4m3x2(y0 * (1.f + 0x1p-21f), y1 * (1.f + 0x1p-21f));
    if (lo == hi) return lo;
    return f32x2_to_e4m3x2(__fdiv_rn(x0, s), __fdiv_rn(x1, s));
}

// Two e4m3 bytes (lo, hi) -> half2 (lo, hi); exact.
__device__ __forceinline__ uint32_t e4m3x2_to_f16x2(uint16_t v) {
    uint32_t r;
    asm("cvt.rn.f16x2.e4m3x2 %0, %1;" : "=r"(r) : "h"(v));
    return r;
}
__device__ __forceinline__ float e4m3_to_f32(uint8_t v) {
    uint32_t h2 = e4m3x2_to_f16x2(v);
    return __half2float(__ushort_as_half(static_cast<uint16_t>(h2 & 0xffff)));
}

// Byte permute: result byte i = byte sel_i of {b:a} (a = bytes 0..3, b = bytes 4..7).
__device__ __forceinline__ uint32_t prmt(uint32_t a, uint32_t b, uint32_t sel) {
    uint32_t r;
    asm("prmt.b32 %0, %1, %2, %3;" : "=r"(r) : "r"(a), "r"(b), "r"(sel));
    return r;
}
// lop3 with an immediate truth table.
template <int LUT>
__device__ __forceinline__ uint32_t lop3(uint32_t a, uint32_t b, uint32_t c) {
    uint32_t r;
    asm("lop3.b32 %0, %1, %2, %3, %4;" : "=r"(r) : "r"(a), "r"(b), "r"(c), "n"(LUT));
    return r;
}
// (a & b) | c
__device__ __forceinline__ uint32_t and_or(uint32_t a, uint32_t b, uint32_t c) {
    return lop3<(0xF0 & 0xCC) | 0xAA>(a, b, c);
}

__device__ __forceinline__ uint32_t hsub2_u(uint32_t a, uint32_t b) {
    __half2 r = __hsub2(*reinterpret_cast<__half2*>(&a), *reinterpret_cast<__half2*>(&b));
    return *reinterpret_cast<uint32_t*>(&r);
}
__device__ __forceinline__ uint32_t hfma2_u(uint32_t a, uint32_t b, uint32_t c) {
    __half2 r = __hfma2(*reinterpret_cast<__half2*>(&a), *reinterpret_cast<__half2*>(&b),
                        *reinterpret_cast<__half2*>(&c));
    return *reinterpret_cast<uint32_t*>(&r);
}

// Streaming 128-bit global load that bypasses L1 allocation (weights are read once).
__device__ __forceinline__ uint4 ldg_stream(const void* p) {
    uint4 r;
    asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];"
                 : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w)
                 : "l"(p));
    return r;
}

// mma.sync m16n8k16, f16 x f16 -> f32 (D = A*B + C).
// Not volatile: a pure function of its operands, so the compiler may interleave independent
// MMAs (their latency on sm_100 is long).
__device__ __forceinline__ void mma_16816(float (&d)[4], const uint32_t (&a)[4], uint32_t b0,
                                          uint32_t b1) {
    asm(
        "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, "
        "{%8,%9}, {%0,%1,%2,%3};"
        : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

// vLLM silu_and_mul on fp16 tensors: gate/up are the fp16 stores of the GEMM, silu is
// evaluated in fp32 and rounded to fp16, the product is a half*half multiply (the reference's
// moe_silu_and_mul_h, w4a8_fp8_wmma/moe_kernel.hip:555-565; oracle test_moe_experts.py:274-280).
// The same on operands already rounded to fp16.
//
// fp16(g / d) is taken from the fast quotient g * rcp(d) (div.approx: within 2 ulp of the
// IEEE quotient for the d that occur here, 1 <= d < 2^126) whenever the whole interval
// quotient * (1 -/+ 2^-20) rounds to one fp16 value: the IEEE quotient lies inside it and
// rounding is monotonic, so that value is exactly fp16(IEEE quotient). Otherwise (a quotient
// within a few fp32 ulp of an fp16 rounding boundary, about 0.1% of inputs) the IEEE divide
// decides. The result equals fp16(g / (1 + expf(-g))) with an IEEE divide, bit for bit.
__device__ __forceinline__ __half silu_mul_h(__half gh, __half uh) {
    const float g = __half2float(gh);
    const float d = 1.0f + expf(-g);
    const float qa = __fdividef(g, d);
    const float w = fabsf(qa) * 0x1p-20f;
    __half sh = __float2half_rn(qa);
    if (__half_as_ushort(__float2half_rn(qa - w)) != __half_as_ushort(__float2half_rn(qa + w)) ||
        !(d < 0x1p126f))
        sh = __float2half_rn(__fdiv_rn(g, d));
    return __hmul(sh, uh);
}
__device__ __forceinline__ __half silu_and_mul_half(float gate_f, float up_f) {
    return silu_mul_h(__float2half_rn(gate_f), __float2half_rn(up_f));
}

// OCP E2M1 (mxfp4) code -> value; the table is the format definition (bit3 sign,
// bits 2..1 exponent, bit 0 mantissa).
__device__ __forceinline__ float e2m1_value(int code) {
    const int mag = code & 7;
    const float v = (mag < 2) ? 0.5f * mag : (float)((2 + (mag & 1)) << ((mag >> 1) - 1)) * 0.5f;
    return (code & 8) ? -v : v;
}

}  // namespace w4a8
