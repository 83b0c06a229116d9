// tcgen05.cuh — 5th-generation tensor core helpers shared by the tile GEMM (gemm_tc.cu) and the
// decode GEMV (moe_decode.cu): the UMMA shared-memory and instruction descriptors, e4m3 code
// expansion, tensor-memory loads/stores, fp32x2 FMA.
#pragma once

#include "common.cuh"

namespace w4a8 {

// UMMA shared-memory descriptor, K-major with the 128-byte swizzle: 8-row atoms of 128 bytes,
// atoms 1024 bytes apart (SBO); the leading offset is unused for swizzled K-major operands.
static __device__ __forceinline__ uint64_t desc_sw128(uint32_t saddr) {
    uint64_t d = (uint64_t)((saddr >> 4) & 0x3FFFu);
    d |= (uint64_t)1 << 16;
    d |= (uint64_t)((1024u >> 4) & 0x3FFFu) << 32;
    d |= (uint64_t)1 << 46;  // descriptor version (sm_100)
    d |= (uint64_t)2 << 61;  // SWIZZLE_128B
    return d;
}

// kind::f8f6f4 instruction descriptor: fp32 accumulate, A = B = e4m3, both K-major.
static __host__ __device__ constexpr uint32_t umma_idesc(int M, int N) {
    return (1u << 4) | ((uint32_t)(N >> 3) << 17) | ((uint32_t)(M >> 4) << 24);
}

// 8 codes (nibble i of `w` = code i) -> 8 e4m3 bytes of the codes' values, codes 0..3 in `lo`
// and 4..7 in `hi`. prmt looks up 4 bytes at once from the selector's low 4 nibbles; a nibble
// with bit 3 set selects in sign-replicate mode, which yields 0x00 for the positive table
// bytes used here. The first lookup (selector = code) gives e4m3(q) for q < 8 and 0 for
// q >= 8; the second (selector = code ^ 8) gives e4m3(q) = 0x50 + (q - 8) for q >= 8 and 0 for
// q < 8; their OR is e4m3(q) for every code.
static __device__ __forceinline__ void codes8_to_e4m3(uint32_t w, uint32_t& lo, uint32_t& hi) {
    constexpr uint32_t kLo0 = 0x44403800u, kLo1 = 0x4E4C4A48u;  // e4m3(0..7)
    constexpr uint32_t kHi0 = 0x53525150u, kHi1 = 0x57565554u;  // e4m3(8..15)
    const uint32_t wx = w ^ 0x88888888u;
    lo = prmt(kLo0, kLo1, w) | prmt(kHi0, kHi1, wx);
    hi = prmt(kLo0, kLo1, w >> 16) | prmt(kHi0, kHi1, wx >> 16);
}

// Integer multiply-add; with operands the compiler cannot see it issues on the FMA pipe, which
// the expansion below uses to take work off the integer (ALU) pipe.
static __device__ __forceinline__ uint32_t imad(uint32_t a, uint32_t b, uint32_t c) {
    uint32_t d;
    asm("mad.lo.u32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(c));
    return d;
}

// codes8_to_e4m3 with half of its integer work on the FMA pipe. `one` = 1 and `m1` = 0xffffffff
// come from kernel arguments (opaque to the compiler). The second lookup takes the complemented
// selector ~w = w * m1 + m1: a code q >= 8 becomes 15 - q < 8 and selects e4m3(q) from a
// reversed table; q < 8 becomes >= 8, the sign-replicate mode, giving 0x00. The two lookups'
// nonzero bytes are disjoint, so their OR is the sum x * one + y.
static __device__ __forceinline__ void codes8_to_e4m3_fma(uint32_t w, uint32_t one, uint32_t m1,
                                                          uint32_t& lo, uint32_t& hi) {
    constexpr uint32_t kLo0 = 0x44403800u, kLo1 = 0x4E4C4A48u;  // e4m3(0..7)
    constexpr uint32_t kRv0 = 0x54555657u, kRv1 = 0x50515253u;  // byte i: e4m3(15 - i)
    const uint32_t nw = imad(w, m1, m1);
    lo = imad(prmt(kLo0, kLo1, w), one, prmt(kRv0, kRv1, nw));
    const uint32_t wh = w >> 16;
    const uint32_t nwh = imad(wh, m1, m1);
    hi = imad(prmt(kLo0, kLo1, wh), one, prmt(kRv0, kRv1, nwh));
}

// d = a * b + c on two fp32 lanes at once.
static __device__ __forceinline__ float2 ffma2(float2 a, float2 b, float2 c) {
    uint64_t d;
    asm("fma.rn.f32x2 %0, %1, %2, %3;"
        : "=l"(d)
        : "l"(*reinterpret_cast<uint64_t*>(&a)), "l"(*reinterpret_cast<uint64_t*>(&b)),
          "l"(*reinterpret_cast<uint64_t*>(&c)));
    return *reinterpret_cast<float2*>(&d);
}

template <int N>
__device__ __forceinline__ void tmem_ld(uint32_t taddr, uint32_t (&v)[N]);

template <>
__device__ __forceinline__ void tmem_ld<16>(uint32_t taddr, uint32_t (&v)[16]) {
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,"
        "%12,%13,%14,%15}, [%16];"
        : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]),
          "=r"(v[7]), "=r"(v[8]), "=r"(v[9]), "=r"(v[10]), "=r"(v[11]), "=r"(v[12]),
          "=r"(v[13]), "=r"(v[14]), "=r"(v[15])
        : "r"(taddr));
    asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}

template <>
__device__ __forceinline__ void tmem_ld<32>(uint32_t taddr, uint32_t (&v)[32]) {
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,"
        "%12,%13,%14,%15,%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31},"
        " [%32];"
        : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]),
          "=r"(v[7]), "=r"(v[8]), "=r"(v[9]), "=r"(v[10]), "=r"(v[11]), "=r"(v[12]),
          "=r"(v[13]), "=r"(v[14]), "=r"(v[15]), "=r"(v[16]), "=r"(v[17]), "=r"(v[18]),
          "=r"(v[19]), "=r"(v[20]), "=r"(v[21]), "=r"(v[22]), "=r"(v[23]), "=r"(v[24]),
          "=r"(v[25]), "=r"(v[26]), "=r"(v[27]), "=r"(v[28]), "=r"(v[29]), "=r"(v[30]),
          "=r"(v[31])
        : "r"(taddr));
    asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}

static __device__ __forceinline__ void tmem_st32(uint32_t taddr, const uint32_t (&v)[32]) {
    asm volatile(
        "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,"
        "%13,%14,%15,%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31,%32};" ::"r"(
            taddr),
        "r"(v[0]), "r"(v[1]), "r"(v[2]), "r"(v[3]), "r"(v[4]), "r"(v[5]), "r"(v[6]), "r"(v[7]),
        "r"(v[8]), "r"(v[9]), "r"(v[10]), "r"(v[11]), "r"(v[12]), "r"(v[13]), "r"(v[14]),
        "r"(v[15]), "r"(v[16]), "r"(v[17]), "r"(v[18]), "r"(v[19]), "r"(v[20]), "r"(v[21]),
        "r"(v[22]), "r"(v[23]), "r"(v[24]), "r"(v[25]), "r"(v[26]), "r"(v[27]), "r"(v[28]),
        "r"(v[29]), "r"(v[30]), "r"(v[31])
        : "memory");
}



template <>
__device__ __forceinline__ void tmem_ld<8>(uint32_t taddr, uint32_t (&v)[8]) {
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x8.b32 {%0,%1,%2,%3,%4,%5,%6,%7}, [%8];"
        : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]),
          "=r"(v[7])
        : "r"(taddr));
    asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}

// 4 consecutive columns of this warp's 32 lanes; the caller waits (tmem_wait_ld).
static __device__ __forceinline__ void tmem_ld4_nowait(uint32_t taddr, uint32_t (&v)[4]) {
    asm volatile("tcgen05.ld.sync.aligned.32x32b.x4.b32 {%0,%1,%2,%3}, [%4];"
                 : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3])
                 : "r"(taddr));
}
// 16 consecutive columns of this warp's 32 lanes; the caller waits (tmem_wait_ld).
static __device__ __forceinline__ void tmem_ld16_nowait(uint32_t taddr, uint32_t (&v)[16]) {
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,"
        "%12,%13,%14,%15}, [%16];"
        : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]),
          "=r"(v[7]), "=r"(v[8]), "=r"(v[9]), "=r"(v[10]), "=r"(v[11]), "=r"(v[12]),
          "=r"(v[13]), "=r"(v[14]), "=r"(v[15])
        : "r"(taddr));
}
static __device__ __forceinline__ void tmem_wait_ld() {
    asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}

static __device__ __forceinline__ void tmem_st8(uint32_t taddr, const uint32_t (&v)[8]) {
    asm volatile(
        "tcgen05.st.sync.aligned.32x32b.x8.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8};" ::"r"(taddr),
        "r"(v[0]), "r"(v[1]), "r"(v[2]), "r"(v[3]), "r"(v[4]), "r"(v[5]), "r"(v[6]), "r"(v[7])
        : "memory");
}

static __device__ __forceinline__ void tmem_st16(uint32_t taddr, const uint32_t (&v)[16]) {
    asm volatile(
        "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,"
        "%13,%14,%15,%16};" ::"r"(taddr),
        "r"(v[0]), "r"(v[1]), "r"(v[2]), "r"(v[3]), "r"(v[4]), "r"(v[5]), "r"(v[6]), "r"(v[7]),
        "r"(v[8]), "r"(v[9]), "r"(v[10]), "r"(v[11]), "r"(v[12]), "r"(v[13]), "r"(v[14]),
        "r"(v[15])
        : "memory");
}

}  // namespace w4a8
