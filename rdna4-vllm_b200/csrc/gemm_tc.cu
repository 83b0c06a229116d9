// gemm_tc.cu — W4A8 (grouped) GEMM tile path on the 5th-generation tensor cores (tcgen05).
//
// Two launches:
//   1. tc_gather_kernel — copies each sorted row's e4m3 activation row, its activation scale and
//      its per-group sums S into dense sorted-order buffers (padding rows become zeros), so the
//      GEMM reads its token tiles with plain 2D TMA boxes instead of per-row gathers.
//   2. w4_tc_kernel — persistent and warp-specialised, one CTA per SM. A tile is 128 weight
//      rows x NT sorted rows (NT = 64 or 128; a tile never straddles an expert block). Tiles are
//      dealt round-robin to the CTAs; inside a CTA every role walks the same tile sequence and
//      the (tile, K-group) steps flow through mbarrier rings, so the next tile's loads and MMAs
//      overlap the current tile's epilogue.
//
// Roles (16 warps):
//   warp 0      TMA producer: weight codes (2D box, 64-byte swizzle), token tile (2D box,
//               128-byte swizzle = the UMMA K-major SW128 layout), group sums (bulk copy).
//   warp 1      MMA issuer: 4 x tcgen05.mma.kind::f8f6f4 (K = 32 each) per group into one of the
//               TMEM accumulators (512 columns / NT), committed to the stage / A / accumulator barriers.
//   warp 2      owns the tensor-memory allocation.
//   warps 4-7   expand the 4-bit codes to e4m3 bytes in the SW128 A layout (thread = weight row).
//   warps 8-15  fold each group's accumulator into fp32 registers and write the tile's output.
//
// Numerics. The A operand holds e4m3(q) — the unsigned 4-bit code itself, exact in e4m3 — so
// per 128-wide group g the tensor core returns acc = sum_k q_k a_k. With S_g = sum_k a_k the
// reference's group result sum_k (q_k - z) a_k equals acc - z*S_g exactly in real arithmetic,
// and it is folded in fp32 as
//     tot += scale[n,g] * acc - (scale[n,g] * z) * S_g
// then multiplied by the row's activation scale: the reference oracle's association
// (w4a8_fp8_wmma/test_correctness.py:113-119) up to fp32 rounding.
//
// Every mbarrier wait is bounded. When one gives up the kernel records an error code, every
// role stops waiting (the results are then garbage, reported through TcArgs::err), the producer
// waits boundedly for its own copies in flight and the tensor memory is always released.
#include <cudaTypedefs.h>

#include <algorithm>
#include <mutex>

#include "common.cuh"
#include "gemm_common.h"
#include "internal.h"

namespace w4a8 {

namespace {

constexpr int kTcThreads = 512;
constexpr uint32_t kSpinLimit = 1u << 22;
constexpr int kFoldWarps = 8;

template <int NT>
struct TcCfg {
    static constexpr int kStages = NT == 128 ? 5 : 7;  // TMA ring depth (codes + tokens)
    static constexpr int kAStages = NT == 128 ? 4 : 5; // dequantised-A ring depth
    static constexpr int kSStages = 8;                 // group-sum ring depth
    static constexpr int kAcc = 512 / NT;              // TMEM accumulators (all 512 columns)
    static constexpr int kCols = NT / 2;               // accumulator columns per fold thread
    static constexpr uint32_t kTmemCols = 512;
    static constexpr uint32_t kStageBytes = 128 * 64 + NT * 128;
};

template <int NT>
struct TcSmem {
    uint8_t b[TcCfg<NT>::kStages][NT * 128];     // token tiles, SW128 K-major (1024-aligned)
    uint8_t a[TcCfg<NT>::kAStages][128 * 128];   // e4m3 weights, SW128 K-major
    uint8_t raw[TcCfg<NT>::kStages][128 * 64];   // packed codes, SW64 as TMA writes them
    __half otile[NT * 128];                      // epilogue: fp16 results, [column][row]
    float ssum[TcCfg<NT>::kSStages][NT];         // group sums S of the tile's rows
    uint64_t full[TcCfg<NT>::kStages];
    uint64_t empty[TcCfg<NT>::kStages];
    uint64_t sfull[TcCfg<NT>::kSStages];
    uint64_t sempty[TcCfg<NT>::kSStages];
    uint64_t afull[TcCfg<NT>::kAStages];
    uint64_t aempty[TcCfg<NT>::kAStages];
    uint64_t tfull[TcCfg<NT>::kAcc];
    uint64_t tempty[TcCfg<NT>::kAcc];
    uint32_t tmem_base;
    int bad;
};

static_assert(sizeof(TcSmem<128>) + 1024 <= 227 * 1024, "tile kernel shared memory");
static_assert(sizeof(TcSmem<64>) + 1024 <= 227 * 1024, "tile kernel shared memory");

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
    return (uint32_t)__cvta_generic_to_shared(p);
}

// UMMA shared-memory descriptor, K-major with the 128-byte swizzle: 8-row atoms of 128 bytes,
// atoms 1024 bytes apart (SBO); the leading offset is unused for swizzled K-major operands.
__device__ __forceinline__ uint64_t desc_sw128(uint32_t saddr) {
    uint64_t d = (uint64_t)((saddr >> 4) & 0x3FFFu);
    d |= (uint64_t)1 << 16;
    d |= (uint64_t)((1024u >> 4) & 0x3FFFu) << 32;
    d |= (uint64_t)1 << 46;  // descriptor version (sm_100)
    d |= (uint64_t)2 << 61;  // SWIZZLE_128B
    return d;
}

// kind::f8f6f4 instruction descriptor: fp32 accumulate, A = B = e4m3, both K-major.
__host__ __device__ constexpr uint32_t umma_idesc(int M, int N) {
    return (1u << 4) | ((uint32_t)(N >> 3) << 17) | ((uint32_t)(M >> 4) << 24);
}

__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count));
}
__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}
__device__ __forceinline__ void mbar_expect_tx(uint64_t* bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)),
                 "r"(bytes)
                 : "memory");
}
__device__ __forceinline__ bool mbar_try(uint64_t* bar, uint32_t parity) {
    uint32_t done;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(done)
        : "r"(smem_u32(bar)), "r"(parity)
        : "memory");
    return done != 0;
}
// Bounded wait; once any wait in the CTA has given up, later waits return at once.
__device__ __forceinline__ void mbar_wait(uint64_t* bar, uint32_t parity, volatile int* bad) {
    if (*bad) return;
    for (uint32_t i = 0; i < kSpinLimit; ++i)
        if (mbar_try(bar, parity)) return;
    *bad = 1;
}

__device__ __forceinline__ void tma_load_2d(void* dst, const CUtensorMap* map, int x, int y,
                                            uint64_t* bar) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
        " [%0], [%1, {%2, %3}], [%4];" ::"r"(smem_u32(dst)),
        "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(smem_u32(bar))
        : "memory");
}
__device__ __forceinline__ void tma_prefetch_2d(const CUtensorMap* map, int x, int y) {
    asm volatile("cp.async.bulk.prefetch.tensor.2d.L2.global.tile [%0, {%1, %2}];" ::"l"(
                     reinterpret_cast<uint64_t>(map)),
                 "r"(x), "r"(y)
                 : "memory");
}
__device__ __forceinline__ void bulk_load(void* dst, const void* src, uint32_t bytes,
                                          uint64_t* bar) {
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];"
        ::"r"(smem_u32(dst)), "l"(src), "r"(bytes), "r"(smem_u32(bar))
        : "memory");
}

// 4 codes (the low 16 bits of `w`, nibble i = code i) -> 4 e4m3 bytes of the codes' values.
// Bytes of codes 0..7 come from the table {0, 1, 2, 3, 4, 5, 6, 7} in e4m3; codes 8..15 are
// 0x50 + (q - 8) (exponent 3, mantissa q - 8). prmt's sign-replicate mode (selector bit 3)
// turns the high codes into 0x00 in the first lookup and into an all-ones mask in the third.
__device__ __forceinline__ uint32_t codes_to_e4m3(uint32_t w) {
    constexpr uint32_t kLo0 = 0x44403800u, kLo1 = 0x4E4C4A48u;  // e4m3(0..7)
    constexpr uint32_t kHi0 = 0x53525150u, kHi1 = 0x57565554u;  // e4m3(8..15)
    constexpr uint32_t kSign = 0x80808080u;
    const uint32_t lo = prmt(kLo0, kLo1, w);                // q<8: e4m3(q); q>=8: 0x00
    const uint32_t hi = prmt(kHi0, kHi1, w & 0x7777u);      // e4m3(8 + (q & 7))
    const uint32_t m = prmt(kSign, kSign, w);               // q<8: 0x80; q>=8: 0xFF
    return lop3<(0xF0 & 0xCC) | (~0xF0 & 0xAA)>(m, hi, lo); // m ? hi : lo, bitwise
}

// d = a * b + c on two fp32 lanes at once.
__device__ __forceinline__ float2 ffma2(float2 a, float2 b, float2 c) {
    uint64_t d;
    asm("fma.rn.f32x2 %0, %1, %2, %3;"
        : "=l"(d)
        : "l"(*reinterpret_cast<uint64_t*>(&a)), "l"(*reinterpret_cast<uint64_t*>(&b)),
          "l"(*reinterpret_cast<uint64_t*>(&c)));
    return *reinterpret_cast<float2*>(&d);
}

__device__ __forceinline__ void tmem_ld32(uint32_t taddr, uint32_t (&v)[32]) {
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

// Expert of tile row block rb (0 for the dense GEMM).
__device__ __forceinline__ int tile_expert(const TcArgs& a, int rb, int NT) {
    if (!a.expert_ids) return 0;
    return a.expert_ids[(int64_t)rb * NT / a.block_m];
}

template <int NT>
__global__ void __launch_bounds__(kTcThreads, 1)
w4_tc_kernel(const TcArgs a, const __grid_constant__ CUtensorMap tmw,
             const __grid_constant__ CUtensorMap tmx) {
    using C = TcCfg<NT>;
    extern __shared__ uint8_t smem_raw[];
    TcSmem<NT>& sm = *reinterpret_cast<TcSmem<NT>*>(
        (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    volatile int* bad = &sm.bad;

    const int P_valid = a.ntp ? min(a.ntp[0], a.P) : a.P;
    const int nblk = (P_valid + NT - 1) / NT;
    const int n_mt = a.silu ? (a.N / 2) / 64 : (a.N + 127) / 128;
    const int n_tiles = nblk * n_mt;
    const int n_out = a.silu ? a.N / 2 : a.N;

    if (tid == 0) {
        sm.bad = 0;
        for (int s = 0; s < C::kStages; ++s) {
            mbar_init(&sm.full[s], 1);
            mbar_init(&sm.empty[s], 1);
        }
        for (int s = 0; s < C::kSStages; ++s) {
            mbar_init(&sm.sfull[s], 1);
            mbar_init(&sm.sempty[s], kFoldWarps);
        }
        for (int s = 0; s < C::kAStages; ++s) {
            mbar_init(&sm.afull[s], 4);
            mbar_init(&sm.aempty[s], 1);
        }
        for (int s = 0; s < C::kAcc; ++s) {
            mbar_init(&sm.tfull[s], 1);
            mbar_init(&sm.tempty[s], kFoldWarps);
        }
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    if (warp == 2) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                         smem_u32(&sm.tmem_base)),
                     "r"(C::kTmemCols));
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::);
    }
    asm volatile("tcgen05.fence::before_thread_sync;" ::);
    __syncthreads();
    asm volatile("tcgen05.fence::after_thread_sync;" ::);
    const uint32_t tmem = sm.tmem_base;

    if (warp == 0) {
        // ---------------- TMA producer ----------------
        if (lane == 0) {
            uint32_t it = 0;
            for (int t = blockIdx.x; t < n_tiles; t += gridDim.x) {
                const int rb = t / n_mt, mt = t % n_mt;
                const int e = tile_expert(a, rb, NT);
                if (e < 0 || e >= a.E) continue;
                const int r0 = rb * NT;
                // warm L2 with this CTA's next tile (weights and tokens) while this one runs
                const int tn = t + gridDim.x;
                if (tn < n_tiles) {
                    const int rbn = tn / n_mt, mtn = tn % n_mt;
                    const int en = tile_expert(a, rbn, NT);
                    if (en >= 0 && en < a.E)
                        for (int g = 0; g < a.G; ++g) {
                            if (a.silu) {
                                tma_prefetch_2d(&tmw, g * 64, en * a.N + mtn * 64);
                                tma_prefetch_2d(&tmw, g * 64, en * a.N + a.N / 2 + mtn * 64);
                            } else {
                                tma_prefetch_2d(&tmw, g * 64, en * a.N + mtn * 128);
                            }
                            tma_prefetch_2d(&tmx, g * 128, rbn * NT);
                        }
                }
                for (int g = 0; g < a.G; ++g, ++it) {
                    const int s = it % C::kStages;
                    const int ss = it % C::kSStages;
                    mbar_wait(&sm.empty[s], ((it / C::kStages) & 1) ^ 1, bad);
                    mbar_expect_tx(&sm.full[s], C::kStageBytes);
                    if (a.silu) {
                        tma_load_2d(&sm.raw[s][0], &tmw, g * 64, e * a.N + mt * 64, &sm.full[s]);
                        tma_load_2d(&sm.raw[s][64 * 64], &tmw, g * 64,
                                    e * a.N + a.N / 2 + mt * 64, &sm.full[s]);
                    } else {
                        tma_load_2d(&sm.raw[s][0], &tmw, g * 64, e * a.N + mt * 128, &sm.full[s]);
                    }
                    tma_load_2d(&sm.b[s][0], &tmx, g * 128, r0, &sm.full[s]);
                    mbar_wait(&sm.sempty[ss], ((it / C::kSStages) & 1) ^ 1, bad);
                    mbar_expect_tx(&sm.sfull[ss], NT * 4);
                    bulk_load(&sm.ssum[ss][0], a.ssum + (int64_t)g * a.P_pad + r0, NT * 4,
                              &sm.sfull[ss]);
                }
            }
            // leave no copy in flight: wait (boundedly) for the last ring's worth of loads
            if (*bad) {
                const uint32_t first = it > (uint32_t)C::kStages ? it - C::kStages : 0;
                for (uint32_t j = first; j < it; ++j)
                    for (uint32_t i = 0; i < kSpinLimit; ++i)
                        if (mbar_try(&sm.full[j % C::kStages], (j / C::kStages) & 1)) break;
                const uint32_t sfirst = it > (uint32_t)C::kSStages ? it - C::kSStages : 0;
                for (uint32_t j = sfirst; j < it; ++j)
                    for (uint32_t i = 0; i < kSpinLimit; ++i)
                        if (mbar_try(&sm.sfull[j % C::kSStages], (j / C::kSStages) & 1)) break;
            }
        }
    } else if (warp == 1) {
        // ---------------- MMA issuer ----------------
        if (lane == 0) {
            constexpr uint32_t idesc = umma_idesc(128, NT);
            uint32_t it = 0;
            for (int t = blockIdx.x; t < n_tiles; t += gridDim.x) {
                const int e = tile_expert(a, t / n_mt, NT);
                if (e < 0 || e >= a.E) continue;
                for (int g = 0; g < a.G; ++g, ++it) {
                    const int s = it % C::kStages;
                    const int as = it % C::kAStages;
                    const int tb = it % C::kAcc;
                    mbar_wait(&sm.full[s], (it / C::kStages) & 1, bad);
                    mbar_wait(&sm.afull[as], (it / C::kAStages) & 1, bad);
                    mbar_wait(&sm.tempty[tb], ((it / C::kAcc) & 1) ^ 1, bad);
                    asm volatile("tcgen05.fence::after_thread_sync;" ::);
                    const uint32_t a0 = smem_u32(&sm.a[as][0]);
                    const uint32_t b0 = smem_u32(&sm.b[s][0]);
                    const uint32_t d = tmem + (uint32_t)(tb * NT);
#pragma unroll
                    for (int kk = 0; kk < 4; ++kk) {
                        const uint64_t da = desc_sw128(a0 + kk * 32);
                        const uint64_t db = desc_sw128(b0 + kk * 32);
                        const uint32_t acc = kk > 0 ? 1u : 0u;
                        asm volatile(
                            "{\n\t.reg .pred p;\n\t"
                            "setp.ne.b32 p, %4, 0;\n\t"
                            "tcgen05.mma.cta_group::1.kind::f8f6f4 [%0], %1, %2, %3, p;\n\t}" ::"r"(d),
                            "l"(da), "l"(db), "r"(idesc), "r"(acc));
                    }
                    asm volatile(
                        "tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];"
                        ::"r"(smem_u32(&sm.empty[s])));
                    asm volatile(
                        "tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];"
                        ::"r"(smem_u32(&sm.aempty[as])));
                    asm volatile(
                        "tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];"
                        ::"r"(smem_u32(&sm.tfull[tb])));
                }
            }
        }
    } else if (warp >= 4 && warp < 8) {
        // ---------------- code expansion: thread = weight row ----------------
        const int m = tid - 128;
        const int sw64 = (m >> 1) & 3, sw128 = m & 7;
        uint32_t it = 0;
        for (int t = blockIdx.x; t < n_tiles; t += gridDim.x) {
            const int e = tile_expert(a, t / n_mt, NT);
            if (e < 0 || e >= a.E) continue;
            for (int g = 0; g < a.G; ++g, ++it) {
                const int s = it % C::kStages;
                const int as = it % C::kAStages;
                mbar_wait(&sm.full[s], (it / C::kStages) & 1, bad);
                mbar_wait(&sm.aempty[as], ((it / C::kAStages) & 1) ^ 1, bad);
                const uint8_t* rr = &sm.raw[s][m * 64];
                uint8_t* ar = &sm.a[as][m * 128];
#pragma unroll
                for (int j = 0; j < 4; ++j) {  // 32 codes -> two 16-byte e4m3 chunks
                    const uint4 w = *reinterpret_cast<const uint4*>(rr + ((j ^ sw64) << 4));
                    uint4 o0, o1;
                    o0.x = codes_to_e4m3(w.x);
                    o0.y = codes_to_e4m3(w.x >> 16);
                    o0.z = codes_to_e4m3(w.y);
                    o0.w = codes_to_e4m3(w.y >> 16);
                    o1.x = codes_to_e4m3(w.z);
                    o1.y = codes_to_e4m3(w.z >> 16);
                    o1.z = codes_to_e4m3(w.w);
                    o1.w = codes_to_e4m3(w.w >> 16);
                    *reinterpret_cast<uint4*>(ar + (((2 * j) ^ sw128) << 4)) = o0;
                    *reinterpret_cast<uint4*>(ar + (((2 * j + 1) ^ sw128) << 4)) = o1;
                }
                asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
                __syncwarp();
                if (lane == 0) mbar_arrive(&sm.afull[as]);
            }
        }
    } else if (warp >= 8) {
        // ---------------- fold + epilogue ----------------
        constexpr int kCols = C::kCols;
        const int q = warp & 3;                     // TMEM lane quadrant
        const int c0 = ((warp - 8) >> 2) * kCols;   // column half
        const int m = q * 32 + lane;                // tile row = TMEM lane
        const bool up_row = a.silu && m >= 64;
        uint32_t it = 0;
        for (int t = blockIdx.x; t < n_tiles; t += gridDim.x) {
            const int rb = t / n_mt, mt = t % n_mt;
            const int e = tile_expert(a, rb, NT);
            const int r0 = rb * NT;
            int n;
            if (a.silu) n = up_row ? a.N / 2 + mt * 64 + (m - 64) : mt * 64 + m;
            else n = mt * 128 + m;
            const int n_store = a.silu ? mt * 64 + (m & 63) : n;
            if (e < 0 || e >= a.E) {  // non-local expert: zeros
                if (!up_row && n_store < n_out)
#pragma unroll 4
                    for (int c = 0; c < kCols; ++c)
                        if (r0 + c0 + c < P_valid)
                            a.out16[(int64_t)(r0 + c0 + c) * n_out + n_store] = __float2half_rn(0.f);
                continue;
            }
            const int nn = n < a.N ? n : 0;
            const __half* srow = a.scales + ((int64_t)e * a.N + nn) * a.G;
            const int32_t* zrow =
                a.zeros ? a.zeros + ((int64_t)e * (a.N / 8) + (nn >> 3)) * a.G : nullptr;
            const int zsh = (nn & 7) * 4;
            // activation scales of the tile's columns: lane l holds columns c0 + l (+ 32)
            float asc_l[kCols / 32];
#pragma unroll
            for (int i = 0; i < kCols / 32; ++i) asc_l[i] = __ldg(a.asc_s + r0 + c0 + i * 32 + lane);
            float tot[kCols];
#pragma unroll
            for (int c = 0; c < kCols; ++c) tot[c] = 0.f;
            float s_cur = __half2float(srow[0]);
            float z_cur = zrow ? (float)((__ldg(zrow) >> zsh) & 0xF) : 8.f;
            for (int g = 0; g < a.G; ++g, ++it) {
                const int ss = it % C::kSStages;
                const int tb = it % C::kAcc;
                float s_nx = 0.f, z_nx = 8.f;
                if (g + 1 < a.G) {
                    s_nx = __half2float(srow[g + 1]);
                    if (zrow) z_nx = (float)((__ldg(zrow + g + 1) >> zsh) & 0xF);
                }
                mbar_wait(&sm.sfull[ss], (it / C::kSStages) & 1, bad);
                mbar_wait(&sm.tfull[tb], (it / C::kAcc) & 1, bad);
                __syncwarp();
                asm volatile("tcgen05.fence::after_thread_sync;" ::);
                const float2 sv = make_float2(s_cur, s_cur);
                const float nz = -s_cur * z_cur;
                const float2 nsz = make_float2(nz, nz);
                const float* S = &sm.ssum[ss][c0];
#pragma unroll
                for (int cc = 0; cc < kCols; cc += 32) {
                    uint32_t v[32];
                    tmem_ld32(tmem + ((uint32_t)(q * 32) << 16) + (uint32_t)(tb * NT + c0 + cc), v);
#pragma unroll
                    for (int j = 0; j < 32; j += 4) {
                        const float4 s4 = *reinterpret_cast<const float4*>(S + cc + j);
                        float2 t0 = make_float2(tot[cc + j], tot[cc + j + 1]);
                        float2 t1 = make_float2(tot[cc + j + 2], tot[cc + j + 3]);
                        t0 = ffma2(nsz, make_float2(s4.x, s4.y), t0);
                        t1 = ffma2(nsz, make_float2(s4.z, s4.w), t1);
                        t0 = ffma2(sv, make_float2(__uint_as_float(v[j]), __uint_as_float(v[j + 1])), t0);
                        t1 = ffma2(sv, make_float2(__uint_as_float(v[j + 2]), __uint_as_float(v[j + 3])), t1);
                        tot[cc + j] = t0.x;
                        tot[cc + j + 1] = t0.y;
                        tot[cc + j + 2] = t1.x;
                        tot[cc + j + 3] = t1.y;
                    }
                }
                asm volatile("tcgen05.fence::before_thread_sync;" ::);
                __syncwarp();
                if (lane == 0) {
                    mbar_arrive(&sm.tempty[tb]);
                    mbar_arrive(&sm.sempty[ss]);
                }
                s_cur = s_nx;
                z_cur = z_nx;
            }
            // ---- epilogue: fp16(tot * a_scale) into the shared tile, then row-contiguous
            // stores by all fold threads (SiLU(gate) * up for the fused gate_up op) ----
#pragma unroll
            for (int c = 0; c < kCols; ++c)
                sm.otile[(c0 + c) * 128 + m] = __float2half_rn(
                    tot[c] * __shfl_sync(0xffffffffu, asc_l[c >> 5], c & 31));
            asm volatile("bar.sync 1, %0;" ::"n"(kFoldWarps * 32));
            const int fw = warp - 8;
            if (a.silu) {
                const int n = mt * 64 + 2 * lane;  // two outputs per lane
#pragma unroll 2
                for (int c = fw; c < NT; c += kFoldWarps) {
                    const int r = r0 + c;
                    if (r >= P_valid) break;
                    const __half2 gh = *reinterpret_cast<const __half2*>(&sm.otile[c * 128 + 2 * lane]);
                    const __half2 uh = *reinterpret_cast<const __half2*>(&sm.otile[c * 128 + 64 + 2 * lane]);
                    __half2 o;
                    o.x = silu_mul_h(__low2half(gh), __low2half(uh));
                    o.y = silu_mul_h(__high2half(gh), __high2half(uh));
                    *reinterpret_cast<__half2*>(a.out16 + (int64_t)r * n_out + n) = o;
                }
            } else {
                const int n = mt * 128 + 4 * lane;  // four outputs per lane
                if (n < n_out)
#pragma unroll 2
                    for (int c = fw; c < NT; c += kFoldWarps) {
                        const int r = r0 + c;
                        if (r >= P_valid) break;
                        *reinterpret_cast<uint2*>(a.out16 + (int64_t)r * n_out + n) =
                            *reinterpret_cast<const uint2*>(&sm.otile[c * 128 + 4 * lane]);
                    }
            }
            asm volatile("bar.sync 1, %0;" ::"n"(kFoldWarps * 32));
        }
    }

    asm volatile("tcgen05.fence::before_thread_sync;" ::);
    __syncthreads();
    if (tid == 0 && sm.bad && a.err) atomicOr(a.err, 1);
    if (warp == 2) {
        asm volatile("tcgen05.fence::after_thread_sync;" ::);
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem),
                     "r"(C::kTmemCols));
    }
}

// One warp per sorted row: dense sorted-order operand rows for the tile kernel. Rows past the
// last valid one (up to the tile-rounded count) and rows with a sentinel id are zero-filled.
__global__ void __launch_bounds__(256) tc_gather_kernel(const TcArgs a, int NT) {
    const int lane = threadIdx.x & 31;
    const int64_t r = (int64_t)blockIdx.x * 8 + (threadIdx.x >> 5);
    const int P_valid = a.ntp ? min(a.ntp[0], a.P) : a.P;
    const int64_t rows = (int64_t)(P_valid + NT - 1) / NT * NT;
    if (r >= rows) return;
    int src = -1;
    if (r < P_valid) {
        const int e = a.expert_ids ? a.expert_ids[r / a.block_m] : 0;
        const int sid = a.sorted_ids ? a.sorted_ids[r] : (int)r;
        if (e >= 0 && e < a.E && sid >= 0 && sid < a.num_valid)
            src = a.src_identity ? (int)r : sid / a.top_k;
    }
    uint4* dst = reinterpret_cast<uint4*>(a.xs + r * a.K);
    const int64_t nv = a.K / 16;
    if (src >= 0) {
        const uint4* sp = reinterpret_cast<const uint4*>(a.xq + (int64_t)src * a.K);
        for (int64_t i = lane; i < nv; i += 32) dst[i] = __ldg(sp + i);
        for (int g = lane; g < a.G; g += 32)
            a.ssum[(int64_t)g * a.P_pad + r] = a.xsum[(int64_t)src * a.G + g].y;
        if (lane == 0) a.asc_s[r] = a.act_scales[src];
    } else {
        for (int64_t i = lane; i < nv; i += 32) dst[i] = make_uint4(0, 0, 0, 0);
        for (int g = lane; g < a.G; g += 32) a.ssum[(int64_t)g * a.P_pad + r] = 0.f;
        if (lane == 0) a.asc_s[r] = 0.f;
    }
}

// ---- tensor maps ----
PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
    static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
    static std::once_flag once;
    std::call_once(once, [] {
        void* p = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) ==
                cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
    });
    return fn;
}

// 2D u8 map over rows x row_bytes (row stride row_bytes), box box_bytes x box_rows.
bool make_map(CUtensorMap* map, const void* base, uint64_t rows, uint64_t row_bytes,
              uint32_t box_bytes, uint32_t box_rows, CUtensorMapSwizzle sw) {
    auto fn = encode_fn();
    if (!fn) return false;
    const cuuint64_t dims[2] = {row_bytes, rows};
    const cuuint64_t strides[1] = {row_bytes};
    const cuuint32_t box[2] = {box_bytes, box_rows};
    const cuuint32_t estr[2] = {1, 1};
    return fn(map, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<void*>(base), dims, strides, box,
              estr, CU_TENSOR_MAP_INTERLEAVE_NONE, sw, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
              CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

int sm_count() {
    int dev = 0, n = 0;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
    return n > 0 ? n : 148;
}

template <int NT>
int launch_tc_t(const TcArgs& a, cudaStream_t stream) {
    const int64_t rows_max = (int64_t)(a.P + NT - 1) / NT * NT;
    tc_gather_kernel<<<(unsigned)((rows_max + 7) / 8), 256, 0, stream>>>(a, NT);
    if (int rc = launch_status()) return rc;
    CUtensorMap tmw, tmx;
    if (!make_map(&tmw, a.w, (uint64_t)a.E * a.N, (uint64_t)a.K / 2, 64, a.silu ? 64 : 128,
                  CU_TENSOR_MAP_SWIZZLE_64B) ||
        !make_map(&tmx, a.xs, (uint64_t)a.P_pad, (uint64_t)a.K, 128, NT,
                  CU_TENSOR_MAP_SWIZZLE_128B))
        return set_error("tile path: tensor map encoding failed");
    const size_t smem = sizeof(TcSmem<NT>) + 1024;
    auto kern = w4_tc_kernel<NT>;
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         (int)smem);
    if (e != cudaSuccess) return (int)e;
    const int n_mt = a.silu ? (a.N / 2) / 64 : (a.N + 127) / 128;
    const int64_t tiles_max = rows_max / NT * n_mt;
    const int grid = (int)std::min<int64_t>(tiles_max, sm_count());
    if (grid <= 0) return W4A8_OK;
    kern<<<grid, kTcThreads, smem, stream>>>(a, tmw, tmx);
    return launch_status();
}

}  // namespace

bool tc_path_ok(int64_t K, int group_size, int e2m1, const void* w, int block_m) {
    return !e2m1 && group_size == 128 && K % 128 == 0 && K >= 128 &&
           (reinterpret_cast<uintptr_t>(w) & 15) == 0 && block_m % 64 == 0;
}

size_t tc_scratch_bytes(int64_t P, int64_t K) {
    const int64_t P_pad = (P + 127) / 128 * 128;
    const int64_t G = std::max<int64_t>(K / 128, 1);
    return align_up((size_t)(P_pad * K), 256) + align_up((size_t)P_pad * 4, 256) +
           align_up((size_t)(G * P_pad) * 4, 256);
}

void tc_carve(void* base, int64_t P, int64_t K, TcArgs& t) {
    const int64_t P_pad = (P + 127) / 128 * 128;
    uint8_t* p = static_cast<uint8_t*>(base);
    t.xs = p;
    p += align_up((size_t)(P_pad * K), 256);
    t.asc_s = reinterpret_cast<float*>(p);
    p += align_up((size_t)P_pad * 4, 256);
    t.ssum = reinterpret_cast<float*>(p);
    t.P_pad = (int)P_pad;
}

int launch_w4_tc(TcArgs a, cudaStream_t stream) {
    if (a.P <= 0) return W4A8_OK;
    if (a.silu && (a.N / 2) % 64 != 0) return set_error("tile path: inter must be a multiple of 64");
    if (a.block_m % 128 == 0) return launch_tc_t<128>(a, stream);
    return launch_tc_t<64>(a, stream);
}

}  // namespace w4a8
