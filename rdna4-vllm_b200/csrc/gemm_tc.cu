// gemm_tc.cu — W4A8 (grouped) GEMM tile path on the 5th-generation tensor cores (tcgen05).
//
// Tile = 128 weight rows x NT activation rows (NT = 64 or 128, never straddling an expert
// block of the padded-sorted layout). The MMA runs "swap-AB": A = the 128 dequantised weight
// rows (TMEM lanes), B = the NT gathered e4m3 activation rows (TMEM columns), both K-major in
// the no-swizzle core-matrix layout, one tcgen05.mma.cta_group::1.kind::f8f6f4 per 32-wide K
// slice, fp32 accumulators in tensor memory.
//
// Numerics. The weight operand holds e4m3(q) — the unsigned 4-bit code itself, exact in e4m3 —
// so per 128-wide group g the tensor core returns acc = sum_k q_k a_k. With S_g = sum_k a_k
// (from the operand quantiser) the reference's group result sum_k (q_k - z) a_k equals
// acc - z*S_g exactly in real arithmetic, and it is folded in fp32 as
//     tot += scale[n,g] * acc - (scale[n,g] * z) * S_g
// then multiplied by the row's activation scale: the reference oracle's association
// (w4a8_fp8_wmma/test_correctness.py:113-119) up to fp32 rounding.
//
// Pipeline per K group g (all 256 threads, one CTA per tile):
//   1. cp.async ring (3 stages) already holds group g's packed codes, token tile and sums;
//   2. threads expand the codes to e4m3 bytes in shared memory (3 prmt + 1 lop3 per 4 codes);
//   3. one thread issues the 4 MMAs of group g into TMEM buffer g%2 and commits them to an
//      mbarrier; meanwhile every thread folds group g-1 from the other TMEM buffer
//      (tcgen05.ld) and issues the cp.async of group g+2.
// Every mbarrier wait is bounded; on timeout the kernel records an error code and finishes
// without further waits, always releasing its tensor memory.
#include <algorithm>

#include "common.cuh"
#include "gemm_common.h"
#include "internal.h"

namespace w4a8 {

namespace {

constexpr int kTcThreads = 256;
constexpr int kStages = 3;          // cp.async ring depth
constexpr int kRawStride = 64;      // bytes per weight row in the raw-code ring

// 16-byte chunk j of raw row m is stored at chunk j ^ ((m >> 1) & 3): the expansion step reads
// 8 consecutive rows per quarter-warp without bank conflicts.
__device__ __forceinline__ int raw_off(int m, int j) { return m * 64 + ((j ^ ((m >> 1) & 3)) << 4); }
constexpr uint32_t kSpinLimit = 1u << 24;

template <int NT>
struct TcSmem {
    uint8_t a[2][128 * 128];                 // e4m3 weights, core-matrix layout
    uint8_t b[kStages][NT * 128];            // e4m3 activations, core-matrix layout
    uint8_t raw[kStages][128 * kRawStride];  // packed int4 codes of the tile's 128 rows
    float ssum[kStages + 1][NT];             // per-group activation sums S
    float asc[NT];
    int src[NT];
    uint64_t mbar[2];
    uint32_t tmem_base;
    int any;
    int bad;                                 // a bounded wait gave up
};

// Byte offset of (row r, 16-byte K chunk j) in a 128-byte-wide K-major core-matrix tile:
// core matrices are 8 rows x 16 bytes contiguous; K-adjacent ones are 128 B apart (LBO),
// 8-row groups are 1024 B apart (SBO).
__device__ __forceinline__ int cm_off(int r, int j) {
    return ((r >> 3) * 8 + j) * 128 + (r & 7) * 16;
}

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
    return (uint32_t)__cvta_generic_to_shared(p);
}

__device__ __forceinline__ uint64_t umma_desc(uint32_t saddr) {
    uint64_t d = (uint64_t)((saddr >> 4) & 0x3FFFu);
    d |= (uint64_t)((128u >> 4) & 0x3FFFu) << 16;   // leading byte offset (K direction)
    d |= (uint64_t)((1024u >> 4) & 0x3FFFu) << 32;  // stride byte offset (8-row groups)
    d |= (uint64_t)1 << 46;                         // descriptor version for sm_100
    return d;                                       // base offset 0, SWIZZLE_NONE
}

// kind::f8f6f4 instruction descriptor: fp32 accumulate, A = B = e4m3, both K-major.
__host__ __device__ constexpr uint32_t umma_idesc(int M, int N) {
    return (1u << 4) | ((uint32_t)(N >> 3) << 17) | ((uint32_t)(M >> 4) << 24);
}

__device__ __forceinline__ void cp_async16(void* smem, const void* gmem, bool pred) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(smem_u32(smem)),
                 "l"(gmem), "r"(pred ? 16 : 0));
}
__device__ __forceinline__ void cp_async4(void* smem, const void* gmem, bool pred) {
    asm volatile("cp.async.ca.shared.global [%0], [%1], 4, %2;" ::"r"(smem_u32(smem)),
                 "l"(gmem), "r"(pred ? 4 : 0));
}

__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity) {
    const uint32_t addr = smem_u32(bar);
    for (uint32_t i = 0; i < kSpinLimit; ++i) {
        uint32_t done;
        asm volatile(
            "{\n\t.reg .pred p;\n\t"
            "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
            "selp.u32 %0, 1, 0, p;\n\t}"
            : "=r"(done)
            : "r"(addr), "r"(parity)
            : "memory");
        if (done) return true;
    }
    return false;
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

template <int NT>
__device__ __forceinline__ void issue_stage(const TcArgs& a, TcSmem<NT>& sm, int e, int mt, int g,
                                            int st, int ss, int r0) {
    const int tid = threadIdx.x;
    if (g < a.G) {
        // token tile: NT rows x 8 chunks of 16 bytes
        for (int i = tid; i < NT * 8; i += kTcThreads) {
            const int r = i >> 3, j = i & 7;
            const int src = sm.src[r];
            const uint8_t* gp = a.xq + (int64_t)max(src, 0) * a.K + (int64_t)g * 128 + j * 16;
            cp_async16(&sm.b[st][cm_off(r, j)], gp, src >= 0);
        }
        // packed codes: 128 rows x 4 chunks of 16 bytes
        const int64_t kw = a.K / 8;
        for (int i = tid; i < 128 * 4; i += kTcThreads) {
            const int m = i >> 2, j = i & 3;
            int n;
            if (a.silu) n = (m < 64) ? mt * 64 + m : a.N / 2 + mt * 64 + (m - 64);
            else n = mt * 128 + m;
            const bool ok = n < a.N;
            const int32_t* gp = a.w + ((int64_t)e * a.N + (ok ? n : 0)) * kw + g * 16 + j * 4;
            cp_async16(&sm.raw[st][raw_off(m, j)], gp, ok);
        }
        // activation sums S of the group
        for (int i = tid; i < NT; i += kTcThreads) {
            const int src = sm.src[i];
            const float* gp = reinterpret_cast<const float*>(a.xsum + (int64_t)max(src, 0) * a.G + g) + 1;
            cp_async4(&sm.ssum[ss][i], gp, src >= 0);
        }
    }
    asm volatile("cp.async.commit_group;" ::);
}

template <int NT>
__global__ void __launch_bounds__(kTcThreads, 2) w4_tc_kernel(const TcArgs a) {
    extern __shared__ __align__(1024) uint8_t smem_raw[];
    TcSmem<NT>& sm = *reinterpret_cast<TcSmem<NT>*>(smem_raw);
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int mt = blockIdx.x;
    const int r0 = blockIdx.y * NT;
    const int n_out = a.silu ? a.N / 2 : a.N;
    const int P_valid = a.ntp ? min(a.ntp[0], a.P) : a.P;
    if (r0 >= P_valid) return;  // rows past num_tokens_post_padded are unspecified
    const int e = a.expert_ids ? a.expert_ids[r0 / a.block_m] : 0;
    if (tid == 0) {
        sm.any = 0;
        sm.bad = 0;
    }
    __syncthreads();
    for (int i = tid; i < NT; i += kTcThreads) {
        const int r = r0 + i;
        int src = -1;
        float asc = 0.f;
        if (r < P_valid && e >= 0 && e < a.E) {
            const int sid = a.sorted_ids ? a.sorted_ids[r] : r;
            if (sid >= 0 && sid < a.num_valid) {
                src = a.src_identity ? r : sid / a.top_k;
                asc = a.act_scales[src];
                sm.any = 1;
            }
        }
        sm.src[i] = src;
        sm.asc[i] = asc;
    }
    __syncthreads();
    // output rows handled by this thread in the epilogue
    const int lg = warp & 3;        // TMEM lane group: lanes 32*lg .. 32*lg+31
    const int half = warp >> 2;     // column half
    const int m = lg * 32 + lane;   // tile row = TMEM lane
    int n;                          // weight row of m
    bool up_row = false;
    if (a.silu) {
        up_row = m >= 64;
        n = up_row ? a.N / 2 + mt * 64 + (m - 64) : mt * 64 + m;
    } else {
        n = mt * 128 + m;
    }
    const int n_store = a.silu ? mt * 64 + (m & 63) : n;
    constexpr int kCols = NT / 2;
    const int c0 = half * kCols;
    if (!sm.any) {  // all-padding tile or non-local expert: zeros
        if (!(a.silu && up_row) && n_store < n_out)
#pragma unroll 1
            for (int c = 0; c < kCols; ++c)
                if (r0 + c0 + c < P_valid)
                    a.out16[(int64_t)(r0 + c0 + c) * n_out + n_store] = __float2half_rn(0.f);
        return;
    }

    // ---- tensor memory + barriers ----
    constexpr uint32_t kTmemCols = 2 * NT;
    if (warp == 0) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                         smem_u32(&sm.tmem_base)),
                     "r"(kTmemCols));
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::);
    }
    if (tid == 0) {
        asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;" ::"r"(smem_u32(&sm.mbar[0])));
        asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;" ::"r"(smem_u32(&sm.mbar[1])));
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    asm volatile("tcgen05.fence::before_thread_sync;" ::);
    __syncthreads();
    asm volatile("tcgen05.fence::after_thread_sync;" ::);
    const uint32_t tmem = sm.tmem_base;

    const bool row_ok = n < a.N;
    const int64_t sc_base = ((int64_t)e * a.N + (row_ok ? n : 0)) * a.G;
    const int32_t* zrow = a.zeros ? a.zeros + ((int64_t)e * (a.N / 8) + ((row_ok ? n : 0) >> 3)) * a.G
                                  : nullptr;
    const int zsh = ((row_ok ? n : 0) & 7) * 4;
    float tot[kCols];
#pragma unroll
    for (int c = 0; c < kCols; ++c) tot[c] = 0.f;

    for (int s = 0; s < kStages - 1; ++s) issue_stage<NT>(a, sm, e, mt, s, s, s, r0);
    // scale/zero of group g-1 (folded in iteration g) and of group g (loaded one ahead)
    float s_fold = 0.f, z_fold = 8.f;
    float s_next = __half2float(a.scales[sc_base]);
    float z_next = zrow ? (float)((__ldg(zrow) >> zsh) & 0xF) : 8.f;
    const uint32_t idesc = umma_idesc(128, NT);
    bool bad = false;

    auto fold = [&](int gf, float sv, float zv) {
        // wait for the MMAs of group gf, then fold its TMEM buffer
        if (!bad && !mbar_wait(&sm.mbar[gf & 1], (uint32_t)((gf >> 1) & 1))) {
            bad = true;
            atomicOr(&sm.bad, 1);
        }
        asm volatile("tcgen05.fence::after_thread_sync;" ::);
        const float sz = sv * zv;
        const float* S = sm.ssum[gf % (kStages + 1)] + c0;
#pragma unroll
        for (int cc = 0; cc < kCols; cc += 32) {
            uint32_t v[32];
            const uint32_t taddr =
                tmem + ((uint32_t)(lg * 32) << 16) + (uint32_t)((gf & 1) * NT + c0 + cc);
            asm volatile(
                "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,"
                "%12,%13,%14,%15,%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31},"
                " [%32];"
                : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]),
                  "=r"(v[6]), "=r"(v[7]), "=r"(v[8]), "=r"(v[9]), "=r"(v[10]), "=r"(v[11]),
                  "=r"(v[12]), "=r"(v[13]), "=r"(v[14]), "=r"(v[15]), "=r"(v[16]), "=r"(v[17]),
                  "=r"(v[18]), "=r"(v[19]), "=r"(v[20]), "=r"(v[21]), "=r"(v[22]), "=r"(v[23]),
                  "=r"(v[24]), "=r"(v[25]), "=r"(v[26]), "=r"(v[27]), "=r"(v[28]), "=r"(v[29]),
                  "=r"(v[30]), "=r"(v[31])
                : "r"(taddr));
            asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
            for (int j = 0; j < 32; j += 4) {
                const float4 s4 = *reinterpret_cast<const float4*>(S + cc + j);
                tot[cc + j + 0] = fmaf(sv, __uint_as_float(v[j + 0]), fmaf(-sz, s4.x, tot[cc + j + 0]));
                tot[cc + j + 1] = fmaf(sv, __uint_as_float(v[j + 1]), fmaf(-sz, s4.y, tot[cc + j + 1]));
                tot[cc + j + 2] = fmaf(sv, __uint_as_float(v[j + 2]), fmaf(-sz, s4.z, tot[cc + j + 2]));
                tot[cc + j + 3] = fmaf(sv, __uint_as_float(v[j + 3]), fmaf(-sz, s4.w, tot[cc + j + 3]));
            }
        }
        asm volatile("tcgen05.fence::before_thread_sync;" ::);
    };

    for (int g = 0; g < a.G; ++g) {
        const int st = g % kStages;
        asm volatile("cp.async.wait_group %0;" ::"n"(kStages - 2));
        __syncthreads();  // group g's codes, tokens and sums have landed for everyone
        {
            // expand codes -> e4m3 bytes: thread handles row mm, 32 codes (half hh of the group)
            const int mm = tid & 127, hh = tid >> 7;
            const uint4 rw0 = *reinterpret_cast<const uint4*>(&sm.raw[st][raw_off(mm, 2 * hh)]);
            const uint4 rw1 = *reinterpret_cast<const uint4*>(&sm.raw[st][raw_off(mm, 2 * hh + 1)]);
            const uint32_t wv[8] = {rw0.x, rw0.y, rw0.z, rw0.w, rw1.x, rw1.y, rw1.z, rw1.w};
#pragma unroll
            for (int q = 0; q < 4; ++q) {  // 16 codes -> one 16-byte chunk
                uint4 o;
                o.x = codes_to_e4m3(wv[2 * q]);
                o.y = codes_to_e4m3(wv[2 * q] >> 16);
                o.z = codes_to_e4m3(wv[2 * q + 1]);
                o.w = codes_to_e4m3(wv[2 * q + 1] >> 16);
                *reinterpret_cast<uint4*>(&sm.a[g & 1][cm_off(mm, hh * 4 + q)]) = o;
            }
        }
        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
        __syncthreads();
        if (tid == 0) {
            asm volatile("tcgen05.fence::after_thread_sync;" ::);
            const uint32_t a0 = smem_u32(&sm.a[g & 1][0]);
            const uint32_t b0 = smem_u32(&sm.b[st][0]);
            const uint32_t d = tmem + (uint32_t)((g & 1) * NT);
#pragma unroll
            for (int kk = 0; kk < 4; ++kk) {
                const uint64_t da = umma_desc(a0 + kk * 256);
                const uint64_t db = umma_desc(b0 + kk * 256);
                const uint32_t acc = kk > 0 ? 1u : 0u;
                asm volatile(
                    "{\n\t.reg .pred p;\n\t"
                    "setp.ne.b32 p, %4, 0;\n\t"
                    "tcgen05.mma.cta_group::1.kind::f8f6f4 [%0], %1, %2, %3, p;\n\t}" ::"r"(d),
                    "l"(da), "l"(db), "r"(idesc), "r"(acc));
            }
            asm volatile(
                "tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
                    smem_u32(&sm.mbar[g & 1])));
        }
        if (g > 0) fold(g - 1, s_fold, z_fold);  // overlaps the MMAs of group g
        s_fold = s_next;
        z_fold = z_next;
        if (g + 1 < a.G) {
            s_next = __half2float(a.scales[sc_base + g + 1]);
            if (zrow) z_next = (float)((__ldg(zrow + g + 1) >> zsh) & 0xF);
        }
        issue_stage<NT>(a, sm, e, mt, g + kStages - 1, (g + kStages - 1) % kStages,
                        (g + kStages - 1) % (kStages + 1), r0);
    }
    fold(a.G - 1, s_fold, z_fold);
    asm volatile("cp.async.wait_all;" ::);
    __syncthreads();

    // ---- epilogue: out[row][n] = fp16(tot * a_scale) (or SiLU of the gate/up pair) ----
    if (a.silu) {
        __half* up = reinterpret_cast<__half*>(&sm.a[0][0]);  // 64 x NT halves
        if (up_row)
#pragma unroll
            for (int c = 0; c < kCols; ++c)
                up[(m - 64) * NT + c0 + c] = __float2half_rn(tot[c] * sm.asc[c0 + c]);
        __syncthreads();
        if (!up_row && n_store < n_out)
#pragma unroll
            for (int c = 0; c < kCols; ++c) {
                const int r = r0 + c0 + c;
                if (r >= P_valid) continue;
                __half v = __float2half_rn(0.f);
                if (sm.src[c0 + c] >= 0)
                    v = silu_and_mul_half(tot[c] * sm.asc[c0 + c],
                                          __half2float(up[m * NT + c0 + c]));
                a.out16[(int64_t)r * n_out + n_store] = v;
            }
    } else if (n_store < n_out) {
#pragma unroll
        for (int c = 0; c < kCols; ++c) {
            const int r = r0 + c0 + c;
            if (r >= P_valid) break;
            const float v = sm.src[c0 + c] >= 0 ? tot[c] * sm.asc[c0 + c] : 0.f;
            a.out16[(int64_t)r * n_out + n_store] = __float2half_rn(v);
        }
    }
    if (tid == 0 && sm.bad && a.err) atomicOr(a.err, 1);
    asm volatile("tcgen05.fence::before_thread_sync;" ::);
    __syncthreads();
    if (warp == 0) {
        asm volatile("tcgen05.fence::after_thread_sync;" ::);
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem),
                     "r"(kTmemCols));
    }
}

template <int NT>
int launch_tc_t(const TcArgs& a, cudaStream_t stream) {
    const size_t smem = sizeof(TcSmem<NT>) + 128;
    auto kern = w4_tc_kernel<NT>;
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         (int)smem);
    if (e != cudaSuccess) return (int)e;
    const int n_tiles = a.silu ? (a.N / 2) / 64 : (a.N + 127) / 128;
    const dim3 grid((unsigned)n_tiles, (unsigned)((a.P + NT - 1) / NT));
    kern<<<grid, kTcThreads, smem, stream>>>(a);
    return launch_status();
}

}  // namespace

bool tc_path_ok(int64_t K, int group_size, int e2m1, const void* w, int block_m) {
    return !e2m1 && group_size == 128 && K % 128 == 0 && K >= 128 &&
           (reinterpret_cast<uintptr_t>(w) & 15) == 0 && block_m % 64 == 0;
}

int launch_w4_tc(TcArgs a, cudaStream_t stream) {
    if (a.P <= 0) return W4A8_OK;
    if (a.silu && (a.N / 2) % 64 != 0) return set_error("tile path: inter must be a multiple of 64");
    if (a.block_m % 128 == 0) return launch_tc_t<128>(a, stream);
    return launch_tc_t<64>(a, stream);
}

}  // namespace w4a8
