// gemm_mma.cu — W4A8 GEMM / grouped-MoE GEMM with the weights dequantised straight into
// tensor-core operand registers (no shared-memory staging of the weights).
//
// One CTA owns 64 output channels (4 warps x 16) x 8*NT activation rows of one expert, and
// optionally WK warps splitting K. Per 128-wide K group (g = 128), each lane streams 16 bytes
// (32 codes) of two channel rows with a 128-bit non-allocating load, expands them to exact fp16
// (q - z) with the 0x6400 magic-number trick, and issues 8 mma.sync.m16n8k16 (fp16 x fp16 ->
// fp32) per 8-row activation tile. The activations are e4m3 bytes converted to fp16 (exact) in a
// shared-memory tile. The group's fp32 accumulator is folded with the group scale into a running
// fp32 total, the same association the reference oracle uses
// (w4a8_fp8_wmma/test_correctness.py:113-119): out = (sum_g partial_g * scale_g) * a_scale.
//
// The K permutation. A lane of quad position c holds K codes [32c, 32c+32) of its 128-wide
// block. Word i (codes 8i..8i+7) expands to half2 pairs (0,4),(1,5),(2,6),(3,7); MMA 2i takes
// pairs (0,4) and (1,5) as its k = {2c,2c+1} and {2c+8,2c+9} slots, MMA 2i+1 takes (2,6),(3,7).
// A dot product is invariant under a permutation of k applied to both operands, so the
// activation tile is stored with the same pairing inside every 8-code unit.
//
// Group sizes other than 128, mxfp4 (E2M1) codes and the scalar golden id go to
// w4_scalar_kernel, one thread per (row, channel) (the reference's v0 scheme,
// moe_kernel.hip:134-204).
#include <algorithm>

#include "common.cuh"
#include "gemm_common.h"
#include "internal.h"

namespace w4a8 {

namespace {

constexpr int kNW = 4;                        // warps along N per CTA (16 channels each)
constexpr int kActSmemBudget = 64 * 1024;     // activation tile bytes per CTA

struct RowInfo {
    int32_t src;    // activation row in x_fp8 (-1 = invalid / padding)
    int32_t sid;    // sorted token id (slot) for scatter
    float ascale;   // activation scale of src
};

__device__ __forceinline__ void load_rows(const GemmArgs& a, int r0, int nrows, RowInfo* info,
                                          int* any_valid) {
    const int P_valid = a.ntp ? min(a.ntp[0], a.P) : a.P;
    for (int i = threadIdx.x; i < nrows; i += blockDim.x) {
        const int r = r0 + i;
        RowInfo ri{-1, 0, 0.f};
        if (r < P_valid) {
            const int sid = a.sorted_ids ? a.sorted_ids[r] : r;
            if (sid >= 0 && sid < a.num_valid) {
                ri.src = a.src_identity ? r : sid / a.top_k;
                ri.sid = sid;
                ri.ascale = a.act_scales[ri.src];
                *any_valid = 1;
            }
        }
        info[i] = ri;
    }
}

// Shared-memory byte offset of the 16-byte unit `u` (0..3) of chunk `c` (0..3) of k-block `kb`
// inside one activation row. The XOR keeps the quarter-warp LDS.128 phases bank-conflict free
// together with a row stride of 32 (mod 128) bytes.
__device__ __forceinline__ int act_unit_offset(int kb, int c, int u) {
    return kb * 256 + c * 64 + ((u ^ ((c >> 1) & 1)) << 4);
}

// Expand one 32-bit word of 8 codes to 4 half2 (pairs (0,4),(1,5),(2,6),(3,7)) of (q - z).
__device__ __forceinline__ void dequant_word(uint32_t w, uint32_t z1024, uint32_t z64,
                                             uint32_t (&h)[4]) {
    constexpr uint32_t kMagic = 0x64006400u;  // fp16 1024.0 in both halves
    constexpr uint32_t kSixteenth = 0x2C002C00u;  // fp16 1/16 in both halves
    const uint32_t w8 = w >> 8;
    h[0] = hsub2_u(and_or(w, 0x000F000Fu, kMagic), z1024);
    h[1] = hfma2_u(and_or(w, 0x00F000F0u, kMagic), kSixteenth, z64);
    h[2] = hsub2_u(and_or(w8, 0x000F000Fu, kMagic), z1024);
    h[3] = hfma2_u(and_or(w8, 0x00F000F0u, kMagic), kSixteenth, z64);
}

// Per-(channel, group) constants: half2(1024+z) for the subtract, half2(-(64+z)) for the fma.
__device__ __forceinline__ void zero_consts(int z, uint32_t& z1024, uint32_t& z64) {
    const __half a = __int2half_rn(1024 + z);
    const __half b = __int2half_rn(-(64 + z));
    z1024 = (uint32_t)__half_as_ushort(a) * 0x10001u;
    z64 = (uint32_t)__half_as_ushort(b) * 0x10001u;
}

struct WeightSlice {
    uint4 w0, w1;      // rows r and r+8: 32 codes each
    int z0, z1;        // zero points
    float s0, s1;      // group scales
};

__device__ __forceinline__ void load_slice(const GemmArgs& a, const int32_t* wq_e,
                                           const __half* sc_e, const int32_t* zr_e, int row0,
                                           int row1, int kb, int c, WeightSlice& ws) {
    const int64_t kw = a.K / 8;  // int32 words per channel row
    ws.w0 = ldg_stream(wq_e + (int64_t)row0 * kw + kb * 16 + c * 4);
    ws.w1 = ldg_stream(wq_e + (int64_t)row1 * kw + kb * 16 + c * 4);
    ws.s0 = __half2float(sc_e[(int64_t)row0 * a.G + kb]);
    ws.s1 = __half2float(sc_e[(int64_t)row1 * a.G + kb]);
    if (zr_e) {
        ws.z0 = (__ldg(zr_e + (int64_t)(row0 >> 3) * a.G + kb) >> ((row0 & 7) * 4)) & 0xF;
        ws.z1 = (__ldg(zr_e + (int64_t)(row1 >> 3) * a.G + kb) >> ((row1 & 7) * 4)) & 0xF;
    } else {
        ws.z0 = ws.z1 = 8;
    }
}

// One 128-wide K block: dequantise and run 8 MMAs per activation tile, fold with the scales.
template <int NT>
__device__ __forceinline__ void compute_block(const WeightSlice& ws, const uint8_t* act_tile,
                                              int row_stride, int kbl, int lane,
                                              float (&tot)[NT][4]) {
    uint32_t za0, zb0, za1, zb1;
    zero_consts(ws.z0, za0, zb0);
    zero_consts(ws.z1, za1, zb1);
    const uint32_t w0[4] = {ws.w0.x, ws.w0.y, ws.w0.z, ws.w0.w};
    const uint32_t w1[4] = {ws.w1.x, ws.w1.y, ws.w1.z, ws.w1.w};
    uint32_t h0[4][4], h1[4][4];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        dequant_word(w0[i], za0, zb0, h0[i]);
        dequant_word(w1[i], za1, zb1, h1[i]);
    }
    const int c = lane & 3;
    const int tok = lane >> 2;
#pragma unroll
    for (int t = 0; t < NT; ++t) {
        const uint8_t* rowp = act_tile + (t * 8 + tok) * row_stride;
        float acc[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            const uint4 b = *reinterpret_cast<const uint4*>(rowp + act_unit_offset(kbl, c, i));
            const uint32_t a0[4] = {h0[i][0], h1[i][0], h0[i][1], h1[i][1]};
            mma_16816(acc, a0, b.x, b.y);
            const uint32_t a1[4] = {h0[i][2], h1[i][2], h0[i][3], h1[i][3]};
            mma_16816(acc, a1, b.z, b.w);
        }
        tot[t][0] = fmaf(acc[0], ws.s0, tot[t][0]);
        tot[t][1] = fmaf(acc[1], ws.s0, tot[t][1]);
        tot[t][2] = fmaf(acc[2], ws.s1, tot[t][2]);
        tot[t][3] = fmaf(acc[3], ws.s1, tot[t][3]);
    }
}

// Fill the activation tile for k range [k0, k0+kc) of the CTA's rows (e4m3 -> fp16, permuted).
template <int NT>
__device__ __forceinline__ void fill_act_tile(const GemmArgs& a, const RowInfo* info,
                                              uint8_t* act_tile, int row_stride, int k0,
                                              int kc) {
    const int units = kc / 16;  // 16 e4m3 bytes per unit
    const int total = NT * 8 * units;
    for (int idx = threadIdx.x; idx < total; idx += blockDim.x) {
        const int rr = idx / units;
        const int uu = idx - rr * units;
        const int src = info[rr].src;
        uint4 v = make_uint4(0, 0, 0, 0);
        if (src >= 0) v = __ldg(reinterpret_cast<const uint4*>(a.x_fp8 + (int64_t)src * a.K + k0) + uu);
        const uint32_t wds[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
        for (int half = 0; half < 2; ++half) {
            const uint32_t lo = wds[half * 2], hi = wds[half * 2 + 1];
            const uint32_t p0 = prmt(lo, hi, 0x5140u);  // bytes b0 b4 b1 b5
            const uint32_t p1 = prmt(lo, hi, 0x7362u);  // bytes b2 b6 b3 b7
            uint4 o;
            o.x = e4m3x2_to_f16x2((uint16_t)(p0 & 0xffff));
            o.y = e4m3x2_to_f16x2((uint16_t)(p0 >> 16));
            o.z = e4m3x2_to_f16x2((uint16_t)(p1 & 0xffff));
            o.w = e4m3x2_to_f16x2((uint16_t)(p1 >> 16));
            const int q = uu * 2 + half;  // 8-code unit index inside the chunk
            const int off = act_unit_offset(q >> 4, (q >> 2) & 3, q & 3);
            *reinterpret_cast<uint4*>(act_tile + rr * row_stride + off) = o;
        }
    }
}

template <int NT, int WK, int EPI>
__global__ void __launch_bounds__(kNW * WK * 32)
w4_mma_kernel(const GemmArgs a) {
    extern __shared__ __align__(16) uint8_t smem[];
    constexpr int R = NT * 8;
    constexpr bool kSilu = (EPI == kEpiSilu);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int wn = warp % kNW, wk = warp / kNW;
    const int r0 = blockIdx.y * R;
    const int n_out = kSilu ? a.N / 2 : a.N;   // output channels
    const int nb = blockIdx.x * (kNW * 16) + wn * 16;

    // Shared-memory carve-up.
    const int kc = a.kc;
    const int row_stride = kc * 2 + 32;
    uint8_t* act_tile = smem;
    RowInfo* info = reinterpret_cast<RowInfo*>(smem + a.info_off);
    __shared__ int any_valid;
    __shared__ int expert_sh;
    if (threadIdx.x == 0) {
        any_valid = 0;
        int e = 0;
        if (a.expert_ids) e = a.expert_ids[r0 / a.block_m];
        expert_sh = e;
    }
    __syncthreads();
    const int e = expert_sh;
    if (e >= 0 && e < a.E) load_rows(a, r0, R, info, &any_valid);
    __syncthreads();
    if (!any_valid) {
        if (EPI != kEpiScatter && (!a.ntp || r0 < a.ntp[0])) {
            // Rows of an all-padding tile (or of a non-local expert) are written as zeros.
            for (int idx = threadIdx.x; idx < R * kNW * 16; idx += blockDim.x) {
                const int rr = idx / (kNW * 16), nn = blockIdx.x * kNW * 16 + idx % (kNW * 16);
                if (r0 + rr < a.P && nn < n_out)
                    a.out16[(int64_t)(r0 + rr) * n_out + nn] = __float2half_rn(0.f);
            }
        }
        return;
    }

    const int64_t kw = a.K / 8;
    const int32_t* wq_e = a.w + (int64_t)e * a.N * kw;
    const __half* sc_e = a.scales + (int64_t)e * a.N * a.G;
    const int32_t* zr_e = a.zeros ? a.zeros + (int64_t)e * (a.N / 8) * a.G : nullptr;

    const int c = lane & 3;
    const int rlo = nb + (lane >> 2);
    const int row0 = min(rlo, n_out - 1), row1 = min(rlo + 8, n_out - 1);

    float tot[NT][4];
    float totu[NT][4];
#pragma unroll
    for (int t = 0; t < NT; ++t)
#pragma unroll
        for (int j = 0; j < 4; ++j) tot[t][j] = 0.f;
#pragma unroll
    for (int t = 0; t < NT; ++t)
#pragma unroll
        for (int j = 0; j < 4; ++j) totu[t][j] = 0.f;

    constexpr int PF = kSilu ? 2 : 4;  // register prefetch depth (k-blocks)
    const int nkb_chunk = kc / 128;
    for (int k0 = 0; k0 < a.K; k0 += kc) {
        const int kb0 = k0 / 128;
        // This warp's k-blocks in the chunk: kbl = wk, wk + WK, ...
        const int my_n = (nkb_chunk - wk + WK - 1) / WK;
        WeightSlice ring[PF];
        WeightSlice ringu[kSilu ? PF : 1];
#pragma unroll
        for (int j = 0; j < PF; ++j) {
            if (j < my_n) {
                const int kb = kb0 + wk + j * WK;
                load_slice(a, wq_e, sc_e, zr_e, row0, row1, kb, c, ring[j]);
                if (kSilu) load_slice(a, wq_e, sc_e, zr_e, row0 + n_out, row1 + n_out, kb, c, ringu[j]);
            }
        }
        if (k0 > 0) __syncthreads();  // previous chunk fully consumed
        fill_act_tile<NT>(a, info, act_tile, row_stride, k0, kc);
        __syncthreads();
        for (int i0 = 0; i0 < my_n; i0 += PF) {
#pragma unroll
            for (int j = 0; j < PF; ++j) {
                const int i = i0 + j;
                if (i < my_n) {
                    const int kbl = wk + i * WK;
                    compute_block<NT>(ring[j], act_tile, row_stride, kbl, lane, tot);
                    if (kSilu) compute_block<NT>(ringu[j], act_tile, row_stride, kbl, lane, totu);
                    if (i + PF < my_n) {
                        const int kb = kb0 + wk + (i + PF) * WK;
                        load_slice(a, wq_e, sc_e, zr_e, row0, row1, kb, c, ring[j]);
                        if (kSilu)
                            load_slice(a, wq_e, sc_e, zr_e, row0 + n_out, row1 + n_out, kb, c, ringu[j]);
                    }
                }
            }
        }
    }

    // Split-K reduction across the WK warps sharing (wn): fixed order wk = 0..WK-1.
    if constexpr (WK > 1) {
        __syncthreads();
        float* red = reinterpret_cast<float*>(smem);  // reuse the activation tile
        constexpr int per_thread = NT * 4 * (kSilu ? 2 : 1);
        if (wk > 0) {
            float* dst = red + ((wk - 1) * kNW * 32 + wn * 32 + lane) * per_thread;
#pragma unroll
            for (int t = 0; t < NT; ++t)
#pragma unroll
                for (int j = 0; j < 4; ++j) {
                    dst[t * 4 + j] = tot[t][j];
                    if (kSilu) dst[NT * 4 + t * 4 + j] = totu[t][j];
                }
        }
        __syncthreads();
        if (wk > 0) return;
        for (int s = 1; s < WK; ++s) {
            const float* srcp = red + ((s - 1) * kNW * 32 + wn * 32 + lane) * per_thread;
#pragma unroll
            for (int t = 0; t < NT; ++t)
#pragma unroll
                for (int j = 0; j < 4; ++j) {
                    tot[t][j] += srcp[t * 4 + j];
                    if (kSilu) totu[t][j] += srcp[NT * 4 + t * 4 + j];
                }
        }
    }

    // Epilogue: tot[t][0..1] -> channel rlo, rows t*8 + 2c + {0,1}; tot[t][2..3] -> rlo + 8.
#pragma unroll
    for (int t = 0; t < NT; ++t) {
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            const int rr = t * 8 + 2 * c + (j & 1);
            const int n = rlo + (j >> 1) * 8;
            const int r = r0 + rr;
            if (n >= n_out || r >= a.P) continue;
            const RowInfo ri = info[rr];
            if (EPI == kEpiScatter) {
                if (ri.src < 0) continue;
                const int token = ri.sid / a.out_top_k;
                const float wgt = a.topk_weights[ri.sid];
                atomicAdd(a.out32 + (int64_t)token * a.N + n, wgt * tot[t][j] * ri.ascale);
            } else if (kSilu) {
                if (a.ntp && r >= a.ntp[0]) continue;
                __half v = __float2half_rn(0.f);
                if (ri.src >= 0)
                    v = silu_and_mul_half(tot[t][j] * ri.ascale, totu[t][j] * ri.ascale);
                a.out16[(int64_t)r * n_out + n] = v;
            } else {
                if (a.ntp && r >= a.ntp[0]) continue;
                const float v = ri.src >= 0 ? tot[t][j] * ri.ascale : 0.f;
                a.out16[(int64_t)r * n_out + n] = __float2half_rn(v);
            }
        }
    }
}

// ---------------------------------------------------------------------------------------
// Generic scalar kernel: any group size (multiple of 8 dividing K), int4 or E2M1 codes.
// One thread per (padded row, output channel); the golden arithmetic of the reference's v0.
// ---------------------------------------------------------------------------------------
template <int EPI>
__global__ void __launch_bounds__(256)
w4_scalar_kernel(const GemmArgs a) {
    constexpr bool kSilu = (EPI == kEpiSilu);
    const int n_out = kSilu ? a.N / 2 : a.N;
    const int n = blockIdx.x * 32 + (threadIdx.x & 31);
    const int r = blockIdx.y * 8 + (threadIdx.x >> 5);
    if (n >= n_out || r >= a.P) return;
    const int P_valid = a.ntp ? min(a.ntp[0], a.P) : a.P;
    if (r >= P_valid) return;
    const int sid = a.sorted_ids ? a.sorted_ids[r] : r;
    const int e = a.expert_ids ? a.expert_ids[r / a.block_m] : 0;
    const bool valid = sid >= 0 && sid < a.num_valid && e >= 0 && e < a.E;
    if (!valid) {
        if (EPI != kEpiScatter) a.out16[(int64_t)r * n_out + n] = __float2half_rn(0.f);
        return;
    }
    const int src = a.src_identity ? r : sid / a.top_k;
    const float asc = a.act_scales[src];
    const int64_t kw = a.K / 8;
    const int32_t* wq_e = a.w + (int64_t)e * a.N * kw;
    const __half* sc_e = a.scales + (int64_t)e * a.N * a.G;
    const int32_t* zr_e = a.zeros ? a.zeros + (int64_t)e * (a.N / 8) * a.G : nullptr;
    const uint8_t* xr = a.x_fp8 + (int64_t)src * a.K;
    const int gsz = a.K / a.G;
    float res[2];
    for (int half = 0; half < (kSilu ? 2 : 1); ++half) {
        const int col = n + half * n_out;
        float acc = 0.f;
        for (int g = 0; g < a.G; ++g) {
            const float wsc = __half2float(sc_e[(int64_t)col * a.G + g]);
            int zp = 8;
            if (zr_e) zp = (zr_e[(int64_t)(col >> 3) * a.G + g] >> ((col & 7) * 4)) & 0xF;
            float gacc = 0.f;
            for (int kk = 0; kk < gsz; ++kk) {
                const int k = g * gsz + kk;
                const int code = (wq_e[(int64_t)col * kw + (k >> 3)] >> ((k & 7) * 4)) & 0xF;
                const float wf = a.e2m1 ? e2m1_value(code) : (float)(code - zp);
                gacc = fmaf(wf, e4m3_to_f32(xr[k]), gacc);
            }
            acc = fmaf(gacc, wsc, acc);
        }
        res[half] = acc;
    }
    if (EPI == kEpiScatter) {
        const int token = sid / a.out_top_k;
        atomicAdd(a.out32 + (int64_t)token * a.N + n, a.topk_weights[sid] * res[0] * asc);
    } else if (kSilu) {
        a.out16[(int64_t)r * n_out + n] = silu_and_mul_half(res[0] * asc, res[1] * asc);
    } else {
        a.out16[(int64_t)r * n_out + n] = __float2half_rn(res[0] * asc);
    }
}

template <int NT, int WK, int EPI>
int launch_mma_t(GemmArgs a, cudaStream_t stream) {
    constexpr int R = NT * 8;
    int kc = (kActSmemBudget / (R * 2)) / 128 * 128;
    kc = std::max(128, std::min(kc, (int)a.K));
    while (a.K % kc) kc -= 128;  // chunks tile K exactly
    a.kc = kc;
    const int row_stride = kc * 2 + 32;
    // Region 0 holds the activation tile and, after the main loop, the split-K partials.
    size_t region = (size_t)R * row_stride;
    if (WK > 1) {
        const size_t red = (size_t)(WK - 1) * kNW * 32 * NT * 4 * (EPI == kEpiSilu ? 2 : 1) * 4;
        region = std::max(region, red);
    }
    region = align_up(region, 16);
    a.info_off = (int)region;
    const size_t smem = region + R * sizeof(RowInfo);
    auto kern = w4_mma_kernel<NT, WK, EPI>;
    if (smem > 48 * 1024)
        cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    const int n_out = (EPI == kEpiSilu) ? a.N / 2 : a.N;
    const dim3 grid((n_out + kNW * 16 - 1) / (kNW * 16), (a.P + R - 1) / R);
    kern<<<grid, kNW * WK * 32, smem, stream>>>(a);
    return launch_status();
}

template <int NT, int EPI>
int launch_mma_wk(GemmArgs a, int wk, cudaStream_t stream) {
    if constexpr (NT <= 2) {
        if (wk >= 4) return launch_mma_t<NT, 4, EPI>(a, stream);
        if (wk == 2) return launch_mma_t<NT, 2, EPI>(a, stream);
    }
    return launch_mma_t<NT, 1, EPI>(a, stream);
}

template <int EPI>
int launch_mma_nt(GemmArgs a, int nt, int wk, cudaStream_t stream) {
    switch (nt) {
        case 1: return launch_mma_wk<1, EPI>(a, wk, stream);
        case 2: return launch_mma_wk<2, EPI>(a, wk, stream);
        case 4: return launch_mma_wk<4, EPI>(a, wk, stream);
        default:
            if constexpr (EPI == kEpiSilu) return launch_mma_wk<4, EPI>(a, wk, stream);
            else return launch_mma_wk<8, EPI>(a, wk, stream);
    }
}

}  // namespace

bool mma_path_ok(const GemmArgs& a) {
    return !a.e2m1 && a.G > 0 && a.K == (int64_t)a.G * 128 &&
           (reinterpret_cast<uintptr_t>(a.w) & 15) == 0 &&
           (reinterpret_cast<uintptr_t>(a.x_fp8) & 15) == 0;
}

int launch_w4_gemm(GemmArgs a, int epi, int row_tile, bool scalar, int64_t est_rows,
                   cudaStream_t stream) {
    if (a.P <= 0) return W4A8_OK;
    if (scalar || !mma_path_ok(a)) {
        const int n_out = (epi == kEpiSilu) ? a.N / 2 : a.N;
        const dim3 grid((n_out + 31) / 32, (a.P + 7) / 8);
        switch (epi) {
            case kEpiStore: w4_scalar_kernel<kEpiStore><<<grid, 256, 0, stream>>>(a); break;
            case kEpiSilu: w4_scalar_kernel<kEpiSilu><<<grid, 256, 0, stream>>>(a); break;
            default: w4_scalar_kernel<kEpiScatter><<<grid, 256, 0, stream>>>(a); break;
        }
        return launch_status();
    }
    // Row tile (8*NT rows) must not straddle an expert block.
    int nt = std::max(1, std::min(row_tile, 64) / 8);
    while (nt > 1 && ((a.block_m % (nt * 8)) != 0 || nt == 3 || nt > 4 && nt != 8)) --nt;
    // Split K across warps when the grid would otherwise under-fill the 148 SMs.
    const int n_out = (epi == kEpiSilu) ? a.N / 2 : a.N;
    const int64_t ctas = (int64_t)((n_out + 63) / 64) * std::max<int64_t>(1, (est_rows + nt * 8 - 1) / (nt * 8));
    int wk = 1;
    while (nt <= 2 && wk < 4 && ctas * kNW * wk < 148 * 16 && a.G >= 2 * wk) wk *= 2;
    switch (epi) {
        case kEpiStore: return launch_mma_nt<kEpiStore>(a, nt, wk, stream);
        case kEpiSilu: return launch_mma_nt<kEpiSilu>(a, nt, wk, stream);
        default: return launch_mma_nt<kEpiScatter>(a, nt, wk, stream);
    }
}

}  // namespace w4a8
