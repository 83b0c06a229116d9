// gemv_stream.cu — persistent W4A8 GEMV for decode-sized row counts.
//
// Work item = (8-row block b of the padded-sorted rows, K split ks of 4 groups, 128-row group
// rg of the weight rows). One CTA per SM walks items round-robin. A producer warp streams each
// item into a ring of shared-memory stages, so several items' weights are in flight per SM:
//   - the 128 x 256-byte weight tile: two 2D TMA boxes with the 128-byte swizzle;
//   - the 8 activation rows (fp16 operand, 1 KB each) and their group sums: bulk copies
//     straight from the source rows (the gather happens in the copy);
//   - scales and zero points: cp.async, completing on the same mbarrier.
// Eight compute warps each take 16 weight rows of the item (mma.sync.m16n8k16, 8 token
// columns) and release the stage.
//
// Arithmetic. Per 128-code group a lane expands 2 weight rows x 32 codes with the fp16
// magic-number trick without subtracting the zero point: pairs (0,4),(2,6) of every 8-code word
// become 1024 + q and pairs (1,5),(3,7) become 1024 + 16q, all exact in fp16. The activation
// operand (fp16 copies of the e4m3 bytes, exact) carries a / 16 at the (1,5),(3,7) positions
// (exact: a power-of-two scale), so one mma.sync.m16n8k16 (fp16 x fp16 -> fp32) chain yields
//     acc = sum_k q_k a_k + K0,   K0 = 1024 * sum_{even pairs} a + 64 * sum_{odd pairs} a.
// With S = sum_k a_k the group result is sum_k (q_k - z) a_k = acc - K0 - z*S; it is folded as
//     tot += scale[n,g] * (acc - K0 - z*S)
// and multiplied by the row's activation scale in the epilogue: the reference's per-group fp32
// association (w4a8_fp8_wmma/test_correctness.py:113-119). K0 and S are per (activation row,
// group) sums computed once by the operand quantiser. The 1024-offset terms are removed in
// fp32, which leaves a relative error near 1e-4 of the group sum (well inside the 1e-2 bar).
//
// K splits write fp32 partials [ks][row][n]; w4_stream_finish_kernel sums them in fixed order
// (results do not depend on scheduling) and applies the epilogue. One split: direct epilogue.
// Every mbarrier wait is bounded (sm100.cuh); once one gives up, later waits are skipped, the
// kernel finishes and sets bit 1 of StreamArgs::counter.
#include <algorithm>

#include "common.cuh"
#include "gemm_common.h"
#include "internal.h"
#include "sm100.cuh"
#include "stream_core.cuh"

namespace w4a8 {

namespace {

constexpr int kWarps = 8;                        // compute warps
constexpr int kStreamThreads = (kWarps + 1) * 32;
constexpr int kSpi = 4;                          // K blocks (groups of 128) per item
constexpr int kRowsPerItem = kWarps * 16;        // 128 weight rows
constexpr int kActStride = kSpi * 256 + 32;      // bytes per activation row in shared memory
constexpr int kStages = 5;

struct ItemMeta {
    int any;      // 1 when at least one of the 8 rows is live
    int e;        // expert
    int b, ks, rg;
    int src[8];   // activation row per token column (-1: padding)
    int sid[8];
};

struct StreamSmem {
    uint8_t wt[kStages][2][128 * 128];       // weight tile halves, SW128 (1024-aligned)
    uint8_t act[kStages][8][kActStride];     // activation rows
    float2 xs[kStages][8][kSpi];             // {K0, S} per (token column, group)
    __half sc[kStages][kRowsPerItem][kSpi];
    uint32_t zr[kStages][kRowsPerItem / 8][kSpi];
    ItemMeta meta[kStages];
    uint64_t full[kStages];
    uint64_t empty[kStages];
    int bad;
};

// Routing values of one item, loaded one item ahead of their use by the producer.
struct ItemRoute {
    int sid, e;
};
__device__ __forceinline__ ItemRoute fetch_route(const StreamArgs& a, int item, int per_b,
                                                 int P_valid, int total) {
    const int lane = threadIdx.x & 31;
    ItemRoute r{-1, -1};
    if (item < total) {
        const int b = item / per_b;
        const int row = b * 8 + lane;
        if (lane < 8 && row < P_valid) r.sid = a.sorted_ids ? a.sorted_ids[row] : row;
        r.e = a.expert_ids ? a.expert_ids[(b * 8) / a.block_m] : 0;
    }
    return r;
}

// Producer (whole warp): item metadata, then the item's copies into stage `st`.
__device__ __forceinline__ void produce_item(const StreamArgs& a, StreamSmem& sm,
                                             const CUtensorMap* tmw, int item, int per_b,
                                             int P_valid, int st, const ItemRoute& rt) {
    const int lane = threadIdx.x & 31;
    const int b = item / per_b, rem = item - b * per_b;
    const int ks = rem / a.rg_n, rg = rem - ks * a.rg_n;
    const int row = b * 8 + lane;
    const int sid = rt.sid;
    const int e = rt.e;
    const bool live = e >= 0 && e < a.E;
    const bool ok = live && lane < 8 && sid >= 0 && sid < a.num_valid;
    const int src = ok ? (a.src_identity ? row : sid / a.top_k) : -1;
    const int any = __any_sync(0xffffffffu, ok);
    const uint32_t okm = __ballot_sync(0xffffffffu, ok);
    ItemMeta& m = sm.meta[st];
    if (lane < 8) {
        m.src[lane] = src;
        m.sid[lane] = ok ? sid : 0;
    }
    if (any) {
        const int kb0 = ks * kSpi;
        const int n0 = rg * kRowsPerItem;
#pragma unroll
        for (int i = 0; i < kRowsPerItem / 32; ++i) {  // scales: 128 rows x 4 groups (8 B)
            const int r = lane + 32 * i, n = n0 + r;
            const bool nok = n < a.N;
            cp_async8_bar(&sm.sc[st][r][0], a.scales + ((int64_t)e * a.N + (nok ? n : 0)) * a.G + kb0,
                          nok);
        }
        if (lane < kRowsPerItem / 8) {  // zero points: 16 words x 4 groups
            const int n8 = n0 / 8 + lane;
            const bool zok = a.zeros && n8 < a.N / 8;
            cp_async16_bar(&sm.zr[st][lane][0],
                           zok ? (const void*)(a.zeros + ((int64_t)e * (a.N / 8) + n8) * a.G + kb0)
                               : (const void*)a.scales,
                           zok);
        }
    }
    __syncwarp();
    if (lane == 0) {
        m.any = any;
        m.e = e;
        m.b = b;
        m.ks = ks;
        m.rg = rg;
        uint64_t* fb = &sm.full[st];
        if (any) {
            const uint32_t bytes = 2 * 128 * 128 + (uint32_t)__popc(okm) * (kSpi * 256 + kSpi * 8);
            mbar_expect_tx(fb, bytes);
            const int y = e * a.N + rg * kRowsPerItem;
            tma_load_2d(&sm.wt[st][0][0], tmw, ks * 256, y, fb);
            tma_load_2d(&sm.wt[st][1][0], tmw, ks * 256 + 128, y, fb);
            for (int c = 0; c < 8; ++c) {
                if (!(okm >> c & 1u)) continue;
                const int srow = m.src[c];
                bulk_load(&sm.act[st][c][0], a.xh + (int64_t)srow * a.K + (int64_t)ks * kSpi * 128,
                          kSpi * 256, fb);
                bulk_load(&sm.xs[st][c][0], a.xsum + (int64_t)srow * a.G + ks * kSpi, kSpi * 8, fb);
            }
        } else {
            mbar_arrive(fb);
        }
    }
    cp_async_arrive(&sm.full[st]);
}

// Compute one item (this warp's 16 weight rows) from stage `st`; emit partials or the epilogue.
__device__ __forceinline__ void compute_item(const StreamArgs& a, const StreamSmem& sm, int st,
                                             int warp, int lane, int P_valid) {
    const ItemMeta& m = sm.meta[st];
    const int c = lane & 3, tok = lane >> 2;
    const int m_any = m.any, m_b = m.b, m_ks = m.ks, m_rg = m.rg;
    const int nl = warp * 16 + tok;              // local row (0..127) of the item
    const int n0 = m_rg * kRowsPerItem + nl;
    if (m_rg * kRowsPerItem + warp * 16 >= a.N) return;   // warp beyond N
    float tot[4] = {0.f, 0.f, 0.f, 0.f};
    if (!m_any) {
        // all-padding block or non-local expert: rows are zeros for the direct store epilogue
        if (a.mode == kStreamStore && !a.force_part) {
#pragma unroll
            for (int jj = 0; jj < 4; ++jj) {
                const int rr = m_b * 8 + 2 * c + (jj & 1), n = n0 + (jj >> 1) * 8;
                if (rr < P_valid && n < a.N) a.out16[(int64_t)rr * a.N + n] = __float2half_rn(0.f);
            }
        }
        return;
    }
    const int src_c[2] = {m.src[2 * c], m.src[2 * c + 1]};
    const int sid_c[2] = {m.sid[2 * c], m.sid[2 * c + 1]};
    const uint8_t* rowp = &sm.act[st][tok][0];
    const int sh0 = (n0 & 7) * 4, sh1 = ((n0 + 8) & 7) * 4;
    const int r0 = nl, r1 = nl + 8;              // tile rows of this lane
#pragma unroll
    for (int j = 0; j < kSpi; ++j) {
        // weight chunk (16 B) c of group j: tile half j / 2, chunk (j % 2) * 4 + c, swizzled
        const uint8_t* wh = &sm.wt[st][j >> 1][0];
        const int u = (j & 1) * 4 + c;
        const uint4 q0 = *reinterpret_cast<const uint4*>(wh + r0 * 128 + ((u ^ (r0 & 7)) << 4));
        const uint4 q1 = *reinterpret_cast<const uint4*>(wh + r1 * 128 + ((u ^ (r1 & 7)) << 4));
        const uint32_t w0[4] = {q0.x, q0.y, q0.z, q0.w};
        const uint32_t w1[4] = {q1.x, q1.y, q1.z, q1.w};
        // two independent accumulator chains (words 0,2 and 1,3) halve the MMA dependency depth
        float acc[2][4] = {{0.f, 0.f, 0.f, 0.f}, {0.f, 0.f, 0.f, 0.f}};
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            uint32_t h0[4], h1[4];
            expand_word(w0[i], h0);
            expand_word(w1[i], h1);
            const uint4 bq = *reinterpret_cast<const uint4*>(rowp + act_off(j, c, i));
            const uint32_t a0[4] = {h0[0], h1[0], h0[1], h1[1]};
            mma_16816(acc[i & 1], a0, bq.x, bq.y);
            const uint32_t a1[4] = {h0[2], h1[2], h0[3], h1[3]};
            mma_16816(acc[i & 1], a1, bq.z, bq.w);
        }
#pragma unroll
        for (int v = 0; v < 4; ++v) acc[0][v] += acc[1][v];
        float z0 = 8.f, z1 = 8.f;
        if (a.zeros) {
            // nibble -> float through the 2^23 magic (one LOP3 + one FADD, no conversion unit)
            z0 = __uint_as_float(0x4B000000u | ((sm.zr[st][nl >> 3][j] >> sh0) & 0xF)) - 8388608.f;
            z1 = __uint_as_float(0x4B000000u | ((sm.zr[st][(nl + 8) >> 3][j] >> sh1) & 0xF)) -
                 8388608.f;
        }
        const float2 xa = sm.xs[st][2 * c][j], xb = sm.xs[st][2 * c + 1][j];  // {K0, S}
        const float s0 = __half2float(sm.sc[st][nl][j]);
        const float s1 = __half2float(sm.sc[st][nl + 8][j]);
        tot[0] = fmaf(s0, fmaf(-z0, xa.y, acc[0][0] - xa.x), tot[0]);
        tot[1] = fmaf(s0, fmaf(-z0, xb.y, acc[0][1] - xb.x), tot[1]);
        tot[2] = fmaf(s1, fmaf(-z1, xa.y, acc[0][2] - xa.x), tot[2]);
        tot[3] = fmaf(s1, fmaf(-z1, xb.y, acc[0][3] - xb.x), tot[3]);
    }
    // tot[0..1]: row n0, token columns 2c, 2c+1; tot[2..3]: row n0 + 8.
#pragma unroll
    for (int jj = 0; jj < 4; ++jj) {
        const int col = 2 * c + (jj & 1);
        const int n = n0 + (jj >> 1) * 8;
        if (n >= a.N) continue;
        const int src = src_c[jj & 1];
        const int rr = m_b * 8 + col;
        if (a.force_part) {
            if (src >= 0) a.part[((int64_t)m_ks * a.P + rr) * a.N + n] = tot[jj];
        } else if (a.mode == kStreamScatter) {
            if (src >= 0) {
                const int sid = sid_c[jj & 1];
                atomicAdd(a.out32 + (int64_t)(sid / a.out_top_k) * a.N + n,
                          a.topk_weights[sid] * tot[jj] * a.act_scales[src]);
            }
        } else {  // store
            if (rr < P_valid)
                a.out16[(int64_t)rr * a.N + n] =
                    __float2half_rn(src >= 0 ? tot[jj] * a.act_scales[src] : 0.f);
        }
    }
}

__global__ void __launch_bounds__(kStreamThreads, 1)
w4_stream_kernel(const StreamArgs a, const __grid_constant__ CUtensorMap tmw) {
    extern __shared__ uint8_t smem_raw[];
    // 1024-byte alignment by offsetting the __shared__ array itself (a round trip through an
    // integer would lose the shared address space and turn every access into a generic one)
    StreamSmem& sm = *reinterpret_cast<StreamSmem*>(
        smem_raw + ((1024u - (smem_u32(smem_raw) & 1023u)) & 1023u));
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    volatile int* bad = &sm.bad;
    const int P_valid = a.ntp ? min(a.ntp[0], a.P) : a.P;
    const int per_b = a.ks_n * a.rg_n;
    const int total = ((P_valid + 7) / 8) * per_b;
    if ((int)blockIdx.x >= total) return;
    if (threadIdx.x == 0) {
        sm.bad = 0;
        for (int s = 0; s < kStages; ++s) {
            mbar_init(&sm.full[s], 1 + 32);  // producer lane 0 (+ tx bytes) and 32 cp.async arrivals
            mbar_init(&sm.empty[s], kWarps);
        }
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    __syncthreads();
    uint32_t st = 0, ph = 0;
    if (warp == kWarps) {
        // ---------------- producer ----------------
        ItemRoute rt = fetch_route(a, blockIdx.x, per_b, P_valid, total);
        for (int item = blockIdx.x; item < total; item += gridDim.x) {
            const ItemRoute nx = fetch_route(a, item + gridDim.x, per_b, P_valid, total);
            if (lane == 0) mbar_wait(&sm.empty[st], ph ^ 1, bad);
            __syncwarp();
            produce_item(a, sm, &tmw, item, per_b, P_valid, (int)st, rt);
            rt = nx;
            if (++st == kStages) {
                st = 0;
                ph ^= 1;
            }
        }
        // the compute warps consume every stage issued, so no copy outlives the CTA unless a
        // wait gave up; then wait (boundedly) for the last stages to land
        if (*bad && lane == 0) {
            const uint64_t t0 = global_ns();
            for (int s = 0; s < kStages; ++s)
                while (!mbar_try(&sm.full[s], ph ^ (s < (int)st ? 0u : 1u)) &&
                       global_ns() - t0 < kWaitLimitNs) {
                }
        }
    } else {
        // ---------------- compute warps ----------------
        for (int item = blockIdx.x; item < total; item += gridDim.x) {
            mbar_wait(&sm.full[st], ph, bad);
            __syncwarp();
            compute_item(a, sm, (int)st, warp, lane, P_valid);
            __syncwarp();
            if (lane == 0) mbar_arrive(&sm.empty[st]);
            if (++st == kStages) {
                st = 0;
                ph ^= 1;
            }
        }
    }
    __syncthreads();
    if (threadIdx.x == 0 && sm.bad && a.counter) atomicOr(a.counter, 2);
}

__global__ void __launch_bounds__(256) operand_quant_kernel(const __half* __restrict__ x,
                                                            OperandOut o, int64_t M, int64_t K,
                                                            const int32_t* row_limit) {
    __shared__ float red[32];
    const int64_t row = blockIdx.x;
    if (row >= M || (row_limit && row >= row_limit[0])) return;
    quant_operand_row(x + row * K, K, row, o, red);
}

// ---------------------------------------------------------------------------------------
// Finish: sum the K-split partials in fixed order and apply the epilogue. One CTA per row.
// kStreamSiluQuant additionally quantises the SiLU row as the next GEMM's operand.
// ---------------------------------------------------------------------------------------
__global__ void __launch_bounds__(256) w4_stream_finish_kernel(const StreamArgs a) {
    extern __shared__ __align__(16) __half silu_row[];
    __shared__ float red[32];
    const int r = blockIdx.x;
    const int P_valid = a.ntp ? min(a.ntp[0], a.P) : a.P;
    if (r >= P_valid) return;
    const int sid = a.sorted_ids ? a.sorted_ids[r] : r;
    const int e = a.expert_ids ? a.expert_ids[r / a.block_m] : 0;
    const bool valid = sid >= 0 && sid < a.num_valid && e >= 0 && e < a.E;
    const int src = valid ? (a.src_identity ? r : sid / a.top_k) : -1;
    const float asc = valid ? a.act_scales[src] : 0.f;
    const bool silu = a.mode == kStreamSilu || a.mode == kStreamSiluQuant;
    const int n_out = silu ? a.N / 2 : a.N;
    for (int n = threadIdx.x; n < n_out; n += blockDim.x) {
        __half hv = __float2half_rn(0.f);
        if (valid) {
            float v = 0.f, u = 0.f;
            for (int ks = 0; ks < a.ks_n; ++ks) {
                const float* p = a.part + ((int64_t)ks * a.P + r) * a.N;
                v += p[n];
                if (silu) u += p[n + n_out];
            }
            if (silu) {
                hv = silu_and_mul_half(v * asc, u * asc);
            } else if (a.mode == kStreamScatter) {
                atomicAdd(a.out32 + (int64_t)(sid / a.out_top_k) * a.N + n,
                          a.topk_weights[sid] * v * asc);
                continue;
            } else {
                hv = __float2half_rn(v * asc);
            }
        } else if (a.mode == kStreamScatter) {
            continue;
        }
        if (a.mode == kStreamSiluQuant) {
            silu_row[n] = hv;
            if (a.out_silu) a.out_silu[(int64_t)r * n_out + n] = hv;
        } else {
            a.out16[(int64_t)r * n_out + n] = hv;
        }
    }
    if (a.mode == kStreamSiluQuant) {
        __syncthreads();
        quant_operand_row(silu_row, n_out, r, a.next, red);
    }
}

}  // namespace

bool stream_path_ok(int64_t K, int G, int e2m1, const void* w) {
    return !e2m1 && G > 0 && K == (int64_t)G * 128 && (G % kSpi) == 0 &&
           (reinterpret_cast<uintptr_t>(w) & 15) == 0;
}

size_t stream_partials_bytes(int64_t P, int64_t N, int64_t K) {
    const int64_t G = std::max<int64_t>(K / 128, 1);
    const int64_t ks = (G + kSpi - 1) / kSpi;
    return align_up((size_t)(ks * P * N) * 4, 256);
}

int launch_operand_quant(const void* x, OperandOut o, int64_t M, int64_t K,
                         const int32_t* row_limit, cudaStream_t stream) {
    if (M <= 0) return W4A8_OK;
    if (K % 128 != 0 || (reinterpret_cast<uintptr_t>(x) & 15) != 0)
        return set_error("operand quant needs K % 128 == 0 and 16-byte aligned rows");
    operand_quant_kernel<<<(unsigned)M, 256, 0, stream>>>(static_cast<const __half*>(x), o, M, K,
                                                         row_limit);
    return launch_status();
}

int launch_w4_stream(StreamArgs a, cudaStream_t stream) {
    if (a.P <= 0) return W4A8_OK;
    a.ks_n = (a.G + kSpi - 1) / kSpi;
    a.rg_n = (a.N + kRowsPerItem - 1) / kRowsPerItem;
    // K splits and the SiLU epilogues (gate row n pairs with up row n + N/2, computed by other
    // warps) go through the fp32 partials and the finish kernel.
    const bool silu = a.mode == kStreamSilu || a.mode == kStreamSiluQuant;
    a.force_part = (a.ks_n > 1 || silu) ? 1 : 0;
    if (a.force_part && !a.part) return set_error("internal: stream path needs a partials buffer");
    if (a.mode == kStreamSiluQuant && (a.N / 2) % 128 != 0)
        return set_error("internal: SiLU-quant needs inter % 128 == 0");
    int dev = 0, sms = 148;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    CUtensorMap tmw;
    if (!make_tma_map_u8(&tmw, a.w, (uint64_t)a.E * a.N, (uint64_t)a.K / 2, 128, kRowsPerItem,
                         CU_TENSOR_MAP_SWIZZLE_128B))
        return set_error("stream path: tensor map encoding failed");
    const size_t smem = sizeof(StreamSmem) + 1024;
    cudaError_t ce = cudaFuncSetAttribute(w4_stream_kernel,
                                          cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (ce != cudaSuccess) return (int)ce;
    w4_stream_kernel<<<sms, kStreamThreads, smem, stream>>>(a, tmw);
    if (int rc = launch_status()) return rc;
    if (a.force_part) {
        const size_t smem = a.mode == kStreamSiluQuant ? (size_t)(a.N / 2) * 2 : 0;
        if (smem > 48 * 1024)
            cudaFuncSetAttribute(w4_stream_finish_kernel,
                                 cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
        w4_stream_finish_kernel<<<a.P, 256, smem, stream>>>(a);
        return launch_status();
    }
    return W4A8_OK;
}

}  // namespace w4a8
