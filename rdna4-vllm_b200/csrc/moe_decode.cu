// moe_decode.cu — the gated MoE layer at decode sizes in three launches.
//
// Same result as the decode branch of the reference's composition (_run_grouped_moe, M <= 96,
// w4a8_fp8_wmma/w4a8_fp8_wmma/moe_experts.py:563-648) and its oracle
// (w4a8_fp8_wmma/test_moe_experts.py:155-191): per (token, slot) gate_up GEMM -> fp16 gate/up ->
// silu_and_mul -> per-token e4m3 re-quantisation -> down GEMM -> fp16 row, then the fp32
// topk-weighted sum over the token's slots in slot order.
//
//   1. decode_prep_kernel   CTA 0 groups the valid (token, slot) pairs by expert (no block
//                           padding) and resets the counters of launches 2-3; CTAs 1..T
//                           quantise one token row each into the GEMV operand format.
//   2. gate_up GEMV         work unit = (expert, 64 gate rows + the matching 64 up rows, all of
//                           K); SiLU-and-mul in the epilogue, fp16 SiLU rows per slot.
//   3. down GEMV            work unit = (expert, 128 output channels); fp16 rows per slot, then
//                           the fp32 topk-weighted sum over each token's slots in slot order.
//
// Two implementations of launches 2-3 share the stage stream (a persistent CTA per SM; units
// dealt round-robin, heavy experts first; 512-wide K chunks through a shared-memory ring fed by
// one producer warp; <= 16 activation rows per pass):
//   - prepacked weights (w4a8_stream_pack): decode_tc_kernel, the 5th-generation tensor cores.
//     The codes are expanded to exact e4m3 values into tensor memory and multiplied with
//     tcgen05.mma (kind::f8f6f4, M 128 x N 16 x K 32); the accumulators are folded per 128-group
//     in fp32 (scale, zero point times the operand's group sum). The down launch is cooperative:
//     it first quantises every SiLU row once (grid-wide), and after its units a grid barrier
//     precedes the slot-order combine.
//   - op-layout weights: decode_gemv_kernel, mma.sync m16n8k32 on e4m3 operands (see
//     dec_compute_t); its down operand is quantised per stage by two warps and its combine is
//     done by the last arrival per (token, 16-channel chunk).
// Both fold in the reference oracle's association (w4a8_fp8_wmma/test_correctness.py:113-119)
// up to fp32 rounding. The intermediates (SiLU rows, the down operand, the per-slot down rows)
// are a few hundred KB and stay in L2. No result depends on scheduling: every sum has a fixed
// order.
//
// Every mbarrier wait and the grid barrier are bounded (sm100.cuh); a wait that gives up sets
// the error word and the kernel finishes without waiting further.
#include <algorithm>
#include <cstddef>
#include <type_traits>
#include <string>

#include "common.cuh"
#include "gemm_common.h"
#include "internal.h"
#include "sm100.cuh"
#include "e4_operand.cuh"
#include "stream_core.cuh"
#include "tcgen05.cuh"

namespace w4a8 {

namespace {

constexpr int kDW = 8;                        // compute warps; then 1 producer, 2 quant warps
constexpr int kDThreads = (kDW + 3) * 32;
constexpr int kDStages = 5;
constexpr int kDSpi = 4;                      // 128-groups per stage (512 K)
constexpr int kDMaxRows = 16;                 // activation rows per pass (2 token groups of 8)
constexpr int kDActStride = kDSpi * 128 + 16;  // e4m3 operand bytes per row + bank padding
constexpr int kPrepThreads = 256;
constexpr int kMaxSlots = 1 << 16;
constexpr int kMaxExperts = 4096;

enum DecMode : int { kGateUp = 0, kDown = 1 };

// Meta word indices.
enum : int {
    kMetaActive = 0, kMetaUnit1 = 1, kMetaUnit2 = 2, kMetaErr = 3,
    kMetaSync = 4,  // CTAs of the tensor-core down launch that finished their units
    kMetaWords = 5
};

struct DecArgs {
    const int32_t* topk_ids;   // row t's slot j at topk_ids[t * ids_stride + j]
    const float* topk_w;       // row t's weight j at topk_w[t * ids_stride + j]
    int T, top_k, E;
    int ids_stride;            // elements between rows of topk_ids / topk_w (top_k when dense)
    int64_t xe_stride;         // bytes between gate_up operand rows (K when dense)
    int64_t xs_stride;         // floats between rows of the group sums (K/128 when dense)
    int64_t asc_stride;        // floats between activation scales (1 when dense)
    int out_f32;               // the layer output is fp32 (else fp16)
    uint32_t one, m1;          // 1 and 0xffffffff (multipliers of codes8_to_e4m3_fma)
    int32_t* off;              // [E + 1] sorted-row offset of each expert
    int32_t* active;           // [E] experts with rows, heavy (> kDMaxRows rows) first
    int32_t* meta;             // kMeta*
    int4* act_tab;             // [E] per active expert i: {expert, first row, end row, 0}
    int32_t* sorted_tok;       // [S] token of sorted row p
    int32_t* sorted_slot;      // [S] slot at sorted row p
    int32_t* slot_pos;         // [S] sorted row of slot s, -1 if the slot's expert is invalid
    int32_t* nslot;            // [T] valid slots of each token
    int32_t* tok_done;         // [T * H/16] finished down rows per (token, 16-channel chunk)
    float* amax;               // [S] max |SiLU row| (atomicMax on the bits; zeroed by prep)
    const int32_t* w;          // this launch's weights (E, N, K/8)
    const __half* scales;      // (E, N, K/128)
    const int32_t* zeros;      // (E, N/8, K/128) or null
    const uint8_t* packed;     // packed blocks (w4a8_stream_pack) or null: then w/scales/zeros
    int64_t K;
    int N, G, H, I;
    const uint8_t* xe;         // e4m3 operand rows (GEMV byte order): gate_up by token, down by
                               // sorted row
    const float* xsum;         // per (row, 128-group) sum S of the row's e4m3 values
    const float* asc;          // per-row activation scale
    __half* silu;              // (S, I) fp16 SiLU rows (gate_up output)
    __half* out2;              // (S, H) fp16 down rows
    void* out;                 // (T, H) layer output, fp16 or fp32 (out_f32)
    const __half* x;           // (T, H) fp16 input (prep)
};

// ---------------------------------------------------------------------------------------
// Launch 1: routing sort + token quantisation.
// ---------------------------------------------------------------------------------------
// Exclusive scan of v over the block (kPrepThreads threads, one value each); returns the
// prefix and writes the total to *total.
__device__ __forceinline__ int block_excl_scan(int v, int* red, int* total) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    int inc = v;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
        const int n = __shfl_up_sync(0xffffffffu, inc, o);
        if (lane >= o) inc += n;
    }
    if (lane == 31) red[warp] = inc;
    __syncthreads();
    if (warp == 0) {
        int s = lane < (kPrepThreads >> 5) ? red[lane] : 0;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            const int n = __shfl_up_sync(0xffffffffu, s, o);
            if (lane >= o) s += n;
        }
        if (lane < (kPrepThreads >> 5)) red[lane] = s;  // inclusive warp totals
    }
    __syncthreads();
    const int base = warp > 0 ? red[warp - 1] : 0;
    *total = red[(kPrepThreads >> 5) - 1];
    __syncthreads();
    return base + inc - v;
}

#ifdef W4A8_DEC_TRACE
__device__ unsigned long long g_prep_trace[8];
#define PREP_MARK(i)                                     \
    do {                                                 \
        if (threadIdx.x == 0) g_prep_trace[i] = global_ns(); \
    } while (0)
#else
#define PREP_MARK(i) \
    do {             \
    } while (0)
#endif

__global__ void __launch_bounds__(kPrepThreads) decode_prep_kernel(const DecArgs a) {
    extern __shared__ int prep_smem[];
    __shared__ float red[32];
    __shared__ int ired[32];
    const int tid = threadIdx.x;
    if (blockIdx.x > 0) {
        // one token row -> GEMV operand (e4m3 rounding of the oracle, fp16 operand copy, group
        // sums, scale)
        const int t = blockIdx.x - 1;
        quant_row_e4<false>(a.x + (int64_t)t * a.H, a.H, t, const_cast<uint8_t*>(a.xe),
                            const_cast<float*>(a.xsum), const_cast<float*>(a.asc), red);
        return;
    }
    PREP_MARK(0);
    const int E = a.E, S = a.T * a.top_k;
    const int n16 = a.H / 16;
    int* cnt = prep_smem;             // [E]
    int* cur = prep_smem + E;         // [E]
    int* ns = prep_smem + 2 * E;      // [T]
    for (int i = tid; i < E; i += kPrepThreads) cnt[i] = 0;
    if (tid < kMetaWords) a.meta[tid] = 0;
    for (int i = tid; i < a.T * n16; i += kPrepThreads) a.tok_done[i] = 0;
    for (int i = tid; i < S; i += kPrepThreads) a.amax[i] = 0.f;
    PREP_MARK(1);
    __syncthreads();
    auto slot_id = [&](int s) { return a.topk_ids[(int64_t)(s / a.top_k) * a.ids_stride + s % a.top_k]; };
    for (int s = tid; s < S; s += kPrepThreads) {
        const int e = slot_id(s);
        if (e >= 0 && e < E) atomicAdd(&cnt[e], 1);
    }
    for (int t = tid; t < a.T; t += kPrepThreads) {
        int n = 0;
        for (int j = 0; j < a.top_k; ++j) {
            const int e = a.topk_ids[(int64_t)t * a.ids_stride + j];
            n += (e >= 0 && e < E);
        }
        a.nslot[t] = n;
        ns[t] = n;
    }
    PREP_MARK(2);
    __syncthreads();
    // offsets (expert order) and the active list (heavy experts first, then the rest; each part
    // in expert order): each thread owns a contiguous run of experts
    const int per = (E + kPrepThreads - 1) / kPrepThreads;
    const int e0 = min(E, tid * per), e1 = min(E, e0 + per);
    int my_rows = 0, my_heavy = 0, my_light = 0;
    for (int e = e0; e < e1; ++e) {
        my_rows += cnt[e];
        my_heavy += cnt[e] > kDMaxRows;
        my_light += (cnt[e] > 0 && cnt[e] <= kDMaxRows);
    }
    PREP_MARK(3);
    int tot_rows, tot_heavy, tot_light;
    int base_rows = block_excl_scan(my_rows, ired, &tot_rows);
    int base_heavy = block_excl_scan(my_heavy, ired, &tot_heavy);
    int base_light = block_excl_scan(my_light, ired, &tot_light) + tot_heavy;
    PREP_MARK(4);
    for (int e = e0; e < e1; ++e) {
        a.off[e] = base_rows;
        cur[e] = base_rows;
        const int4 tab = make_int4(e, base_rows, base_rows + cnt[e], 0);
        base_rows += cnt[e];
        if (cnt[e] > kDMaxRows) {
            a.act_tab[base_heavy] = tab;
            a.active[base_heavy++] = e;
        } else if (cnt[e] > 0) {
            a.act_tab[base_light] = tab;
            a.active[base_light++] = e;
        }
    }
    if (tid == 0) {
        a.off[E] = tot_rows;
        a.meta[kMetaActive] = tot_heavy + tot_light;
    }
    __syncthreads();
    PREP_MARK(5);
    // placement: one shared-memory atomic per slot. The order of rows inside an expert's
    // range does not change any result (each row is its own accumulator column and the combine
    // reads rows through slot_pos in slot order), so it need not be stable.
    for (int s = tid; s < S; s += kPrepThreads) {
        const int e = slot_id(s);
        if (e >= 0 && e < E) {
            const int p = atomicAdd(&cur[e], 1);
            a.slot_pos[s] = p;
            a.sorted_slot[p] = s;
            a.sorted_tok[p] = s / a.top_k;
        } else {
            a.slot_pos[s] = -1;
        }
    }
    PREP_MARK(6);
    // tokens without a valid slot: the layer output is zero
    for (int t = 0; t < a.T; ++t)
        if (ns[t] == 0)
            for (int n = tid; n < a.H; n += kPrepThreads) {
                if (a.out_f32) static_cast<float*>(a.out)[(int64_t)t * a.H + n] = 0.f;
                else static_cast<__half*>(a.out)[(int64_t)t * a.H + n] = __float2half_rn(0.f);
            }
    PREP_MARK(7);
}

// The first three members are one packed weight block (w4a8_stream_pack): a stage of packed
// weights lands with a single bulk copy.
struct alignas(1024) DStage {
    uint8_t wt[2][128 * 128];                 // weight rows, two 128-byte K halves, SW128
    __half sc[128][kDSpi];                    // scales per (weight row, group)
    uint32_t zr[16][kDSpi];                   // packed zero points per (8 weight rows, group)
    uint8_t act[kDMaxRows][kDActStride];      // e4m3 operand rows (GEMV byte order)
    float xs[kDMaxRows][kDSpi];               // S per (row, group)
    float asc[kDMaxRows];                     // down: activation scale per row
};
constexpr uint32_t kPackBlock = 2 * 128 * 128 + 128 * kDSpi * 2 + 16 * kDSpi * 4;  // 34,048 B
static_assert(offsetof(DStage, act) >= kPackBlock, "packed block layout");

struct DMeta {
    int e, sl, p0, nrows, chunk, last;
};

struct DSmem {
    DStage st[kDStages];
    DMeta meta[kDStages];
    uint64_t full[kDStages];
    uint64_t empty[kDStages];
    int bad;
};

#ifdef W4A8_DEC_TRACE
// Experiment builds only: per CTA (first 8), per stage event (issue, landed, computed), ns.
constexpr int kTrCtas = 8, kTrStages = 64;
__device__ unsigned long long g_dec_trace[2][kTrCtas][kTrStages][12];
#define DEC_TRACE(mode, stage, ev)                                                              \
    do {                                                                                       \
        if (blockIdx.x < kTrCtas && (stage) < kTrStages)                                       \
            g_dec_trace[mode][blockIdx.x][stage][ev] = global_ns();                            \
    } while (0)
#else
#define DEC_TRACE(mode, stage, ev) \
    do {                           \
    } while (0)
#endif

// Smem weight row m (0..127) of unit slice sl -> weight row n of the expert.
template <int MODE>
__device__ __forceinline__ int unit_row(const DecArgs& a, int sl, int m) {
    if (MODE == kGateUp) return m < 64 ? sl * 64 + m : a.I + sl * 64 + (m - 64);
    return sl * 128 + m;
}

// The static unit schedule every role of a CTA walks: unit u = blockIdx.x + i * gridDim.x,
// heavy experts first; a unit is ceil(rows / kDMaxRows) passes of K / 512 stages.
struct UnitWalk {
    int u, units, nsl;
    __device__ __forceinline__ int4 tab(const DecArgs& a, int uu) const {
        return uu < units ? a.act_tab[uu / nsl] : make_int4(-1, 0, 0, 0);
    }
};

// Producer: one stage of one unit pass. `src` is lane r's activation row (r < nrows) for the
// gate_up operand copies (the token); the down operand is built by the quantisation warps.
// The weight copy goes first: it needs no lookup.
template <int MODE, bool PACKED>
__device__ __forceinline__ void dec_produce(const DecArgs& a, DSmem& sm, const CUtensorMap* tmw,
                                            int st, int e, int sl, int p0, int nrows, int chunk,
                                            int nchunk, int src) {
    const int lane = threadIdx.x & 31;
    DMeta& m = sm.meta[st];
    DStage& S = sm.st[st];
    constexpr uint32_t kActBytes = MODE == kGateUp ? kDSpi * 128 + kDSpi * 4 : 0;
    if (lane == 0) {
        m.e = e;
        m.sl = sl;
        m.p0 = p0;
        m.nrows = nrows;
        m.chunk = chunk;
        m.last = chunk == nchunk - 1;
        uint64_t* fb = &sm.full[st];
        mbar_expect_tx(fb, (PACKED ? kPackBlock : 2 * 128 * 128) + (uint32_t)nrows * kActBytes);
        if (PACKED) {
            const int nsl = MODE == kGateUp ? a.I / 64 : a.H / 128;
            const int64_t blk = ((int64_t)e * nsl + sl) * nchunk + chunk;
            bulk_load(&S.wt[0][0], a.packed + blk * kPackBlock, kPackBlock, fb);
        } else {
            const int kx = chunk * 256;  // byte column of the chunk's first half
            if (MODE == kGateUp) {
                const int yg = e * a.N + sl * 64, yu = e * a.N + a.I + sl * 64;
                tma_load_2d(&S.wt[0][0], tmw, kx, yg, fb);
                tma_load_2d(&S.wt[0][64 * 128], tmw, kx, yu, fb);
                tma_load_2d(&S.wt[1][0], tmw, kx + 128, yg, fb);
                tma_load_2d(&S.wt[1][64 * 128], tmw, kx + 128, yu, fb);
            } else {
                const int y = e * a.N + sl * 128;
                tma_load_2d(&S.wt[0][0], tmw, kx, y, fb);
                tma_load_2d(&S.wt[1][0], tmw, kx + 128, y, fb);
            }
        }
    }
    if (!PACKED) {
#pragma unroll
        for (int i = 0; i < 4; ++i) {  // scales: 128 rows x 4 groups (8 B each)
            const int r = lane + 32 * i;
            const int n = unit_row<MODE>(a, sl, r);
            cp_async8_bar(&S.sc[r][0], a.scales + ((int64_t)e * a.N + n) * a.G + chunk * kDSpi, true);
        }
        if (lane < 16) {  // zero points: 16 words (8 rows each) x 4 groups
            const int n8 = unit_row<MODE>(a, sl, lane * 8) >> 3;
            const bool zok = a.zeros != nullptr;
            cp_async16_bar(&S.zr[lane][0],
                           zok ? (const void*)(a.zeros + ((int64_t)e * (a.N / 8) + n8) * a.G + chunk * kDSpi)
                               : (const void*)a.scales,
                           zok);
        }
    }
    __syncwarp();  // expect_tx precedes every lane's bulk copy
    if (MODE == kGateUp && lane < nrows) {
        bulk_load(&S.act[lane][0], a.xe + (int64_t)src * a.xe_stride + (int64_t)chunk * kDSpi * 128,
                  kDSpi * 128, &sm.full[st]);
        bulk_load(&S.xs[lane][0], a.xsum + (int64_t)src * a.xs_stride + chunk * kDSpi, kDSpi * 4,
                  &sm.full[st]);
    }
    if (PACKED) {
        if (lane == 0) mbar_arrive(&sm.full[st]);
    } else {
        cp_async_arrive(&sm.full[st]);
    }
}


// Down-operand quantisation warp: the 512-wide chunk `chunk` of SiLU row p (fp16, written by the
// gate_up launch) with scale max(amax[p], 4.48e-6) / 448 -> stage row r: e4m3 bytes in GEMV
// order, group sums S, scale. Lane l handles 8-element units l and l + 32. The row's data is
// fetched (fetch_row) before the stage slot is free, so its latency overlaps the wait.
struct QRow {
    float amax;
    uint4 v0, v1;
};
__device__ __forceinline__ QRow fetch_row(const DecArgs& a, int p, int chunk) {
    const int lane = threadIdx.x & 31;
    const uint4* src = reinterpret_cast<const uint4*>(a.silu + (int64_t)p * a.I + (int64_t)chunk * 512);
    QRow q;
    q.amax = __uint_as_float(__ldcg(reinterpret_cast<const unsigned*>(a.amax) + p));
    q.v0 = __ldcg(src + lane);
    q.v1 = __ldcg(src + lane + 32);
    return q;
}
template <class Stage>
__device__ __forceinline__ void quant_stage_row(Stage& S, int r, const QRow& row) {
    const int lane = threadIdx.x & 31;
    const float s = __fdiv_rn(fmaxf(row.amax, kAmaxFloor), kE4m3Max);
    const float rcp = __frcp_rn(s);
#pragma unroll
    for (int k = 0; k < 2; ++k) {
        const uint4 v = k ? row.v1 : row.v0;
        const uint32_t w[4] = {v.x, v.y, v.z, v.w};
        uint32_t q[2];
        float sum = 0.f;
#pragma unroll
        for (int j = 0; j < 4; j += 2) {
            const float2 f0 = __half22float2(*reinterpret_cast<const __half2*>(&w[j]));
            const float2 f1 = __half22float2(*reinterpret_cast<const __half2*>(&w[j + 1]));
            const uint16_t p0 = quant_pair(f0.x, f0.y, s, rcp);
            const uint16_t p1 = quant_pair(f1.x, f1.y, s, rcp);
            q[j / 2] = (uint32_t)p0 | ((uint32_t)p1 << 16);
            const uint32_t e0 = e4m3x2_to_f16x2(p0), e1 = e4m3x2_to_f16x2(p1);
            const float2 d0 = __half22float2(*reinterpret_cast<const __half2*>(&e0));
            const float2 d1 = __half22float2(*reinterpret_cast<const __half2*>(&e1));
            sum += (d0.x + d0.y) + (d1.x + d1.y);
        }
        const int unit = lane + 32 * k;  // 8-element unit of the chunk; group = unit / 16
        *reinterpret_cast<uint2*>(&S.act[r][unit * 8]) =
            make_uint2(prmt(q[0], q[1], 0x6420u), prmt(q[0], q[1], 0x7531u));
#pragma unroll
        for (int o = 8; o > 0; o >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, o);
        if ((lane & 15) == 0) S.xs[r][unit / 16] = sum;
    }
    if (lane == 0) S.asc[r] = s;
}

// mma.sync m16n8k32 with e4m3 operands, D = A*B + D.
__device__ __forceinline__ void mma_e4m3(float (&d)[4], const uint32_t (&a)[4], uint32_t b0,
                                         uint32_t b1) {
    asm("mma.sync.aligned.m16n8k32.row.col.f32.e4m3.e4m3.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, "
        "{%8,%9}, {%0,%1,%2,%3};"
        : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

// One warp's share of one stage: tile rows r0 (first 8 MMA rows) and r1 (last 8), ntg token
// groups of 8; accumulates into tot[tg][4].
//
// Weights. Thread (g, t) loads 16 bytes (4 words, codes [32t, 32t+32) of the 128-group) of
// rows r0 and r1; MMA i takes word i. Of a word w (codes c0..c7, nibble k = code k) one LOP3
// each forms four e4m3 operands:
//   L_e = (w & 0x07070707) | 0x50505050 -> bytes 8 + (c & 7) of codes 0,2,4,6   (exact)
//   V_e = (w & 0x08080808) | 0x50505050 -> bytes 8 + 8 * (c >> 3) of the same codes
//   L_o, V_o: the same on w >> 4, codes 1,3,5,7
// so L + V = 16 + c, and the two MMAs (A = L, A = V) on the same activations accumulate
//   acc = sum_k c_k a_k + 16 S,   S = sum_k a_k  (the group's e4m3 activation sum).
// Activations: the operand quantiser stores each 8-element unit as elements 0,2,4,6,1,3,5,7,
// so b0/b1 of MMA i are the unit of word i (same permutation on both sides of the dot
// product). The group fold is tot += scale * (acc - (16 + z) * S).
template <int NTG>
__device__ __forceinline__ void dec_compute_t(const DStage& S, int r0, int r1, bool has_z,
                                              float (&tot)[2][4]) {
    const int lane = threadIdx.x & 31;
    const int c = lane & 3, tok = lane >> 2;
    const int sh0 = (r0 & 7) * 4, sh1 = (r1 & 7) * 4;
#pragma unroll
    for (int j = 0; j < kDSpi; ++j) {
        const uint8_t* wh = &S.wt[j >> 1][0];
        const int u = (j & 1) * 4 + c;
        const uint4 q0 = *reinterpret_cast<const uint4*>(wh + r0 * 128 + ((u ^ (r0 & 7)) << 4));
        const uint4 q1 = *reinterpret_cast<const uint4*>(wh + r1 * 128 + ((u ^ (r1 & 7)) << 4));
        const uint32_t w0[4] = {q0.x, q0.y, q0.z, q0.w};
        const uint32_t w1[4] = {q1.x, q1.y, q1.z, q1.w};
        uint4 b[NTG][2];
#pragma unroll
        for (int tg = 0; tg < NTG; ++tg) {
            const uint8_t* ar = &S.act[tg * 8 + tok][j * 128 + c * 32];
            b[tg][0] = *reinterpret_cast<const uint4*>(ar);
            b[tg][1] = *reinterpret_cast<const uint4*>(ar + 16);
        }
        float z0 = 8.f, z1 = 8.f;
        if (has_z) {
            z0 = __uint_as_float(0x4B000000u | ((S.zr[r0 >> 3][j] >> sh0) & 0xF)) - 8388608.f;
            z1 = __uint_as_float(0x4B000000u | ((S.zr[r1 >> 3][j] >> sh1) & 0xF)) - 8388608.f;
        }
        const float s0 = __half2float(S.sc[r0][j]);
        const float s1 = __half2float(S.sc[r1][j]);
        float acc[NTG][2][4] = {};
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            constexpr uint32_t kL = 0x07070707u, kV = 0x08080808u, kE = 0x50505050u;
            const uint32_t o0 = w0[i] >> 4, o1 = w1[i] >> 4;
            const uint32_t aL[4] = {and_or(w0[i], kL, kE), and_or(w1[i], kL, kE), and_or(o0, kL, kE),
                                    and_or(o1, kL, kE)};
            const uint32_t aV[4] = {and_or(w0[i], kV, kE), and_or(w1[i], kV, kE), and_or(o0, kV, kE),
                                    and_or(o1, kV, kE)};
#pragma unroll
            for (int tg = 0; tg < NTG; ++tg) {
                const uint32_t bl = (i & 1) ? (i & 2 ? b[tg][1].z : b[tg][0].z)
                                            : (i & 2 ? b[tg][1].x : b[tg][0].x);
                const uint32_t bh = (i & 1) ? (i & 2 ? b[tg][1].w : b[tg][0].w)
                                            : (i & 2 ? b[tg][1].y : b[tg][0].y);
                mma_e4m3(acc[tg][0], aL, bl, bh);
                mma_e4m3(acc[tg][1], aV, bl, bh);
            }
        }
#pragma unroll
        for (int tg = 0; tg < NTG; ++tg) {
            const float sa = S.xs[tg * 8 + 2 * c][j], sb = S.xs[tg * 8 + 2 * c + 1][j];
            const float za = 16.f + z0, zb = 16.f + z1;
            tot[tg][0] = fmaf(s0, fmaf(-za, sa, acc[tg][0][0] + acc[tg][1][0]), tot[tg][0]);
            tot[tg][1] = fmaf(s0, fmaf(-za, sb, acc[tg][0][1] + acc[tg][1][1]), tot[tg][1]);
            tot[tg][2] = fmaf(s1, fmaf(-zb, sa, acc[tg][0][2] + acc[tg][1][2]), tot[tg][2]);
            tot[tg][3] = fmaf(s1, fmaf(-zb, sb, acc[tg][0][3] + acc[tg][1][3]), tot[tg][3]);
        }
    }
}

__device__ __forceinline__ void dec_compute(const DStage& S, int r0, int r1, int ntg, bool has_z,
                                            float (&tot)[2][4]) {
    if (ntg > 1) dec_compute_t<2>(S, r0, r1, has_z, tot);
    else dec_compute_t<1>(S, r0, r1, has_z, tot);
}

// atomicAdd with acquire-release semantics at GPU scope: orders this warp's earlier stores
// (made visible to it by a __syncwarp) before the count, and the rows counted by other
// arrivals before this thread's later loads. The warp need not wait for the result.
__device__ __forceinline__ int atomic_add_acq_rel_gpu(int* p, int v) {
    int old;
    asm volatile("atom.add.acq_rel.gpu.s32 %0, [%1], %2;" : "=r"(old) : "l"(p), "r"(v) : "memory");
    return old;
}

__device__ __forceinline__ int ld_acquire_gpu(const int* p) {
    int v;
    asm volatile("ld.acquire.gpu.global.s32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}

// out[t, n .. n+7] = sum_{j ascending} w[t, j] * out2[row(t, j), n .. n+7], fp32 multiply then
// add (the oracle's slot-order reduce); the rows come from L2 (written by other CTAs).
__device__ __forceinline__ void combine8(const DecArgs& a, int t, int n) {
    float acc[8] = {};
    for (int j0 = 0; j0 < a.top_k; j0 += 8) {  // eight slots' rows in flight at once
        int pos[8];
        float wt[8];
        uint4 v[8];
#pragma unroll
        for (int q = 0; q < 8; ++q) {
            const bool ok = j0 + q < a.top_k;
            pos[q] = ok ? __ldg(a.slot_pos + t * a.top_k + j0 + q) : -1;
            wt[q] = ok ? __ldg(a.topk_w + (int64_t)t * a.ids_stride + j0 + q) : 0.f;
        }
#pragma unroll
        for (int q = 0; q < 8; ++q)
            if (pos[q] >= 0)
                v[q] = __ldcg(reinterpret_cast<const uint4*>(a.out2 + (int64_t)pos[q] * a.H + n));
#pragma unroll
        for (int q = 0; q < 8; ++q) {
            if (pos[q] < 0) continue;
            const uint32_t u[4] = {v[q].x, v[q].y, v[q].z, v[q].w};
#pragma unroll
            for (int c = 0; c < 4; ++c) {
                const float2 f = __half22float2(*reinterpret_cast<const __half2*>(&u[c]));
                acc[2 * c] = __fadd_rn(acc[2 * c], __fmul_rn(wt[q], f.x));
                acc[2 * c + 1] = __fadd_rn(acc[2 * c + 1], __fmul_rn(wt[q], f.y));
            }
        }
    }
    if (a.out_f32) {
        float4* o = reinterpret_cast<float4*>(static_cast<float*>(a.out) + (int64_t)t * a.H + n);
        o[0] = make_float4(acc[0], acc[1], acc[2], acc[3]);
        o[1] = make_float4(acc[4], acc[5], acc[6], acc[7]);
    } else {
        uint4 h;
        uint32_t* hw = reinterpret_cast<uint32_t*>(&h);
#pragma unroll
        for (int c = 0; c < 4; ++c) {
            const __half2 p = __floats2half2_rn(acc[2 * c], acc[2 * c + 1]);
            hw[c] = *reinterpret_cast<const uint32_t*>(&p);
        }
        *reinterpret_cast<uint4*>(static_cast<__half*>(a.out) + (int64_t)t * a.H + n) = h;
    }
}

// out[t, n, n+1] = fp16(sum_{j ascending} w[t, j] * out2[row(t, j), n, n+1]), fp32 multiply
// then add (the oracle's slot-order reduce); rows are fetched four slots at a time.
constexpr int kCombMaxK = 16;
__device__ __forceinline__ void combine_pair(const DecArgs& a, int t, int n) {
    float acc0 = 0.f, acc1 = 0.f;
    for (int j0 = 0; j0 < a.top_k; j0 += 4) {
        int pos[4];
        float wt[4];
        uint32_t v[4];
#pragma unroll
        for (int q = 0; q < 4; ++q) {
            const bool ok = j0 + q < a.top_k;
            pos[q] = ok ? __ldg(a.slot_pos + t * a.top_k + j0 + q) : -1;
            wt[q] = ok ? __ldg(a.topk_w + (int64_t)t * a.ids_stride + j0 + q) : 0.f;
        }
#pragma unroll
        for (int q = 0; q < 4; ++q)
            if (pos[q] >= 0)
                v[q] = __ldcg(reinterpret_cast<const unsigned*>(a.out2 + (int64_t)pos[q] * a.H + n));
#pragma unroll
        for (int q = 0; q < 4; ++q) {
            if (pos[q] >= 0) {
                const float2 f = __half22float2(*reinterpret_cast<const __half2*>(&v[q]));
                acc0 = __fadd_rn(acc0, __fmul_rn(wt[q], f.x));
                acc1 = __fadd_rn(acc1, __fmul_rn(wt[q], f.y));
            }
        }
    }
    if (a.out_f32)
        *reinterpret_cast<float2*>(static_cast<float*>(a.out) + (int64_t)t * a.H + n) =
            make_float2(acc0, acc1);
    else
        *reinterpret_cast<__half2*>(static_cast<__half*>(a.out) + (int64_t)t * a.H + n) =
            __floats2half2_rn(acc0, acc1);
}

// The previous pass's arrivals: every lane whose count completed its (token, chunk) has the
// warp sum that token's slot rows over the chunk's 16 channels.
__device__ __forceinline__ void resolve_pending(const DecArgs& a, int old, int t, int chunk,
                                                int ns, int lane) {
    const bool mine = old >= 0 && old == ns - 1;  // (token t, chunk) completed by this lane
    unsigned todo = __ballot_sync(0xffffffffu, mine);
    if (!todo) return;
    __threadfence();  // the other arrivals' rows (paired with their release)
    // four (token, chunk) items at a time: lanes 8i .. 8i+7 take the i-th remaining item
    while (todo) {
        const unsigned src = __fns(todo, 0, (lane >> 3) + 1);  // 0xffffffff: no such item
        const int tt = __shfl_sync(0xffffffffu, t, src & 31);
        const int cc = __shfl_sync(0xffffffffu, chunk, src & 31);
        if (src < 32) combine_pair(a, tt, cc * 16 + 2 * (lane & 7));
#pragma unroll
        for (int i = 0; i < 4; ++i) todo &= todo - 1;
    }
}

template <int MODE, bool PACKED>
__global__ void __launch_bounds__(kDThreads, 1)
decode_gemv_kernel(const DecArgs a, const __grid_constant__ CUtensorMap tmw) {
    extern __shared__ uint8_t smem_raw[];
    DSmem& sm = *reinterpret_cast<DSmem*>(smem_raw +
                                          ((1024u - (smem_u32(smem_raw) & 1023u)) & 1023u));
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    volatile int* bad = &sm.bad;
    const int nsl = MODE == kGateUp ? a.I / 64 : a.H / 128;
    const int n_active = a.meta[kMetaActive];
    const int units = n_active * nsl;
    const int nchunk = (int)(a.K / 512);
    // full: the producer's expect_tx arrive + its completion arrive (packed) or 32 cp.async
    // arrivals (op layout), + one arrival of the stage's quantisation warp (down)
    constexpr uint32_t kQuantArrive = MODE == kDown ? 1 : 0;
    if (threadIdx.x == 0) {
        sm.bad = 0;
        for (int s = 0; s < kDStages; ++s) {
            mbar_init(&sm.full[s], (PACKED ? 2 : 1 + 32) + kQuantArrive);
            mbar_init(&sm.empty[s], kDW);
        }
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    __syncthreads();
    const UnitWalk walk{0, units, nsl};
    const int G = gridDim.x;
    uint32_t st = 0, ph = 0;
    if (warp == kDW) {
        // ---------------- producer ----------------
        // The unit table entry of the unit after next and the first pass's token rows of the
        // next unit are loaded while the current unit's stages are issued.
        auto src_of = [&](int p, int end) {  // lane's token row for the pass at p (gate_up)
            const int q = p + lane;
            return (MODE == kGateUp && q < end) ? a.sorted_tok[q] : 0;
        };
        int n_issued = 0;
        int n_iss = 0;
        int4 cur = walk.tab(a, blockIdx.x);
        int4 nxt = walk.tab(a, blockIdx.x + G);
        int src_cur = cur.x >= 0 ? src_of(cur.y, cur.z) : 0;
        for (int u = blockIdx.x; u < units; u += G) {
            const int4 nn = walk.tab(a, u + 2 * G);
            const int src_nxt = nxt.x >= 0 ? src_of(nxt.y, nxt.z) : 0;
            const int e = cur.x, sl = u % nsl, q0 = cur.y, q1 = cur.z;
            for (int p0 = q0; p0 < q1; p0 += kDMaxRows) {
                const int nrows = min(kDMaxRows, q1 - p0);
                const int src = p0 == q0 ? src_cur : src_of(p0, q1);
                for (int ch = 0; ch < nchunk; ++ch) {
                    if (lane == 0) mbar_wait(&sm.empty[st], ph ^ 1, bad);
                    __syncwarp();
                    if (lane == 0) DEC_TRACE(MODE, n_issued, 0);
                    ++n_issued;
                    dec_produce<MODE, PACKED>(a, sm, &tmw, (int)st, e, sl, p0, nrows, ch, nchunk,
                                              src);
                    if (++st == kDStages) {
                        st = 0;
                        ph ^= 1;
                    }
                }
            }
            cur = nxt;
            nxt = nn;
            src_cur = src_nxt;
        }
        // a sentinel stage tells the compute warps to stop
        if (lane == 0) mbar_wait(&sm.empty[st], ph ^ 1, bad);
        __syncwarp();
        if (lane == 0) {
            sm.meta[st].e = -1;
            mbar_arrive(&sm.full[st]);
            if (PACKED) mbar_arrive(&sm.full[st]);
        }
        if (!PACKED) cp_async_arrive(&sm.full[st]);
        if (*bad && lane == 0) {
            const uint64_t t0 = global_ns();
            for (int s = 0; s < kDStages; ++s)
                while (!mbar_try(&sm.full[s], ph ^ (s <= (int)st ? 0u : 1u)) &&
                       global_ns() - t0 < kWaitLimitNs) {
                }
        }
    } else if (warp > kDW) {
        // ---------------- down: operand quantisation warps (stages alternate between them) ---
        if (MODE == kDown) {
            const int qw = warp - kDW - 1;  // 0 or 1
            int stage_no = 0;
            for (int u = blockIdx.x; u < units; u += G) {
                const int4 cur = walk.tab(a, u);
                for (int p0 = cur.y; p0 < cur.z; p0 += kDMaxRows) {
                    const int nrows = min(kDMaxRows, cur.z - p0);
                    for (int ch = 0; ch < nchunk; ++ch, ++stage_no) {
                        if ((stage_no & 1) == qw) {
                            QRow q0 = fetch_row(a, p0, ch);
                            QRow q1 = fetch_row(a, p0 + (nrows > 1 ? 1 : 0), ch);
                            if (lane == 0) mbar_wait(&sm.empty[st], ph ^ 1, bad);
                            __syncwarp();
                            for (int r = 0; r < nrows; r += 2) {
                                const QRow c0 = q0, c1 = q1;
                                if (r + 2 < nrows) {  // next pair in flight during this pair
                                    q0 = fetch_row(a, p0 + r + 2, ch);
                                    q1 = fetch_row(a, p0 + (r + 3 < nrows ? r + 3 : r + 2), ch);
                                }
                                quant_stage_row(sm.st[st], r, c0);
                                if (r + 1 < nrows) quant_stage_row(sm.st[st], r + 1, c1);
                            }
                            __syncwarp();
                            if (lane == 0) mbar_arrive(&sm.full[st]);
                        }
                        if (++st == kDStages) {
                            st = 0;
                            ph ^= 1;
                        }
                    }
                }
            }
            // the sentinel stage: the second quantisation arrival
            if ((stage_no & 1) == qw) {
                if (lane == 0) mbar_wait(&sm.empty[st], ph ^ 1, bad);
                __syncwarp();
                if (lane == 0) mbar_arrive(&sm.full[st]);
            }
        }
    } else {
        // ---------------- compute warps ----------------
        const int c = lane & 3, tok = lane >> 2;
        int r0, r1;
        if (MODE == kGateUp) {
            r0 = warp * 8 + tok;
            r1 = 64 + warp * 8 + tok;
        } else {
            r0 = warp * 16 + tok;
            r1 = warp * 16 + 8 + tok;
        }
        float tot[2][4] = {};
        int pend_old = -1, pend_t = 0, pend_chunk = 0, pend_nslot = 0;  // down: pending arrival
        int n_done = 0;
        for (;;) {
            mbar_wait(&sm.full[st], ph, bad);
            __syncwarp();
            if (warp == 0 && lane == 0) DEC_TRACE(MODE, n_done, 1);
            const DMeta& m = sm.meta[st];
            const int e = m.e;
            if (e < 0 || *bad) break;
            const int ntg = (m.nrows + 7) >> 3;
            const int sl = m.sl, p0 = m.p0, nrows = m.nrows;
            const bool last = m.last;
            // epilogue operands, requested before the stage's MMAs so their latency hides there
            float asc_c[2][2] = {};
            int my_t = 0, my_ns = 0;  // down: token of row `lane` and its valid slot count
            if (last) {
#pragma unroll
                for (int tg = 0; tg < 2; ++tg)
#pragma unroll
                    for (int q = 0; q < 2; ++q) {
                        const int rl = tg * 8 + 2 * c + q;
                        if (rl < nrows)
                            asc_c[tg][q] = MODE == kGateUp
                                               ? __ldg(a.asc + __ldg(a.sorted_tok + p0 + rl) * a.asc_stride)
                                               : sm.st[st].asc[rl];
                    }
                if (MODE == kDown && lane < nrows) {
                    my_t = __ldg(a.sorted_tok + p0 + lane);
                    my_ns = __ldg(a.nslot + my_t);
                }
            }
            if (m.chunk == 0) {
#pragma unroll
                for (int tg = 0; tg < 2; ++tg)
#pragma unroll
                    for (int v = 0; v < 4; ++v) tot[tg][v] = 0.f;
            }
            if (warp == 0 && lane == 0) DEC_TRACE(MODE, n_done, 3);
            dec_compute(sm.st[st], r0, r1, ntg, PACKED || a.zeros != nullptr, tot);
            __syncwarp();
            if (warp == 0 && lane == 0) DEC_TRACE(MODE, n_done, 2);
            __syncwarp();
            if (lane == 0) mbar_arrive(&sm.empty[st]);
            if (warp == 0 && lane == 0) DEC_TRACE(MODE, n_done, 2);
            ++n_done;
            if (++st == kDStages) {
                st = 0;
                ph ^= 1;
            }
            if (!last) continue;
            // ---- pass epilogue (warp-local: no barrier with the other warps) ----
            if (MODE == kGateUp) {
                // SiLU rows (fp16) and their per-row amax for the down operand's scale
                const int n = sl * 64 + warp * 8 + tok;  // gate channel == SiLU channel
#pragma unroll
                for (int tg = 0; tg < 2; ++tg) {
                    float mx[2] = {0.f, 0.f};
#pragma unroll
                    for (int q = 0; q < 2; ++q) {
                        const int rl = tg * 8 + 2 * c + q;
                        if (rl < nrows) {
                            const float as = asc_c[tg][q];
                            const __half h = silu_and_mul_half(tot[tg][q] * as, tot[tg][2 + q] * as);
                            a.silu[(int64_t)(p0 + rl) * a.I + n] = h;
                            mx[q] = fabsf(__half2float(h));
                        }
                    }
#pragma unroll
                    for (int q = 0; q < 2; ++q) {
#pragma unroll
                        for (int o = 4; o < 32; o <<= 1)
                            mx[q] = fmaxf(mx[q], __shfl_xor_sync(0xffffffffu, mx[q], o));
                        const int rl = tg * 8 + 2 * c + q;
                        if (tok == 0 && rl < nrows)
                            atomicMax(reinterpret_cast<unsigned*>(a.amax) + p0 + rl,
                                      __float_as_uint(mx[q]));
                    }
                }
            } else {
                const int n = sl * 128 + warp * 16 + tok;
#pragma unroll
                for (int tg = 0; tg < 2; ++tg)
#pragma unroll
                    for (int q = 0; q < 2; ++q) {
                        const int rl = tg * 8 + 2 * c + q;
                        if (rl < nrows) {
                            const float as = asc_c[tg][q];
                            __half* o = a.out2 + (int64_t)(p0 + rl) * a.H + n;
                            o[0] = __float2half_rn(tot[tg][q] * as);
                            o[8] = __float2half_rn(tot[tg][2 + q] * as);
                        }
                    }
                // per (token, 16-channel chunk) arrival of this warp's rows; the last arrival
                // of a chunk sums the token's slot rows there. The count's result is consumed
                // one pass later (or at the end), so the warp does not wait for it here.
                __syncwarp();
                resolve_pending(a, pend_old, pend_t, pend_chunk, pend_nslot, lane);
                pend_chunk = sl * 8 + warp;
                if (lane < nrows) {
                    pend_t = my_t;
                    pend_nslot = my_ns;
                    pend_old = atomic_add_acq_rel_gpu(
                        &a.tok_done[(int64_t)my_t * (a.H / 16) + pend_chunk], 1);
                } else {
                    pend_old = -1;
                }
            }
        }
        if (MODE == kDown) resolve_pending(a, pend_old, pend_t, pend_chunk, pend_nslot, lane);
    }
    __syncthreads();
    if (threadIdx.x == 0 && sm.bad) atomicOr(a.meta + kMetaErr, 2);
}

struct DecLayout {
    size_t off_off, off_active, off_tab, off_stok, off_meta, off_sorted, off_pos, off_nslot,
        off_amax, off_tokdone, off_xh1, off_xs1, off_sc1, off_silu, off_out2, off_xh2, off_xs2,
        off_sc2, total;
};

DecLayout dec_layout(int64_t T, int64_t top_k, int64_t E, int64_t H, int64_t I) {
    DecLayout L{};
    const int64_t S = T * top_k;
    size_t o = 0;
    auto take = [&](size_t bytes) {
        const size_t at = o;
        o += align_up(std::max<size_t>(bytes, 1), 256);
        return at;
    };
    L.off_off = take((size_t)(E + 1) * 4);
    L.off_active = take((size_t)E * 4);
    L.off_tab = take((size_t)E * 16);
    L.off_stok = take((size_t)S * 4);
    L.off_meta = take(kMetaWords * 4);
    L.off_sorted = take((size_t)S * 4);
    L.off_pos = take((size_t)S * 4);
    L.off_nslot = take((size_t)T * 4);
    L.off_amax = take((size_t)S * 4);
    L.off_tokdone = take((size_t)T * (H / 16) * 4);
    L.off_xh1 = take((size_t)T * H);
    L.off_xs1 = take((size_t)T * (H / 128) * 4);
    L.off_sc1 = take((size_t)T * 4);
    L.off_silu = take((size_t)S * I * 2);
    L.off_out2 = take((size_t)S * H * 2);
    L.off_xh2 = take((size_t)S * I);            // the down operand (tensor-core path)
    L.off_xs2 = take((size_t)S * (I / 128) * 4);
    L.off_sc2 = take((size_t)S * 4);
    L.total = o;
    return L;
}

int sm_count_dev() {
    int dev = 0, n = 0;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
    return n > 0 ? n : 148;
}

template <int MODE, bool PACKED>
int launch_dec_gemv_t(const DecArgs& a, int units_max, cudaStream_t st) {
    CUtensorMap tmw{};
    if (!PACKED) {
        const uint32_t box_rows = MODE == kGateUp ? 64 : 128;
        if (!make_tma_map_u8(&tmw, a.w, (uint64_t)a.E * a.N, (uint64_t)a.K / 2, 128, box_rows,
                             CU_TENSOR_MAP_SWIZZLE_128B))
            return set_error("moe_decode: tensor map encoding failed");
    }
    const size_t smem = sizeof(DSmem) + 1024;
    cudaError_t ce = cudaFuncSetAttribute(decode_gemv_kernel<MODE, PACKED>,
                                          cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (ce != cudaSuccess) return (int)ce;
    const int grid = std::max(1, std::min(units_max, sm_count_dev()));
    decode_gemv_kernel<MODE, PACKED><<<grid, kDThreads, smem, st>>>(a, tmw);
    return launch_status();
}


// ---------------------------------------------------------------------------------------
// The decode GEMV on the 5th-generation tensor cores (prepacked weights).
//
// Roles (16 warps): 8 math warps, 1 producer (as above), 1 MMA warp (owns the tensor memory;
// lane 0 issues), 2 down-operand quantisation warps, 4 epilogue warps. Per stage (128 weight
// rows x 512 K), in two half-stages of two 128-groups:
//   - the math warps copy the stage's token rows into four SW128 K-major B tiles (16 rows x
//     128 K each); per group each thread expands a quarter of its weight row's 128 codes
//     (thread = weight row = TMEM lane; the quarters are warps w, w + 4, w + 8, w + 12; four
//     warps per scheduler hide the expansion's latency) to their exact e4m3 values
//     (codes8_to_e4m3; the prepack stores each word's codes in the operand's byte order) and
//     stores them to one of three tensor-memory A buffers (tcgen05.st);
//   - the MMA thread issues per group 4 x tcgen05.mma.kind::f8f6f4 (M 128, N 16, K 32; A from
//     tensor memory, B from shared memory) into one of four accumulator buffers and commits
//     per half-stage (and, after the stage's second half, to the stage's empty barrier). On
//     B200 such an MMA occupies the tensor pipe about 48 cycles whatever N <= 64, so one MMA
//     per 32 K (not the two a split of the codes would need) keeps it under the HBM rate;
//   - the math warps fold the accumulators of half-stage hc - 2 (tcgen05.ld) into fp32
//     registers, tot += scale * (acc - z * S), while the MMAs of hc - 1 and hc run;
//   - at a pass end the math warps write tot to a shared-memory tile and the epilogue warps
//     do the global work (SiLU-and-mul, row amax, down rows, combine arrivals), so no math
//     warp waits on global memory.
// A gate_up block interleaves gate and up rows (w4a8_stream_pack), so SiLU-and-mul is one
// shuffle between adjacent lanes; a down block's 16-channel chunks lie inside one warp.
// ---------------------------------------------------------------------------------------
constexpr int kTW = 16;                       // math warps
constexpr int kTQ = kTW / 4;                  // math warps per TMEM lane quarter
constexpr int kTCodes = 128 / kTQ;            // codes of a 128-group one thread expands
constexpr int kTE = 4;                        // fold warps (one per TMEM lane quarter)
constexpr int kTThreads = (kTW + 2 + kTE) * 32;  // + producer, MMA, fold warps
constexpr int kTStages = 4;
constexpr int kTN = 16;                       // token columns per MMA (= kDMaxRows)
constexpr int kTHalf = kDSpi / 2;             // groups per half-stage
constexpr int kTABufs = 3;                    // A buffers (half-stages in flight)
constexpr int kTDBufs = 4;                    // accumulator buffers
constexpr uint32_t kTmemCols = 512;           // A: 3 x 2 groups x 32 = 192 columns;
constexpr uint32_t kDCol0 = kTABufs * kTHalf * 32;  // D: 4 x 2 groups x 16 = 128 columns
static_assert(kDCol0 + kTDBufs * kTHalf * kTN <= kTmemCols, "tensor memory overflow");

struct alignas(1024) TStage {
    uint8_t wt[2][128 * 128];                 // the packed block: codes, scales, zero points
    __half sc[128][kDSpi];
    uint32_t zr[16][kDSpi];
    uint8_t pad_[34816 - 34048];
    uint8_t bsw[kDSpi][kTN * 128];            // B tiles per 128-group, SW128 K-major (1024-aligned)
    uint8_t act[kDMaxRows][kDActStride];      // token rows as copied / quantised (linear)
    float xs[kDMaxRows][kDSpi];               // S per (row, group)
    float asc[kDMaxRows];                     // down: activation scale per row
};
static_assert(offsetof(TStage, bsw) % 1024 == 0, "B tiles must be 1024-byte aligned");

struct TSmem {
    TStage st[kTStages];
    DMeta meta[kTStages];
    uint64_t full[kTStages];
    uint64_t empty[kTStages];
    uint64_t afull[kTABufs], dfull[kTDBufs], dempty[kTDBufs];
    uint32_t tmem_base;
    int bad;
};

__device__ __forceinline__ void umma_f8(uint32_t d, uint32_t a_tmem, uint64_t b_desc,
                                        uint32_t idesc, uint32_t acc) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f8f6f4 [%0], [%1], %2, %3, p;\n\t}" ::"r"(d),
        "r"(a_tmem), "l"(b_desc), "r"(idesc), "r"(acc));
}
__device__ __forceinline__ void umma_commit(uint64_t* bar) {
    asm volatile(
        "tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
            smem_u32(bar)));
}

// Grid barrier of a cooperative launch on the counter meta[kMetaSync] (zeroed by the prep
// launch): each CTA adds one, then waits until it reaches `target` (gridDim.x times the barrier's
// ordinal). Gives up after kWaitLimitNs, setting the error word and *bad.
__device__ __forceinline__ void grid_barrier(const DecArgs& a, int target, volatile int* bad) {
    __syncthreads();
    if (threadIdx.x == 0) {
        __threadfence();
        atomicAdd(a.meta + kMetaSync, 1);
        const uint64_t t0 = global_ns();
        while (ld_acquire_gpu(a.meta + kMetaSync) < target) {
            if (global_ns() - t0 > kWaitLimitNs) {
                atomicOr(a.meta + kMetaErr, 4);
                *bad = 1;
                break;
            }
            __nanosleep(64);
        }
        __threadfence();
    }
    __syncthreads();
    // the rows other CTAs stored are next read by bulk copies (the async proxy)
    asm volatile("fence.proxy.async.global;" ::: "memory");
}

template <int MODE>
__global__ void __launch_bounds__(kTThreads, 1)
decode_tc_kernel(const DecArgs a) {
    extern __shared__ uint8_t smem_raw[];
    TSmem& sm = *reinterpret_cast<TSmem*>(smem_raw +
                                          ((1024u - (smem_u32(smem_raw) & 1023u)) & 1023u));
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    volatile int* bad = &sm.bad;
    const int nsl = MODE == kGateUp ? a.I / 64 : a.H / 128;
    const int n_active = a.meta[kMetaActive];
    const int units = n_active * nsl;
    const int nchunk = (int)(a.K / 512);
    if (threadIdx.x == 0) {
        sm.bad = 0;
        for (int s = 0; s < kTStages; ++s) {
            mbar_init(&sm.full[s], 2);
            mbar_init(&sm.empty[s], kTE + 1);
        }
        for (int s = 0; s < kTABufs; ++s) mbar_init(&sm.afull[s], kTW);
        for (int s = 0; s < kTDBufs; ++s) {
            mbar_init(&sm.dfull[s], 1);
            mbar_init(&sm.dempty[s], kTE);
        }
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    if (warp == kTW + 1) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                         smem_u32(&sm.tmem_base)),
                     "r"(kTmemCols));
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::);
    }
    asm volatile("tcgen05.fence::before_thread_sync;" ::);
    __syncthreads();
    asm volatile("tcgen05.fence::after_thread_sync;" ::);
    const uint32_t tmem = sm.tmem_base;
    if (MODE == kDown) {
        // the down operand: every SiLU row quantised once (one warp per row over the grid),
        // then a grid barrier (the launch is cooperative, so every CTA is resident)
        const int rows = a.off[a.E];
        constexpr int kWarps = kTThreads / 32;
        for (int p = blockIdx.x * kWarps + warp; p < rows; p += gridDim.x * kWarps)
            quant_row_e4<true>(a.silu + (int64_t)p * a.I, a.I, p, const_cast<uint8_t*>(a.xe),
                               const_cast<float*>(a.xsum), const_cast<float*>(a.asc), nullptr);
        grid_barrier(a, (int)gridDim.x, &sm.bad);
    }
    const UnitWalk walk{0, units, nsl};
    const int G = gridDim.x;
    uint32_t st = 0, ph = 0;
    if (warp == kTW) {
        // ---------------- producer: the same stage stream as decode_gemv_kernel ----------------
        int n_iss = 0;
        auto src_of = [&](int p, int end) {
            const int q = p + lane;
            return q < end ? (MODE == kGateUp ? a.sorted_tok[q] : q) : 0;
        };
        // units are taken from a grid-wide counter (heavy experts come first in the unit
        // order). Three are queued: a counter result and a table entry are first used one
        // unit after they were requested, so a one-stage unit (down) does not wait on them.
        int* const ctr = a.meta + (MODE == kGateUp ? kMetaUnit1 : kMetaUnit2);
        auto grab = [&]() {
            int v = 0;
            if (lane == 0) v = atomicAdd(ctr, 1);
            return __shfl_sync(0xffffffffu, v, 0);
        };
        int u = grab();
        int u_nxt = u < units ? grab() : units;
        int u_nn = u_nxt < units ? grab() : units;
        int4 cur = walk.tab(a, u);
        int4 nxt = walk.tab(a, u_nxt);
        int src_cur = cur.x >= 0 ? src_of(cur.y, cur.z) : 0;
        while (u < units) {
            // lane 0's counter result: shuffled out only in the next iteration
            int pend = 0;
            if (lane == 0 && u_nn < units) pend = atomicAdd(ctr, 1);
            const int4 nn = walk.tab(a, u_nn);
            const int src_nxt = nxt.x >= 0 ? src_of(nxt.y, nxt.z) : 0;
            const int e = cur.x, sl = u % nsl, q0 = cur.y, q1 = cur.z;
            for (int p0 = q0; p0 < q1; p0 += kDMaxRows) {
                const int nrows = min(kDMaxRows, q1 - p0);
                const int src = p0 == q0 ? src_cur : src_of(p0, q1);
                for (int ch = 0; ch < nchunk; ++ch) {
                    if (lane == 0) mbar_wait(&sm.empty[st], ph ^ 1, bad);
                    __syncwarp();
                    if (lane == 0) DEC_TRACE(MODE, n_iss, 0);
                    ++n_iss;
                    DMeta& m = sm.meta[st];
                    TStage& S = sm.st[st];
                    if (lane == 0) {
                        m.e = e;
                        m.sl = sl;
                        m.p0 = p0;
                        m.nrows = nrows;
                        m.chunk = ch;
                        m.last = ch == nchunk - 1;
                        constexpr uint32_t kActBytes = kDSpi * 128 + kDSpi * 4;
                        mbar_expect_tx(&sm.full[st], kPackBlock + (uint32_t)nrows * kActBytes);
                        const int64_t blk = ((int64_t)e * nsl + sl) * nchunk + ch;
                        bulk_load(&S.wt[0][0], a.packed + blk * kPackBlock, kPackBlock, &sm.full[st]);
                    }
                    __syncwarp();
                    if (lane < nrows) {
                        bulk_load(&S.act[lane][0],
                                  a.xe + (int64_t)src * a.xe_stride + (int64_t)ch * kDSpi * 128,
                                  kDSpi * 128, &sm.full[st]);
                        bulk_load(&S.xs[lane][0], a.xsum + (int64_t)src * a.xs_stride + ch * kDSpi,
                                  kDSpi * 4, &sm.full[st]);
                    }
                    if (lane == 0) mbar_arrive(&sm.full[st]);
                    if (++st == kTStages) {
                        st = 0;
                        ph ^= 1;
                    }
                }
            }
            u = u_nxt;
            u_nxt = u_nn;
            u_nn = u_nn < units ? __shfl_sync(0xffffffffu, pend, 0) : units;
            cur = nxt;
            nxt = nn;
            src_cur = src_nxt;
        }
        if (lane == 0) mbar_wait(&sm.empty[st], ph ^ 1, bad);
        __syncwarp();
        if (lane == 0) {
            sm.meta[st].e = -1;
            mbar_arrive(&sm.full[st]);
            mbar_arrive(&sm.full[st]);
        }
    } else if (warp == kTW + 1) {
        // ---------------- MMA issuer: one handshake per half-stage ----------------
        if (lane == 0) {
            constexpr uint32_t idesc = umma_idesc(128, kTN);
            uint32_t hc = 0;  // half-stages issued
            uint32_t ab = 0, abph = 0;  // A buffer of half hc and its barrier phase
            for (;;) {
                        // the stage's metadata (the end marker has expert -1)
                        mbar_wait(&sm.full[st], ph, bad);
                        if (sm.meta[st].e < 0 || *bad) break;
                        const uint32_t b_base = smem_u32(&sm.st[st].bsw[0][0]);
                        for (int k = 0; k < 2; ++k, ++hc) {
                            const uint32_t db = hc % kTDBufs;
                            mbar_wait(&sm.afull[ab], abph, bad);
                            mbar_wait(&sm.dempty[db], ((hc / kTDBufs) & 1) ^ 1, bad);
                            asm volatile("tcgen05.fence::after_thread_sync;" ::);
#pragma unroll
                            for (int jj = 0; jj < kTHalf; ++jj) {
                                const int j = k * kTHalf + jj;
                                const uint32_t ta = tmem + (ab * kTHalf + jj) * 32;
                                const uint32_t d = tmem + kDCol0 + (db * kTHalf + jj) * kTN;
#pragma unroll
                                for (int kk = 0; kk < 4; ++kk) {
                                    const uint64_t dd = desc_sw128(b_base + j * (kTN * 128) + kk * 32);
                                    umma_f8(d, ta + kk * 8, dd, idesc, kk > 0 ? 1u : 0u);
                                }
                            }
                            umma_commit(&sm.dfull[db]);
                            if (k == 1) umma_commit(&sm.empty[st]);
                            if (++ab == kTABufs) {
                                ab = 0;
                                abph ^= 1;
                            }
                        }
                        if (++st == kTStages) {
                            st = 0;
                            ph ^= 1;
                        }
            }
        }
    } else if (warp >= kTW + 2) {
        // ---------------- fold warps ----------------
        // Warp fw = warp % 4 reads TMEM lane quarter fw: thread = weight row m, all token columns of the
        // pass. Per half-stage: the accumulators (only the pass's live columns) -> fp32 totals,
        // tot += scale * (acc - z * S); at a pass end the epilogue (gate_up: lanes 2c / 2c+1
        // hold gate / up of one channel; down: the fp16 down row of each token).
        static_assert(kTE == 4, "four consecutive fold warps, one per lane quarter");
        const int fw = warp & 3;  // a warp reaches TMEM lanes [32 (warp % 4), +32) only
        const int m = fw * 32 + lane;
        const uint32_t lane_base = (uint32_t)(fw * 32) << 16;
        const int sh = (m & 7) * 4;
        float tot[kTN];
#pragma unroll
        for (int t = 0; t < kTN; ++t) tot[t] = 0.f;
        uint32_t hc = 0;                                   // half-stages folded
        float asc_l = 0.f;                                 // lane t: the pass's row t scale
        for (;;) {
                    const uint32_t stage = hc >> 1;
                    const uint32_t slot = stage % kTStages;
                    if (lane == 0) mbar_wait(&sm.full[slot], (stage / kTStages) & 1, bad);
                    __syncwarp();
                    const DMeta md = sm.meta[slot];
                    if (md.e < 0 || *bad) break;
                    const int sl = md.sl, p0 = md.p0, nrows = md.nrows;
                    const TStage& P = sm.st[slot];
                    if (md.chunk == 0) {
                        // the pass's activation scales, needed only at its end (down: written
                        // by this launch, so not through the read-only path)
                        asc_l = lane < nrows
                            ? __ldcg(a.asc + (int64_t)(MODE == kGateUp ? __ldg(a.sorted_tok + p0 + lane)
                                                                       : p0 + lane) * a.asc_stride)
                            : 0.f;
                    }
                    for (int k = 0; k < 2; ++k, ++hc) {
                        const uint32_t db = hc % kTDBufs;
                        if (lane == 0) mbar_wait(&sm.dfull[db], (hc / kTDBufs) & 1, bad);
                        __syncwarp();
                        asm volatile("tcgen05.fence::after_thread_sync;" ::);
                        uint32_t v[kTHalf][kTN];
                        const uint32_t d0 = tmem + lane_base + kDCol0 + db * kTHalf * kTN;
                        if (nrows <= 4) {
#pragma unroll
                            for (int jj = 0; jj < kTHalf; ++jj)
                                tmem_ld4_nowait(d0 + jj * kTN, *reinterpret_cast<uint32_t(*)[4]>(&v[jj][0]));
                        } else {
#pragma unroll
                            for (int jj = 0; jj < kTHalf; ++jj) tmem_ld16_nowait(d0 + jj * kTN, v[jj]);
                        }
                        tmem_wait_ld();
                        asm volatile("tcgen05.fence::before_thread_sync;" ::);
                        __syncwarp();
                        if (lane == 0) mbar_arrive(&sm.dempty[db]);
                        static_assert(kTHalf == 2, "the fold reads group pairs");
                        const float2 sc = __half22float2(*reinterpret_cast<const __half2*>(&P.sc[m][2 * k]));
                        const uint2 zw = *reinterpret_cast<const uint2*>(&P.zr[m >> 3][2 * k]);
                        const float nz0 = -(float)((zw.x >> sh) & 0xF), nz1 = -(float)((zw.y >> sh) & 0xF);
                        auto fold = [&](auto ncols) {
#pragma unroll
                            for (int t = 0; t < decltype(ncols)::value; ++t) {
                                const float2 xs = *reinterpret_cast<const float2*>(&P.xs[t][2 * k]);
                                tot[t] = fmaf(sc.x, fmaf(nz0, xs.x, __uint_as_float(v[0][t])), tot[t]);
                                tot[t] = fmaf(sc.y, fmaf(nz1, xs.y, __uint_as_float(v[1][t])), tot[t]);
                            }
                        };
                        if (nrows <= 4) fold(std::integral_constant<int, 4>{});
                        else fold(std::integral_constant<int, kTN>{});
                    }
                    if (md.last) {
                        // the pass epilogue
                        if (MODE == kGateUp) {
                            const int nch = sl * 64 + 16 * fw + (lane >> 1);
#pragma unroll
                            for (int t = 0; t < kTN; ++t) {
                                if (t < nrows) {
                                    const float scl = __shfl_sync(0xffffffffu, asc_l, t);
                                    const float other = __shfl_xor_sync(0xffffffffu, tot[t], 1);
                                    if (!(lane & 1))
                                        a.silu[(int64_t)(p0 + t) * a.I + nch] =
                                            silu_and_mul_half(tot[t] * scl, other * scl);
                                }
                            }
                        } else {
                            // the down rows; the slot-order combine runs after the closing
                            // grid barrier
                            const int nch = sl * 128 + m;
#pragma unroll
                            for (int t = 0; t < kTN; ++t) {
                                if (t < nrows) {
                                    const float scl = __shfl_sync(0xffffffffu, asc_l, t);
                                    a.out2[(int64_t)(p0 + t) * a.H + nch] = __float2half_rn(tot[t] * scl);
                                }
                            }
                        }
#pragma unroll
                        for (int t = 0; t < kTN; ++t) tot[t] = 0.f;
                    }
                    __syncwarp();
                    if (lane == 0) mbar_arrive(&sm.empty[slot]);
        }
    } else {
        // ---------------- expansion warps ----------------
        // Half-stage hc (groups 2k, 2k+1 of a stage) goes to A buffer hc % 3, free once the
        // MMAs of half hc - 3 completed.
        const int q = warp & 3, h = warp >> 2;             // lane quarter, code quarter
        const int m = q * 32 + lane;                       // weight row = TMEM lane
        const uint32_t lane_base = (uint32_t)(q * 32) << 16;
        uint32_t n = 0;                                    // stages consumed
        uint32_t hc = 0;                                   // half-stages expanded
        uint32_t ab = 0;                                   // A buffer of half hc
        for (;;) {
            if (lane == 0) mbar_wait(&sm.full[st], ph, bad);
            __syncwarp();
            if (warp == 0 && lane == 0) DEC_TRACE(MODE, n, 1);
            const int e = sm.meta[st].e;
            if (e < 0 || *bad) break;
            TStage& S = sm.st[st];
            // token rows -> SW128 B tiles (16-byte unit u of row r at u ^ (r & 7)); the rows
            // from nrows on feed accumulator columns no one reads
            const int nb = sm.meta[st].nrows * (kDSpi * 8);
            for (int i = threadIdx.x; i < nb; i += kTW * 32) {
                const int r = i >> 5, v = i & 31, kb = v >> 3, uu = v & 7;
                *reinterpret_cast<uint4*>(&S.bsw[kb][r * 128 + ((uu ^ (r & 7)) << 4)]) =
                    *reinterpret_cast<const uint4*>(&S.act[r][v * 16]);
            }
            asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
            if (warp == 0 && lane == 0) DEC_TRACE(MODE, n, 4);
            for (int k = 0; k < 2; ++k, ++hc) {
                if (hc >= (uint32_t)kTABufs) {
                    const uint32_t hp = hc - kTABufs;
                    if (lane == 0) mbar_wait(&sm.dfull[hp % kTDBufs], (hp / kTDBufs) & 1, bad);
                    __syncwarp();
                    asm volatile("tcgen05.fence::after_thread_sync;" ::);
                }
#pragma unroll
                for (int jj = 0; jj < kTHalf; ++jj) {
                    const int j = k * kTHalf + jj;
                    // codes [32 h, 32 h + 32) of group j of row m: 16-byte unit h of the group
                    const uint8_t* wh = &S.wt[j >> 1][0];
                    const int u0 = (j & 1) * 4 + h;
                    const uint4 qa = *reinterpret_cast<const uint4*>(wh + m * 128 + ((u0 ^ (m & 7)) << 4));
                    const uint32_t w[4] = {qa.x, qa.y, qa.z, qa.w};
                    uint32_t A[8];
#pragma unroll
                    for (int i = 0; i < 4; ++i) codes8_to_e4m3_fma(w[i], a.one, a.m1, A[2 * i], A[2 * i + 1]);
                    tmem_st8(tmem + lane_base + (ab * kTHalf + jj) * 32 + 8 * h, A);
                }
                if (warp == 0 && lane == 0 && k == 0) DEC_TRACE(MODE, n, 5);
                asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
                asm volatile("tcgen05.fence::before_thread_sync;" ::);
                __syncwarp();
                if (lane == 0) mbar_arrive(&sm.afull[ab]);
                if (++ab == kTABufs) ab = 0;
                if (warp == 0 && lane == 0 && k == 0) DEC_TRACE(MODE, n, 3);
            }
            if (warp == 0 && lane == 0) DEC_TRACE(MODE, n, 2);
            ++n;
            if (++st == kTStages) {
                st = 0;
                ph ^= 1;
            }
        }
    }
    asm volatile("tcgen05.fence::before_thread_sync;" ::);
    __syncthreads();
    if (threadIdx.x == 0 && sm.bad) atomicOr(a.meta + kMetaErr, 2);
    if (warp == kTW + 1) {
        asm volatile("tcgen05.fence::after_thread_sync;" ::);
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem),
                     "r"(kTmemCols));
    }
    if (threadIdx.x == 0) DEC_TRACE(MODE, 0, 10);
    if (MODE == kDown) {
        // grid barrier (the launch is cooperative, so every CTA is resident), then the
        // slot-order combine of all tokens over the whole grid
        grid_barrier(a, 2 * (int)gridDim.x, &sm.bad);
        if (threadIdx.x == 0) DEC_TRACE(MODE, 0, 11);
        if (sm.bad) return;
        const int n8 = a.H / 8;
        const int items = a.T * n8;
        for (int i = blockIdx.x * kTThreads + threadIdx.x; i < items; i += gridDim.x * kTThreads)
            combine8(a, i / n8, (i % n8) * 8);
    }
}

template <int MODE>
int launch_dec_tc(const DecArgs& a, int units_max, cudaStream_t st) {
    static_assert(sizeof(TSmem) + 1024 <= 227 * 1024, "tensor-core decode shared memory");
    const size_t smem = sizeof(TSmem) + 1024;
    cudaError_t ce = cudaFuncSetAttribute(decode_tc_kernel<MODE>,
                                          cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (ce != cudaSuccess) return (int)ce;
    const int grid = std::max(1, std::min(units_max, sm_count_dev()));
    if (MODE == kDown) {
        // cooperative: the closing grid barrier needs every CTA resident (one per SM)
        DecArgs args = a;
        void* params[] = {&args};
        ce = cudaLaunchCooperativeKernel(reinterpret_cast<const void*>(decode_tc_kernel<MODE>),
                                         dim3(grid), dim3(kTThreads), params, smem, st);
        if (ce != cudaSuccess) return (int)ce;
        return launch_status();
    }
    decode_tc_kernel<MODE><<<grid, kTThreads, smem, st>>>(a);
    return launch_status();
}

template <int MODE>
int launch_dec_gemv(const DecArgs& a, int units_max, cudaStream_t st) {
    // prepacked weights: the tensor-core kernel; op layout: the mma.sync kernel
    return a.packed ? launch_dec_tc<MODE>(a, units_max, st)
                    : launch_dec_gemv_t<MODE, false>(a, units_max, st);
}

// ---------------------------------------------------------------------------------------
// Weight prepack for the decode GEMV: op layout -> one contiguous block per (expert, unit
// slice, 512-wide K chunk), in the exact shared-memory image of a DStage's weight part:
//   codes  [2 halves][128 rows][8 x 16 B], 16-byte unit u of row m stored at u ^ (m & 7)
//          (the 128-byte swizzle the compute warps read); within each 32-bit word the eight
//          codes are reordered c0 c2 c4 c6 c1 c3 c5 c7 (gemv_nibble_order);
//   scales [128 rows][4 groups] fp16;  zeros [16 (8-row words)][4 groups] u32 (8 when absent).
// Row m of a gate_up block is gate row sl*64 + m/2 (m even) or the matching up row
// inter + sl*64 + (m-1)/2 (m odd), so every gate/up pair sits in adjacent TMEM lanes.
// ---------------------------------------------------------------------------------------
// Codes c0..c7 of a word (nibble i = c_i) -> nibble order c0 c2 c4 c6 c1 c3 c5 c7, the GEMV
// byte order of the e4m3 operand rows, so that nibble i expands to operand byte i.
__device__ __forceinline__ uint32_t gemv_nibble_order(uint32_t w) {
    const uint32_t ev = w & 0x0F0F0F0Fu, od = (w >> 4) & 0x0F0F0F0Fu;  // c0 c2 c4 c6 / c1 c3 c5 c7
    const uint32_t e2 = (ev | (ev >> 4)) & 0x00FF00FFu, o2 = (od | (od >> 4)) & 0x00FF00FFu;
    return ((e2 | (e2 >> 8)) & 0xFFFFu) | (((o2 | (o2 >> 8)) & 0xFFFFu) << 16);
}

__global__ void __launch_bounds__(256)
stream_pack_kernel(const int32_t* __restrict__ w, const __half* __restrict__ scales,
                   const int32_t* __restrict__ zeros, int64_t K, int N, int G, int inter,
                   int nsl, int nch, uint8_t* __restrict__ packed) {
    const int64_t blk = blockIdx.x;
    const int ch = (int)(blk % nch);
    const int sl = (int)((blk / nch) % nsl);
    const int64_t e = blk / ((int64_t)nch * nsl);
    uint8_t* dst = packed + blk * kPackBlock;
    const uint8_t* wb = reinterpret_cast<const uint8_t*>(w);
    auto row_of = [&](int m) {  // gate_up: gate row 64 sl + m/2 (m even), its up row (m odd)
        if (inter > 0) return (m & 1) ? inter + sl * 64 + (m >> 1) : sl * 64 + (m >> 1);
        return sl * 128 + m;
    };
    for (int idx = threadIdx.x; idx < 2048; idx += blockDim.x) {
        const int h = idx >> 10, m = (idx >> 3) & 127, u = idx & 7;
        const int n = row_of(m);
        uint4 v = __ldg(reinterpret_cast<const uint4*>(
            wb + ((int64_t)e * N + n) * (K / 2) + (int64_t)ch * 256 + h * 128 + u * 16));
        v.x = gemv_nibble_order(v.x);
        v.y = gemv_nibble_order(v.y);
        v.z = gemv_nibble_order(v.z);
        v.w = gemv_nibble_order(v.w);
        *reinterpret_cast<uint4*>(dst + h * 16384 + m * 128 + ((u ^ (m & 7)) << 4)) = v;
    }
    if (threadIdx.x < 128) {
        const int m = threadIdx.x, n = row_of(m);
        const uint2 v = *reinterpret_cast<const uint2*>(scales + ((int64_t)e * N + n) * G + ch * 4);
        *reinterpret_cast<uint2*>(dst + 32768 + m * 8) = v;
    } else if (threadIdx.x < 144) {
        // zero points of block rows 8 m8 .. 8 m8 + 7, nibble (m % 8), 4 groups
        const int m8 = threadIdx.x - 128;
        uint32_t zw[4] = {0x88888888u, 0x88888888u, 0x88888888u, 0x88888888u};
        if (zeros) {
#pragma unroll
            for (int g = 0; g < 4; ++g) {
                uint32_t v = 0;
                for (int i = 0; i < 8; ++i) {
                    const int n = row_of(m8 * 8 + i);
                    const uint32_t zz =
                        (uint32_t)(zeros[((int64_t)e * (N / 8) + (n >> 3)) * G + ch * 4 + g] >> ((n & 7) * 4)) & 0xF;
                    v |= zz << (4 * i);
                }
                zw[g] = v;
            }
        }
        *reinterpret_cast<uint4*>(dst + 32768 + 1024 + m8 * 16) = make_uint4(zw[0], zw[1], zw[2], zw[3]);
    }
}

}  // namespace

bool fused_decode_ok(int64_t T, int64_t top_k, int64_t E, int64_t H, int64_t I) {
    return T * top_k <= kMaxSlots && E <= kMaxExperts && H % 512 == 0 && I % 512 == 0 &&
           T <= 65535 && top_k <= kCombMaxK;
}

size_t fused_decode_workspace(int64_t T, int64_t top_k, int64_t E, int64_t H, int64_t I) {
    return dec_layout(T, top_k, E, H, I).total;
}

// The three launches of the fused decode layer (arguments checked by the caller).
size_t stream_pack_bytes(int64_t E, int64_t N, int64_t K) {
    return (size_t)E * (size_t)(N / 128) * (size_t)(K / 512) * kPackBlock;
}

int launch_stream_pack(const int32_t* w, const void* scales, const int32_t* zeros, int64_t E,
                       int64_t N, int64_t K, int gate_up, void* packed, cudaStream_t st) {
    const int nsl = (int)(gate_up ? (N / 2) / 64 : N / 128);
    const int nch = (int)(K / 512);
    const int64_t blocks = E * nsl * nch;
    if (blocks <= 0) return W4A8_OK;
    stream_pack_kernel<<<(unsigned)blocks, 256, 0, st>>>(
        w, static_cast<const __half*>(scales), zeros, K, (int)N, (int)(K / 128),
        gate_up ? (int)(N / 2) : 0, nsl, nch, static_cast<uint8_t*>(packed));
    return launch_status();
}

namespace {
// Operand source of the gate_up launch: fp16 token rows quantised by the prep launch, or
// expert-parallel payload rows that already hold the e4m3 operand (w4a8_ep_pack).
struct DecInput {
    const void* x;             // fp16 (T, H) or payload rows
    int64_t row_bytes;         // 0: fp16 rows; else payload row size
    const int32_t* topk_ids;
    const float* topk_w;
};
int run_fused_decode(const DecInput& in, int64_t T, int64_t top_k, int64_t E,
                     const int32_t* w13, const void* s13, const int32_t* z13, const int32_t* w2,
                     const void* s2, const int32_t* z2, int64_t H, int64_t I, void* out,
                     bool out_f32, void* workspace, cudaStream_t st, const void* p13,
                     const void* p2);
}  // namespace

int launch_fused_decode(const void* x, const int32_t* topk_ids, const float* topk_weights,
                        int64_t T, int64_t top_k, int64_t E, const int32_t* w13, const void* s13,
                        const int32_t* z13, const int32_t* w2, const void* s2, const int32_t* z2,
                        int64_t H, int64_t I, void* out, void* workspace, cudaStream_t st,
                        const void* p13, const void* p2) {
    return run_fused_decode(DecInput{x, 0, topk_ids, topk_weights}, T, top_k, E, w13, s13, z13,
                            w2, s2, z2, H, I, out, false, workspace, st, p13, p2);
}

int launch_fused_decode_rows(const void* rows, int64_t row_bytes, int64_t R, int64_t top_k,
                             int64_t E, const void* p13, const void* p2, int64_t H, int64_t I,
                             float* out, void* workspace, cudaStream_t st) {
    const int64_t G = H / 128;
    const uint8_t* b = static_cast<const uint8_t*>(rows);
    const int64_t off_ids = H + 4 * G + 4;
    return run_fused_decode(DecInput{rows, row_bytes, reinterpret_cast<const int32_t*>(b + off_ids),
                                     reinterpret_cast<const float*>(b + off_ids + 4 * top_k)},
                            R, top_k, E, nullptr, nullptr, nullptr, nullptr, nullptr, nullptr, H,
                            I, out, true, workspace, st, p13, p2);
}

namespace {
int run_fused_decode(const DecInput& in, int64_t T, int64_t top_k, int64_t E,
                     const int32_t* w13, const void* s13, const int32_t* z13, const int32_t* w2,
                     const void* s2, const int32_t* z2, int64_t H, int64_t I, void* out,
                     bool out_f32, void* workspace, cudaStream_t st, const void* p13,
                     const void* p2) {
    const void* x = in.x;
    const int32_t* topk_ids = in.topk_ids;
    const float* topk_weights = in.topk_w;
    static_assert(sizeof(DSmem) + 1024 <= 227 * 1024, "decode GEMV shared memory");
    const DecLayout L = dec_layout(T, top_k, E, H, I);
    uint8_t* ws = static_cast<uint8_t*>(workspace);
    DecArgs a{};
    a.topk_ids = topk_ids;
    a.topk_w = topk_weights;
    a.T = (int)T;
    a.top_k = (int)top_k;
    a.E = (int)E;
    a.off = reinterpret_cast<int32_t*>(ws + L.off_off);
    a.active = reinterpret_cast<int32_t*>(ws + L.off_active);
    a.act_tab = reinterpret_cast<int4*>(ws + L.off_tab);
    a.sorted_tok = reinterpret_cast<int32_t*>(ws + L.off_stok);
    a.meta = reinterpret_cast<int32_t*>(ws + L.off_meta);
    a.sorted_slot = reinterpret_cast<int32_t*>(ws + L.off_sorted);
    a.slot_pos = reinterpret_cast<int32_t*>(ws + L.off_pos);
    a.nslot = reinterpret_cast<int32_t*>(ws + L.off_nslot);
    a.amax = reinterpret_cast<float*>(ws + L.off_amax);
    a.tok_done = reinterpret_cast<int32_t*>(ws + L.off_tokdone);
    a.H = (int)H;
    a.I = (int)I;
    a.silu = reinterpret_cast<__half*>(ws + L.off_silu);
    a.out2 = reinterpret_cast<__half*>(ws + L.off_out2);
    a.out = out;
    a.out_f32 = out_f32 ? 1 : 0;
    a.one = 1u;
    a.m1 = 0xffffffffu;
    a.x = static_cast<const __half*>(x);
    const int64_t G1 = H / 128;
    if (in.row_bytes == 0) {
        a.ids_stride = (int)top_k;
        a.xe = ws + L.off_xh1;
        a.xsum = reinterpret_cast<const float*>(ws + L.off_xs1);
        a.asc = reinterpret_cast<const float*>(ws + L.off_sc1);
        a.xe_stride = H;
        a.xs_stride = G1;
        a.asc_stride = 1;
    } else {  // payload rows: [H e4m3 bytes][G sums][scale][top_k ids][top_k weights]
        a.ids_stride = (int)(in.row_bytes / 4);
        const uint8_t* b = static_cast<const uint8_t*>(x);
        a.xe = b;
        a.xsum = reinterpret_cast<const float*>(b + H);
        a.asc = reinterpret_cast<const float*>(b + H + 4 * G1);
        a.xe_stride = in.row_bytes;
        a.xs_stride = in.row_bytes / 4;
        a.asc_stride = in.row_bytes / 4;
    }
    // 1. routing sort (+ token quantisation of fp16 input rows)
    const size_t prep_smem = (size_t)E * 8 + (size_t)T * 4;
    if (prep_smem > 48 * 1024)
        cudaFuncSetAttribute(decode_prep_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             (int)prep_smem);
    decode_prep_kernel<<<(unsigned)(1 + (in.row_bytes ? 0 : T)), kPrepThreads, prep_smem, st>>>(a);
    if (int rc = launch_status()) return rc;
    // 2. gate_up GEMV + SiLU (+ the down operand, by each expert's last unit)
    a.packed = static_cast<const uint8_t*>(p13);
    a.w = w13;
    a.scales = static_cast<const __half*>(s13);
    a.zeros = z13;
    a.K = H;
    a.N = (int)(2 * I);
    a.G = (int)(H / 128);
    const int64_t S = T * top_k;
    const int64_t max_active = std::min<int64_t>(E, S);
    if (int rc = launch_dec_gemv<kGateUp>(a, (int)std::min<int64_t>(max_active * (I / 64), 1 << 30), st))
        return rc;
    // 3. down GEMV + the slot-order reduce (by each (token, slice)'s last arrival)
    a.packed = static_cast<const uint8_t*>(p2);
    a.w = w2;
    a.scales = static_cast<const __half*>(s2);
    a.zeros = z2;
    a.K = I;
    a.N = (int)H;
    a.G = (int)(I / 128);
    if (p2) {  // the tensor-core down launch quantises each SiLU row once into these
        a.xe = ws + L.off_xh2;
        a.xsum = reinterpret_cast<const float*>(ws + L.off_xs2);
        a.asc = reinterpret_cast<const float*>(ws + L.off_sc2);
        a.xe_stride = I;
        a.xs_stride = I / 128;
        a.asc_stride = 1;
    } else {  // the mma.sync down launch's quantisation warps build it per stage
        a.xe = nullptr;
        a.xsum = nullptr;
        a.asc = nullptr;
    }
    return launch_dec_gemv<kDown>(a, (int)std::min<int64_t>(max_active * (H / 128), 1 << 30), st);
}
}  // namespace

}  // namespace w4a8

#ifdef W4A8_DEC_TRACE
extern "C" W4A8_API int w4a8_debug_dec_trace(void* host, size_t bytes) {
    return (int)cudaMemcpyFromSymbol(host, w4a8::g_dec_trace, bytes);
}
extern "C" W4A8_API int w4a8_debug_prep_trace(void* host) {
    return (int)cudaMemcpyFromSymbol(host, w4a8::g_prep_trace, sizeof(w4a8::g_prep_trace));
}
#endif
