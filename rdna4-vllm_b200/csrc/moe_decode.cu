// moe_decode.cu — the gated MoE layer at decode sizes in three launches.
//
// Same result as the decode branch of the reference's composition (_run_grouped_moe, M <= 96,
// w4a8_fp8_wmma/w4a8_fp8_wmma/moe_experts.py:563-648) and its oracle
// (w4a8_fp8_wmma/test_moe_experts.py:155-191): per (token, slot) gate_up GEMM -> fp16 gate/up ->
// silu_and_mul -> per-token e4m3 re-quantisation -> down GEMM -> fp16 row, then the fp32
// topk-weighted sum over the token's slots in slot order.
//
//   1. decode_prep_kernel   CTA 0 sorts the valid (token, slot) pairs by expert (stable, no
//                           block padding) and resets the counters of launches 2-3; CTAs 1..T
//                           quantise one token row each into the GEMV operand format.
//   2. decode_gemv_kernel<gate_up>
//                           work unit = (expert, 64 gate rows + the matching 64 up rows, all of
//                           K). Every warp's m16 tile holds 8 gate rows and the same 8 up rows,
//                           so each thread ends with gate and up of the same (row, token) and
//                           applies SiLU-and-mul in registers. The last unit to finish an expert
//                           (a per-expert counter) quantises that expert's SiLU rows as the down
//                           GEMM's operand.
//   3. decode_gemv_kernel<down>
//                           work unit = (expert, 128 output channels). Rows are rounded to fp16
//                           (the oracle's per-slot fp16 store); the last unit to finish a
//                           (token, 128-channel slice) — a per-(token, slice) counter — sums the
//                           token's slot rows in slot order (fp32 multiply, then add) and writes
//                           the fp16 output.
// The intermediates (SiLU rows, the down operand, the per-slot down rows) are a few hundred KB
// and stay in L2. The results do not depend on scheduling: every sum has a fixed order.
//
// GEMV core (both kernels): persistent, one CTA per SM, 8 compute warps + 1 producer warp. Units
// are dealt round-robin (heavy experts first); the producer streams each unit's K in 512-wide
// chunks through a 4-stage shared-memory ring: the 128 weight rows with their scales and zero
// points (one bulk copy of a prepacked block, or TMA + cp.async from the op layout), the unit's
// e4m3 activation rows (<= 16 per pass; more rows take more passes) and their group sums by
// bulk copies. The tensor-core arithmetic is mma.sync m16n8k32 on e4m3 operands (see
// dec_compute_t), folded per 128-group in fp32 with the group scale, then multiplied by the
// row's activation scale: the reference oracle's association
// (w4a8_fp8_wmma/test_correctness.py:113-119) up to fp32 rounding.
//
// Every mbarrier wait is bounded (sm100.cuh); a wait that gives up sets bit 1 of the error word
// and the kernel finishes without waiting further. There are no cross-CTA spin-waits: the
// last-arriver steps are decided by atomic counters.
#include <algorithm>
#include <cstddef>
#include <string>

#include "common.cuh"
#include "gemm_common.h"
#include "internal.h"
#include "sm100.cuh"
#include "e4_operand.cuh"
#include "stream_core.cuh"

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
enum : int { kMetaActive = 0, kMetaUnit1 = 1, kMetaUnit2 = 2, kMetaErr = 3, kMetaWords = 4 };

struct DecArgs {
    const int32_t* topk_ids;   // row t's slot j at topk_ids[t * ids_stride + j]
    const float* topk_w;       // row t's weight j at topk_w[t * ids_stride + j]
    int T, top_k, E;
    int ids_stride;            // elements between rows of topk_ids / topk_w (top_k when dense)
    int64_t xe_stride;         // bytes between gate_up operand rows (K when dense)
    int64_t xs_stride;         // floats between rows of the group sums (K/128 when dense)
    int64_t asc_stride;        // floats between activation scales (1 when dense)
    int out_f32;               // the layer output is fp32 (else fp16)
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
    const int E = a.E, S = a.T * a.top_k;
    const int n16 = a.H / 16;
    int* cnt = prep_smem;             // [E]
    int* cur = prep_smem + E;         // [E]
    int* ns = prep_smem + 2 * E;      // [T]
    for (int i = tid; i < E; i += kPrepThreads) cnt[i] = 0;
    if (tid < kMetaWords) a.meta[tid] = 0;
    for (int i = tid; i < a.T * n16; i += kPrepThreads) a.tok_done[i] = 0;
    for (int i = tid; i < S; i += kPrepThreads) a.amax[i] = 0.f;
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
    int tot_rows, tot_heavy, tot_light;
    int base_rows = block_excl_scan(my_rows, ired, &tot_rows);
    int base_heavy = block_excl_scan(my_heavy, ired, &tot_heavy);
    int base_light = block_excl_scan(my_light, ired, &tot_light) + tot_heavy;
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
    // stable placement: slots in ascending order, warps of a chunk in turn
    const int lane = tid & 31, warp = tid >> 5;
    for (int c0 = 0; c0 < S; c0 += kPrepThreads) {
        const int s = c0 + tid;
        int e = s < S ? slot_id(s) : -1;
        if (!(e >= 0 && e < E)) e = -1;
        if (s < S && e < 0) a.slot_pos[s] = -1;
        for (int w = 0; w < kPrepThreads / 32; ++w) {
            if (warp == w) {
                const unsigned m = __match_any_sync(0xffffffffu, e);
                const int leader = __ffs(m) - 1;
                const int rank = __popc(m & ((1u << lane) - 1));
                int base = 0;
                if (e >= 0 && lane == leader) base = cur[e];
                base = __shfl_sync(0xffffffffu, base, leader);
                if (e >= 0) {
                    const int p = base + rank;
                    a.slot_pos[s] = p;
                    a.sorted_slot[p] = s;
                    a.sorted_tok[p] = s / a.top_k;
                    if (lane == leader) cur[e] = base + __popc(m);
                }
            }
            __syncthreads();
        }
    }
    // tokens without a valid slot: the layer output is zero
    for (int t = 0; t < a.T; ++t)
        if (ns[t] == 0)
            for (int n = tid; n < a.H; n += kPrepThreads) {
                if (a.out_f32) static_cast<float*>(a.out)[(int64_t)t * a.H + n] = 0.f;
                else static_cast<__half*>(a.out)[(int64_t)t * a.H + n] = __float2half_rn(0.f);
            }
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
// order, group sums S, scale. Lane l handles 8-element units l and l + 32.
__device__ __forceinline__ void quant_stage_row(const DecArgs& a, DStage& S, int r, int p,
                                                int chunk) {
    const int lane = threadIdx.x & 31;
    const float amax = __uint_as_float(__ldcg(reinterpret_cast<const unsigned*>(a.amax) + p));
    const float s = __fdiv_rn(fmaxf(amax, kAmaxFloor), kE4m3Max);
    const float rcp = __frcp_rn(s);
    const uint4* src = reinterpret_cast<const uint4*>(a.silu + (int64_t)p * a.I + (int64_t)chunk * 512);
    const uint4 v0 = __ldcg(src + lane), v1 = __ldcg(src + lane + 32);
#pragma unroll
    for (int k = 0; k < 2; ++k) {
        const uint4 v = k ? v1 : v0;
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
#pragma unroll 2
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
                            if (lane == 0) mbar_wait(&sm.empty[st], ph ^ 1, bad);
                            __syncwarp();
                            for (int r = 0; r < nrows; ++r)
                                quant_stage_row(a, sm.st[st], r, p0 + r, ch);
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
        for (;;) {
            mbar_wait(&sm.full[st], ph, bad);
            __syncwarp();
            const DMeta& m = sm.meta[st];
            const int e = m.e;
            if (e < 0 || *bad) break;
            const int ntg = (m.nrows + 7) >> 3;
            const int sl = m.sl, p0 = m.p0, nrows = m.nrows;
            const bool last = m.last;
            // epilogue operands, requested before the stage's MMAs so their latency hides there
            float asc_c[2][2] = {};
            int my_t = 0;  // down: token of row `lane`
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
                if (MODE == kDown && lane < nrows) my_t = __ldg(a.sorted_tok + p0 + lane);
            }
            if (m.chunk == 0) {
#pragma unroll
                for (int tg = 0; tg < 2; ++tg)
#pragma unroll
                    for (int v = 0; v < 4; ++v) tot[tg][v] = 0.f;
            }
#ifndef W4A8_DEC_SKIP_COMPUTE
            dec_compute(sm.st[st], r0, r1, ntg, PACKED || a.zeros != nullptr, tot);
#endif
            __syncwarp();
            if (lane == 0) mbar_arrive(&sm.empty[st]);
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
                // of a chunk sums the token's slot rows there
                __syncwarp();
                bool mine = false;
                const int chunk16 = sl * 8 + warp;
                if (lane < nrows) {
                    __threadfence();  // release: the warp's rows (ordered by the syncwarp)
                    const int old = atomicAdd(&a.tok_done[(int64_t)my_t * (a.H / 16) + chunk16], 1);
                    mine = old == __ldg(a.nslot + my_t) - 1;
                }
                unsigned todo = __ballot_sync(0xffffffffu, mine);
                if (todo) __threadfence();  // acquire: the other arrivals' rows
                while (todo) {
                    const int src_lane = __ffs(todo) - 1;
                    todo &= todo - 1;
                    const int t = __shfl_sync(0xffffffffu, my_t, src_lane);
                    if (lane < 8) combine_pair(a, t, chunk16 * 16 + 2 * lane);
                }
            }
        }
    }
    __syncthreads();
    if (threadIdx.x == 0 && sm.bad) atomicOr(a.meta + kMetaErr, 2);
}

struct DecLayout {
    size_t off_off, off_active, off_tab, off_stok, off_meta, off_sorted, off_pos, off_nslot,
        off_amax, off_tokdone, off_xh1, off_xs1, off_sc1, off_silu, off_out2, total;
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

template <int MODE>
int launch_dec_gemv(const DecArgs& a, int units_max, cudaStream_t st) {
    return a.packed ? launch_dec_gemv_t<MODE, true>(a, units_max, st)
                    : launch_dec_gemv_t<MODE, false>(a, units_max, st);
}

// ---------------------------------------------------------------------------------------
// Weight prepack for the decode GEMV: op layout -> one contiguous block per (expert, unit
// slice, 512-wide K chunk), in the exact shared-memory image of a DStage's weight part:
//   codes  [2 halves][128 rows][8 x 16 B], 16-byte unit u of row m stored at u ^ (m & 7)
//          (the 128-byte swizzle the compute warps read);
//   scales [128 rows][4 groups] fp16;  zeros [16 (8-row words)][4 groups] u32 (8 when absent).
// Row m of a gate_up block is gate row sl*64 + m (m < 64) or up row inter + sl*64 + m - 64.
// ---------------------------------------------------------------------------------------
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
    auto row_of = [&](int m) {
        if (inter > 0) return m < 64 ? sl * 64 + m : inter + sl * 64 + (m - 64);
        return sl * 128 + m;
    };
    for (int idx = threadIdx.x; idx < 2048; idx += blockDim.x) {
        const int h = idx >> 10, m = (idx >> 3) & 127, u = idx & 7;
        const int n = row_of(m);
        const uint4 v = __ldg(reinterpret_cast<const uint4*>(
            wb + ((int64_t)e * N + n) * (K / 2) + (int64_t)ch * 256 + h * 128 + u * 16));
        *reinterpret_cast<uint4*>(dst + h * 16384 + m * 128 + ((u ^ (m & 7)) << 4)) = v;
    }
    if (threadIdx.x < 128) {
        const int m = threadIdx.x, n = row_of(m);
        const uint2 v = *reinterpret_cast<const uint2*>(scales + ((int64_t)e * N + n) * G + ch * 4);
        *reinterpret_cast<uint2*>(dst + 32768 + m * 8) = v;
    } else if (threadIdx.x < 144) {
        const int m8 = threadIdx.x - 128, n8 = row_of(m8 * 8) >> 3;
        uint4 v = make_uint4(0x88888888u, 0x88888888u, 0x88888888u, 0x88888888u);
        if (zeros)
            v = *reinterpret_cast<const uint4*>(zeros + ((int64_t)e * (N / 8) + n8) * G + ch * 4);
        *reinterpret_cast<uint4*>(dst + 32768 + 1024 + m8 * 16) = v;
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
    a.xe = nullptr;  // the down operand is built by the quantisation warps
    a.xsum = nullptr;
    a.asc = nullptr;
    return launch_dec_gemv<kDown>(a, (int)std::min<int64_t>(max_active * (H / 128), 1 << 30), st);
}
}  // namespace

}  // namespace w4a8
