// gemm_tc.cu — W4A8 (grouped) GEMM tile path on the 5th-generation tensor cores (tcgen05).
//
// Two launches:
//   1. tc_quant_rows_kernel — quantises each sorted row's source activations to e4m3 (per-token
//      scale) and writes them, the scale and the per-group sums S into dense sorted-order
//      buffers (padding rows become zeros), so the GEMM reads its token tiles with plain 2D
//      TMA boxes instead of per-row gathers.
//   2. w4_tc_kernel — persistent and warp-specialised, one CTA per SM. A tile is 128 weight
//      rows x NT sorted rows (NT = 64 or 128; a tile never straddles an expert block). Tiles are
//      dealt round-robin to the CTAs; inside a CTA every role walks the same tile sequence and
//      the (tile, K-group) steps flow through mbarrier rings, so the next tile's loads and MMAs
//      overlap the current tile's epilogue.
//
// Roles (16 warps). In the expansion and fold roles one leader thread waits on the mbarriers
// and a named barrier releases the role's other warps.
//   warp 0      TMA producer: weight codes (2D box, 64-byte swizzle), token tile (2D box,
//               128-byte swizzle = the UMMA K-major SW128 layout), group sums (bulk copy).
//   warp 1      MMA issuer: 4 x tcgen05.mma.kind::f8f6f4 (K = 32 each) per group, A from tensor
//               memory, B from shared memory, into one of the TMEM accumulators, committed to
//               the stage / A / accumulator barriers.
//   warp 2      owns the tensor-memory allocation; loads each group's weight scales and zeros
//               into a shared ring as {s, -s*z}.
//   warps 4-7   expand the 4-bit codes to e4m3 bytes and store them to the A tile in tensor
//               memory (thread = weight row = TMEM lane).
//   warps 8-15  fold each group's accumulator into fp32 registers (4 lane quadrants x 2 column
//               halves) and write the finished tiles' outputs.
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
#include "sm100.cuh"
#include "tcgen05.cuh"

namespace w4a8 {

namespace {

constexpr int kTcThreads = 512;
constexpr int kFoldWarps = 8;

template <int NT>
struct TcCfg {
    static constexpr int kStages = NT == 128 ? 6 : 11; // TMA ring depth (codes + tokens)
    static constexpr int kSStages = 8;                 // group-sum ring depth
    // Tensor memory (512 columns): kAcc fp32 accumulators of NT columns, then kAStages
    // dequantised A tiles of 32 columns (128 rows x 128 e4m3 bytes each).
    static constexpr int kAcc = NT == 128 ? 3 : 4;
    static constexpr int kAStages = (512 - kAcc * NT) / 32;
    static constexpr uint32_t kACol0 = kAcc * NT;
    static constexpr int kCols = NT / 2;               // accumulator columns per fold thread
    static constexpr uint32_t kTmemCols = 512;
    static constexpr uint32_t kStageBytes = 128 * 64 + NT * 128;
};

template <int NT>
struct TcSmem {
    uint8_t b[TcCfg<NT>::kStages][NT * 128];     // token tiles, SW128 K-major (1024-aligned)
    uint8_t raw[TcCfg<NT>::kStages][128 * 64];   // packed codes, SW64 as TMA writes them
    __half otile[2][NT * 128];                   // finished tiles, fp16, [column][row]
    float ssum[TcCfg<NT>::kSStages][NT];         // group sums S of the tile's rows
    float2 meta[TcCfg<NT>::kSStages][128];       // per weight row: {scale, -scale * zero}
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

// Stage index + phase bit of a barrier ring, advanced one step per K group.
template <int N>
struct RingPos {
    uint32_t idx = 0, phase = 0;
    __device__ __forceinline__ void next() {
        if (++idx == N) {
            idx = 0;
            phase ^= 1;
        }
    }
};

// The tile sequence of one CTA: t = blockIdx.x + i * gridDim.x, t = rb * n_mt + mt, walked
// without per-step division. `expert` is the tile's expert (0 for the dense GEMM).
struct TileWalk {
    int rb, mt, drb, dmt, n_mt, nblk, bpe;
    __device__ __forceinline__ TileWalk(int n_mt_, int nblk_, int bpe_)
        : rb(blockIdx.x / n_mt_), mt(blockIdx.x % n_mt_), drb(gridDim.x / n_mt_),
          dmt(gridDim.x % n_mt_), n_mt(n_mt_), nblk(nblk_), bpe(bpe_) {}
    __device__ __forceinline__ bool more() const { return rb < nblk; }
    __device__ __forceinline__ void next() {
        rb += drb;
        mt += dmt;
        if (mt >= n_mt) {
            mt -= n_mt;
            ++rb;
        }
    }
    __device__ __forceinline__ int expert(const TcArgs& a) const {
        return a.expert_ids ? a.expert_ids[rb / bpe] : 0;
    }
};

template <int NT>
__global__ void __launch_bounds__(kTcThreads, 1)
w4_tc_kernel(const TcArgs a, const __grid_constant__ CUtensorMap tmw,
             const __grid_constant__ CUtensorMap tmx) {
    using C = TcCfg<NT>;
    extern __shared__ uint8_t smem_raw[];
    // 1024-byte alignment by offsetting the __shared__ array itself (a round trip through an
    // integer would lose the shared address space and turn every access into a generic one)
    TcSmem<NT>& sm = *reinterpret_cast<TcSmem<NT>*>(
        smem_raw + ((1024u - (smem_u32(smem_raw) & 1023u)) & 1023u));
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    volatile int* bad = &sm.bad;

    const int P_valid = a.ntp ? min(a.ntp[0], a.P) : a.P;
    const int nblk = (P_valid + NT - 1) / NT;
    const int n_mt = a.silu ? (a.N / 2) / 64 : (a.N + 127) / 128;
    const int n_out = a.silu ? a.N / 2 : a.N;
    const int bpe = a.expert_ids ? a.block_m / NT : 1;  // tile row blocks per expert block
    const int G = a.G;

    if (tid == 0) {
        sm.bad = 0;
        for (int s = 0; s < C::kStages; ++s) {
            mbar_init(&sm.full[s], 1);
            mbar_init(&sm.empty[s], 1);
        }
        for (int s = 0; s < C::kSStages; ++s) {
            mbar_init(&sm.sfull[s], 1 + 32);  // producer's bulk copy + the meta warp's lanes
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
            RingPos<C::kStages> st;
            RingPos<C::kSStages> ss;
            uint32_t issued = 0;
            for (TileWalk tw(n_mt, nblk, bpe); tw.more(); tw.next()) {
                const int e = tw.expert(a);
                if (e < 0 || e >= a.E) continue;
                const int r0 = tw.rb * NT, mt = tw.mt;
                // warm L2 with this CTA's next tile (weights and tokens) while this one runs
                TileWalk nx = tw;
                nx.next();
                if (nx.more()) {
                    const int en = nx.expert(a);
                    if (en >= 0 && en < a.E)
                        for (int g = 0; g < G; ++g) {
                            if (a.silu) {
                                tma_prefetch_2d(&tmw, g * 64, en * a.N + nx.mt * 64);
                                tma_prefetch_2d(&tmw, g * 64, en * a.N + a.N / 2 + nx.mt * 64);
                            } else {
                                tma_prefetch_2d(&tmw, g * 64, en * a.N + nx.mt * 128);
                            }
                            tma_prefetch_2d(&tmx, g * 128, nx.rb * NT);
                        }
                }
                for (int g = 0; g < G; ++g) {
                    uint64_t* fb = &sm.full[st.idx];
                    mbar_wait(&sm.empty[st.idx], st.phase ^ 1, bad);
                    mbar_expect_tx(fb, C::kStageBytes);
                    uint8_t* raw = &sm.raw[st.idx][0];
                    if (a.silu) {
                        tma_load_2d(raw, &tmw, g * 64, e * a.N + mt * 64, fb);
                        tma_load_2d(raw + 64 * 64, &tmw, g * 64, e * a.N + a.N / 2 + mt * 64, fb);
                    } else {
                        tma_load_2d(raw, &tmw, g * 64, e * a.N + mt * 128, fb);
                    }
                    tma_load_2d(&sm.b[st.idx][0], &tmx, g * 128, r0, fb);
                    mbar_wait(&sm.sempty[ss.idx], ss.phase ^ 1, bad);
                    mbar_expect_tx(&sm.sfull[ss.idx], NT * 4);
                    bulk_load(&sm.ssum[ss.idx][0], a.ssum + (int64_t)g * a.P_pad + r0, NT * 4,
                              &sm.sfull[ss.idx]);
                    st.next();
                    ss.next();
                    ++issued;
                }
            }
            // leave no copy in flight: wait (boundedly) for the last ring's worth of loads
            if (*bad) {
                const uint64_t t0 = global_ns();
                for (uint32_t j = 0; j < (uint32_t)C::kStages && j < issued; ++j)
                    while (!mbar_try(&sm.full[j], ((issued - 1 - j) / C::kStages) & 1) &&
                           global_ns() - t0 < kWaitLimitNs) {
                    }
                for (uint32_t j = 0; j < (uint32_t)C::kSStages && j < issued; ++j)
                    while (!mbar_try(&sm.sfull[j], ((issued - 1 - j) / C::kSStages) & 1) &&
                           global_ns() - t0 < kWaitLimitNs) {
                    }
            }
        }
    } else if (warp == 1) {
        // ---------------- MMA issuer ----------------
        if (lane == 0) {
            constexpr uint32_t idesc = umma_idesc(128, NT);
            RingPos<C::kStages> st;
            RingPos<C::kAStages> as;
            RingPos<C::kAcc> tb;
            for (TileWalk tw(n_mt, nblk, bpe); tw.more(); tw.next()) {
                const int e = tw.expert(a);
                if (e < 0 || e >= a.E) continue;
                for (int g = 0; g < G; ++g) {
                    mbar_wait(&sm.full[st.idx], st.phase, bad);
                    mbar_wait(&sm.afull[as.idx], as.phase, bad);
                    mbar_wait(&sm.tempty[tb.idx], tb.phase ^ 1, bad);
                    asm volatile("tcgen05.fence::after_thread_sync;" ::);
                    const uint32_t ta = tmem + C::kACol0 + as.idx * 32;
                    const uint32_t b0 = smem_u32(&sm.b[st.idx][0]);
                    const uint32_t d = tmem + tb.idx * NT;
#pragma unroll
                    for (int kk = 0; kk < 4; ++kk) {  // K = 32 e4m3 = 8 TMEM columns of A
                        const uint64_t db = desc_sw128(b0 + kk * 32);
                        const uint32_t acc = kk > 0 ? 1u : 0u;
                        asm volatile(
                            "{\n\t.reg .pred p;\n\t"
                            "setp.ne.b32 p, %4, 0;\n\t"
                            "tcgen05.mma.cta_group::1.kind::f8f6f4 [%0], [%1], %2, %3, p;\n\t}" ::"r"(d),
                            "r"(ta + kk * 8), "l"(db), "r"(idesc), "r"(acc));
                    }
                    asm volatile(
                        "tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];"
                        ::"r"(smem_u32(&sm.empty[st.idx])));
                    asm volatile(
                        "tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];"
                        ::"r"(smem_u32(&sm.aempty[as.idx])));
                    asm volatile(
                        "tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];"
                        ::"r"(smem_u32(&sm.tfull[tb.idx])));
                    st.next();
                    as.next();
                    tb.next();
                }
            }
        }
    } else if (warp == 2) {
        // ---------------- per-row group scales / zeros -> {s, -s*z} ----------------
        // Lane l serves rows l, l+32, l+64, l+96. Loads run one chunk of up to 4 groups ahead
        // of the stores, so their latency hides behind the fold of the previous chunk.
        const int cg = (G % 4 == 0) ? 4 : 1;
        RingPos<C::kSStages> ss;
        TileWalk tw(n_mt, nblk, bpe);
        auto skip_invalid = [&](TileWalk& w) {
            while (w.more()) {
                const int e = w.expert(a);
                if (e >= 0 && e < a.E) break;
                w.next();
            }
        };
        skip_invalid(tw);
        float sc[4][4], sn[4][4];  // current / next chunk: [row][group]
        int zc[4][4], zn[4][4];
        auto load = [&](float (&sd)[4][4], int (&zd)[4][4], const TileWalk& w, int gg) {
            const int e = w.expert(a);
#pragma unroll
            for (int r = 0; r < 4; ++r) {
                const int m = lane + 32 * r;
                int n;
                if (a.silu) n = m >= 64 ? a.N / 2 + w.mt * 64 + (m - 64) : w.mt * 64 + m;
                else n = w.mt * 128 + m;
                const int nn = n < a.N ? n : 0;
                const __half* sp = a.scales + ((int64_t)e * a.N + nn) * G + gg;
                const int32_t* zp =
                    a.zeros ? a.zeros + ((int64_t)e * (a.N / 8) + (nn >> 3)) * G + gg : nullptr;
#pragma unroll
                for (int j = 0; j < 4; ++j) {
                    if (j < cg) {
                        sd[r][j] = __half2float(sp[j]);
                        zd[r][j] = zp ? ((__ldg(zp + j) >> ((nn & 7) * 4)) & 0xF) : 8;
                    }
                }
            }
        };
        int g0 = 0;
        if (tw.more()) load(sc, zc, tw, 0);
        while (tw.more()) {
            TileWalk wn = tw;  // next chunk's coordinates, then its loads
            int gn = g0 + cg;
            if (gn >= G) {
                gn = 0;
                wn.next();
                skip_invalid(wn);
            }
            if (wn.more()) load(sn, zn, wn, gn);
#pragma unroll
            for (int j = 0; j < 4; ++j) {
                if (j < cg) {
                    if (lane == 0) mbar_wait(&sm.sempty[ss.idx], ss.phase ^ 1, bad);
                    __syncwarp();
#pragma unroll
                    for (int r = 0; r < 4; ++r) {
                        const float sv = sc[r][j];
                        sm.meta[ss.idx][lane + 32 * r] = make_float2(sv, -sv * (float)zc[r][j]);
                    }
                    mbar_arrive(&sm.sfull[ss.idx]);
                    ss.next();
                }
            }
            tw = wn;
            g0 = gn;
#pragma unroll
            for (int r = 0; r < 4; ++r)
#pragma unroll
                for (int j = 0; j < 4; ++j) {
                    sc[r][j] = sn[r][j];
                    zc[r][j] = zn[r][j];
                }
        }
    } else if (warp >= 4 && warp < 8) {
        // ---------------- code expansion: thread = weight row = TMEM lane ----------------
        // Warp 4's lane 0 waits for the stage and the A slot; a named barrier releases the rest.
        const int m = tid - 128;
        const int sw64 = (m >> 1) & 3;
        const uint32_t lane_base = (uint32_t)((warp & 3) * 32) << 16;
        RingPos<C::kStages> st;
        RingPos<C::kAStages> as;
        for (TileWalk tw(n_mt, nblk, bpe); tw.more(); tw.next()) {
            const int e = tw.expert(a);
            if (e < 0 || e >= a.E) continue;
            for (int g = 0; g < G; ++g) {
                if (tid == 128) {
                    mbar_wait(&sm.full[st.idx], st.phase, bad);
                    mbar_wait(&sm.aempty[as.idx], as.phase ^ 1, bad);
                }
                asm volatile("bar.sync 2, 128;" ::: "memory");
                // row m of the A tile = TMEM lane m; column j holds e4m3 bytes k = 4j..4j+3
                const uint8_t* rr = &sm.raw[st.idx][m * 64];
                uint32_t o[32];
#pragma unroll
                for (int j = 0; j < 4; ++j) {  // 16 raw bytes = 32 codes = 8 TMEM columns
                    const uint4 w = *reinterpret_cast<const uint4*>(rr + ((j ^ sw64) << 4));
                    codes8_to_e4m3(w.x, o[8 * j + 0], o[8 * j + 1]);
                    codes8_to_e4m3(w.y, o[8 * j + 2], o[8 * j + 3]);
                    codes8_to_e4m3(w.z, o[8 * j + 4], o[8 * j + 5]);
                    codes8_to_e4m3(w.w, o[8 * j + 6], o[8 * j + 7]);
                }
                tmem_st32(tmem + lane_base + C::kACol0 + as.idx * 32, o);
                asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
                asm volatile("tcgen05.fence::before_thread_sync;" ::);
                __syncwarp();
                if (lane == 0) mbar_arrive(&sm.afull[as.idx]);
                st.next();
                as.next();
            }
        }
    } else if (warp >= 8) {
        // ---------------- fold + epilogue ----------------
        // Warp w folds TMEM lane quadrant w % 4, columns [h * kCols, (h + 1) * kCols). Warp 8's
        // lane 0 waits for the group's sums and accumulator; a named barrier releases the rest.
        // A finished tile goes to a shared fp16 tile, double buffered so that a warp may park
        // the next tile while others still store this one; all fold warps then write it out
        // row-contiguously (SiLU(gate) * up for the fused op).
        constexpr int kCols = C::kCols;
        const int q = warp & 3;
        const int fw = warp - 8;
        const int c0 = (fw >> 2) * kCols;
        const int m = q * 32 + lane;  // tile row = TMEM lane
        const uint32_t lane_base = (uint32_t)(q * 32) << 16;
        RingPos<C::kSStages> ss;
        RingPos<C::kAcc> tb;
        int tiles_done = 0;
        // the parked tile (buffer pend_buf, rows r0.., weight tile mt) to global memory
        auto drain = [&](int pend_buf, int pend_r0, int pend_mt) {
            const int c_lo = 0, c_hi = NT;
            const __half* ot = sm.otile[pend_buf];
            if (a.silu) {
                const int n = pend_mt * 64 + 2 * lane;
                for (int c = c_lo + fw; c < c_hi; c += kFoldWarps) {
                    const int r = pend_r0 + c;
                    if (r >= P_valid) break;
                    const __half2 gh = *reinterpret_cast<const __half2*>(&ot[c * 128 + 2 * lane]);
                    const __half2 uh = *reinterpret_cast<const __half2*>(&ot[c * 128 + 64 + 2 * lane]);
                    __half2 o;
                    o.x = silu_mul_h(__low2half(gh), __low2half(uh));
                    o.y = silu_mul_h(__high2half(gh), __high2half(uh));
                    *reinterpret_cast<__half2*>(a.out16 + (int64_t)r * n_out + n) = o;
                }
            } else {
                const int n = pend_mt * 128 + 4 * lane;
                if (n < n_out)
                    for (int c = c_lo + fw; c < c_hi; c += kFoldWarps) {
                        const int r = pend_r0 + c;
                        if (r >= P_valid) break;
                        *reinterpret_cast<uint2*>(a.out16 + (int64_t)r * n_out + n) =
                            *reinterpret_cast<const uint2*>(&ot[c * 128 + 4 * lane]);
                    }
            }
        };
        for (TileWalk tw(n_mt, nblk, bpe); tw.more(); tw.next()) {
            const int e = tw.expert(a);
            const int r0 = tw.rb * NT, mt = tw.mt;
            if (e < 0 || e >= a.E) {  // non-local expert: zero rows
                const int n = a.silu ? mt * 64 + 2 * lane : mt * 128 + 4 * lane;
                for (int c = fw; c < NT; c += kFoldWarps) {
                    const int r = r0 + c;
                    if (r >= P_valid) break;
                    if (a.silu)
                        *reinterpret_cast<uint32_t*>(a.out16 + (int64_t)r * n_out + n) = 0u;
                    else if (n < n_out)
                        *reinterpret_cast<uint2*>(a.out16 + (int64_t)r * n_out + n) = make_uint2(0u, 0u);
                }
                continue;
            }
            // activation scales of the tile's columns: lane l holds columns c0 + l (+ 32)
            float asc_l[kCols / 32];
#pragma unroll
            for (int i = 0; i < kCols / 32; ++i) asc_l[i] = __ldg(a.asc_s + r0 + c0 + i * 32 + lane);
            float tot[kCols];
#pragma unroll
            for (int c = 0; c < kCols; ++c) tot[c] = 0.f;
            for (int g = 0; g < G; ++g) {
                if (tid == 256) {
                    mbar_wait(&sm.sfull[ss.idx], ss.phase, bad);
                    mbar_wait(&sm.tfull[tb.idx], tb.phase, bad);
                }
                asm volatile("bar.sync 3, %0;" ::"n"(kFoldWarps * 32) : "memory");
                asm volatile("tcgen05.fence::after_thread_sync;" ::);
                const float2 md = sm.meta[ss.idx][m];
                const float2 sv = make_float2(md.x, md.x);
                const float2 nsz = make_float2(md.y, md.y);
                const float* S = &sm.ssum[ss.idx][c0];
#pragma unroll
                for (int cc = 0; cc < kCols; cc += 32) {
                    uint32_t v[32];
                    tmem_ld<32>(tmem + lane_base + tb.idx * NT + c0 + cc, v);
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
                    mbar_arrive(&sm.tempty[tb.idx]);
                    mbar_arrive(&sm.sempty[ss.idx]);
                }
                ss.next();
                tb.next();
            }
            // park the finished tile: fp16(tot * a_scale) into the free shared tile
            const int buf = tiles_done & 1;
#pragma unroll
            for (int c = 0; c < kCols; ++c)
                sm.otile[buf][(c0 + c) * 128 + m] = __float2half_rn(
                    tot[c] * __shfl_sync(0xffffffffu, asc_l[c >> 5], c & 31));
            asm volatile("bar.sync 1, %0;" ::"n"(kFoldWarps * 32) : "memory");
            drain(buf, r0, mt);
            ++tiles_done;
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

// One warp quantises one row per token to e4m3 exactly as act_quant_fp8 does (a_scale =
// max(amax, 4.48e-6) / 448, q = e4m3_rn(x / a_scale) with the IEEE quotient;
// w4a8_fp8_wmma/test_correctness.py:74-76): bytes in natural order, the per-group sums S of
// the e4m3 values (sum[g * sum_stride]) and the scale. K % 256 == 0.
__device__ __forceinline__ void quant_row_nat_warp(const __half* src, int64_t K, uint8_t* dst,
                                                   float* sum, int64_t sum_stride, float* scale) {
    const int lane = threadIdx.x & 31;
    const uint4* xr = reinterpret_cast<const uint4*>(src);
    const int nch = (int)(K / 8);  // 8-element chunks; chunk i belongs to group i / 16
    float amax = 0.f;
    for (int i = lane; i < nch; i += 32) {
        const uint4 v = __ldg(xr + i);
        const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            const __half2 h = __habs2(*reinterpret_cast<const __half2*>(&w[j]));
            amax = fmaxf(amax, fmaxf(__low2float(h), __high2float(h)));
        }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
    const float s = __fdiv_rn(fmaxf(amax, kAmaxFloor), kE4m3Max);
    const float rcp = __frcp_rn(s);
    if (lane == 0) *scale = s;
    uint2* d2 = reinterpret_cast<uint2*>(dst);
    for (int i0 = 0; i0 < nch; i0 += 32) {  // nch % 32 == 0: lanes 0-15 / 16-31 = one group each
        const int i = i0 + lane;
        const uint4 v = __ldg(xr + i);
        const uint32_t w[4] = {v.x, v.y, v.z, v.w};
        uint32_t q[2];
        float acc = 0.f;
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
            acc += (d0.x + d0.y) + (d1.x + d1.y);
        }
        d2[i] = make_uint2(q[0], q[1]);
#pragma unroll
        for (int o = 8; o > 0; o >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, o);
        if ((lane & 15) == 0) sum[(int64_t)(i / 16) * sum_stride] = acc;
    }
}

// Gather case: every source row once (tokens), into the token-level operand.
__global__ void __launch_bounds__(256) tc_quant_tokens_kernel(const TcArgs a) {
    const int64_t t = (int64_t)blockIdx.x * 8 + (threadIdx.x >> 5);
    if (t >= a.x_rows) return;
    quant_row_nat_warp(a.x + t * a.K, a.K, a.tq + t * a.K, a.tq_sum + t * a.G, 1, a.tq_scale + t);
}

// One warp per sorted row: writes the row's e4m3 bytes, scale and group sums in sorted order, so
// the tile kernel reads its token tiles with plain 2D TMA boxes. With a token-level operand the
// row is a copy of its token's; otherwise the source row is quantised here. Rows past the last
// valid one (up to the tile-rounded count) and rows with a sentinel id are zero-filled.
__global__ void __launch_bounds__(256) tc_quant_rows_kernel(const TcArgs a, int NT) {
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
    const int n16 = (int)(a.K / 16);
    if (src < 0) {
        for (int i = lane; i < n16; i += 32) dst[i] = make_uint4(0u, 0u, 0u, 0u);
        for (int g = lane; g < a.G; g += 32) a.ssum[(int64_t)g * a.P_pad + r] = 0.f;
        if (lane == 0) a.asc_s[r] = 0.f;
        return;
    }
    if (a.tq) {
        const uint4* srow = reinterpret_cast<const uint4*>(a.tq + (int64_t)src * a.K);
        for (int i = lane; i < n16; i += 32) dst[i] = srow[i];
        for (int g = lane; g < a.G; g += 32)
            a.ssum[(int64_t)g * a.P_pad + r] = a.tq_sum[(int64_t)src * a.G + g];
        if (lane == 0) a.asc_s[r] = a.tq_scale[src];
        return;
    }
    quant_row_nat_warp(a.x + (int64_t)src * a.K, a.K, a.xs + r * a.K, a.ssum + r, a.P_pad,
                       a.asc_s + r);
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
    if (a.tq && a.x_rows > 0) {
        tc_quant_tokens_kernel<<<(unsigned)((a.x_rows + 7) / 8), 256, 0, stream>>>(a);
        if (int rc = launch_status()) return rc;
    }
    tc_quant_rows_kernel<<<(unsigned)((rows_max + 7) / 8), 256, 0, stream>>>(a, NT);
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

bool make_tma_map_u8(CUtensorMap* map, const void* base, uint64_t rows, uint64_t row_bytes,
                     uint32_t box_bytes, uint32_t box_rows, CUtensorMapSwizzle sw) {
    return make_map(map, base, rows, row_bytes, box_bytes, box_rows, sw);
}

bool tc_path_ok(int64_t K, int group_size, int e2m1, const void* w, int block_m) {
    return !e2m1 && group_size == 128 && K % 256 == 0 && K >= 256 &&
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
