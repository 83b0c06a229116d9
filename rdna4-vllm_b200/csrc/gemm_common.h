// gemm_common.h — argument block shared by the W4A8 GEMM kernels.
#pragma once

#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

namespace w4a8 {

enum Epilogue : int {
    kEpiStore = 0,    // out16[r, n] = fp16(acc * a_scale)
    kEpiSilu = 1,     // out16[r, n] = silu_and_mul(gate n, up n + N/2)
    kEpiScatter = 2,  // out32[sid / out_top_k, n] += topk_w[sid] * acc * a_scale (atomic)
};

// Rows are padded-sorted positions r in [0, P). Row r is live when r < ntp (or P when ntp is
// null) and sid = sorted_ids[r] (r when null) < num_valid; its activation row is r when
// src_identity, else sid / top_k; its expert is expert_ids[r / block_m] (0 when null).
struct GemmArgs {
    const uint8_t* x_fp8;
    const float* act_scales;
    const int32_t* w;
    const __half* scales;
    const int32_t* zeros;       // null = symmetric zero point 8
    const int32_t* sorted_ids;  // null = identity (dense)
    const int32_t* expert_ids;  // null = expert 0
    const int32_t* ntp;         // null = P
    const float* topk_weights;  // scatter only
    __half* out16;
    float* out32;
    int64_t K;
    int N;          // weight rows per expert (2*inter for the fused SiLU)
    int G;          // K groups
    int E;
    int P;
    int num_valid;
    int top_k;
    int out_top_k;
    int block_m;
    int src_identity;
    int e2m1;
    int kc;         // activation chunk (set by the launcher)
    int info_off;   // byte offset of the per-row table in dynamic shared memory (launcher)
};

bool mma_path_ok(const GemmArgs& a);

// ---- persistent streaming GEMV (gemv_stream.cu) ----
enum StreamMode : int {
    kStreamStore = 0,      // out16[r, n] = fp16(acc * a_scale)
    kStreamSilu = 1,       // out16[r, n] = silu_and_mul(gate n, up n + N/2)   (N/2 columns)
    kStreamScatter = 2,    // out32[sid / out_top_k, n] += topk_w[sid] * acc * a_scale
    kStreamSiluQuant = 3,  // finish only: SiLU row, then quantise it as the next GEMM's operand
};

// Output block of the operand quantiser (e4m3 bytes, scales, fp16 operand copy, group sums).
struct OperandOut {
    uint8_t* xq;
    float* scales;
    __half* xh;
    float2* xsum;
};

struct StreamArgs {
    const __half* xh;           // (rows, K) fp16 operand copy of the e4m3 activations
    const float2* xsum;         // (rows, G) per-group {K0, S} activation sums (see gemv_stream.cu)
    const float* act_scales;    // (rows,)
    const int32_t* w;
    const __half* scales;
    const int32_t* zeros;
    const int32_t* sorted_ids;
    const int32_t* expert_ids;
    const int32_t* ntp;
    const float* topk_weights;
    __half* out16;
    float* out32;
    float* part;                // fp32 partials [ks][P][N]
    int* counter;               // unused by the static schedule; kept zero
    int64_t K;
    int N, G, E, P, num_valid, top_k, out_top_k, block_m, src_identity, mode;
    int ks_n, rg_n, force_part; // set by the launcher
    OperandOut next;            // kStreamSiluQuant: where the quantised SiLU rows go
    __half* out_silu;           // kStreamSiluQuant: optional fp16 SiLU rows (P, N/2)
};

bool stream_path_ok(int64_t K, int G, int e2m1, const void* w);
size_t stream_partials_bytes(int64_t P, int64_t N, int64_t K);
int launch_w4_stream(StreamArgs a, cudaStream_t stream);

// ---- tcgen05 tile GEMM (gemm_tc.cu) ----
// Rows as in GemmArgs; activations are the operand quantiser's e4m3 bytes plus group sums.
struct TcArgs {
    const __half* x;            // (x_rows, K) fp16 source rows (tokens, or the SiLU rows)
    uint8_t* xs;                // scratch (P_pad, K): sorted-order e4m3 rows (tc_carve)
    float* asc_s;               // scratch (P_pad,): sorted-order activation scales
    float* ssum;                // scratch (K/128, P_pad): sorted-order group sums, group-major
    // Token-level operand (gather case, x_rows < P): each source row quantised once, then
    // gathered into sorted order. Null: every sorted row is quantised from x.
    uint8_t* tq;                // (x_rows, K) e4m3 bytes
    float* tq_scale;            // (x_rows,)
    float* tq_sum;              // (x_rows, K/128)
    int x_rows;
    const int32_t* w;
    const __half* scales;
    const int32_t* zeros;
    const int32_t* sorted_ids;
    const int32_t* expert_ids;
    const int32_t* ntp;
    __half* out16;
    int* err;                   // set to a non-zero code when a bounded wait gives up
    int64_t K;
    int N, G, E, P, P_pad, num_valid, top_k, block_m, src_identity, silu;
};
bool tc_path_ok(int64_t K, int group_size, int e2m1, const void* w, int block_m);
// Scratch of the tile path for P sorted rows: carved by tc_carve into xs / asc_s / ssum.
size_t tc_scratch_bytes(int64_t P, int64_t K);
void tc_carve(void* base, int64_t P, int64_t K, TcArgs& t);
int launch_w4_tc(TcArgs a, cudaStream_t stream);
// Quantise rows [0, min(M, row_limit)) of x (fp16) into the streaming GEMV operand format.
int launch_operand_quant(const void* x, OperandOut o, int64_t M, int64_t K,
                         const int32_t* row_limit, cudaStream_t stream);
int launch_w4_gemm(GemmArgs a, int epi, int row_tile, bool scalar, int64_t est_rows,
                   cudaStream_t stream);

}  // namespace w4a8
