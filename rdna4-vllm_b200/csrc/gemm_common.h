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
};

bool mma_path_ok(const GemmArgs& a);
int launch_w4_gemm(GemmArgs a, int epi, int row_tile, bool scalar, int64_t est_rows,
                   cudaStream_t stream);

}  // namespace w4a8
