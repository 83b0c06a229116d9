// internal.h — launchers shared between the translation units of libw4a8_b200.so.
#pragma once

#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stddef.h>
#include <stdint.h>

namespace w4a8 {

// row_limit (optional, device): rows at or past row_limit[0] are skipped.
int launch_act_quant(const void* x, uint8_t* xq, float* scales, int64_t M, int64_t K,
                     cudaStream_t stream, const int32_t* row_limit = nullptr);

// moe_align_block_size; slot_to_row (optional) receives each placed slot's padded row.
int launch_moe_align(const int32_t* topk_ids, int64_t num_slots, int32_t num_experts,
                     int32_t num_local_experts, int32_t block_m, const int32_t* expert_map,
                     int32_t* sorted_token_ids, int64_t sorted_capacity, int32_t* expert_ids,
                     int32_t* num_tokens_post_padded, void* workspace, size_t workspace_bytes,
                     int32_t* slot_to_row, cudaStream_t stream);

// Gather-reduce with a prebuilt slot->row map (-1 = absent); fp32 or fp16 output.
int launch_gather_reduce(const __half* out2, const int32_t* slot_to_row, const float* topk_w,
                         void* out, bool out_half, int64_t M, int64_t N, int top_k,
                         cudaStream_t stream);

}  // namespace w4a8
