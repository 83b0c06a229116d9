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

// Fused decode layer (moe_decode.cu): three launches, see there.
bool fused_decode_ok(int64_t T, int64_t top_k, int64_t E, int64_t H, int64_t I);
size_t fused_decode_workspace(int64_t T, int64_t top_k, int64_t E, int64_t H, int64_t I);
int launch_fused_decode(const void* x, const int32_t* topk_ids, const float* topk_weights,
                        int64_t T, int64_t top_k, int64_t E, const int32_t* w13, const void* s13,
                        const int32_t* z13, const int32_t* w2, const void* s2, const int32_t* z2,
                        int64_t H, int64_t I, void* out, void* workspace, cudaStream_t st,
                        const void* p13 = nullptr, const void* p2 = nullptr);
// The same layer on expert-parallel payload rows (w4a8_ep_pack layout); fp32 (R, H) output.
int launch_fused_decode_rows(const void* rows, int64_t row_bytes, int64_t R, int64_t top_k,
                             int64_t E, const void* p13, const void* p2, int64_t H, int64_t I,
                             float* out, void* workspace, cudaStream_t st);
size_t stream_pack_bytes(int64_t E, int64_t N, int64_t K);
int launch_stream_pack(const int32_t* w, const void* scales, const int32_t* zeros, int64_t E,
                       int64_t N, int64_t K, int gate_up, void* packed, cudaStream_t st);

}  // namespace w4a8
