/*
 * w4a8_b200.h — C ABI of the B200 (sm_100a) W4A8 GEMM / MoE library.
 *
 * Every entry point takes plain device pointers, sizes and a cudaStream_t, launches on that
 * stream, never synchronises the host and never allocates device memory: scratch comes from
 * the caller through a (workspace, workspace_bytes) pair whose size the matching
 * *_workspace_size() query returns. This keeps every call capturable into a CUDA graph and
 * lets the torch shim hand out memory from its caching allocator.
 *
 * Data formats (identical to the reference op surface, w4a8_fp8_wmma/bindings.cpp:389-412):
 *   x            fp16 (rows, K), row-major, contiguous.
 *   w_packed     int32 (N, K/8) dense or (E, N, K/8) grouped; nibble j of word w holds the
 *                unsigned 4-bit code of input channel k = 8w + j (low nibble first).
 *   scales       fp16 (N, K/g) or (E, N, K/g), per (output channel, K group).
 *   w_zeros      int32 (N/8, K/g) or (E, N/8, K/g); nibble (n % 8) of word [n/8][g] is the
 *                zero point of channel n. NULL selects the symmetric uint4b8 zero point 8.
 *   routing      sorted_token_ids (P,), expert_ids (P/block_m,), num_tokens_post_padded (1,),
 *                all int32, in the moe_align_block_size contract (expert-sorted, each expert's
 *                run padded to block_m with the sentinel num_slots = T*top_k).
 *
 * Arithmetic (the reference's torch oracle, test_correctness.py:92-119):
 *   a_scale[r] = max(amax_k |x[r,k]|, 4.48e-6f) / 448   (IEEE fp32 divide)
 *   xq[r,k]    = e4m3_rn(x[r,k] / a_scale[r])            (IEEE fp32 divide, RNE, satfinite)
 *   out[r,n]   = fp16( (sum_g scale[n,g] * sum_{k in g} xq[r,k] * (q[n,k] - z[n,g])) * a_scale[r] )
 *
 * Return value: 0 on success, W4A8_ERR_INVALID (-1) for a rejected argument (message in
 * w4a8_last_error()), or a positive cudaError_t from the launch.
 */
#ifndef W4A8_B200_H
#define W4A8_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef struct CUstream_st* w4a8_stream_t; /* == cudaStream_t */

#if defined(__GNUC__)
#define W4A8_API __attribute__((visibility("default")))
#else
#define W4A8_API
#endif

#define W4A8_OK 0
#define W4A8_ERR_INVALID (-1)

/* Kernel ids carried over the ABI, equal to the reference's enums (kernel_names.h:18-46). */
#define W4A8_DENSE_REFERENCE_SCALAR 0
#define W4A8_DENSE_PREFILL_WMMA 5
#define W4A8_DENSE_PREFILL_WMMA_ASHUFFLE 10
#define W4A8_DENSE_DECODE_GEMV 11
#define W4A8_MOE_SCALAR 0
#define W4A8_MOE_WMMA 6
#define W4A8_MOE_GEMV 7

/* Message describing the last W4A8_ERR_INVALID returned on this host thread. */
W4A8_API const char* w4a8_last_error(void);

/* Library version string, e.g. "w4a8_b200 0.1 sm_100a". */
W4A8_API const char* w4a8_version(void);

/*
 * Per-token e4m3 activation quantisation.
 * Replaces moe_compute_act_fp8_kernel (w4a8_fp8_wmma/moe_kernel.hip:87-130) and
 * compute_act_fp8_and_scales_kernel (w4a8_fp8_wmma/w4a8_fp8_wmma_kernel.hip:153-201), with the
 * oracle's divide-based rounding (test_correctness.py:74-76) rather than the kernels' reciprocal.
 *   x (M, K) fp16 -> x_fp8 (M, K) e4m3 bytes, act_scales (M,) fp32.
 */
W4A8_API int w4a8_act_quant_fp8(const void* x, uint8_t* x_fp8, float* act_scales, int64_t M, int64_t K,
                       w4a8_stream_t stream);

/*
 * moe_align_block_size: sort the (token, slot) pairs by expert, ascending slot id inside each
 * expert, pad each expert's run to a multiple of block_m with the sentinel num_slots.
 * Replaces vLLM's moe_align_block_size as called at w4a8_fp8_wmma/moe_experts.py:587-589;
 * order defined by the reference's Python moe_align (test_moe_correctness.py:49-67).
 *   topk_ids (num_slots,) int32 expert per slot (slot = t*top_k + j).
 *   expert_map (num_experts,) int32 global->local expert id (-1 = not local) or NULL.
 *   num_local_experts: experts after mapping (== num_experts when expert_map is NULL).
 *   sorted_token_ids (sorted_capacity,), expert_ids (sorted_capacity/block_m,),
 *   num_tokens_post_padded (1,). Entries past num_tokens_post_padded are set to the sentinel
 *   (sorted ids) and -1 (expert ids). sorted_capacity must be a multiple of block_m and at
 *   least num_slots + num_local_experts*(block_m-1).
 */
W4A8_API size_t w4a8_moe_align_workspace_size(int32_t num_local_experts);
W4A8_API int w4a8_moe_align_block_size(const int32_t* topk_ids, int64_t num_slots, int32_t num_experts,
                              int32_t num_local_experts, int32_t block_m,
                              const int32_t* expert_map, int32_t* sorted_token_ids,
                              int64_t sorted_capacity, int32_t* expert_ids,
                              int32_t* num_tokens_post_padded, void* workspace,
                              size_t workspace_bytes, w4a8_stream_t stream);

/*
 * moe_align_block_size without a workspace argument, for callers that cannot allocate device
 * memory when they route (a framework's private memory pool, a binding with no allocator, a
 * deployment that bans cudaMalloc after start-up). No counterpart in the reference: its align
 * comes from vLLM. The per-expert offsets live in a fixed 16 KB device array inside the
 * library, so num_local_experts is limited to 4095 (larger values return W4A8_ERR_INVALID).
 * The first call on each device looks the array's address up (cudaGetSymbolAddress) with that
 * device current; make that first call before any stream capture. The address is cached for the
 * life of the process, which assumes the device's primary context lives as long (no
 * cudaDeviceReset between calls). A failed lookup returns W4A8_ERR_INVALID with the CUDA error
 * in w4a8_last_error(). The array is shared by all calls on a device: calls that overlap on the
 * GPU (different streams, no ordering) race.
 * Arguments and results are those of w4a8_moe_align_block_size.
 */
W4A8_API int w4a8_moe_align_block_size_noalloc(const int32_t* topk_ids, int64_t num_slots,
                                               int32_t num_experts, int32_t num_local_experts,
                                               int32_t block_m, const int32_t* expert_map,
                                               int32_t* sorted_token_ids,
                                               int64_t sorted_capacity, int32_t* expert_ids,
                                               int32_t* num_tokens_post_padded,
                                               w4a8_stream_t stream);

/*
 * Dense W4A8 GEMM: out (M, N) fp16 = x (M, K) fp16 @ dequant(w)^T.
 * Replaces launch_mmq_fp8_gemm_gfx1201 (w4a8_fp8_wmma/w4a8_fp8_wmma_kernel.hip:2507-2994) behind
 * the op mmq_fp8_gemm (bindings.cpp:98-146). kernel: 0 scalar golden, 5/10 tile path, 11 decode
 * GEMV path; every id computes the same function.
 */
W4A8_API size_t w4a8_mmq_fp8_gemm_workspace_size(int64_t M, int64_t N, int64_t K);
W4A8_API int w4a8_mmq_fp8_gemm(const void* x, const int32_t* w_packed, const void* scales,
                      const int32_t* w_zeros, void* out, int64_t M, int64_t N, int64_t K,
                      int64_t group_size, int32_t kernel, int32_t weight_is_e2m1,
                      void* workspace, size_t workspace_bytes, w4a8_stream_t stream);

/*
 * Grouped MoE GEMM: for each padded sorted row r < num_tokens_post_padded with
 * s = sorted_token_ids[r] < T*top_k:  out[r] = x[s / top_k] @ dequant(W[expert_ids[r/block_m]])^T.
 * Padding rows are written as zeros. out is (P, N) fp16.
 * Replaces launch_mmq_fp8_moe_gemm_gfx1201 (w4a8_fp8_wmma/moe_kernel.hip:1358) behind the op
 * mmq_fp8_moe_gemm (bindings.cpp:178-228). kernel: 0 scalar, 6 tile ("wmma"), 7 GEMV.
 */
/* Workspace of the three grouped GEMM entry points: x_rows = T for mmq_fp8_moe_gemm and
 * mmq_fp8_moe_gemm1_silu (activations gathered by token), x_rows = P for the scatter op. */
W4A8_API size_t w4a8_moe_gemm_workspace_size(int64_t x_rows, int64_t P, int64_t N, int64_t K);
W4A8_API int w4a8_mmq_fp8_moe_gemm(const void* x, const int32_t* w_packed, const void* scales,
                          const int32_t* w_zeros, const int32_t* sorted_token_ids,
                          const int32_t* expert_ids, const int32_t* num_tokens_post_padded,
                          void* out, int64_t T, int64_t E, int64_t N, int64_t K, int64_t P,
                          int64_t group_size, int64_t top_k, int64_t block_m, int32_t kernel,
                          int32_t weight_is_e2m1, void* workspace, size_t workspace_bytes,
                          w4a8_stream_t stream);

/*
 * Fused gate_up GEMM + SiLU-and-mul: w_packed is (E, 2*inter, K/8) = [gate | up] rows; out is
 * (P, inter) fp16 = fp16(silu(fp16(gate))) * fp16(up), bit-identical to mmq_fp8_moe_gemm
 * followed by vLLM silu_and_mul. Replaces run_moe_gemm1_silu
 * (w4a8_fp8_wmma/moe_kernel.hip:1264-1325, epilogue :555-565) behind mmq_fp8_moe_gemm1_silu
 * (bindings.cpp:234-288). Uses the same workspace size as w4a8_mmq_fp8_moe_gemm. The C ABI
 * accepts kernel ids 0, 6 and 7; the torch op keeps the reference's 'wmma'-only check.
 */
W4A8_API int w4a8_mmq_fp8_moe_gemm1_silu(const void* x, const int32_t* w_packed, const void* scales,
                                const int32_t* w_zeros, const int32_t* sorted_token_ids,
                                const int32_t* expert_ids, const int32_t* num_tokens_post_padded,
                                void* out, int64_t T, int64_t E, int64_t N, int64_t K, int64_t P,
                                int64_t group_size, int64_t top_k, int64_t block_m,
                                int32_t kernel, int32_t weight_is_e2m1, void* workspace,
                                size_t workspace_bytes, w4a8_stream_t stream);

/*
 * Down GEMM + topk-weighted atomic scatter: x is the (P, K) post-activation buffer (row r is
 * gathered by identity); for each valid row r with s = sorted_token_ids[r]:
 *   output[s / top_k, :] += topk_weights[s] * (x[r] @ dequant(W[e])^T)   (fp32 atomics)
 * output is (M_out, N) fp32 and must be pre-zeroed by the caller.
 * Replaces the SCATTER=true path of run_moe_gemm (w4a8_fp8_wmma/moe_kernel.hip:1044-1056,
 * 1400-1436) behind mmq_fp8_moe_gemm_scatter (bindings.cpp:293-353).
 */
W4A8_API int w4a8_mmq_fp8_moe_gemm_scatter(const void* x, const int32_t* w_packed, const void* scales,
                                  const int32_t* w_zeros, const int32_t* sorted_token_ids,
                                  const int32_t* expert_ids,
                                  const int32_t* num_tokens_post_padded,
                                  const float* topk_weights, float* output, int64_t M_out,
                                  int64_t E, int64_t N, int64_t K, int64_t P, int64_t group_size,
                                  int64_t top_k, int64_t block_m, int32_t kernel,
                                  int32_t weight_is_e2m1, void* workspace,
                                  size_t workspace_bytes, w4a8_stream_t stream);

/*
 * Topk-weighted gather-reduce: out[t, n] = sum_{j<top_k} topk_weights[t*top_k+j] *
 * out2[row(t*top_k+j), n] in fp32, j ascending, where row(slot) is the padded row holding
 * that slot (missing slots contribute nothing). out2 (P, N) fp16 -> out (M, N) fp32, every
 * element written. Replaces moe_build_inverse_map_kernel + moe_gather_reduce_kernel
 * (w4a8_fp8_wmma/moe_kernel.hip:1230-1262, launcher :1437-1464) behind
 * mmq_fp8_moe_gather_reduce (bindings.cpp:358-379).
 */
W4A8_API size_t w4a8_moe_gather_reduce_workspace_size(int64_t M, int64_t top_k);
W4A8_API int w4a8_moe_gather_reduce(const void* out2, const int32_t* sorted_token_ids,
                           const float* topk_weights, const int32_t* num_tokens_post_padded,
                           float* out, int64_t M, int64_t N, int64_t P, int64_t top_k,
                           void* workspace, size_t workspace_bytes, w4a8_stream_t stream);

/*
 * silu_and_mul on fp16 rows: x (M, 2*inter) [gate | up] -> out (M, inter),
 * out = fp16(g / (1 + expf(-g))) * up with g the fp16 gate (IEEE divide, half*half product).
 * The unfused composition's activation step between gate_up and down, which the reference
 * takes from vLLM (apply_moe_activation, w4a8_fp8_wmma/w4a8_fp8_wmma/moe_experts.py:620-630);
 * the fused gate_up op applies the same arithmetic in its epilogue.
 */
W4A8_API int w4a8_silu_and_mul(const void* x, void* out, int64_t M, int64_t inter,
                               w4a8_stream_t stream);

/*
 * MoE router in one launch: logits (num_tokens, num_experts) of dtype 0 = fp32, 1 = fp16,
 * 2 = bf16 -> topk_ids (num_tokens, top_k) int32 and topk_weights (num_tokens, top_k) fp32:
 * softmax over the experts (fp32), the top_k largest in descending order (ties: lower expert
 * index first), divided by their sum when renormalize != 0. expert_counts (num_experts,) int32,
 * optional (may be null), receives the number of slots routed to each expert (zeroed first).
 * Replaces the router vLLM runs before the reference's moe_align call
 * (w4a8_fp8_wmma/w4a8_fp8_wmma/moe_experts.py:587-589 takes its topk_ids / topk_weights).
 * Limits: num_experts <= 1024, top_k <= 16.
 */
W4A8_API int w4a8_route_topk(const void* logits, int32_t logits_dtype, int64_t num_tokens,
                             int32_t num_experts, int32_t top_k, int32_t renormalize,
                             int32_t* topk_ids, float* topk_weights, int32_t* expert_counts,
                             w4a8_stream_t stream);

/*
 * Expert-parallel dispatch (no counterpart in the reference, which has no expert parallelism;
 * its expert_map is only forwarded to vLLM's align, w4a8_fp8_wmma/w4a8_fp8_wmma/
 * moe_experts.py:587-589). Each of the T tokens is quantised once (the oracle's per-token e4m3
 * rounding) and written once per rank that owns one of its top_k experts (rank d owns global
 * experts [d*experts_per_rank, (d+1)*experts_per_rank)), as one payload row of
 * w4a8_ep_row_bytes(H, top_k) bytes:
 *   [H e4m3 bytes][H/128 fp32 group sums][fp32 scale][top_k int32 local ids][top_k fp32 weights]
 * (local id -1 = that slot is on another rank). send_rows is (world, T) rows: chunk d holds
 * rank d's rows in token order; rows no token claims get ids -1. pos (world, T) int32 receives
 * each token's row in chunk d or -1. own_rows (T rows, or NULL) receives every token once more
 * with the single slot shared_local_id at weight 1 (a replicated shared expert). Ids outside
 * [0, world*experts_per_rank) are dropped. H % 256 == 0, top_k <= 16, world <= 32.
 */
W4A8_API size_t w4a8_ep_row_bytes(int64_t H, int64_t top_k);
W4A8_API int w4a8_ep_pack(const void* x, const int32_t* topk_ids, const float* topk_weights,
                          int64_t T, int64_t top_k, int64_t H, int32_t experts_per_rank,
                          int32_t world, int32_t shared_local_id, void* send_rows,
                          void* own_rows, int32_t* pos, w4a8_stream_t stream);

/*
 * The gated MoE layer on R payload rows (received rows, then the own shared-expert rows): for
 * every row, out[r] = sum over its valid local slots j (ascending) of
 * w_j * fp16(down_e(silu_and_mul(gate_up_e(row)))) in fp32, with the expert weights prepacked
 * by w4a8_stream_pack (E local experts). out is (R, H) fp32; rows without a valid slot are 0.
 * Same arithmetic as w4a8_moe_decode. Workspace: w4a8_ep_moe_rows_workspace_size.
 */
W4A8_API size_t w4a8_ep_moe_rows_workspace_size(int64_t R, int64_t top_k, int64_t E, int64_t H,
                                                int64_t I);
W4A8_API int w4a8_ep_moe_rows(const void* rows, int64_t R, int64_t top_k, int64_t E,
                              const void* p13, const void* p2, int64_t H, int64_t I, float* out,
                              void* workspace, size_t workspace_bytes, w4a8_stream_t stream);

/*
 * Expert-parallel gather: out[t] = sum over ranks d ascending with pos[d, t] >= 0 of
 * back[d*T + pos[d, t]] (fp32 rows returned by the owners), then + own_out[t] (the shared
 * expert's fp32 row) when own_out is not NULL. out is (T, H) fp32.
 */
W4A8_API int w4a8_ep_gather(const float* back, const int32_t* pos, const float* own_out,
                            float* out, int64_t T, int32_t world, int64_t H,
                            w4a8_stream_t stream);

/*
 * Whole gated MoE layer at decode sizes in one call: moe_align (block 8) -> gate_up GEMV ->
 * silu_and_mul -> down GEMV -> topk-weighted reduce, the decode branch of the reference's
 * composition _run_grouped_moe (w4a8_fp8_wmma/w4a8_fp8_wmma/moe_experts.py:563-648), which
 * there takes four ops plus vLLM's align and activation.
 *   x (T, H) fp16; topk_ids (T, top_k) int32; topk_weights (T, top_k) fp32;
 *   w13 (E, 2I, H/8) int32 [gate | up], s13 (E, 2I, H/128) fp16, z13 (E, 2I/8, H/128) or NULL;
 *   w2 (E, H, I/8), s2 (E, H, I/128), z2 (E, H/8, I/128) or NULL;
 *   out (T, H) fp16 = sum_j topk_weights[t, j] * fp16(down_j(silu_and_mul(gate_up_j(x_t)))).
 * group_size must be 128 and H, I multiples of 512.
 */
W4A8_API size_t w4a8_moe_decode_workspace_size(int64_t T, int64_t top_k, int64_t E, int64_t H,
                                               int64_t I);
W4A8_API int w4a8_moe_decode(const void* x, const int32_t* topk_ids, const float* topk_weights,
                             int64_t T, int64_t top_k, int64_t E, const int32_t* w13,
                             const void* s13, const int32_t* z13, const int32_t* w2,
                             const void* s2, const int32_t* z2, int64_t H, int64_t I,
                             int64_t group_size, void* out, void* workspace,
                             size_t workspace_bytes, w4a8_stream_t stream);

/*
 * Load-time weight prepack for the decode GEMV (no counterpart kernel in the reference; it is
 * the device-side analogue of the reference's load-time layout converters,
 * w4a8_fp8_wmma/w4a8_fp8_wmma/moe_experts.py:331-482). One GEMM operand (w13 with
 * gate_up = 1, or w2 with gate_up = 0) in the op layout above becomes one contiguous
 * 34,048-byte block per (expert, 128-row slice, 512-wide K chunk): the slice's codes in the
 * GEMV's swizzled shared-memory order, then its fp16 scales and packed zero points (8 when
 * w_zeros is NULL). A gate_up slice holds gate rows [64s, 64s+64) and the matching up rows.
 * Needs K % 512 == 0, N % 128 == 0. Size: w4a8_stream_pack_size.
 */
W4A8_API size_t w4a8_stream_pack_size(int64_t E, int64_t N, int64_t K);
W4A8_API int w4a8_stream_pack(const int32_t* w_packed, const void* scales, const int32_t* w_zeros,
                              int64_t E, int64_t N, int64_t K, int32_t gate_up, void* packed,
                              size_t packed_bytes, w4a8_stream_t stream);

/*
 * w4a8_moe_decode on prepacked weights (p13 from w4a8_stream_pack(w13, gate_up = 1), p2 from
 * w4a8_stream_pack(w2, gate_up = 0)): the same arithmetic and result, in three launches
 * (routing sort + token quantisation; gate_up GEMV with SiLU; down GEMV with the slot-order
 * reduce). Needs hidden and inter multiples of 512, top_k <= 16, T*top_k <= 65536,
 * E <= 4096. Workspace: w4a8_moe_decode_workspace_size.
 */
W4A8_API int w4a8_moe_decode_packed(const void* x, const int32_t* topk_ids,
                                    const float* topk_weights, int64_t T, int64_t top_k,
                                    int64_t E, const void* p13, const void* p2, int64_t H,
                                    int64_t I, void* out, void* workspace,
                                    size_t workspace_bytes, w4a8_stream_t stream);

#ifdef __cplusplus
}
#endif

#endif /* W4A8_B200_H */
