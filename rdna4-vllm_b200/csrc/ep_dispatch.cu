// ep_dispatch.cu — expert-parallel dispatch and gather around the two NCCL all-to-alls.
//
// Protocol (rank r of `world`, experts split experts_per_rank per rank, T tokens per rank):
//   pack   — each token is quantised once (the oracle's per-token e4m3 rounding) and sent once
//            to every rank that owns at least one of its top_k experts, as one payload row:
//              [H e4m3 bytes (GEMV byte order)][H/128 group sums][scale]
//              [top_k local expert ids, -1 = slot not on that rank][top_k routing weights]
//            Chunk d of the send buffer holds rank d's rows in token order (row pos_d(t) = the
//            number of earlier tokens bound for d); unused rows keep id -1. pos (world, T) keeps
//            each token's row per rank (-1 = not sent). A second copy of every row, with the
//            shared expert as its only slot (weight 1), goes to the rank's own row block.
//   (all-to-all of the send buffer; the owner runs the decode layer on its received rows plus
//    its own shared-expert rows, which produces one fp32 row per payload row: the slot-order
//    weighted sum over the row's local experts)
//   gather — out[t] = sum over ranks d ascending of back[d, pos_d(t)] (fp32), then + the
//            rank's own shared-expert row.
// The reference has no expert parallelism (its expert_map is only forwarded to vLLM's align,
// w4a8_fp8_wmma/w4a8_fp8_wmma/moe_experts.py:587-589).
#include <algorithm>
#include <string>

#include "common.cuh"
#include "e4_operand.cuh"
#include "internal.h"

namespace w4a8 {

namespace {

constexpr int kPackThreads = 256;
constexpr int kMaxWorld = 32;
constexpr int kMaxTopK = 16;

__host__ __device__ inline int64_t ep_row_bytes(int64_t H, int64_t k) {
    return (H + 4 * (H / 128) + 4 + 8 * k + 15) / 16 * 16;
}

// Destination mask of token t: bit d set when one of its valid slots is owned by rank d.
__device__ __forceinline__ uint32_t dest_mask(const int32_t* ids, int64_t t, int k, int per_rank,
                                              int E) {
    uint32_t m = 0;
    for (int j = 0; j < k; ++j) {
        const int e = ids[t * k + j];
        if (e >= 0 && e < E) m |= 1u << (e / per_rank);
    }
    return m;
}

__global__ void __launch_bounds__(kPackThreads)
ep_pack_kernel(const __half* __restrict__ x, const int32_t* __restrict__ ids,
               const float* __restrict__ wts, int T, int k, int H, int per_rank, int world,
               int shared_id, uint8_t* __restrict__ send, uint8_t* __restrict__ own,
               int32_t* __restrict__ pos) {
    extern __shared__ __align__(16) uint8_t row[];  // the token's payload prefix
    __shared__ float red[32];
    __shared__ int cnt[kMaxWorld];
    const int t = blockIdx.x, tid = threadIdx.x;
    const int G = H / 128;
    const int E = per_rank * world;
    const int64_t rb = ep_row_bytes(H, k);
    if (tid < kMaxWorld) cnt[tid] = 0;
    // 1. quantise the row once: e4m3 bytes (GEMV order), group sums, scale
    float* xs = reinterpret_cast<float*>(row + H);
    quant_row_e4_block(x + (int64_t)t * H, H, row, xs, xs + G, red);
    // 2. rows of earlier tokens per destination
    const uint32_t mine = dest_mask(ids, t, k, per_rank, E);
    for (int u = tid; u < t; u += kPackThreads) {
        uint32_t m = dest_mask(ids, u, k, per_rank, E) & mine;
        while (m) {
            atomicAdd(&cnt[__ffs(m) - 1], 1);
            m &= m - 1;
        }
    }
    __syncthreads();
    // 3. one payload row per destination rank (+ the shared-expert row)
    const int prefix = H + 4 * G + 4;  // bytes of the e4m3 row, sums and scale
    for (int d = 0; d < world; ++d) {
        const bool has = (mine >> d) & 1u;
        if (tid == 0) pos[(int64_t)d * T + t] = has ? cnt[d] : -1;
        if (!has) continue;
        uint8_t* dst = send + ((int64_t)d * T + cnt[d]) * rb;
        for (int i = tid; i < prefix / 4; i += kPackThreads)
            reinterpret_cast<uint32_t*>(dst)[i] = reinterpret_cast<const uint32_t*>(row)[i];
        if (tid < k) {
            const int e = ids[(int64_t)t * k + tid];
            const bool here = e >= 0 && e < E && e / per_rank == d;
            reinterpret_cast<int32_t*>(dst + prefix)[tid] = here ? e - d * per_rank : -1;
            reinterpret_cast<float*>(dst + prefix + 4 * k)[tid] = here ? wts[(int64_t)t * k + tid] : 0.f;
        }
    }
    if (own) {
        uint8_t* dst = own + (int64_t)t * rb;
        for (int i = tid; i < prefix / 4; i += kPackThreads)
            reinterpret_cast<uint32_t*>(dst)[i] = reinterpret_cast<const uint32_t*>(row)[i];
        if (tid < k) {
            reinterpret_cast<int32_t*>(dst + prefix)[tid] = tid == 0 ? shared_id : -1;
            reinterpret_cast<float*>(dst + prefix + 4 * k)[tid] = tid == 0 ? 1.f : 0.f;
        }
    }
}

// out[t, n..n+3] = sum_{d ascending, pos[d,t] >= 0} back[d*T + pos[d,t], n..] (+ own[t, n..]).
__global__ void __launch_bounds__(256)
ep_gather_kernel(const float* __restrict__ back, const int32_t* __restrict__ pos,
                 const float* __restrict__ own, float* __restrict__ out, int T, int world, int H) {
    const int t = blockIdx.y;
    const int n = (blockIdx.x * blockDim.x + threadIdx.x) * 4;
    if (n >= H) return;
    float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
    for (int d = 0; d < world; ++d) {
        const int p = __ldg(pos + (int64_t)d * T + t);
        if (p < 0) continue;
        const float4 v = __ldg(reinterpret_cast<const float4*>(back + ((int64_t)d * T + p) * H + n));
        acc.x = __fadd_rn(acc.x, v.x);
        acc.y = __fadd_rn(acc.y, v.y);
        acc.z = __fadd_rn(acc.z, v.z);
        acc.w = __fadd_rn(acc.w, v.w);
    }
    if (own) {
        const float4 v = __ldg(reinterpret_cast<const float4*>(own + (int64_t)t * H + n));
        acc.x = __fadd_rn(acc.x, v.x);
        acc.y = __fadd_rn(acc.y, v.y);
        acc.z = __fadd_rn(acc.z, v.z);
        acc.w = __fadd_rn(acc.w, v.w);
    }
    *reinterpret_cast<float4*>(out + (int64_t)t * H + n) = acc;
}

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; }

}  // namespace

}  // namespace w4a8

using namespace w4a8;

extern "C" size_t w4a8_ep_row_bytes(int64_t H, int64_t top_k) {
    if (H <= 0 || top_k <= 0) return 0;
    return (size_t)ep_row_bytes(H, top_k);
}

extern "C" int w4a8_ep_pack(const void* x, const int32_t* topk_ids, const float* topk_weights,
                            int64_t T, int64_t top_k, int64_t H, int32_t experts_per_rank,
                            int32_t world, int32_t shared_local_id, void* send_rows,
                            void* own_rows, int32_t* pos, w4a8_stream_t stream) {
    const std::string o = "ep_pack";
    if (T < 0 || top_k <= 0 || top_k > kMaxTopK || H <= 0 || experts_per_rank <= 0 ||
        world <= 0 || world > kMaxWorld)
        return set_error(o + ": bad sizes (top_k 1..16, world 1..32)");
    if (H % 256 != 0) return set_error(o + ": hidden size must be a multiple of 256");
    if ((int64_t)world * T * ep_row_bytes(H, top_k) > ((int64_t)1 << 40))
        return set_error(o + ": size overflow");
    if (T == 0) return W4A8_OK;
    if (!x || !topk_ids || !topk_weights || !send_rows || !pos) return set_error(o + ": null pointer");
    if (!aligned16(x) || !aligned16(send_rows) || (own_rows && !aligned16(own_rows)))
        return set_error(o + ": rows must be 16-byte aligned");
    cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
    const int64_t rb = ep_row_bytes(H, top_k);
    const int64_t prefix = H + 4 * (H / 128) + 4;
    // every row's ids (and weights) start as -1 (NaN): rows no token claims are skipped
    cudaError_t e = cudaMemset2DAsync(static_cast<uint8_t*>(send_rows) + prefix, (size_t)rb, 0xFF,
                                      (size_t)(8 * top_k), (size_t)(world * T), st);
    if (e != cudaSuccess) return (int)e;
    const size_t smem = (size_t)prefix + 16;
    if (smem > 48 * 1024)
        cudaFuncSetAttribute(ep_pack_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    ep_pack_kernel<<<(unsigned)T, kPackThreads, smem, st>>>(
        static_cast<const __half*>(x), topk_ids, topk_weights, (int)T, (int)top_k, (int)H,
        experts_per_rank, world, shared_local_id, static_cast<uint8_t*>(send_rows),
        static_cast<uint8_t*>(own_rows), pos);
    return launch_status();
}

extern "C" size_t w4a8_ep_moe_rows_workspace_size(int64_t R, int64_t top_k, int64_t E, int64_t H,
                                                 int64_t I) {
    if (R < 0 || top_k <= 0 || E <= 0 || H <= 0 || I <= 0) return 0;
    return fused_decode_workspace(R, top_k, E, H, I);
}

extern "C" int w4a8_ep_moe_rows(const void* rows, int64_t R, int64_t top_k, int64_t E,
                                const void* p13, const void* p2, int64_t H, int64_t I,
                                float* out, void* workspace, size_t workspace_bytes,
                                w4a8_stream_t stream) {
    const std::string o = "ep_moe_rows";
    if (R < 0 || top_k <= 0 || E <= 0 || H <= 0 || I <= 0) return set_error(o + ": bad sizes");
    if (!fused_decode_ok(R, top_k, E, H, I))
        return set_error(o + ": needs hidden, inter % 512 == 0, top_k <= 16, rows*top_k <= 65536");
    if (R == 0) return W4A8_OK;
    if (!rows || !p13 || !p2 || !out) return set_error(o + ": null pointer");
    if (!aligned16(rows) || !aligned16(p13) || !aligned16(p2) || !aligned16(out))
        return set_error(o + ": buffers must be 16-byte aligned");
    if (!workspace || workspace_bytes < fused_decode_workspace(R, top_k, E, H, I))
        return set_error(o + ": workspace too small");
    return launch_fused_decode_rows(rows, ep_row_bytes(H, top_k), R, top_k, E, p13, p2, H, I, out,
                                    workspace, reinterpret_cast<cudaStream_t>(stream));
}

extern "C" int w4a8_ep_gather(const float* back, const int32_t* pos, const float* own_out,
                              float* out, int64_t T, int32_t world, int64_t H,
                              w4a8_stream_t stream) {
    if (T < 0 || world <= 0 || world > kMaxWorld || H <= 0 || H % 4 != 0)
        return set_error("ep_gather: bad sizes");
    if (T == 0) return W4A8_OK;
    if (!back || !pos || !out) return set_error("ep_gather: null pointer");
    if (!aligned16(back) || !aligned16(out) || (own_out && !aligned16(own_out)))
        return set_error("ep_gather: rows must be 16-byte aligned");
    const dim3 grid((unsigned)((H / 4 + 255) / 256), (unsigned)T);
    ep_gather_kernel<<<grid, 256, 0, reinterpret_cast<cudaStream_t>(stream)>>>(
        back, pos, own_out, out, (int)T, world, (int)H);
    return launch_status();
}
