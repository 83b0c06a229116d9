// ep_dispatch.cu — expert-parallel dispatch and combine around the NCCL all-to-alls.
//
// Dispatch: slot s = t*top_k + j goes to rank d = topk_ids[s] / experts_per_rank (clamped to
// [0, world)). Its send row is d*capacity + pos, pos = the number of earlier slots (in slot
// order) bound for d, so every chunk keeps slot order. One CTA per slot counts those earlier
// slots, then copies token t's fp16 row into the send buffer and writes the local expert id.
// Rows no slot claims keep id -1 (set by a memset before the launch) and are skipped by the
// receiver's layer.
//
// Combine: out[t, n] = sum_{j ascending} w[t*top_k+j] * back[row(t*top_k+j), n] in fp32 (fmul
// then fadd), then + fp32(shared[t, n]) when a shared-expert output (fp16) is given: the same
// operations in the same order as the slot-order gather-reduce followed by the shared add.
#include <algorithm>

#include "common.cuh"
#include "internal.h"

namespace w4a8 {

namespace {

__device__ __forceinline__ int slot_dest(const int32_t* ids, int64_t s, int per_rank, int world) {
    const int d = ids[s] / per_rank;
    return d < 0 ? 0 : (d >= world ? world - 1 : d);
}

__global__ void __launch_bounds__(256)
ep_dispatch_kernel(const __half* __restrict__ x, const int32_t* __restrict__ topk_ids,
                   int64_t num_slots, int top_k, int64_t H, int per_rank, int world,
                   int64_t capacity, __half* __restrict__ send_x, int32_t* __restrict__ send_id,
                   int32_t* __restrict__ slot_row) {
    __shared__ int32_t part[8];
    __shared__ int32_t row_s;
    const int64_t s = blockIdx.x;
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int d = slot_dest(topk_ids, s, per_rank, world);
    int32_t cnt = 0;
    for (int64_t i = tid; i < s; i += blockDim.x) cnt += slot_dest(topk_ids, i, per_rank, world) == d;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) cnt += __shfl_xor_sync(0xffffffffu, cnt, o);
    if (lane == 0) part[warp] = cnt;
    __syncthreads();
    if (tid == 0) {
        int32_t pos = 0;
        for (int w = 0; w < (int)(blockDim.x >> 5); ++w) pos += part[w];
        const int32_t row = (int32_t)(d * capacity + pos);
        row_s = row;
        slot_row[s] = row;
        send_id[row] = topk_ids[s] - d * per_rank;
    }
    __syncthreads();
    const int64_t row = row_s;
    const int64_t t = s / top_k;
    const uint4* src = reinterpret_cast<const uint4*>(x + t * H);
    uint4* dst = reinterpret_cast<uint4*>(send_x + row * H);
    for (int64_t i = tid; i < H / 8; i += blockDim.x) dst[i] = __ldg(src + i);
}

constexpr int kMaxTopK = 16;

__global__ void __launch_bounds__(256)
ep_combine_kernel(const __half* __restrict__ back, const int32_t* __restrict__ slot_row,
                  const float* __restrict__ topk_w, const __half* __restrict__ shared,
                  float* __restrict__ out, int64_t H, int top_k) {
    __shared__ int32_t rows[kMaxTopK];
    __shared__ float wts[kMaxTopK];
    const int64_t t = blockIdx.y;
    if (threadIdx.x < top_k) {
        rows[threadIdx.x] = slot_row[t * top_k + threadIdx.x];
        wts[threadIdx.x] = topk_w[t * top_k + threadIdx.x];
    }
    __syncthreads();
    const int64_t n = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) * 8;
    if (n >= H) return;
    uint4 v[kMaxTopK];
#pragma unroll
    for (int j = 0; j < kMaxTopK; ++j)
        if (j < top_k) v[j] = __ldg(reinterpret_cast<const uint4*>(back + (int64_t)rows[j] * H + n));
    float acc[8];
#pragma unroll
    for (int c = 0; c < 8; ++c) acc[c] = 0.f;
#pragma unroll
    for (int j = 0; j < kMaxTopK; ++j) {
        if (j < top_k) {
            const float w = wts[j];
            const uint32_t h[4] = {v[j].x, v[j].y, v[j].z, v[j].w};
#pragma unroll
            for (int c = 0; c < 4; ++c) {
                const float2 f = __half22float2(*reinterpret_cast<const __half2*>(&h[c]));
                acc[2 * c] = __fadd_rn(acc[2 * c], __fmul_rn(w, f.x));
                acc[2 * c + 1] = __fadd_rn(acc[2 * c + 1], __fmul_rn(w, f.y));
            }
        }
    }
    if (shared) {
        const uint4 sv = *reinterpret_cast<const uint4*>(shared + t * H + n);
        const uint32_t h[4] = {sv.x, sv.y, sv.z, sv.w};
#pragma unroll
        for (int c = 0; c < 4; ++c) {
            const float2 f = __half22float2(*reinterpret_cast<const __half2*>(&h[c]));
            acc[2 * c] = __fadd_rn(acc[2 * c], f.x);
            acc[2 * c + 1] = __fadd_rn(acc[2 * c + 1], f.y);
        }
    }
    float4* o = reinterpret_cast<float4*>(out + t * H + n);
    o[0] = make_float4(acc[0], acc[1], acc[2], acc[3]);
    o[1] = make_float4(acc[4], acc[5], acc[6], acc[7]);
}

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; }

}  // namespace

}  // namespace w4a8

using namespace w4a8;

extern "C" int w4a8_ep_dispatch(const void* x, const int32_t* topk_ids, int64_t T, int64_t top_k,
                                int64_t H, int32_t experts_per_rank, int32_t world,
                                int64_t capacity, void* send_x, int32_t* send_id,
                                int32_t* slot_row, w4a8_stream_t stream) {
    if (T < 0 || top_k <= 0 || H <= 0 || experts_per_rank <= 0 || world <= 0 || capacity < 0)
        return set_error("ep_dispatch: bad sizes");
    if (H % 8 != 0) return set_error("ep_dispatch: hidden size must be a multiple of 8");
    if (capacity < T * top_k) return set_error("ep_dispatch: capacity < T * top_k");
    if ((int64_t)world * capacity > INT32_MAX) return set_error("ep_dispatch: size overflow");
    if (T == 0) return W4A8_OK;
    if (!x || !topk_ids || !send_x || !send_id || !slot_row)
        return set_error("ep_dispatch: null pointer");
    if (!aligned16(x) || !aligned16(send_x)) return set_error("ep_dispatch: rows must be 16-byte aligned");
    cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
    cudaError_t e = cudaMemsetAsync(send_id, 0xFF, (size_t)(world * capacity) * sizeof(int32_t), st);
    if (e != cudaSuccess) return (int)e;
    ep_dispatch_kernel<<<(unsigned)(T * top_k), 256, 0, st>>>(
        static_cast<const __half*>(x), topk_ids, T * top_k, (int)top_k, H, experts_per_rank,
        world, capacity, static_cast<__half*>(send_x), send_id, slot_row);
    return launch_status();
}

extern "C" int w4a8_ep_combine(const void* back, const int32_t* slot_row,
                               const float* topk_weights, const void* shared, float* out,
                               int64_t T, int64_t top_k, int64_t H, w4a8_stream_t stream) {
    if (T < 0 || top_k <= 0 || top_k > kMaxTopK || H <= 0)
        return set_error("ep_combine: bad sizes (top_k must be 1..16)");
    if (H % 8 != 0) return set_error("ep_combine: hidden size must be a multiple of 8");
    if (T == 0) return W4A8_OK;
    if (!back || !slot_row || !topk_weights || !out) return set_error("ep_combine: null pointer");
    if (!aligned16(back) || !aligned16(out) || (shared && !aligned16(shared)))
        return set_error("ep_combine: rows must be 16-byte aligned");
    const dim3 grid((unsigned)((H / 8 + 255) / 256), (unsigned)T);
    ep_combine_kernel<<<grid, 256, 0, reinterpret_cast<cudaStream_t>(stream)>>>(
        static_cast<const __half*>(back), slot_row, topk_weights,
        static_cast<const __half*>(shared), out, H, (int)top_k);
    return launch_status();
}
