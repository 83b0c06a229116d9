// moe_align.cu — deterministic moe_align_block_size.
//
// Order contract (the reference's Python moe_align, w4a8_fp8_wmma/test_moe_correctness.py:49-67):
// experts ascending; inside an expert, slot ids (t*top_k + j) ascending; each expert's run is
// padded up to a multiple of block_m with the sentinel num_slots; an expert with no slots gets
// no block; num_tokens_post_padded = total padded length.
//
// Two launches:
//   1. align_count_kernel (one CTA): per-expert histogram in shared memory, exclusive scan of
//      the padded counts into `offsets` (workspace), expert_ids per block, the tail fill.
//   2. align_place_kernel (one warp per local expert): each warp walks the slot list in order
//      with __ballot_sync and writes its expert's slots at offsets[e] + running rank, which is
//      stable by construction. For many slots (prefill) align_place_chunked_kernel ranks
//      2048-slot chunks in parallel instead. The padding sentinels come from the count kernel.
// The slot list is staged in shared memory as int16 local expert ids when it fits.
#include "common.cuh"
#include "internal.h"

namespace w4a8 {

namespace {

constexpr int kCountThreads = 1024;
constexpr int kPlaceWarps = 8;
constexpr int64_t kMaxSmemSlots = 96 * 1024 / 2;  // int16 ids in 96 KB of shared memory

__device__ __forceinline__ int local_expert(const int32_t* __restrict__ topk_ids,
                                            const int32_t* __restrict__ expert_map, int64_t i,
                                            int num_experts) {
    const int e = topk_ids[i];
    if (e < 0 || e >= num_experts) return -1;
    return expert_map ? expert_map[e] : e;
}

__global__ void __launch_bounds__(kCountThreads)
align_count_kernel(const int32_t* __restrict__ topk_ids, int64_t num_slots, int num_experts,
                   int num_local, int block_m, const int32_t* __restrict__ expert_map,
                   int32_t* __restrict__ sorted_ids, int64_t capacity,
                   int32_t* __restrict__ expert_ids, int32_t* __restrict__ ntp_out,
                   int32_t* __restrict__ offsets) {
    extern __shared__ int32_t counts[];  // num_local entries
    __shared__ int32_t partial[kCountThreads];
    const int tid = threadIdx.x;
    for (int e = tid; e < num_local; e += kCountThreads) counts[e] = 0;
    __syncthreads();
    for (int64_t i = tid; i < num_slots; i += kCountThreads) {
        const int le = local_expert(topk_ids, expert_map, i, num_experts);
        if (le >= 0 && le < num_local) atomicAdd(&counts[le], 1);
    }
    __syncthreads();
    // Contiguous chunk of experts per thread -> local padded sum -> block exclusive scan.
    const int per = (num_local + kCountThreads - 1) / kCountThreads;
    const int e0 = min(tid * per, num_local), e1 = min(e0 + per, num_local);
    int32_t local = 0;
    for (int e = e0; e < e1; ++e) local += (counts[e] + block_m - 1) / block_m * block_m;
    partial[tid] = local;
    __syncthreads();
    for (int off = 1; off < kCountThreads; off <<= 1) {  // Hillis-Steele inclusive scan
        const int32_t v = tid >= off ? partial[tid - off] : 0;
        __syncthreads();
        partial[tid] += v;
        __syncthreads();
    }
    int32_t run = partial[tid] - local;  // exclusive prefix of this thread's chunk
    const int32_t sentinel = (int32_t)num_slots;
    for (int e = e0; e < e1; ++e) {
        offsets[e] = run;
        const int32_t padded = (counts[e] + block_m - 1) / block_m * block_m;
        for (int32_t b = run / block_m; b < (run + padded) / block_m; ++b) expert_ids[b] = e;
        for (int32_t p = run + counts[e]; p < run + padded; ++p) sorted_ids[p] = sentinel;
        run += padded;
    }
    const int32_t total = partial[kCountThreads - 1];
    if (tid == 0) {
        offsets[num_local] = total;
        ntp_out[0] = total;
    }
    for (int64_t i = total + tid; i < capacity; i += kCountThreads) sorted_ids[i] = sentinel;
    for (int64_t b = total / block_m + tid; b < capacity / block_m; b += kCountThreads)
        expert_ids[b] = -1;
}

template <bool kSmem>
__global__ void __launch_bounds__(kPlaceWarps * 32)
align_place_kernel(const int32_t* __restrict__ topk_ids, int64_t num_slots, int num_experts,
                   int num_local, const int32_t* __restrict__ expert_map,
                   const int32_t* __restrict__ offsets, int32_t* __restrict__ sorted_ids,
                   int32_t* __restrict__ slot_to_row) {
    extern __shared__ int16_t ids[];
    if (kSmem) {
        for (int64_t i = threadIdx.x; i < num_slots; i += blockDim.x)
            ids[i] = (int16_t)local_expert(topk_ids, expert_map, i, num_experts);
        __syncthreads();
    }
    const int lane = threadIdx.x & 31;
    const int e = blockIdx.x * kPlaceWarps + (threadIdx.x >> 5);
    if (e >= num_local) return;
    const int32_t base = offsets[e];
    const uint32_t lt = (1u << lane) - 1u;
    int32_t run = base;
    for (int64_t c = 0; c < num_slots; c += 32) {
        const int64_t i = c + lane;
        int le = -1;
        if (i < num_slots) le = kSmem ? (int)ids[i] : local_expert(topk_ids, expert_map, i, num_experts);
        const uint32_t m = __ballot_sync(0xffffffffu, le == e);
        if (le == e) {
            const int32_t pos = run + __popc(m & lt);
            sorted_ids[pos] = (int32_t)i;
            if (slot_to_row) slot_to_row[i] = pos;  // inverse map for the gather-reduce
        }
        run += __popc(m);
    }
}

// Chunked stable placement, for many slots and up to kChunkMaxExperts local experts. CTA c
// owns slots [c*kChunk, (c+1)*kChunk). It counts each expert's slots in the chunks before it
// (shared-memory histogram), then ranks its own slots in rounds of 1024 in slot order:
// __match_any_sync gives the rank among equal experts inside a warp, and a per-expert
// exclusive scan over the 32 warps gives the warp's offset. The padding sentinels are written
// by the count kernel.
constexpr int kChunk = 2048;
constexpr int kChunkThreads = 1024;
constexpr int kChunkMaxExperts = 512;
__global__ void __launch_bounds__(kChunkThreads)
align_place_chunked_kernel(const int32_t* __restrict__ topk_ids, int64_t num_slots,
                           int num_experts, int num_local, const int32_t* __restrict__ expert_map,
                           const int32_t* __restrict__ offsets, int32_t* __restrict__ sorted_ids,
                           int32_t* __restrict__ slot_to_row) {
    extern __shared__ int32_t csm[];
    int32_t* base = csm;                          // [num_local] running position per expert
    int32_t* tot = base + num_local;              // [num_local] count in the current round
    int32_t* wcnt = tot + num_local;              // [32][num_local] per-warp counts -> prefixes
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int64_t c0 = (int64_t)blockIdx.x * kChunk;
    const int64_t c1 = c0 + kChunk < num_slots ? c0 + kChunk : num_slots;
    for (int e = tid; e < num_local; e += kChunkThreads) base[e] = 0;
    __syncthreads();
    for (int64_t i = tid; i < c0; i += kChunkThreads) {
        const int le = local_expert(topk_ids, expert_map, i, num_experts);
        if (le >= 0 && le < num_local) atomicAdd(&base[le], 1);
    }
    __syncthreads();
    for (int e = tid; e < num_local; e += kChunkThreads) base[e] += offsets[e];
    const uint32_t lt = (1u << lane) - 1u;
    for (int64_t r0 = c0; r0 < c1; r0 += kChunkThreads) {
        for (int e = tid; e < 32 * num_local; e += kChunkThreads) wcnt[e] = 0;
        __syncthreads();
        const int64_t i = r0 + tid;
        int le = -1;
        if (i < c1) le = local_expert(topk_ids, expert_map, i, num_experts);
        if (le >= num_local) le = -1;
        const uint32_t peers = __match_any_sync(0xffffffffu, le);
        const int rank = __popc(peers & lt);
        if (le >= 0 && rank == 0) wcnt[warp * num_local + le] = __popc(peers);
        __syncthreads();
        for (int e = tid; e < num_local; e += kChunkThreads) {  // exclusive scan over warps
            int32_t run = 0;
            for (int w = 0; w < 32; ++w) {
                const int32_t v = wcnt[w * num_local + e];
                wcnt[w * num_local + e] = run;
                run += v;
            }
            tot[e] = run;
        }
        __syncthreads();
        if (le >= 0) {
            const int32_t pos = base[le] + wcnt[warp * num_local + le] + rank;
            sorted_ids[pos] = (int32_t)i;
            if (slot_to_row) slot_to_row[i] = pos;
        }
        __syncthreads();
        for (int e = tid; e < num_local; e += kChunkThreads) base[e] += tot[e];
    }
}

}  // namespace

}  // namespace w4a8

extern "C" size_t w4a8_moe_align_workspace_size(int32_t num_local_experts) {
    return w4a8::align_up(((size_t)num_local_experts + 1) * sizeof(int32_t), 256);
}

namespace w4a8 {

int launch_moe_align(const int32_t* topk_ids, int64_t num_slots, int32_t num_experts,
                     int32_t num_local_experts, int32_t block_m, const int32_t* expert_map,
                     int32_t* sorted_token_ids, int64_t sorted_capacity, int32_t* expert_ids,
                     int32_t* num_tokens_post_padded, void* workspace, size_t workspace_bytes,
                     int32_t* slot_to_row, cudaStream_t stream) {
    if (num_slots < 0 || num_experts <= 0 || num_local_experts <= 0 || block_m <= 0)
        return set_error("moe_align: sizes must be positive");
    if (num_slots >= (int64_t)INT32_MAX) return set_error("moe_align: too many slots");
    if (num_local_experts > 32767) return set_error("moe_align: at most 32767 local experts");
    if (!expert_map && num_local_experts != num_experts)
        return set_error("moe_align: num_local_experts must equal num_experts without a map");
    if (sorted_capacity % block_m != 0)
        return set_error("moe_align: sorted capacity must be a multiple of block_m");
    const int64_t need = num_slots + (int64_t)num_local_experts * (block_m - 1);
    if (sorted_capacity < need)
        return set_error("moe_align: sorted capacity " + std::to_string(sorted_capacity) +
                         " < num_slots + E*(block_m-1) = " + std::to_string(need));
    if (!topk_ids || !sorted_token_ids || !expert_ids || !num_tokens_post_padded)
        return set_error("moe_align: null pointer");
    if (workspace_bytes < w4a8_moe_align_workspace_size(num_local_experts) || !workspace)
        return set_error("moe_align: workspace too small");
    int32_t* offsets = static_cast<int32_t*>(workspace);
    const size_t count_smem = (size_t)num_local_experts * sizeof(int32_t);
    if (count_smem > 48 * 1024) {
        cudaFuncSetAttribute(align_count_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             (int)count_smem);
    }
    align_count_kernel<<<1, kCountThreads, count_smem, stream>>>(
        topk_ids, num_slots, num_experts, num_local_experts, block_m, expert_map,
        sorted_token_ids, sorted_capacity, expert_ids, num_tokens_post_padded, offsets);
    int st = launch_status();
    if (st) return st;
    if (num_slots > 4 * kChunk && num_local_experts <= kChunkMaxExperts) {
        const size_t smem = (size_t)34 * num_local_experts * sizeof(int32_t);
        cudaError_t ce = cudaFuncSetAttribute(align_place_chunked_kernel,
                                              cudaFuncAttributeMaxDynamicSharedMemorySize,
                                              (int)smem);
        if (ce != cudaSuccess) return (int)ce;
        const unsigned grid = (unsigned)((num_slots + kChunk - 1) / kChunk);
        align_place_chunked_kernel<<<grid, kChunkThreads, smem, stream>>>(
            topk_ids, num_slots, num_experts, num_local_experts, expert_map, offsets,
            sorted_token_ids, slot_to_row);
        return launch_status();
    }
    const dim3 grid((num_local_experts + kPlaceWarps - 1) / kPlaceWarps);
    if (num_slots <= kMaxSmemSlots) {
        const size_t smem = align_up((size_t)num_slots * sizeof(int16_t), 16);
        cudaFuncSetAttribute(align_place_kernel<true>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             (int)(kMaxSmemSlots * sizeof(int16_t)));
        align_place_kernel<true><<<grid, kPlaceWarps * 32, smem, stream>>>(
            topk_ids, num_slots, num_experts, num_local_experts, expert_map, offsets,
            sorted_token_ids, slot_to_row);
    } else {
        align_place_kernel<false><<<grid, kPlaceWarps * 32, 0, stream>>>(
            topk_ids, num_slots, num_experts, num_local_experts, expert_map, offsets,
            sorted_token_ids, slot_to_row);
    }
    return launch_status();
}

}  // namespace w4a8

extern "C" int w4a8_moe_align_block_size(const int32_t* topk_ids, int64_t num_slots,
                                         int32_t num_experts, int32_t num_local_experts,
                                         int32_t block_m, const int32_t* expert_map,
                                         int32_t* sorted_token_ids, int64_t sorted_capacity,
                                         int32_t* expert_ids, int32_t* num_tokens_post_padded,
                                         void* workspace, size_t workspace_bytes,
                                         w4a8_stream_t stream) {
    return w4a8::launch_moe_align(topk_ids, num_slots, num_experts, num_local_experts, block_m,
                                  expert_map, sorted_token_ids, sorted_capacity, expert_ids,
                                  num_tokens_post_padded, workspace, workspace_bytes, nullptr,
                                  reinterpret_cast<cudaStream_t>(stream));
}

// ---------------------------------------------------------------------------------------------
// Allocation-free variant of moe_align_block_size.
//
// Some callers cannot allocate device memory at the point where they route tokens: code that
// runs inside another framework's memory pool without a handle to it, plugins whose host
// language binding exposes no allocator, or deployments that forbid cudaMalloc after start-up
// because it synchronises the device. For them the per-expert offsets that the ordinary entry
// point keeps in caller workspace live in this fixed device array instead. It holds up to
// kNoAllocMaxExperts + 1 offsets (16 KB); every GPU that loads the library keeps it until the
// process exits.
// ---------------------------------------------------------------------------------------------
#include <mutex>

namespace {

constexpr int32_t kNoAllocMaxExperts = 4095;
static __device__ __align__(256) int32_t g_align_noalloc_scratch[kNoAllocMaxExperts + 1];

// Device address of the array, looked up once per device with that device current. The name
// g_align_noalloc_scratch is only a host-side stand-in in host code; kernels must get this
// address instead.
int noalloc_scratch(void** out) {
    constexpr int kMaxDevices = 64;
    static std::mutex mu;
    static void* addr[kMaxDevices] = {};
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess)
        return w4a8::set_error(std::string("moe_align_noalloc: cudaGetDevice failed: ") +
                               cudaGetErrorString(e));
    if (dev < 0 || dev >= kMaxDevices) return w4a8::set_error("moe_align_noalloc: device index out of range");
    std::lock_guard<std::mutex> lock(mu);
    if (!addr[dev]) {
        void* p = nullptr;
        e = cudaGetSymbolAddress(&p, g_align_noalloc_scratch);
        if (e != cudaSuccess)
            return w4a8::set_error(
                std::string("moe_align_noalloc: cudaGetSymbolAddress failed: ") +
                cudaGetErrorString(e));
        addr[dev] = p;
    }
    *out = addr[dev];
    return W4A8_OK;
}

}  // namespace

extern "C" int w4a8_moe_align_block_size_noalloc(const int32_t* topk_ids, int64_t num_slots,
                                                 int32_t num_experts, int32_t num_local_experts,
                                                 int32_t block_m, const int32_t* expert_map,
                                                 int32_t* sorted_token_ids,
                                                 int64_t sorted_capacity, int32_t* expert_ids,
                                                 int32_t* num_tokens_post_padded,
                                                 w4a8_stream_t stream) {
    if (num_local_experts > kNoAllocMaxExperts)
        return w4a8::set_error("moe_align_noalloc: at most " +
                               std::to_string(kNoAllocMaxExperts) +
                               " local experts (fixed device scratch); got " +
                               std::to_string(num_local_experts));
    void* scratch = nullptr;
    if (int rc = noalloc_scratch(&scratch)) return rc;
    // The count kernel writes every offset it uses before the place kernel reads it, so the
    // array needs no clearing between calls.
    return w4a8::launch_moe_align(topk_ids, num_slots, num_experts, num_local_experts, block_m,
                                  expert_map, sorted_token_ids, sorted_capacity, expert_ids,
                                  num_tokens_post_padded, scratch,
                                  sizeof(int32_t) * (kNoAllocMaxExperts + 1), nullptr,
                                  reinterpret_cast<cudaStream_t>(stream));
}
