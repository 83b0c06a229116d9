// moe_layer.cu — the whole gated MoE layer at decode sizes behind one C-ABI call.
//
// Same result as the reference's decode composition (_run_grouped_moe, M <= 96 branch,
// w4a8_fp8_wmma/w4a8_fp8_wmma/moe_experts.py:563-648): moe_align(block 8) -> gate_up GEMV ->
// silu_and_mul -> down GEMV -> topk-weighted reduce, in seven launches and no host sync:
//   1. align count          2. align place (also writes the slot -> padded-row map)
//   3. operand quant of x   4. gate_up streaming GEMV (fp32 K-split partials)
//   5. finish: sum partials, fp16 gate/up, SiLU-and-mul, quantise the row as the down GEMM's
//      operand (the separate act-quant launch of the down GEMM disappears)
//   6. down streaming GEMV -> fp16 rows (P, H)
//   7. gather-reduce in slot order -> (T, H) fp16 output
// The down output is rounded to fp16 per (token, slot) before the weighted sum, the
// association of the reference oracle (w4a8_fp8_wmma/test_moe_experts.py:182-190).
#include <algorithm>
#include <string>

#include "common.cuh"
#include "gemm_common.h"
#include "internal.h"

namespace w4a8 {
namespace {

constexpr int kDecodeBlockM = 8;

struct DecodeLayout {
    int64_t cap;  // padded sorted capacity
    size_t off_align, off_sorted, off_eids, off_ntp, off_map, off_s1, off_xh1, off_xs1, off_part,
        off_s2, off_xh2, off_xs2, off_out2, total;
};

DecodeLayout decode_layout(int64_t T, int64_t top_k, int64_t E, int64_t H, int64_t I) {
    DecodeLayout L{};
    const int64_t slots = T * top_k;
    L.cap = (slots + E * (kDecodeBlockM - 1) + kDecodeBlockM - 1) / kDecodeBlockM * kDecodeBlockM;
    size_t o = 0;
    auto take = [&](size_t bytes) {
        const size_t at = o;
        o += align_up(bytes, 256);
        return at;
    };
    L.off_align = take(((size_t)E + 1) * 4);
    L.off_sorted = take((size_t)L.cap * 4);
    L.off_eids = take((size_t)(L.cap / kDecodeBlockM) * 4);
    L.off_ntp = take(4);
    L.off_map = take((size_t)slots * 4);
    L.off_s1 = take((size_t)T * 4);
    L.off_xh1 = take((size_t)T * H * 2);
    L.off_xs1 = take((size_t)T * (H / 128) * 8);
    L.off_part = take(stream_partials_bytes(L.cap, 2 * I, H));
    L.off_s2 = take((size_t)L.cap * 4);
    L.off_xh2 = take((size_t)L.cap * I * 2);
    L.off_xs2 = take((size_t)L.cap * (I / 128) * 8);
    L.off_out2 = take((size_t)L.cap * H * 2);
    L.total = o;
    return L;
}

}  // namespace
}  // namespace w4a8

using namespace w4a8;

extern "C" size_t w4a8_moe_decode_workspace_size(int64_t T, int64_t top_k, int64_t E, int64_t H,
                                                 int64_t I) {
    if (T < 0 || top_k <= 0 || E <= 0 || H <= 0 || I <= 0) return 0;
    size_t b = decode_layout(T, top_k, E, H, I).total;
    if (fused_decode_ok(T, top_k, E, H, I)) b = std::max(b, fused_decode_workspace(T, top_k, E, H, I));
    return b;
}

extern "C" int w4a8_moe_decode(const void* x, const int32_t* topk_ids, const float* topk_weights,
                               int64_t T, int64_t top_k, int64_t E, const int32_t* w13,
                               const void* s13, const int32_t* z13, const int32_t* w2,
                               const void* s2, const int32_t* z2, int64_t H, int64_t I,
                               int64_t group_size, void* out, void* workspace,
                               size_t workspace_bytes, w4a8_stream_t stream) {
    const std::string o = "moe_decode";
    if (T < 0 || top_k <= 0 || E <= 0 || H <= 0 || I <= 0) return set_error(o + ": bad sizes");
    if (group_size != 128) return set_error(o + ": the fused decode layer serves group_size 128");
    if (H % 512 != 0 || I % 512 != 0)
        return set_error(o + ": hidden and inter must be multiples of 512");
    if (T * top_k > INT32_MAX / 2 || E > 32767) return set_error(o + ": size overflow");
    if (T == 0) return W4A8_OK;
    if (!x || !topk_ids || !topk_weights || !w13 || !s13 || !w2 || !s2 || !out)
        return set_error(o + ": null pointer");
    if (!stream_path_ok(H, (int)(H / 128), 0, w13) || !stream_path_ok(I, (int)(I / 128), 0, w2))
        return set_error(o + ": weights must be 16-byte aligned");
    cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
    if (fused_decode_ok(T, top_k, E, H, I)) {
        if (!workspace || workspace_bytes < fused_decode_workspace(T, top_k, E, H, I))
            return set_error(o + ": workspace too small");
        return launch_fused_decode(x, topk_ids, topk_weights, T, top_k, E, w13, s13, z13, w2, s2,
                                   z2, H, I, out, workspace, st);
    }
    const DecodeLayout L = decode_layout(T, top_k, E, H, I);
    if (!workspace || workspace_bytes < L.total) return set_error(o + ": workspace too small");
    uint8_t* ws = static_cast<uint8_t*>(workspace);
    int32_t* sorted = reinterpret_cast<int32_t*>(ws + L.off_sorted);
    int32_t* eids = reinterpret_cast<int32_t*>(ws + L.off_eids);
    int32_t* ntp = reinterpret_cast<int32_t*>(ws + L.off_ntp);
    int32_t* map = reinterpret_cast<int32_t*>(ws + L.off_map);
    const int64_t slots = T * top_k;

    // 1-2. routing sort + inverse map (slots of out-of-range experts stay -1)
    cudaError_t ce = cudaMemsetAsync(map, 0xFF, (size_t)slots * 4, st);
    if (ce != cudaSuccess) return (int)ce;
    if (int rc = launch_moe_align(topk_ids, slots, (int32_t)E, (int32_t)E, kDecodeBlockM, nullptr,
                                  sorted, L.cap, eids, ntp, ws + L.off_align,
                                  align_up(((size_t)E + 1) * 4, 256), map, st))
        return rc;
    // 3. x -> gate_up operand
    OperandOut op1{nullptr, reinterpret_cast<float*>(ws + L.off_s1),
                   reinterpret_cast<__half*>(ws + L.off_xh1),
                   reinterpret_cast<float2*>(ws + L.off_xs1)};
    if (int rc = launch_operand_quant(x, op1, T, H, nullptr, st)) return rc;
    // 4-5. gate_up GEMV + SiLU + down operand
    OperandOut op2{nullptr, reinterpret_cast<float*>(ws + L.off_s2),
                   reinterpret_cast<__half*>(ws + L.off_xh2),
                   reinterpret_cast<float2*>(ws + L.off_xs2)};
    StreamArgs g1{};
    g1.xh = op1.xh;
    g1.xsum = op1.xsum;
    g1.act_scales = op1.scales;
    g1.w = w13;
    g1.scales = static_cast<const __half*>(s13);
    g1.zeros = z13;
    g1.sorted_ids = sorted;
    g1.expert_ids = eids;
    g1.ntp = ntp;
    g1.part = reinterpret_cast<float*>(ws + L.off_part);
    g1.K = H;
    g1.N = (int)(2 * I);
    g1.G = (int)(H / 128);
    g1.E = (int)E;
    g1.P = (int)L.cap;
    g1.num_valid = (int)slots;
    g1.top_k = (int)top_k;
    g1.out_top_k = (int)top_k;
    g1.block_m = kDecodeBlockM;
    g1.mode = kStreamSiluQuant;
    g1.next = op2;
    if (int rc = launch_w4_stream(g1, st)) return rc;
    // 6. down GEMV on the padded rows (identity gather) -> fp16 rows
    __half* out2 = reinterpret_cast<__half*>(ws + L.off_out2);
    StreamArgs g2{};
    g2.xh = op2.xh;
    g2.xsum = op2.xsum;
    g2.act_scales = op2.scales;
    g2.w = w2;
    g2.scales = static_cast<const __half*>(s2);
    g2.zeros = z2;
    g2.sorted_ids = sorted;
    g2.expert_ids = eids;
    g2.ntp = ntp;
    g2.out16 = out2;
    g2.part = reinterpret_cast<float*>(ws + L.off_part);  // K splits reuse gate_up's partials
    g2.K = I;
    g2.N = (int)H;
    g2.G = (int)(I / 128);
    g2.E = (int)E;
    g2.P = (int)L.cap;
    g2.num_valid = (int)slots;
    g2.top_k = 1;
    g2.out_top_k = (int)top_k;
    g2.block_m = kDecodeBlockM;
    g2.src_identity = 1;
    g2.mode = kStreamStore;
    if (stream_partials_bytes(L.cap, H, I) > stream_partials_bytes(L.cap, 2 * I, H) &&
        (I / 128) > 4)
        return set_error(o + ": internal: partials buffer too small for the down GEMM");
    if (int rc = launch_w4_stream(g2, st)) return rc;
    // 7. topk-weighted gather-reduce in slot order -> fp16
    return launch_gather_reduce(out2, map, topk_weights, out, true, T, H, (int)top_k, st);
}

extern "C" size_t w4a8_stream_pack_size(int64_t E, int64_t N, int64_t K) {
    if (E <= 0 || N <= 0 || K <= 0 || N % 128 != 0 || K % 512 != 0) return 0;
    return stream_pack_bytes(E, N, K);
}

extern "C" int w4a8_stream_pack(const int32_t* w_packed, const void* scales, const int32_t* w_zeros,
                                int64_t E, int64_t N, int64_t K, int32_t gate_up, void* packed,
                                size_t packed_bytes, w4a8_stream_t stream) {
    const std::string o = "stream_pack";
    if (E <= 0 || N <= 0 || K <= 0) return set_error(o + ": bad sizes");
    if (K % 512 != 0 || N % 128 != 0 || (gate_up && (N / 2) % 64 != 0))
        return set_error(o + ": needs K % 512 == 0 and N % 128 == 0");
    if (!w_packed || !scales || !packed) return set_error(o + ": null pointer");
    if ((reinterpret_cast<uintptr_t>(w_packed) & 15) || (reinterpret_cast<uintptr_t>(packed) & 15) ||
        (reinterpret_cast<uintptr_t>(scales) & 7) || (w_zeros && (reinterpret_cast<uintptr_t>(w_zeros) & 15)))
        return set_error(o + ": weights, zeros and the output must be 16-byte aligned");
    if (packed_bytes < stream_pack_bytes(E, N, K)) return set_error(o + ": output too small");
    return launch_stream_pack(w_packed, scales, w_zeros, E, N, K, gate_up ? 1 : 0, packed,
                              reinterpret_cast<cudaStream_t>(stream));
}

extern "C" int w4a8_moe_decode_packed(const void* x, const int32_t* topk_ids,
                                      const float* topk_weights, int64_t T, int64_t top_k,
                                      int64_t E, const void* p13, const void* p2, int64_t H,
                                      int64_t I, void* out, void* workspace,
                                      size_t workspace_bytes, w4a8_stream_t stream) {
    const std::string o = "moe_decode_packed";
    if (T < 0 || top_k <= 0 || E <= 0 || H <= 0 || I <= 0) return set_error(o + ": bad sizes");
    if (!fused_decode_ok(T, top_k, E, H, I))
        return set_error(o + ": needs hidden, inter % 512 == 0, top_k <= 16, T*top_k <= 65536, "
                             "E <= 4096");
    if (T == 0) return W4A8_OK;
    if (!x || !topk_ids || !topk_weights || !p13 || !p2 || !out) return set_error(o + ": null pointer");
    if ((reinterpret_cast<uintptr_t>(p13) & 15) || (reinterpret_cast<uintptr_t>(p2) & 15) ||
        (reinterpret_cast<uintptr_t>(x) & 15))
        return set_error(o + ": x and the packed weights must be 16-byte aligned");
    if (!workspace || workspace_bytes < fused_decode_workspace(T, top_k, E, H, I))
        return set_error(o + ": workspace too small");
    return launch_fused_decode(x, topk_ids, topk_weights, T, top_k, E, nullptr, nullptr, nullptr,
                               nullptr, nullptr, nullptr, H, I, out, workspace,
                               reinterpret_cast<cudaStream_t>(stream), p13, p2);
}
