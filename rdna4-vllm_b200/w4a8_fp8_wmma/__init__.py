"""w4a8_fp8_wmma — B200 (sm_100a) build of the W4A8 FP8 GEMM / MoE op library.

Drop-in for the reference package of the same name (w4a8_fp8_wmma/w4a8_fp8_wmma/__init__.py):
same Python wrappers, kernel-name maps, torch op namespace and schemas, and fake (meta) impls.
The ops run hand-written CUDA kernels from ``libw4a8_b200.so`` through the ``_C.so`` torch shim;
there is no CPU or Triton fallback. Importing the package without the built libraries raises.
"""
from __future__ import annotations

import os

import torch  # must come before loading _C so libtorch is already resident

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_HERE, "libw4a8_b200.so")
SHIM_PATH = os.path.join(_HERE, "_C.so")

if not (os.path.exists(LIB_PATH) and os.path.exists(SHIM_PATH)):
    raise ImportError(
        "w4a8_fp8_wmma: native libraries are not built "
        f"({LIB_PATH}, {SHIM_PATH}); run `python rdna4-vllm_b200/build.py`")
torch.ops.load_library(SHIM_PATH)

# Descriptive kernel names -> the opaque ids carried over the op ABI
# (reference: w4a8_fp8_wmma/w4a8_fp8_wmma/__init__.py:10-22, kernel_names.h:18-46).
_MOE_KERNELS = {"scalar": 0, "wmma": 6, "gemv": 7}
_DENSE_KERNELS = {
    "reference_scalar": 0, "rocwmma_v1": 1, "rocwmma_tiled": 2, "rocwmma_pipe": 4,
    "prefill_wmma": 5, "prefill_wmma_b128": 6, "wmma_tiled_tuned": 7, "wmma_dbuf": 8,
    "wmma_dbuf2": 9, "prefill_wmma_ashuffle": 10, "decode_gemv": 11,
    "splitk_smallm": 12, "regdirect_shuffle": 13, "nsplit_smallm": 14,
}
# Names served by this build; the rest are gfx1201 research kernels and raise in the op.
SERVED_DENSE_KERNELS = ("reference_scalar", "prefill_wmma", "prefill_wmma_ashuffle",
                        "decode_gemv")


def _resolve_dense_kernel(kernel) -> int:
    """Map a dense kernel name to its op id; unknown names and bare ints are rejected."""
    if isinstance(kernel, str):
        try:
            return _DENSE_KERNELS[kernel]
        except KeyError:
            raise ValueError(
                f"unknown dense kernel {kernel!r}; known: {sorted(_DENSE_KERNELS)}") from None
    raise TypeError(
        f"dense kernel must be a name in {sorted(_DENSE_KERNELS)} (the integer "
        f"'version' was removed); got {kernel!r}")


def _resolve_moe_kernel(kernel) -> int:
    """Map a MoE kernel name to its op id; unknown names and bare ints are rejected."""
    if isinstance(kernel, str):
        try:
            return _MOE_KERNELS[kernel]
        except KeyError:
            raise ValueError(
                f"unknown moe kernel {kernel!r}; known: {sorted(_MOE_KERNELS)}") from None
    raise TypeError(
        f"moe kernel must be a name in {sorted(_MOE_KERNELS)} (the integer 'version' was "
        f"removed); got {kernel!r}")


def _empty_zeros(dev) -> torch.Tensor:
    return torch.empty(0, dtype=torch.int32, device=dev)


def mmq_fp8_gemm(x: torch.Tensor, w_packed: torch.Tensor, scales: torch.Tensor,
                 kernel: str = "reference_scalar", w_zeros: torch.Tensor | None = None,
                 weight_is_e2m1: bool = False) -> torch.Tensor:
    """Dense W4A8 GEMM: (M, K) fp16 x (N, K/8) int32 codes -> (M, N) fp16.

    scales (N, K/g) fp16; w_zeros (N/8, K/g) int32 packed zero points or None (zp = 8).
    Every served kernel name computes the same function; "decode_gemv" forces the
    small-M register GEMV, "prefill_wmma*" the tile path, "reference_scalar" the scalar kernel.
    """
    if w_zeros is None:
        w_zeros = _empty_zeros(x.device)
    return torch.ops.w4a8_fp8_wmma.mmq_fp8_gemm(
        x, w_packed, scales, w_zeros, _resolve_dense_kernel(kernel), weight_is_e2m1)


def mmq_fp8_moe_gemm(x, w_packed, scales, sorted_token_ids, expert_ids,
                     num_tokens_post_padded, top_k: int, block_m: int, kernel: str = "wmma",
                     w_zeros=None, weight_is_e2m1: bool = False) -> torch.Tensor:
    """Grouped MoE GEMM: out[r] = x[sorted_token_ids[r] // top_k] @ W[expert(r)]^T.

    x (T, K) fp16; w_packed (E, N, K/8) int32; scales (E, N, K/g) fp16; routing tensors in the
    moe_align_block_size layout. Returns (P, N) fp16; padding rows are zero.
    """
    if w_zeros is None:
        w_zeros = _empty_zeros(x.device)
    return torch.ops.w4a8_fp8_wmma.mmq_fp8_moe_gemm(
        x, w_packed, scales, w_zeros, sorted_token_ids, expert_ids, num_tokens_post_padded,
        top_k, block_m, _resolve_moe_kernel(kernel), weight_is_e2m1)


def mmq_fp8_moe_gemm1_silu(x, w_packed, scales, sorted_token_ids, expert_ids,
                           num_tokens_post_padded, top_k: int, block_m: int,
                           kernel: str = "wmma", w_zeros=None,
                           weight_is_e2m1: bool = False) -> torch.Tensor:
    """Fused gate_up GEMM + silu_and_mul: w_packed (E, 2*inter, K/8) = [gate | up].

    Returns (P, inter) fp16, bit-identical to mmq_fp8_moe_gemm followed by vLLM silu_and_mul
    (fp16 gate/up stores, silu in fp32 rounded to fp16, half*half product).
    """
    if w_zeros is None:
        w_zeros = _empty_zeros(x.device)
    return torch.ops.w4a8_fp8_wmma.mmq_fp8_moe_gemm1_silu(
        x, w_packed, scales, w_zeros, sorted_token_ids, expert_ids, num_tokens_post_padded,
        top_k, block_m, _resolve_moe_kernel(kernel), weight_is_e2m1)


def mmq_fp8_moe_gemm_scatter(x, w_packed, scales, sorted_token_ids, expert_ids,
                             num_tokens_post_padded, topk_weights, output, top_k: int,
                             block_m: int, kernel: str = "wmma", w_zeros=None,
                             weight_is_e2m1: bool = False) -> None:
    """Down GEMM + topk-weighted atomic scatter into the pre-zeroed (M, N) fp32 ``output``.

    x (P, K) fp16 is the post-activation buffer, gathered by row identity; row r adds
    topk_weights[s] * (x[r] @ W[e]^T) into output[s // top_k] with s = sorted_token_ids[r].
    """
    if w_zeros is None:
        w_zeros = _empty_zeros(x.device)
    torch.ops.w4a8_fp8_wmma.mmq_fp8_moe_gemm_scatter(
        x, w_packed, scales, w_zeros, sorted_token_ids, expert_ids, num_tokens_post_padded,
        topk_weights, output, top_k, block_m, _resolve_moe_kernel(kernel), weight_is_e2m1)


def mmq_fp8_moe_gather_reduce(out2, sorted_token_ids, topk_weights, num_tokens_post_padded,
                              top_k):
    """Topk-weighted gather-reduce: (P, N) fp16 rows -> (M, N) fp32, M = numel(w) // top_k."""
    return torch.ops.w4a8_fp8_wmma.mmq_fp8_moe_gather_reduce(
        out2, sorted_token_ids, topk_weights, num_tokens_post_padded, top_k)


# ---- B200-build extras: the two kernels the reference takes from vLLM / runs implicitly ----

def act_quant_fp8(x: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor]:
    """Per-token e4m3 quantisation: (M, K) fp16 -> (uint8 e4m3 bytes (M, K), fp32 scales (M,))."""
    q, s = torch.ops.w4a8_b200.act_quant_fp8(x)
    return q, s


def moe_align_block_size(topk_ids: torch.Tensor, block_m: int, num_experts: int,
                         expert_map: torch.Tensor | None = None,
                         num_local_experts: int | None = None):
    """Deterministic moe_align_block_size -> (sorted_token_ids, expert_ids, ntp).

    Order: experts ascending, slot ids ascending inside an expert, runs padded to block_m with
    the sentinel topk_ids.numel(). With ``expert_map`` (global -> local id, -1 = remote) only
    local slots are kept and expert_ids hold local ids. Capacity is
    round_up(numel + E_local * (block_m - 1), block_m); entries past ntp hold the sentinel / -1.
    """
    ids = topk_ids.to(torch.int32).contiguous()
    n_local = int(num_local_experts) if num_local_experts is not None else int(num_experts)
    s, e, n = torch.ops.w4a8_b200.moe_align_block_size(ids, int(block_m), int(num_experts),
                                                       expert_map, n_local)
    return s, e, n


def silu_and_mul(x: torch.Tensor) -> torch.Tensor:
    """(M, 2*inter) fp16 [gate | up] -> (M, inter): fp16(g / (1 + exp(-g))) * up, the unfused
    activation step between gate_up and down (the fused gate_up op applies the same epilogue)."""
    return torch.ops.w4a8_b200.silu_and_mul(x.contiguous())


def route_topk(logits: torch.Tensor, top_k: int, renormalize: bool = True):
    """The MoE router in one launch: (T, E) fp32/fp16/bf16 logits -> topk_ids (T, top_k) int32,
    topk_weights (T, top_k) fp32 (softmax, the top_k largest with ties to the lower expert,
    renormalised) and expert_counts (E,) int32, the slots routed to each expert. It produces the
    inputs vLLM's router hands to the reference's moe_align call (moe_experts.py:587-589)."""
    ids, w, counts = torch.ops.w4a8_b200.route_topk(logits.contiguous(), int(top_k),
                                                    bool(renormalize))
    return ids, w, counts


# ---- Fake / meta impls (output contracts of the CUDA impls, reference __init__.py:240-297) ----
_register_fake = getattr(getattr(torch, "library", None), "register_fake", None)
if _register_fake is not None:
    @_register_fake("w4a8_fp8_wmma::mmq_fp8_gemm")
    def _fake_mmq_fp8_gemm(x, w_packed, scales, w_zeros, kernel, weight_is_e2m1=False):
        return x.new_empty((x.shape[0], w_packed.shape[0]), dtype=torch.float16)

    @_register_fake("w4a8_fp8_wmma::mmq_regdirect_fp8")
    def _fake_mmq_regdirect_fp8(x, w_rep, scales, w_zeros, N):
        return x.new_empty((x.shape[0], N), dtype=torch.float16)

    @_register_fake("w4a8_fp8_wmma::mmq_regdirect_f16")
    def _fake_mmq_regdirect_f16(x, w_rep, scales, w_zeros, N):
        return x.new_empty((x.shape[0], N), dtype=torch.float16)

    @_register_fake("w4a8_fp8_wmma::mmq_regdirect_w4a16")
    def _fake_mmq_regdirect_w4a16(x, w_rep, scales, w_zeros, N):
        return x.new_empty((x.shape[0], N), dtype=torch.float16)

    @_register_fake("w4a8_fp8_wmma::mmq_fp8_moe_gemm")
    def _fake_mmq_fp8_moe_gemm(x, w_packed, scales, w_zeros, sorted_token_ids, expert_ids,
                               num_tokens_post_padded, top_k, block_m, kernel,
                               weight_is_e2m1=False):
        return x.new_empty((sorted_token_ids.shape[0], w_packed.shape[1]), dtype=torch.float16)

    @_register_fake("w4a8_fp8_wmma::mmq_fp8_moe_gemm1_silu")
    def _fake_mmq_fp8_moe_gemm1_silu(x, w_packed, scales, w_zeros, sorted_token_ids,
                                     expert_ids, num_tokens_post_padded, top_k, block_m, kernel,
                                     weight_is_e2m1=False):
        return x.new_empty((sorted_token_ids.shape[0], w_packed.shape[1] // 2),
                           dtype=torch.float16)

    @_register_fake("w4a8_fp8_wmma::mmq_fp8_moe_gemm_scatter")
    def _fake_mmq_fp8_moe_gemm_scatter(x, w_packed, scales, w_zeros, sorted_token_ids,
                                       expert_ids, num_tokens_post_padded, topk_weights, output,
                                       top_k, block_m, kernel, weight_is_e2m1=False):
        return None

    @_register_fake("w4a8_b200::route_topk")
    def _fake_route_topk(logits, top_k, renormalize):
        T, E = logits.shape
        return [logits.new_empty((T, top_k), dtype=torch.int32),
                logits.new_empty((T, top_k), dtype=torch.float32),
                logits.new_empty((E,), dtype=torch.int32)]

    @_register_fake("w4a8_b200::silu_and_mul")
    def _fake_silu_and_mul(x):
        return x.new_empty((x.shape[0], x.shape[1] // 2), dtype=torch.float16)

    @_register_fake("w4a8_fp8_wmma::mmq_fp8_moe_gather_reduce")
    def _fake_mmq_fp8_moe_gather_reduce(out2, sorted_token_ids, topk_weights,
                                        num_tokens_post_padded, top_k):
        return out2.new_empty((topk_weights.shape[0] // top_k, out2.shape[1]),
                              dtype=torch.float32)
