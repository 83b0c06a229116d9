"""Grouped-MoE composition and checkpoint-layout converters (vLLM-free).

``run_grouped_moe`` mirrors the reference's ``_run_grouped_moe``
(w4a8_fp8_wmma/w4a8_fp8_wmma/moe_experts.py:493-665): moe_align -> gate_up GEMM fused with
silu_and_mul -> down GEMM -> topk-weighted reduce, with the same decode/prefill split
(M <= 96 takes the GEMV kernels with block_m 8 and the atomic-scatter epilogue; larger M takes
the tile kernels with block_m 64, a materialised down output and the gather-reduce) and the same
4096-token chunking. Every step is one of this package's CUDA ops; the routing sort is this
library's deterministic moe_align_block_size instead of vLLM's.

Converters restate the reference's load-time layout changes:
AWQ (moe_experts.py:331-396), compressed-tensors GPTQ (:409-454), MoeWNA16 (:473-482).
"""
from __future__ import annotations

import os
import weakref

import torch

from . import (moe_align_block_size, mmq_fp8_moe_gather_reduce, mmq_fp8_moe_gemm,
               mmq_fp8_moe_gemm_scatter)

AWQ_REVERSE_PACK_ORDER = [0, 4, 1, 5, 2, 6, 3, 7]
GEMV_MAX_M = int(os.environ.get("VLLM_ROCM_W4A8_FP8_WMMA_MOE_GEMV_MAX_M", "96"))
GEMV_BLOCK_M = int(os.environ.get("VLLM_ROCM_W4A8_FP8_WMMA_MOE_GEMV_BLOCK_M", "8"))
# 128-row blocks feed the tcgen05 tile path N=128 MMAs (the reference uses 64 on gfx1201)
TILE_BLOCK_M = int(os.environ.get("VLLM_ROCM_W4A8_FP8_WMMA_MOE_BLOCK_M", "128"))
APPLY_CHUNK = int(os.environ.get("VLLM_ROCM_W4A8_FP8_WMMA_MOE_APPLY_CHUNK", "4096"))

_MOE_IDS = {"scalar": 0, "wmma": 6, "gemv": 7}


def _gemm1_silu(x, w, s, z, sorted_ids, expert_ids, ntp, top_k, block_m, kernel):
    if z is None:
        z = torch.empty(0, dtype=torch.int32, device=x.device)
    return torch.ops.w4a8_b200.moe_gemm1_silu(x, w, s, z, sorted_ids, expert_ids, ntp, top_k,
                                              block_m, _MOE_IDS[kernel], False)


def run_grouped_moe(x: torch.Tensor, w1: torch.Tensor, w2: torch.Tensor, w1_s: torch.Tensor,
                    w2_s: torch.Tensor, w1_zp: torch.Tensor | None, w2_zp: torch.Tensor | None,
                    topk_weights: torch.Tensor, topk_ids: torch.Tensor, kernel: str = "wmma",
                    global_num_experts: int | None = None,
                    expert_map: torch.Tensor | None = None,
                    apply_router_weight_on_input: bool = False,
                    out_dtype: torch.dtype | None = None) -> torch.Tensor:
    """Whole gated MoE in the op layout; returns (M, K) already topk-weighted and reduced.

    w1 (E, 2*inter, K/8) int32 [gate | up], w2 (E, K, inter/8) int32, scales (E, N, K/g) fp16,
    zeros (E, N/8, K/g) int32 or None (symmetric zp 8). ``expert_map`` maps global expert ids
    to local ones (-1 = remote); remote slots contribute nothing.
    """
    M, K = x.shape
    top_k = topk_ids.size(1)
    E_local = w1.size(0)
    E_global = int(global_num_experts) if global_num_experts is not None else E_local
    dev = x.device
    out_dtype = out_dtype or x.dtype
    if APPLY_CHUNK and M > APPLY_CHUNK and not apply_router_weight_on_input:
        out = torch.empty((M, K), dtype=out_dtype, device=dev)
        for lo in range(0, M, APPLY_CHUNK):
            hi = min(lo + APPLY_CHUNK, M)
            out[lo:hi] = run_grouped_moe(x[lo:hi], w1, w2, w1_s, w2_s, w1_zp, w2_zp,
                                         topk_weights[lo:hi], topk_ids[lo:hi], kernel,
                                         global_num_experts, expert_map, False, out_dtype)
        return out
    use_gemv = kernel != "scalar" and M <= GEMV_MAX_M
    if (use_gemv and expert_map is None and not apply_router_weight_on_input
            and _fused_decode_ok(x, w1, w2, w1_s, w2_s, w1_zp, w2_zp, E_global)):
        # whole layer on the prepacked weights: routing sort + token quant -> gate_up+SiLU ->
        # down + slot-order reduce (3 launches)
        y = decode_pack_for(w1, w2, w1_s, w2_s, w1_zp, w2_zp)(x, topk_weights, topk_ids)
        return y if out_dtype == torch.float16 else y.to(out_dtype)
    block_m = GEMV_BLOCK_M if use_gemv else TILE_BLOCK_M
    gver = "gemv" if use_gemv else kernel
    sorted_ids, expert_ids, ntp = moe_align_block_size(
        topk_ids, block_m, E_global, expert_map, E_local)
    x_in = x
    if apply_router_weight_on_input:
        assert top_k == 1, "router-weight-on-input requires top_k == 1"
        x_in = x_in * topk_weights.reshape(M, 1).to(x_in.dtype)
    x16 = x_in.to(torch.float16).contiguous()
    w1_s = w1_s if w1_s.dtype == torch.float16 else w1_s.to(torch.float16)
    w2_s = w2_s if w2_s.dtype == torch.float16 else w2_s.to(torch.float16)
    buf2 = _gemm1_silu(x16, w1, w1_s, w1_zp, sorted_ids, expert_ids, ntp, top_k, block_m, gver)
    if apply_router_weight_on_input:
        tw = torch.ones(M * top_k, dtype=torch.float32, device=dev)
    else:
        tw = topk_weights.reshape(-1).to(torch.float32).contiguous()
    if use_gemv:
        output = torch.zeros((M, K), dtype=torch.float32, device=dev)
        mmq_fp8_moe_gemm_scatter(buf2, w2, w2_s, sorted_ids, expert_ids, ntp, tw, output, top_k,
                                 block_m, kernel=gver, w_zeros=w2_zp)
        return output.to(out_dtype)
    ident = torch.arange(sorted_ids.numel(), dtype=torch.int32, device=dev)
    out2 = mmq_fp8_moe_gemm(buf2, w2, w2_s, ident, expert_ids, ntp, 1, block_m, kernel=kernel,
                            w_zeros=w2_zp)
    acc = mmq_fp8_moe_gather_reduce(out2, sorted_ids, tw, ntp, top_k)
    return acc.to(out_dtype)


class DecodePack:
    """One MoE layer's weights prepacked for the decode path (a load-time step, like the
    reference's layout converters): w13 and w2 as contiguous GEMV stage blocks with their
    scales and zero points (torch.ops.w4a8_b200.stream_pack). The op-layout tensors stay the
    source of truth; the pack is derived from them."""

    def __init__(self, w1, w2, w1_s, w2_s, w1_zp=None, w2_zp=None):
        dev = w1.device
        z1 = w1_zp if w1_zp is not None else torch.empty(0, dtype=torch.int32, device=dev)
        z2 = w2_zp if w2_zp is not None else torch.empty(0, dtype=torch.int32, device=dev)
        self.E = w1.size(0)
        self.inter = w1.size(1) // 2
        self.hidden = w1.size(2) * 8
        self.p13 = torch.ops.w4a8_b200.stream_pack(w1, w1_s.contiguous(), z1, True)
        self.p2 = torch.ops.w4a8_b200.stream_pack(w2, w2_s.contiguous(), z2, False)

    def __call__(self, x, topk_weights, topk_ids):
        return torch.ops.w4a8_b200.moe_decode_packed(
            x.contiguous(), self.p13, self.p2, self.E, self.inter,
            topk_weights.to(torch.float32).contiguous(), topk_ids.to(torch.int32).contiguous())


# Packs built on first use, keyed by the identity (and version) of the op-layout tensors; the
# entry dies with them. A caller that manages its own load step can build DecodePack directly.
_PACKS: dict[int, tuple] = {}


def decode_pack_for(w1, w2, w1_s, w2_s, w1_zp, w2_zp) -> DecodePack:
    key = id(w1)
    srcs = (w1, w2, w1_s, w2_s, w1_zp, w2_zp)
    ent = _PACKS.get(key)
    if ent is not None:
        refs, vers, pack = ent
        if all((r() is t) if t is not None else r is None for r, t in zip(refs, srcs)) and \
                vers == tuple(t._version if t is not None else 0 for t in srcs):
            return pack
    pack = DecodePack(*srcs)
    refs = tuple(weakref.ref(t) if t is not None else None for t in srcs)
    _PACKS[key] = (refs, tuple(t._version if t is not None else 0 for t in srcs), pack)
    weakref.finalize(w1, _PACKS.pop, key, None)
    return pack


def _fused_decode_ok(x, w1, w2, w1_s, w2_s, w1_zp, w2_zp, E_global) -> bool:
    """The fused decode op serves fp16 activations, g128 scales and hidden/inter % 512 == 0."""
    if x.dtype != torch.float16 or w1.size(0) != E_global:
        return False
    H, I = x.size(1), w1.size(1) // 2
    if H % 512 or I % 512 or w1_s.dtype != torch.float16 or w2_s.dtype != torch.float16:
        return False
    if w1_s.size(2) * 128 != H or w2_s.size(2) * 128 != I:
        return False
    return (w1_zp is None) == (w2_zp is None)


# --------------------------------------------------------------------------------------------
# checkpoint layout -> op layout (load time; integer repacking, any device)
# --------------------------------------------------------------------------------------------
def _repack_along_k(codes_nk: torch.Tensor) -> torch.Tensor:
    """(..., N, K) codes -> (..., N, K/8) int32, nibble j = input channel 8w + j."""
    c = codes_nk.to(torch.int32) & 0xF
    out = torch.zeros(c.shape[:-1] + (c.shape[-1] // 8,), dtype=torch.int32, device=c.device)
    for j in range(8):
        out |= c[..., j::8] << (4 * j)
    return out


def _pack_along_n(codes_ng: torch.Tensor) -> torch.Tensor:
    """(..., N, G) codes -> (..., N/8, G) int32, nibble j of word n8 = channel 8*n8 + j."""
    c = codes_ng.to(torch.int32) & 0xF
    out = torch.zeros(c.shape[:-2] + (c.shape[-2] // 8, c.shape[-1]), dtype=torch.int32,
                      device=c.device)
    for j in range(8):
        out |= c[..., j::8, :] << (4 * j)
    return out


def _unpack_awq(p: torch.Tensor) -> torch.Tensor:
    """(..., C/8) int32 in AWQ nibble order -> (..., C) natural-order codes."""
    shifts = torch.arange(0, 32, 4, dtype=torch.int32, device=p.device)
    nib = (p.unsqueeze(-1) >> shifts) & 0xF
    rev = torch.tensor(AWQ_REVERSE_PACK_ORDER, dtype=torch.long, device=p.device)
    return nib[..., rev].reshape(p.shape[:-1] + (p.shape[-1] * 8,))


def awq_moe_to_op_layout(qweight: torch.Tensor, scales: torch.Tensor, qzeros: torch.Tensor):
    """AWQ MoE (E, K, N/8) + scales (E, G, N) + qzeros (E, G, N/8) ->
    op layout w (E, N, K/8), scales (E, N, G) fp16, zeros (E, N/8, G)."""
    w = _repack_along_k(_unpack_awq(qweight).transpose(1, 2))
    s = scales.transpose(1, 2).contiguous().to(torch.float16)
    z = _pack_along_n(_unpack_awq(qzeros).transpose(1, 2))
    return w.contiguous(), s, z.contiguous()


def ct_moe_to_op_layout(qweight: torch.Tensor, scales: torch.Tensor):
    """compressed-tensors GPTQ (E, K/8, N) natural order + scales (E, G, N) ->
    op layout w (E, N, K/8), scales (E, N, G) fp16 (symmetric uint4b8)."""
    E, Kp, N = qweight.shape
    shifts = torch.arange(0, 32, 4, dtype=torch.int32, device=qweight.device)
    codes = ((qweight.unsqueeze(2) >> shifts.view(1, 1, 8, 1)) & 0xF).reshape(E, Kp * 8, N)
    w = _repack_along_k(codes.transpose(1, 2))
    return w.contiguous(), scales.transpose(1, 2).contiguous().to(torch.float16)


def wna16_moe_to_op_layout(qweight_u8: torch.Tensor, scales: torch.Tensor,
                           qzeros_u8: torch.Tensor | None):
    """MoeWNA16 uint8 storage -> op layout (zero-copy view for the weights).
    qweight (E, N, K/2) u8 K-packed; qzeros (E, N/2, K/g) u8 N-packed."""
    w = qweight_u8.contiguous().view(torch.int32)
    s = scales if scales.dtype == torch.float16 else scales.to(torch.float16)
    z = None
    if qzeros_u8 is not None:
        E, Nh, Kg = qzeros_u8.shape
        zi = qzeros_u8.contiguous().to(torch.int32).reshape(E, Nh // 4, 4, Kg)
        z = (zi[:, :, 0] | (zi[:, :, 1] << 8) | (zi[:, :, 2] << 16) | (zi[:, :, 3] << 24))
        z = z.contiguous()
    return w, s, z


def mxfp4_to_op_layout(weight_packed: torch.Tensor, weight_scale: torch.Tensor):
    """OCP mxfp4 (E2M1 codes + E8M0 block exponents) -> op layout, for weight_is_e2m1=True.

    weight_packed (..., N, K/2) uint8, two E2M1 codes per byte with the lower K index in the low
    nibble; weight_scale (..., N, K/32) uint8 E8M0 (value 2^(s-127)). Returns w (..., N, K/8)
    int32 holding the codes unchanged (code j of a word = input channel 8w + j) and fp16 group
    scales 2^(s-127) (group_size 32), the reference's mxfp4/convert.py:convert_mxfp4_moe
    contract. There are no zero points (E2M1 is symmetric). Scales outside fp16's range are
    rejected instead of saturating: the kernels carry fp16 group scales."""
    if weight_packed.dtype != torch.uint8 or weight_scale.dtype != torch.uint8:
        raise TypeError("mxfp4 weight_packed and weight_scale must be uint8")
    K = weight_packed.size(-1) * 2
    if K % 32 or weight_scale.size(-1) != K // 32:
        raise ValueError(f"mxfp4 needs K % 32 == 0 and K/32 scale blocks; got K={K}, "
                         f"{weight_scale.size(-1)} blocks")
    if bool((weight_scale == 0xFF).any()):
        raise ValueError("mxfp4 scale holds the E8M0 NaN code 0xFF")
    exp = weight_scale.to(torch.int32) - 127
    if bool((exp > 15).any()):
        raise ValueError("mxfp4 block scale above 2^15 does not fit the fp16 group scales")
    # two codes per byte, K-packed: four consecutive bytes are one little-endian int32 word
    w = weight_packed.contiguous().view(torch.int32)
    s = torch.ldexp(torch.ones_like(exp, dtype=torch.float32), exp).to(torch.float16)
    return w, s
