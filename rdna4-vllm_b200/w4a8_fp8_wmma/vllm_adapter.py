"""vLLM mixed-precision linear kernel that routes 4-bit weight linears through this library's
dense W4A8 GEMM (torch.ops.w4a8_fp8_wmma.mmq_fp8_gemm) on B200 (sm_100).

The counterpart of the reference's RocmW4A8Fp8WmmaLinearKernel
(w4a8_fp8_wmma/w4a8_fp8_wmma/vllm_adapter.py:390-600), which register() puts at the front of
vLLM's kernel list for the platform. Weight contract (compressed-tensors wNa16 style):
  w_q   (N, K/8) int32, 8 codes per word, low nibble first — or GPTQ's (K/8, N), repacked at
        load time;
  w_s   (N, K/group) fp16/bf16 (GPTQ: (K/group, N), transposed at load time);
  w_zp  (N/8, K/group) int32 packed zero points, or absent for the symmetric uint4b8 type
        (zero point 8);
  g_idx (activation reordering) is not supported.
Activations are quantised per token to e4m3 inside the op; fp16 and bf16 inputs are served
(bf16 is computed through an fp16 copy of the activations, as the op takes fp16).

The reference additionally keeps a Triton fallback copy of the weights and an autotuned
per-shape M crossover for gfx1201; on B200 the op itself picks its decode GEMV (M <= 32) or
its tcgen05 tile path, so neither is kept.
"""
from __future__ import annotations

import torch

from vllm.model_executor.kernels.linear.mixed_precision.MPLinearKernel import (
    MPLinearKernel,
    MPLinearLayerConfig,
)
from vllm.platforms import current_platform
from vllm.scalar_type import scalar_types

SUPPORTED_QUANT_TYPES = [scalar_types.uint4b8, scalar_types.uint4]
MIN_CAPABILITY = 100  # sm_100 (B200)


def check_config(c: MPLinearLayerConfig) -> tuple[bool, str | None]:
    """The shape / type checks of can_implement, without the platform check."""
    if c.weight_type not in SUPPORTED_QUANT_TYPES:
        return False, f"unsupported weight_type {c.weight_type}"
    if c.act_type not in (torch.float16, torch.bfloat16):
        return False, f"act_type must be fp16/bf16, got {c.act_type}"
    if c.has_g_idx:
        return False, "act reordering (g_idx) not supported"
    if c.weight_type == scalar_types.uint4 and not c.zero_points:
        return False, "uint4 weights need zero points"
    gs = c.group_size
    K, N = c.partition_weight_shape
    if gs == -1:
        return False, "per-channel (group_size=-1) not supported"
    if gs % 16 != 0 or gs > 128:
        return False, f"group_size must be a multiple of 16 and <= 128, got {gs}"
    if K % gs != 0 or K % 8 != 0:
        return False, f"K={K} must be a multiple of 8 and of group_size={gs}"
    if N % 8 != 0:
        return False, f"N={N} must be a multiple of 8"
    return True, None


def repack_gptq(wq: torch.Tensor, K: int, N: int) -> torch.Tensor:
    """GPTQ qweight (K/8, N), codes packed along K -> (N, K/8), codes packed along K per row."""
    shifts = (torch.arange(8, device=wq.device, dtype=torch.int32) * 4).view(1, 8, 1)
    codes = ((wq.unsqueeze(1) >> shifts) & 0xF).reshape(K, N).t().contiguous()  # (N, K)
    out = torch.zeros((N, K // 8), dtype=torch.int32, device=wq.device)
    for j in range(8):
        out |= (codes[:, j::8] & 0xF) << (4 * j)
    return out


class B200W4A8LinearKernel(MPLinearKernel):
    """W4A8 (int4 weights, per-token e4m3 activations) linear on B200 tensor cores."""

    SUPPORTED_QUANT_TYPES = SUPPORTED_QUANT_TYPES

    @classmethod
    def get_min_capability(cls) -> int:
        return MIN_CAPABILITY

    @classmethod
    def can_implement(cls, c: MPLinearLayerConfig) -> tuple[bool, str | None]:
        if not current_platform.is_cuda():
            return False, "CUDA only"
        cap = current_platform.get_device_capability()
        if cap is None or cap.to_int() < MIN_CAPABILITY:
            return False, f"requires compute capability >= {MIN_CAPABILITY}"
        return check_config(c)

    def process_weights_after_loading(self, layer: torch.nn.Module) -> None:
        c = self.config
        K, N = c.partition_weight_shape  # (in, out)
        w_q, w_s, w_zp, _ = self._get_weight_params(layer)
        if tuple(w_q.shape) == (K // 8, N) and (K // 8, N) != (N, K // 8):
            self._transform_param(layer, self.w_q_name, lambda p: repack_gptq(p.data, K, N))
            self._transform_param(layer, self.w_s_name, lambda p: p.data.t().contiguous())
        elif tuple(w_q.shape) != (N, K // 8):
            raise RuntimeError(f"unexpected w_q shape {tuple(w_q.shape)}; expected (N, K/8) = "
                               f"{(N, K // 8)} or GPTQ (K/8, N) = {(K // 8, N)}")
        else:
            self._transform_param(layer, self.w_q_name, lambda p: p.data.contiguous())
        _, w_s, _, _ = self._get_weight_params(layer)
        layer._w4a8_b200_scales = w_s.data.to(torch.float16).contiguous()
        if w_zp is not None:
            self._transform_param(layer, self.w_zp_name, lambda p: p.data.contiguous())

    def apply_weights(self, layer: torch.nn.Module, x: torch.Tensor,
                      bias: torch.Tensor | None = None) -> torch.Tensor:
        from . import mmq_fp8_gemm
        c = self.config
        N = c.partition_weight_shape[1]
        w_q, _, w_zp, _ = self._get_weight_params(layer)
        x2 = x.reshape(-1, x.shape[-1])
        x16 = x2.to(torch.float16).contiguous()
        out = mmq_fp8_gemm(x16, w_q, layer._w4a8_b200_scales, kernel="prefill_wmma",
                           w_zeros=w_zp if (c.zero_points and w_zp is not None) else None)
        if out.dtype != x.dtype:
            out = out.to(x.dtype)
        if bias is not None:
            out = out + bias
        return out.reshape(x.shape[:-1] + (N,))
