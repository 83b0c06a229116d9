"""Plain-PyTorch fp32 reference of the MoE layer, for parity at sizes the numpy oracle cannot
finish in seconds (configs[2]: 4096 tokens x 257 experts). TEST INFRASTRUCTURE ONLY.

It restates oracle/w4a8_oracle.py:moe_layer with torch tensors on any device:
  * activation quant — fp32 IEEE divides (tensor by tensor), then torch's float8_e4m3fn
    conversion (the reference oracle's own op, w4a8_fp8_wmma/test_correctness.py:74-76);
  * each GEMM — dequantised weights scale*(q - z) in fp32 times the e4m3 activations, then the
    activation scale, rounded to fp16 (the oracle sums per 128-group first; the two associations
    differ by fp32 rounding only);
  * SiLU — fp16(g / (1 + exp(-g))) * up in fp16 (test_moe_experts.py:274-280);
  * reduce — fp32, slot order (test_moe_experts.py:182-190).
tests/test_torch_ref_cpu.py pins it to the numpy oracle on CPU.
"""
from __future__ import annotations

import torch

_SHIFTS = None


def _shifts(dev):
    return torch.arange(0, 32, 4, dtype=torch.int32, device=dev)


def unpack_int4(p: torch.Tensor) -> torch.Tensor:
    """(..., K/8) int32 -> (..., K) int32 codes (nibble j of word w = channel 8w + j)."""
    c = (p.unsqueeze(-1) >> _shifts(p.device)) & 0xF
    return c.reshape(*p.shape[:-1], p.shape[-1] * 8)


def unpack_zeros(zp: torch.Tensor, N: int) -> torch.Tensor:
    """(N/8, G) int32 -> (N, G) int32 (nibble n % 8 of word n / 8)."""
    c = (zp.unsqueeze(-2) >> _shifts(zp.device).view(8, 1)) & 0xF  # (N/8, 8, G)
    return c.reshape(N, zp.shape[-1])


def dequant(w: torch.Tensor, s: torch.Tensor, z: torch.Tensor | None) -> torch.Tensor:
    """One expert: w (N, K/8), s (N, G) fp16, z (N/8, G) or None -> (N, K) fp32 s*(q - z)."""
    q = unpack_int4(w).float()
    N, K = q.shape
    G = s.shape[1]
    zz = torch.full((N, G), 8.0, device=w.device) if z is None or z.numel() == 0 else \
        unpack_zeros(z, N).float()
    return ((q.view(N, G, K // G) - zz[:, :, None]) * s.float()[:, :, None]).view(N, K)


def act_quant(x: torch.Tensor):
    xf = x.float()
    amax = xf.abs().amax(dim=1).clamp(min=1e-8 * 448.0)
    # tensor / tensor: torch's CUDA divide by a Python scalar multiplies by the reciprocal,
    # which is not the oracle's IEEE divide
    scale = amax / torch.full_like(amax, 448.0)
    q = (xf / scale[:, None]).to(torch.float8_e4m3fn).float()
    return q, scale


def gemm(xq, xs, W):
    return ((xq @ W.t()) * xs[:, None]).half()


def silu_and_mul(o1: torch.Tensor) -> torch.Tensor:
    inter = o1.shape[1] // 2
    g = o1[:, :inter].float()
    return (g / (1.0 + torch.exp(-g))).half() * o1[:, inter:]


@torch.no_grad()
def moe_layer(x, w13, s13, z13, w2, s2, z2, topk_ids, topk_weights) -> torch.Tensor:
    """(T, H) fp32 = sum_j w[t,j] * fp16(down(silu_and_mul(gate_up(x_t)))), op-layout weights."""
    if x.is_cuda:
        prev = torch.backends.cuda.matmul.allow_tf32
        torch.backends.cuda.matmul.allow_tf32 = False
    try:
        T, H = x.shape
        k = topk_ids.shape[1]
        xq, xs = act_quant(x)
        flat = topk_ids.reshape(-1).long()
        y2 = torch.zeros((T * k, H), dtype=torch.float32, device=x.device)
        for e in torch.unique(flat).tolist():
            slots = torch.nonzero(flat == e).squeeze(1)
            t = slots // k
            W1 = dequant(w13[e], s13[e], None if z13 is None else z13[e])
            act = silu_and_mul(gemm(xq[t], xs[t], W1))
            aq, as_ = act_quant(act)
            W2 = dequant(w2[e], s2[e], None if z2 is None else z2[e])
            y2[slots] = gemm(aq, as_, W2).float()
        w = topk_weights.float().reshape(T, k)
        y = torch.zeros((T, H), dtype=torch.float32, device=x.device)
        ar = torch.arange(T, device=x.device) * k
        for j in range(k):
            y += w[:, j:j + 1] * y2[ar + j]
        return y
    finally:
        if x.is_cuda:
            torch.backends.cuda.matmul.allow_tf32 = prev
