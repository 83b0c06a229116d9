"""The vLLM adapter's apply_weights on a B200 against the dense oracle (symmetric uint4b8 and
uint4 with zero points, fp16 and bf16 activations, a leading batch dimension and a bias)."""
import numpy as np
import pytest
import torch

pytest.importorskip("vllm")
from vllm.model_executor.kernels.linear.mixed_precision.MPLinearKernel import (  # noqa: E402
    MPLinearLayerConfig,
)
from vllm.scalar_type import scalar_types  # noqa: E402

import inputs as I  # noqa: E402
import w4a8_oracle as O  # noqa: E402
from helpers import MAX_ABS_REL, max_abs_rel  # noqa: E402

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("asym,act", [(False, torch.float16), (True, torch.bfloat16)])
@pytest.mark.parametrize("M", [3, 200])
def test_apply_weights_vs_oracle(asym, act, M):
    from w4a8_fp8_wmma.vllm_adapter import B200W4A8LinearKernel
    K, N, g = 2048, 1024, 128
    x, c, s, z = I.dense_case(500 + M, M, N, K, g, asym)
    if not asym:
        z = np.full_like(z, 8)
    layer = torch.nn.Module()
    layer.w_q = torch.nn.Parameter(torch.from_numpy(O.pack_int4(c)).cuda(), requires_grad=False)
    layer.w_s = torch.nn.Parameter(torch.from_numpy(s).cuda(), requires_grad=False)
    zp_name = None
    if asym:
        layer.w_zp = torch.nn.Parameter(torch.from_numpy(O.pack_zeros(z)).cuda(),
                                        requires_grad=False)
        zp_name = "w_zp"
    wt = scalar_types.uint4 if asym else scalar_types.uint4b8
    k = B200W4A8LinearKernel(MPLinearLayerConfig((K, N), (K, N), wt, act, g, asym, False),
                             "w_q", "w_s", zp_name)
    k.process_weights_after_loading(layer)
    xt = torch.from_numpy(x).cuda().to(act).reshape(1, M, K)
    bias = torch.linspace(-1, 1, N, device="cuda").to(act)
    out = k.apply_weights(layer, xt, bias)
    assert out.shape == (1, M, N) and out.dtype == act
    x_in = xt.reshape(M, K).half().cpu().numpy()
    ref = O.dense_gemm(x_in, O.pack_int4(c), s, O.pack_zeros(z) if asym else None)
    ref = ref.astype(np.float32) + bias.float().cpu().numpy()[None, :]
    assert max_abs_rel(out.reshape(M, N).float().cpu().numpy(), ref) <= MAX_ABS_REL
