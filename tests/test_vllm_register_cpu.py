"""The vLLM hook: B200W4A8LinearKernel's checks and load-time repack, and register() (the
counterpart of the reference's register.py) — on CPU, against vLLM 0.22's kernel registry."""
import numpy as np
import pytest
import torch

vllm = pytest.importorskip("vllm")
from vllm.model_executor.kernels.linear import _POSSIBLE_KERNELS  # noqa: E402
from vllm.model_executor.kernels.linear.mixed_precision.MPLinearKernel import (  # noqa: E402
    MPLinearLayerConfig,
)
from vllm.platforms import PlatformEnum  # noqa: E402
from vllm.scalar_type import scalar_types  # noqa: E402

import w4a8_oracle as O  # noqa: E402
from w4a8_fp8_wmma import register as R  # noqa: E402
from w4a8_fp8_wmma.vllm_adapter import (B200W4A8LinearKernel, check_config,  # noqa: E402
                                        repack_gptq)


def cfg(K=2048, N=4096, wt=scalar_types.uint4b8, act=torch.float16, g=128, zp=False,
        gidx=False):
    return MPLinearLayerConfig((K, N), (K, N), wt, act, g, zp, gidx)


def test_check_config():
    assert check_config(cfg())[0]
    assert check_config(cfg(act=torch.bfloat16))[0]
    assert check_config(cfg(wt=scalar_types.uint4, zp=True))[0]
    assert not check_config(cfg(wt=scalar_types.uint4, zp=False))[0]
    assert not check_config(cfg(wt=scalar_types.uint8b128))[0]
    assert not check_config(cfg(gidx=True))[0]
    assert not check_config(cfg(g=-1))[0]
    assert not check_config(cfg(g=256))[0]
    assert not check_config(cfg(K=2056, g=16))[0]
    assert not check_config(cfg(N=4100))[0]
    # this container has no GPU: the platform check refuses
    assert not B200W4A8LinearKernel.can_implement(cfg())[0]


def test_repack_gptq_matches_op_layout():
    rng = np.random.default_rng(3)
    K, N = 256, 64
    codes = rng.integers(0, 16, (N, K), dtype=np.uint8)
    gptq = O.pack_int4(codes.T.reshape(K // 8, 8, N).transpose(0, 2, 1))[..., 0]  # (K/8, N)
    got = repack_gptq(torch.from_numpy(gptq), K, N).numpy()
    assert np.array_equal(got, O.pack_int4(codes))


def test_process_weights_gptq_layout():
    K, N, g = 256, 64, 128
    rng = np.random.default_rng(4)
    codes = rng.integers(0, 16, (N, K), dtype=np.uint8)
    s = rng.uniform(1e-3, 2e-2, (N, K // g)).astype(np.float16)
    layer = torch.nn.Module()
    gptq = O.pack_int4(codes.T.reshape(K // 8, 8, N).transpose(0, 2, 1))[..., 0]
    layer.qweight = torch.nn.Parameter(torch.from_numpy(gptq), requires_grad=False)
    layer.scales = torch.nn.Parameter(torch.from_numpy(np.ascontiguousarray(s.T)).to(torch.bfloat16),
                                      requires_grad=False)
    k = B200W4A8LinearKernel(cfg(K=K, N=N), "qweight", "scales")
    k.process_weights_after_loading(layer)
    assert np.array_equal(layer.qweight.numpy(), O.pack_int4(codes))
    assert layer._w4a8_b200_scales.dtype == torch.float16
    assert np.array_equal(layer._w4a8_b200_scales.numpy(),
                          torch.from_numpy(s).to(torch.bfloat16).half().numpy())


def test_register_prepends_once_and_honours_the_switch(monkeypatch):
    lst = _POSSIBLE_KERNELS.setdefault(PlatformEnum.CUDA, [])
    before = list(lst)
    monkeypatch.setattr(R, "_REGISTERED", False)
    try:
        monkeypatch.setenv("VLLM_ROCM_USE_W4A8_FP8_WMMA", "0")
        assert R.register(verbose=False) is False
        assert B200W4A8LinearKernel not in lst
        monkeypatch.delenv("VLLM_ROCM_USE_W4A8_FP8_WMMA")
        assert R.register(verbose=False) is True
        assert lst[0] is B200W4A8LinearKernel
        assert R.register(verbose=False) is True
        assert lst.count(B200W4A8LinearKernel) == 1
    finally:
        lst[:] = before
