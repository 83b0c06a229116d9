"""Register this library's W4A8 linear kernel into vLLM's kernel dispatcher.

The counterpart of the reference's register() (w4a8_fp8_wmma/w4a8_fp8_wmma/register.py:42-175):
call it once, before a quantized model is loaded, and 4-bit linear layers that
B200W4A8LinearKernel.can_implement() accepts run on this library; the others fall through to
vLLM's next kernel. The reference prepends its kernel to _POSSIBLE_KERNELS[ROCM]; on B200 the
list is _POSSIBLE_KERNELS[CUDA].

Usage:
    import w4a8_fp8_wmma
    from w4a8_fp8_wmma.register import register
    register()
    # ... then construct the vLLM engine / load the model

The reference's environment switch is honoured: VLLM_ROCM_USE_W4A8_FP8_WMMA=0 (or this
build's VLLM_USE_W4A8_B200=0) disables the registration. The MoE layers of a model take this
library through run_grouped_moe (the composition vLLM's fused-MoE hook calls); the reference's
MoE method patches, its mxfp4 dense hook and its Triton / attention autotune accelerators are
gfx1201-specific and have no counterpart here.
"""
import os

_REGISTERED = False
_DISABLE_VARS = ("VLLM_ROCM_USE_W4A8_FP8_WMMA", "VLLM_USE_W4A8_B200")


def register(verbose: bool = True) -> bool:
    """Prepend B200W4A8LinearKernel to vLLM's _POSSIBLE_KERNELS[CUDA].

    Returns True if registered (or already registered), False if disabled by environment."""
    global _REGISTERED
    if _REGISTERED:
        return True
    for var in _DISABLE_VARS:
        if os.environ.get(var, "1") != "1":
            if verbose:
                print(f"[w4a8_b200] disabled via {var}={os.environ[var]}")
            return False
    import w4a8_fp8_wmma  # noqa: F401  (loads the native libraries)
    from vllm.model_executor.kernels.linear import _POSSIBLE_KERNELS
    from vllm.platforms import PlatformEnum

    from .vllm_adapter import B200W4A8LinearKernel

    lst = _POSSIBLE_KERNELS.setdefault(PlatformEnum.CUDA, [])
    if B200W4A8LinearKernel not in lst:
        lst.insert(0, B200W4A8LinearKernel)
    _REGISTERED = True
    if verbose:
        print("[w4a8_b200] registered at _POSSIBLE_KERNELS[CUDA][0]:", [k.__name__ for k in lst])
    return True
