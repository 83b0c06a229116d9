"""The fused router (w4a8_route_topk / torch.ops.w4a8_b200.route_topk) against the oracle's
restatement of the softmax -> top-k -> renormalise router (oracle/w4a8_oracle.py:route_topk).

Bars: ids bit-exact (including exact ties, which go to the lower expert index); weights within
1e-6 relative (fp32 softmax, different summation order); expert counts equal to the histogram of
the ids; the C ABI rejects out-of-range sizes."""
import ctypes

import numpy as np
import pytest
import torch

import w4a8_oracle as O

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def w4():
    assert torch.cuda.is_available(), "GPU tests need a CUDA device"
    import w4a8_fp8_wmma
    return w4a8_fp8_wmma


def _check(w4, logits_np, k, renorm, dtype=torch.float32):
    lg = torch.from_numpy(logits_np).cuda().to(dtype)
    ids, w, counts = w4.route_topk(lg, k, renorm)
    ref_in = lg.float().cpu().numpy()  # the oracle sees the same (rounded) logits
    rid, rw = O.route_topk(ref_in, k, renormalize=renorm)
    assert np.array_equal(ids.cpu().numpy(), rid)
    np.testing.assert_allclose(w.cpu().numpy(), rw, rtol=1e-6, atol=1e-7)
    E = logits_np.shape[1]
    assert np.array_equal(counts.cpu().numpy(), np.bincount(rid.ravel(), minlength=E))


@pytest.mark.parametrize("T,E,k,seed", [(32, 256, 8, 0), (4096, 256, 8, 1), (7, 60, 4, 2),
                                        (33, 1000, 16, 3), (1, 8, 8, 4), (129, 257, 9, 5)])
def test_route_topk_vs_oracle(w4, T, E, k, seed):
    rng = np.random.default_rng(seed)
    _check(w4, rng.standard_normal((T, E), dtype=np.float32) * 2, k, True)


@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16])
def test_route_topk_half_logits(w4, dtype):
    rng = np.random.default_rng(11)
    _check(w4, rng.standard_normal((64, 256), dtype=np.float32), 8, True, dtype)


def test_route_topk_ties_and_no_renorm(w4):
    rng = np.random.default_rng(12)
    # few distinct values: many exact ties, which must go to the lower expert index
    lg = rng.integers(-3, 4, (48, 128)).astype(np.float32)
    _check(w4, lg, 8, True)
    _check(w4, lg, 8, False)


def test_route_topk_zipf_biased(w4):
    import inputs as I
    logits, ids, w = I.routing(np.random.default_rng(13), 512, 256, 8, zipf_bias=True)
    _check(w4, logits, 8, True)


def test_route_topk_c_abi_rejects_bad_sizes(w4):
    import os
    lib = ctypes.CDLL(os.path.join(os.path.dirname(w4.__file__), "libw4a8_b200.so"))
    f = lib.w4a8_route_topk
    f.restype = ctypes.c_int
    f.argtypes = [ctypes.c_void_p, ctypes.c_int32, ctypes.c_int64, ctypes.c_int32, ctypes.c_int32,
                  ctypes.c_int32, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p]
    x = torch.zeros(4, 2048, device="cuda")
    ids = torch.empty(4, 17, dtype=torch.int32, device="cuda")
    w = torch.empty(4, 17, device="cuda")
    for E, k, dt in [(2048, 8, 0), (64, 17, 0), (64, 0, 0), (8, 9, 0), (64, 8, 3)]:
        assert f(x.data_ptr(), dt, 4, E, k, 1, ids.data_ptr(), w.data_ptr(), None, None) != 0
