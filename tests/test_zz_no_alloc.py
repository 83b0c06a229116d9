"""The allocation-free moe_align entry point (w4a8_moe_align_block_size_noalloc).

It exists for callers that cannot allocate device memory when they route tokens (code inside
another framework's memory pool, bindings with no allocator, deployments that forbid cudaMalloc
after start-up). It keeps its per-expert offsets in a fixed device array inside the library
instead of caller workspace. Here it is called through the C ABI twice in a row, on different
routings, and each result must equal the ordinary entry point's bit for bit (routing order is
integer work: the tolerance is exact equality). This file sorts last so a stop-at-first-failure
run has already run every other test.
"""
import ctypes

import numpy as np
import pytest
import torch

import inputs as I
from helpers import load_lib

pytestmark = pytest.mark.gpu
c_i64, c_i32, c_vp, c_sz = ctypes.c_int64, ctypes.c_int32, ctypes.c_void_p, ctypes.c_size_t


def _lib():
    assert torch.cuda.is_available(), "needs a CUDA device"
    L = load_lib()
    L.w4a8_last_error.restype = ctypes.c_char_p
    L.w4a8_moe_align_workspace_size.restype = c_sz
    L.w4a8_moe_align_workspace_size.argtypes = [c_i32]
    L.w4a8_moe_align_block_size.argtypes = [c_vp, c_i64, c_i32, c_i32, c_i32, c_vp, c_vp, c_i64,
                                            c_vp, c_vp, c_vp, c_sz, c_vp]
    L.w4a8_moe_align_block_size_noalloc.argtypes = [c_vp, c_i64, c_i32, c_i32, c_i32, c_vp, c_vp,
                                                    c_i64, c_vp, c_vp, c_vp]
    return L


def _outputs(slots, E, bm):
    cap = (slots + E * (bm - 1) + bm - 1) // bm * bm
    return (torch.full((cap,), -7, dtype=torch.int32, device="cuda"),
            torch.full((cap // bm,), -7, dtype=torch.int32, device="cuda"),
            torch.zeros(1, dtype=torch.int32, device="cuda"), cap)


def _stream():
    return c_vp(torch.cuda.current_stream().cuda_stream)


def test_noalloc_align_matches_workspace_align_twice():
    L = _lib()
    cases = [(I.random_topk(21, 32, 256, 8), 256, 8),
             (I.routing(np.random.default_rng(22), 4096, 256, 8, zipf_bias=True)[1], 256, 64)]
    for ids_np, E, bm in cases:  # two calls in a row; the second reuses the shared array
        ids = torch.from_numpy(np.ascontiguousarray(ids_np)).cuda()
        slots = ids.numel()
        s_ref, e_ref, n_ref, cap = _outputs(slots, E, bm)
        ws_n = L.w4a8_moe_align_workspace_size(E)
        ws = torch.empty(ws_n, dtype=torch.uint8, device="cuda")
        rc = L.w4a8_moe_align_block_size(ids.data_ptr(), slots, E, E, bm, None, s_ref.data_ptr(),
                                         cap, e_ref.data_ptr(), n_ref.data_ptr(), ws.data_ptr(),
                                         ws_n, _stream())
        assert rc == 0, L.w4a8_last_error()
        s_new, e_new, n_new, _ = _outputs(slots, E, bm)
        rc = L.w4a8_moe_align_block_size_noalloc(ids.data_ptr(), slots, E, E, bm, None,
                                                 s_new.data_ptr(), cap, e_new.data_ptr(),
                                                 n_new.data_ptr(), _stream())
        assert rc == 0, L.w4a8_last_error()
        torch.cuda.synchronize()
        assert int(n_new.item()) == int(n_ref.item())
        assert torch.equal(s_new, s_ref)
        assert torch.equal(e_new, e_ref)


def test_noalloc_align_rejects_too_many_experts():
    L = _lib()
    ids = torch.zeros(8, dtype=torch.int32, device="cuda")
    s, e, n, cap = _outputs(8, 5000, 8)
    rc = L.w4a8_moe_align_block_size_noalloc(ids.data_ptr(), 8, 5000, 5000, 8, None, s.data_ptr(),
                                             cap, e.data_ptr(), n.data_ptr(), _stream())
    assert rc == -1
    assert b"at most 4095 local experts" in L.w4a8_last_error()
