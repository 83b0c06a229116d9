"""GPU parity through the C ABI itself (ctypes on libw4a8_b200.so): torch only provides device
memory and the stream; results are compared with the CPU oracle."""
import ctypes

import numpy as np
import pytest
import torch

import inputs as I
import w4a8_oracle as O
from helpers import MAX_ABS_REL, load_lib, max_abs_rel

pytestmark = pytest.mark.gpu
c_i64, c_i32, c_vp, c_sz = ctypes.c_int64, ctypes.c_int32, ctypes.c_void_p, ctypes.c_size_t


@pytest.fixture(scope="module")
def lib():
    assert torch.cuda.is_available()
    L = load_lib()
    L.w4a8_last_error.restype = ctypes.c_char_p
    L.w4a8_act_quant_fp8.argtypes = [c_vp, c_vp, c_vp, c_i64, c_i64, c_vp]
    L.w4a8_moe_align_workspace_size.restype = c_sz
    L.w4a8_moe_align_workspace_size.argtypes = [c_i32]
    L.w4a8_moe_align_block_size.argtypes = [c_vp, c_i64, c_i32, c_i32, c_i32, c_vp, c_vp, c_i64,
                                            c_vp, c_vp, c_vp, c_sz, c_vp]
    L.w4a8_mmq_fp8_gemm_workspace_size.restype = c_sz
    L.w4a8_mmq_fp8_gemm_workspace_size.argtypes = [c_i64, c_i64, c_i64]
    L.w4a8_mmq_fp8_gemm.argtypes = [c_vp, c_vp, c_vp, c_vp, c_vp, c_i64, c_i64, c_i64, c_i64,
                                    c_i32, c_i32, c_vp, c_sz, c_vp]
    L.w4a8_moe_gemm_workspace_size.restype = c_sz
    L.w4a8_moe_gemm_workspace_size.argtypes = [c_i64, c_i64, c_i64, c_i64]
    L.w4a8_mmq_fp8_moe_gemm.argtypes = [c_vp] * 8 + [c_i64] * 8 + [c_i32, c_i32, c_vp, c_sz, c_vp]
    return L


def cu(a):
    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


def stream():
    return c_vp(torch.cuda.current_stream().cuda_stream)


def ok(lib, rc):
    assert rc == 0, (rc, lib.w4a8_last_error())


def test_capi_act_quant(lib):
    x, *_ = I.dense_case(1, 33, 8, 2048, 128)
    xd = cu(x)
    q = torch.empty((33, 2048), dtype=torch.uint8, device="cuda")
    s = torch.empty(33, dtype=torch.float32, device="cuda")
    ok(lib, lib.w4a8_act_quant_fp8(xd.data_ptr(), q.data_ptr(), s.data_ptr(), 33, 2048, stream()))
    torch.cuda.synchronize()
    qr, sr = O.act_quant(x)
    assert np.array_equal(q.cpu().numpy(), qr) and np.array_equal(s.cpu().numpy(), sr)


def test_capi_moe_align(lib):
    ids = I.random_topk(3, 32, 256, 8)
    slots, E, bm = ids.size, 256, 8
    cap = slots + E * (bm - 1)
    cap = (cap + bm - 1) // bm * bm
    idd = cu(ids)
    sorted_ = torch.empty(cap, dtype=torch.int32, device="cuda")
    eids = torch.empty(cap // bm, dtype=torch.int32, device="cuda")
    ntp = torch.empty(1, dtype=torch.int32, device="cuda")
    ws_n = lib.w4a8_moe_align_workspace_size(E)
    ws = torch.empty(ws_n, dtype=torch.uint8, device="cuda")
    ok(lib, lib.w4a8_moe_align_block_size(idd.data_ptr(), slots, E, E, bm, None,
                                          sorted_.data_ptr(), cap, eids.data_ptr(),
                                          ntp.data_ptr(), ws.data_ptr(), ws_n, stream()))
    torch.cuda.synchronize()
    rs, re, rn = O.moe_align(ids, bm, E)
    assert int(ntp.item()) == rn
    assert np.array_equal(sorted_.cpu().numpy()[:rn], rs)
    assert np.array_equal(eids.cpu().numpy()[:rn // bm], re)


@pytest.mark.parametrize("kernel", [0, 5, 10, 11])
def test_capi_dense_gemm(lib, kernel):
    M, N, K = 16, 2048, 2048
    x, c, s, z = I.dense_case(0, M, N, K, 128, True)
    xd, wd, sd, zd = cu(x), cu(O.pack_int4(c)), cu(s), cu(O.pack_zeros(z))
    out = torch.empty((M, N), dtype=torch.float16, device="cuda")
    ws_n = lib.w4a8_mmq_fp8_gemm_workspace_size(M, N, K)
    ws = torch.empty(ws_n, dtype=torch.uint8, device="cuda")
    ok(lib, lib.w4a8_mmq_fp8_gemm(xd.data_ptr(), wd.data_ptr(), sd.data_ptr(), zd.data_ptr(),
                                  out.data_ptr(), M, N, K, 128, kernel, 0, ws.data_ptr(), ws_n,
                                  stream()))
    torch.cuda.synchronize()
    ref = O.dense_gemm(x, O.pack_int4(c), s, O.pack_zeros(z)).astype(np.float32)
    assert max_abs_rel(out.cpu().numpy(), ref) <= MAX_ABS_REL


def test_capi_moe_gemm_gemv(lib):
    T, E, N, K, k, bm = 32, 64, 256, 1024, 8, 8
    rng = np.random.default_rng(9)
    x = rng.standard_normal((T, K), dtype=np.float32).astype(np.float16)
    codes, scales, zeros = I.expert_weights(rng, E, N, K, 128, True)
    ids = np.stack([rng.permutation(E)[:k] for _ in range(T)]).astype(np.int32)
    s, e, n = O.moe_align(ids, bm, E)
    P = len(s)
    bufs = [cu(x), cu(O.pack_int4(codes)), cu(scales), cu(O.pack_zeros(zeros)), cu(s), cu(e),
            cu(np.array([n], np.int32))]
    out = torch.empty((P, N), dtype=torch.float16, device="cuda")
    ws_n = lib.w4a8_moe_gemm_workspace_size(T, P, N, K)
    ws = torch.empty(ws_n, dtype=torch.uint8, device="cuda")
    ok(lib, lib.w4a8_mmq_fp8_moe_gemm(*[b.data_ptr() for b in bufs], out.data_ptr(), T, E, N, K,
                                      P, 128, k, bm, 7, 0, ws.data_ptr(), ws_n, stream()))
    torch.cuda.synchronize()
    ref = O.moe_gemm(x, O.pack_int4(codes), scales, O.pack_zeros(zeros), s, e, n, k, bm)
    valid = s < T * k
    assert max_abs_rel(out.cpu().numpy()[valid], ref[valid].astype(np.float32)) <= MAX_ABS_REL
