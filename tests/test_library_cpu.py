"""CPU checks of the native boundary: the C-ABI library loads and exports every symbol the
header declares, argument validation rejects what the reference's bindings reject, and the
torch op surface (namespace, schemas, fakes, name maps) matches the reference's."""
import ctypes

import pytest
import torch

from helpers import header_symbols, load_lib

c_i64, c_i32, c_vp, c_sz = ctypes.c_int64, ctypes.c_int32, ctypes.c_void_p, ctypes.c_size_t


def test_library_exports_every_header_symbol():
    lib = load_lib()
    syms = header_symbols()
    assert len(syms) >= 13
    missing = [s for s in syms if not hasattr(lib, s)]
    assert not missing, missing


def test_version_and_workspace_queries():
    lib = load_lib()
    lib.w4a8_version.restype = ctypes.c_char_p
    assert b"sm_100a" in lib.w4a8_version()
    lib.w4a8_mmq_fp8_gemm_workspace_size.restype = c_sz
    lib.w4a8_mmq_fp8_gemm_workspace_size.argtypes = [c_i64, c_i64, c_i64]
    assert lib.w4a8_mmq_fp8_gemm_workspace_size(16, 2048, 2048) >= 16 * 2048 * 3 + 16 * 4
    lib.w4a8_moe_align_workspace_size.restype = c_sz
    lib.w4a8_moe_align_workspace_size.argtypes = [c_i32]
    assert lib.w4a8_moe_align_workspace_size(256) >= 257 * 4


def _dense(lib, M, N, K, g, kernel, e2m1=0, zeros=None):
    f = lib.w4a8_mmq_fp8_gemm
    f.restype = ctypes.c_int
    f.argtypes = [c_vp, c_vp, c_vp, c_vp, c_vp, c_i64, c_i64, c_i64, c_i64, c_i32, c_i32, c_vp,
                  c_sz, c_vp]
    return f(None, None, None, zeros, None, M, N, K, g, kernel, e2m1, None, 0, None)


def _err(lib):
    lib.w4a8_last_error.restype = ctypes.c_char_p
    return lib.w4a8_last_error().decode()


@pytest.mark.parametrize("g,msg", [(20, "group_size must be a multiple of 16"),
                                    (256, "group_size must be a multiple of 16"),
                                    (24, "K not divisible")])
def test_dense_rejects_bad_group(g, msg):
    lib = load_lib()
    assert _dense(lib, 4, 64, {20: 160, 256: 512, 24: 136}[g], g, 0) == -1
    assert msg in _err(lib)


@pytest.mark.parametrize("kernel,msg", [(3, "dense kernel id invalid"), (15, "dense kernel id invalid"),
                                        (7, "retired gfx1201 research kernel")])
def test_dense_rejects_kernel_ids(kernel, msg):
    lib = load_lib()
    assert _dense(lib, 4, 64, 128, 128, kernel) == -1
    assert msg in _err(lib)


def test_dense_e2m1_with_zeros_rejected():
    lib = load_lib()
    assert _dense(lib, 4, 64, 128, 128, 0, e2m1=1, zeros=1) == -1
    assert "symmetric" in _err(lib)


def test_dense_m0_is_noop():
    lib = load_lib()
    assert _dense(lib, 0, 64, 128, 128, 5) == 0


def _moe(lib, name, P, block_m, kernel, K=256, g=128):
    f = getattr(lib, name)
    f.restype = ctypes.c_int
    f.argtypes = [c_vp] * 8 + [c_i64] * 8 + [c_i32, c_i32, c_vp, c_sz, c_vp]
    return f(None, None, None, None, None, None, None, None, 4, 8, 64, K, P, g, 2, block_m,
             kernel, 0, None, 0, None)


@pytest.mark.parametrize("P,bm,kernel,msg", [
    (30, 16, 6, "not divisible by block_m"), (64, 16, 5, "moe kernel id must be"),
    (64, 8, 6, "wmma block_m must be mult of 16"), (128, 128, 7, "gemv needs block_m"),
])
def test_moe_gemm_validation(P, bm, kernel, msg):
    lib = load_lib()
    assert _moe(lib, "w4a8_mmq_fp8_moe_gemm", P, bm, kernel) == -1
    assert msg in _err(lib)


def test_silu_c_abi_rejects_odd_n():
    lib = load_lib()
    f = lib.w4a8_mmq_fp8_moe_gemm1_silu
    f.restype = ctypes.c_int
    f.argtypes = [c_vp] * 8 + [c_i64] * 8 + [c_i32, c_i32, c_vp, c_sz, c_vp]
    assert f(None, None, None, None, None, None, None, None, 4, 8, 72, 256, 64, 128, 2, 16, 6, 0,
             None, 0, None) == -1
    assert "inter must be a multiple of 8" in _err(lib)


def test_align_validation():
    lib = load_lib()
    f = lib.w4a8_moe_align_block_size
    f.restype = ctypes.c_int
    f.argtypes = [c_vp, c_i64, c_i32, c_i32, c_i32, c_vp, c_vp, c_i64, c_vp, c_vp, c_vp, c_sz, c_vp]
    # capacity too small: 256 slots + 256*(8-1) > 512
    assert f(1, 256, 256, 256, 8, None, 1, 512, 1, 1, 1, 4096, None) == -1
    assert "sorted capacity" in _err(lib)
    assert f(1, 256, 256, 256, 8, None, 1, 2052, 1, 1, 1, 4096, None) == -1
    assert "multiple of block_m" in _err(lib)


def test_ep_c_abi_validation():
    lib = load_lib()
    rb = lib.w4a8_ep_row_bytes
    rb.restype = c_sz
    rb.argtypes = [c_i64, c_i64]
    assert rb(2048, 8) == (2048 + 4 * 16 + 4 + 64 + 15) // 16 * 16
    d = lib.w4a8_ep_pack
    d.restype = ctypes.c_int
    d.argtypes = [c_vp, c_vp, c_vp, c_i64, c_i64, c_i64, c_i32, c_i32, c_i32, c_vp, c_vp, c_vp, c_vp]
    assert d(1, 1, 1, 4, 2, 200, 8, 2, -1, 1, None, 1, None) == -1   # H % 256 != 0
    assert "multiple of 256" in _err(lib)
    assert d(1, 1, 1, 4, 17, 256, 8, 2, -1, 1, None, 1, None) == -1  # top_k > 16
    assert "top_k" in _err(lib)
    assert d(None, None, None, 0, 2, 256, 8, 2, -1, None, None, None, None) == 0   # T = 0
    g = lib.w4a8_ep_gather
    g.restype = ctypes.c_int
    g.argtypes = [c_vp, c_vp, c_vp, c_vp, c_i64, c_i32, c_i64, c_vp]
    assert g(1, 1, None, 1, 4, 33, 64, None) == -1                 # world > 32
    assert g(None, None, None, None, 0, 2, 64, None) == 0          # T = 0: no-op
    m = lib.w4a8_ep_moe_rows
    m.restype = ctypes.c_int
    m.argtypes = [c_vp, c_i64, c_i64, c_i64, c_vp, c_vp, c_i64, c_i64, c_vp, c_vp, c_sz, c_vp]
    assert m(1, 4, 8, 33, 1, 1, 2000, 512, 1, 1, 1 << 20, None) == -1  # hidden % 512
    assert "512" in _err(lib)


def test_silu_and_mul_c_abi_validation():
    lib = load_lib()
    f = lib.w4a8_silu_and_mul
    f.restype = ctypes.c_int
    f.argtypes = [c_vp, c_vp, c_i64, c_i64, c_vp]
    assert f(None, None, -1, 4, None) == -1
    assert "negative" in _err(lib)
    assert f(None, None, 0, 4, None) == 0


# ---------------------------------------------------------------- torch surface ------------
REF_SCHEMAS = {
    "mmq_fp8_gemm": "mmq_fp8_gemm(Tensor x, Tensor w_packed, Tensor scales, Tensor w_zeros, int kernel, bool weight_is_e2m1=False) -> Tensor",
    "mmq_fp8_moe_gemm": "mmq_fp8_moe_gemm(Tensor x, Tensor w_packed, Tensor scales, Tensor w_zeros, Tensor sorted_token_ids, Tensor expert_ids, Tensor num_tokens_post_padded, int top_k, int block_m, int kernel, bool weight_is_e2m1=False) -> Tensor",
    "mmq_fp8_moe_gemm1_silu": "mmq_fp8_moe_gemm1_silu(Tensor x, Tensor w_packed, Tensor scales, Tensor w_zeros, Tensor sorted_token_ids, Tensor expert_ids, Tensor num_tokens_post_padded, int top_k, int block_m, int kernel, bool weight_is_e2m1=False) -> Tensor",
    "mmq_fp8_moe_gemm_scatter": "mmq_fp8_moe_gemm_scatter(Tensor x, Tensor w_packed, Tensor scales, Tensor w_zeros, Tensor sorted_token_ids, Tensor expert_ids, Tensor num_tokens_post_padded, Tensor topk_weights, Tensor(a!) output, int top_k, int block_m, int kernel, bool weight_is_e2m1=False) -> ()",
    "mmq_fp8_moe_gather_reduce": "mmq_fp8_moe_gather_reduce(Tensor out2, Tensor sorted_token_ids, Tensor topk_weights, Tensor num_tokens_post_padded, int top_k) -> Tensor",
    "mmq_regdirect_fp8": "mmq_regdirect_fp8(Tensor x, Tensor w_rep, Tensor scales, Tensor w_zeros, int N) -> Tensor",
}


@pytest.fixture(scope="module")
def pkg():
    import w4a8_fp8_wmma
    return w4a8_fp8_wmma


@pytest.mark.parametrize("name", sorted(REF_SCHEMAS))
def test_op_schemas_match_reference(pkg, name):
    op = getattr(torch.ops.w4a8_fp8_wmma, name).default
    assert str(op._schema) == "w4a8_fp8_wmma::" + REF_SCHEMAS[name]
    assert torch.Tag.pt2_compliant_tag in op.tags


def test_kernel_name_maps(pkg):
    assert pkg._resolve_moe_kernel("gemv") == 7 and pkg._resolve_dense_kernel("decode_gemv") == 11
    with pytest.raises(ValueError):
        pkg._resolve_moe_kernel("v6")
    with pytest.raises(TypeError):
        pkg._resolve_dense_kernel(5)


def test_fake_impls_shapes(pkg):
    from torch._subclasses.fake_tensor import FakeTensorMode
    with FakeTensorMode():
        x = torch.empty(5, 256, dtype=torch.float16, device="cuda")
        w = torch.empty(64, 32, dtype=torch.int32, device="cuda")
        s = torch.empty(64, 2, dtype=torch.float16, device="cuda")
        assert pkg.mmq_fp8_gemm(x, w, s, kernel="decode_gemv").shape == (5, 64)
        we = torch.empty(4, 64, 32, dtype=torch.int32, device="cuda")
        se = torch.empty(4, 64, 2, dtype=torch.float16, device="cuda")
        sti = torch.empty(48, dtype=torch.int32, device="cuda")
        eid = torch.empty(3, dtype=torch.int32, device="cuda")
        ntp = torch.empty(1, dtype=torch.int32, device="cuda")
        assert pkg.mmq_fp8_moe_gemm(x, we, se, sti, eid, ntp, 2, 16).shape == (48, 64)
        assert pkg.mmq_fp8_moe_gemm1_silu(x, we, se, sti, eid, ntp, 2, 16).shape == (48, 32)
        o2 = torch.empty(48, 64, dtype=torch.float16, device="cuda")
        tw = torch.empty(10, dtype=torch.float32, device="cuda")
        r = pkg.mmq_fp8_moe_gather_reduce(o2, sti, tw, ntp, 2)
        assert r.shape == (5, 64) and r.dtype == torch.float32


def test_cpu_tensors_rejected(pkg):
    x = torch.zeros(2, 128, dtype=torch.float16)
    w = torch.zeros(8, 16, dtype=torch.int32)
    s = torch.zeros(8, 1, dtype=torch.float16)
    with pytest.raises((RuntimeError, NotImplementedError)):
        pkg.mmq_fp8_gemm(x, w, s, kernel="prefill_wmma")
