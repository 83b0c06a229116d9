"""Checkpoint-format converters against fixtures made by the reference's own converters
(tests/golden/make_golden.py, section `formats`): compressed-tensors GPTQ
(moe_experts.py:437), MoeWNA16 (moe_experts.py:473) and mxfp4 (mxfp4/convert.py), plus the
oracle's E2M1 GEMM against the reference's mxfp4 dense oracle (mxfp4/test_mxfp4_kernel_gpu.py:64-71).
Integer repacking is bit-exact; the E2M1 GEMM uses the reference test's bar (max |diff| /
max(|ref|, 1) < 5e-3), since that oracle quantises with a reciprocal multiply."""
import os

import numpy as np
import pytest
import torch

import w4a8_oracle as O

F = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden", "formats.npz")


@pytest.fixture(scope="module")
def fx():
    return np.load(F)


def _conv():
    # the converters are pure torch; importing the package without its native libraries is not
    # possible, so load the module file on its own
    import importlib.util
    import sys
    import types
    root = os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))),
                        "rdna4-vllm_b200", "w4a8_fp8_wmma")
    pkg = types.ModuleType("_w4a8_conv_pkg")
    pkg.__path__ = [root]
    pkg.moe_align_block_size = pkg.mmq_fp8_moe_gather_reduce = None
    pkg.mmq_fp8_moe_gemm = pkg.mmq_fp8_moe_gemm_scatter = None
    sys.modules["_w4a8_conv_pkg"] = pkg
    spec = importlib.util.spec_from_file_location("_w4a8_conv_pkg.moe_experts",
                                                  os.path.join(root, "moe_experts.py"))
    m = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(m)
    return m


def test_ct_converter_matches_reference(fx):
    w, s = _conv().ct_moe_to_op_layout(torch.from_numpy(fx["ct_qweight"]),
                                       torch.from_numpy(fx["ct_scales"]))
    assert np.array_equal(w.numpy(), fx["ct_op_w"])
    assert np.array_equal(s.numpy().view(np.uint16), fx["ct_op_s"].view(np.uint16))


def test_wna16_converter_matches_reference(fx):
    w, s, z = _conv().wna16_moe_to_op_layout(torch.from_numpy(fx["wna16_qweight"]),
                                             torch.from_numpy(fx["wna16_scales"]),
                                             torch.from_numpy(fx["wna16_qzeros"]))
    assert np.array_equal(w.numpy(), fx["wna16_op_w"])
    assert np.array_equal(s.numpy().view(np.uint16), fx["wna16_op_s"].view(np.uint16))
    assert np.array_equal(z.numpy(), fx["wna16_op_z"])
    w2, _, z2 = _conv().wna16_moe_to_op_layout(torch.from_numpy(fx["wna16_qweight"]),
                                               torch.from_numpy(fx["wna16_scales"]), None)
    assert z2 is None and np.array_equal(w2.numpy(), fx["wna16_op_w"])


def test_mxfp4_converter_matches_reference(fx):
    w, s = _conv().mxfp4_to_op_layout(torch.from_numpy(fx["mx_packed"]),
                                      torch.from_numpy(fx["mx_scale"]))
    assert np.array_equal(w.numpy(), fx["mx_op_w"])
    assert np.array_equal(s.numpy().view(np.uint16), fx["mx_op_s"].view(np.uint16))


def test_mxfp4_converter_rejects_bad_scales(fx):
    c = _conv()
    bad = torch.from_numpy(fx["mx_scale"]).clone()
    bad[0, 0, 0] = 0xFF
    with pytest.raises(ValueError, match="NaN"):
        c.mxfp4_to_op_layout(torch.from_numpy(fx["mx_packed"]), bad)
    bad[0, 0, 0] = 127 + 16
    with pytest.raises(ValueError, match="fp16"):
        c.mxfp4_to_op_layout(torch.from_numpy(fx["mx_packed"]), bad)


def test_oracle_e2m1_table_is_the_reference_lut_and_exact_in_e4m3():
    # reference LUT (mxfp4/convert.py FP4_E2M1_LUT, tile_config.h:66-67), as bits
    assert np.array_equal(O.e2m1_value_bits(), O.E2M1_VALUES.view(np.uint32))
    assert np.array_equal(O.e4m3_decode(O.e4m3_encode(O.E2M1_VALUES)).view(np.uint32),
                          O.E2M1_VALUES.view(np.uint32))


def test_oracle_e2m1_gemm_vs_reference_mxfp4_oracle(fx):
    out = O.dense_gemm_e2m1(fx["mx_x"], fx["mx_op_w"][0], fx["mx_op_s"][0]).astype(np.float32)
    ref = fx["mx_dense_ref"]
    rel = np.abs(out - ref) / np.maximum(np.abs(ref), 1.0)
    assert rel.max() < 5e-3


def test_oracle_e2m1_integer_codes_equal_int4():
    """The reference's equivalence check (mxfp4/test_mxfp4_kernel_gpu.py:45-61): E2M1 codes of
    integer value v give the same GEMM as int4 code v + 8 with the symmetric zero point."""
    rng = np.random.default_rng(3)
    int_codes = np.array([0, 2, 4, 5, 6, 7, 10, 12, 13, 14, 15])  # values 0,1,2,3,4,6,-1,-2,...
    codes = int_codes[rng.integers(0, len(int_codes), (64, 256))].astype(np.uint8)
    vals = O.E2M1_VALUES[codes]
    c4 = (vals + 8).astype(np.uint8)
    x = (rng.standard_normal((8, 256), dtype=np.float32) * 0.5).astype(np.float16)
    s = rng.uniform(0.25, 0.75, (64, 8)).astype(np.float16)
    a = O.dense_gemm_e2m1(x, O.pack_int4(codes), s)
    b = O.dense_gemm(x, O.pack_int4(c4), s, None)
    assert np.array_equal(a.view(np.uint16), b.view(np.uint16))
