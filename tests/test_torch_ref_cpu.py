"""The torch fp32 layer reference (tests/torch_ref.py) against the numpy oracle on CPU, so the
GPU tests that use it at configs[2] sizes inherit the oracle's pinning."""
import numpy as np
import torch

import inputs as I
import torch_ref as R
import w4a8_oracle as O
from helpers import max_abs_rel


def test_torch_ref_layer_matches_oracle():
    c = I.moe_layer_case(5, 24, 12, 256, 128, 4, 128)
    p13, p2 = O.pack_int4(c["c13"]), O.pack_int4(c["c2"])
    z13, z2 = O.pack_zeros(c["z13"]), O.pack_zeros(c["z2"])
    ref = O.moe_layer(c["x"], p13, c["s13"], z13, p2, c["s2"], z2, c["topk_ids"],
                      c["topk_weights"])
    t = torch.from_numpy
    y = R.moe_layer(t(c["x"]), t(p13), t(c["s13"]), t(z13), t(p2), t(c["s2"]), t(z2),
                    t(c["topk_ids"]), t(c["topk_weights"])).numpy()
    assert max_abs_rel(y, ref) <= 2e-3


def test_torch_ref_act_quant_bit_exact():
    rng = np.random.default_rng(9)
    x = (rng.standard_normal((16, 512), dtype=np.float32) * 5).astype(np.float16)
    x[3] = np.abs(x[3])
    x[4, 7] = np.float16(60000)
    q, s = R.act_quant(torch.from_numpy(x))
    qr, sr = O.act_quant(x)
    assert np.array_equal(s.numpy().view(np.uint32), sr.view(np.uint32))
    assert np.array_equal(q.numpy().view(np.uint32), O.e4m3_decode(qr).view(np.uint32))


def test_torch_ref_unpack_matches_oracle():
    rng = np.random.default_rng(10)
    codes = rng.integers(0, 16, (64, 256)).astype(np.uint8)
    zeros = rng.integers(0, 16, (64, 2)).astype(np.uint8)
    s = rng.uniform(1e-3, 2e-2, (64, 2)).astype(np.float16)
    W = R.dequant(torch.from_numpy(O.pack_int4(codes)), torch.from_numpy(s),
                  torch.from_numpy(O.pack_zeros(zeros))).numpy()
    ref = O.dequant_signed(O.pack_int4(codes), O.pack_zeros(zeros), 128) * \
        np.repeat(s.astype(np.float32), 128, axis=1)
    assert np.array_equal(W, ref)
