"""Pin the CPU oracle against fixtures produced by the reference's own oracle functions
(tests/golden/make_golden.py). Runs on CPU."""
import os

import numpy as np
import pytest
import torch

import inputs as I
import w4a8_oracle as O

G = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")


def _load(name):
    return np.load(os.path.join(G, name))


def test_e4m3_encoder_matches_torch_exhaustively():
    rng = np.random.default_rng(0)
    vals = O.e4m3_decode(np.arange(256, dtype=np.uint8))
    vals = np.sort(np.unique(vals[~np.isnan(vals)]))
    mids = ((vals[:-1].astype(np.float64) + vals[1:]) / 2).astype(np.float32)
    cand = np.concatenate([
        vals, mids, np.nextafter(mids, np.float32(1e9)), np.nextafter(mids, np.float32(-1e9)),
        rng.standard_normal(200_000).astype(np.float32) * 100,
        (rng.random(100_000) * 2 ** -8).astype(np.float32),
        np.array([448, 449, 463.9, 464, 465, 479.9, 480, 1e5, -464, -480, 0, -0.0, 2 ** -10],
                 np.float32)])
    ours = O.e4m3_encode(cand)
    ref = torch.from_numpy(cand).to(torch.float8_e4m3fn).view(torch.uint8).numpy()
    assert np.array_equal(ours, ref)


def test_e4m3_decode_roundtrip():
    codes = np.arange(256, dtype=np.uint8)
    v = O.e4m3_decode(codes)
    ok = ~np.isnan(v)
    assert np.array_equal(O.e4m3_encode(v[ok]), codes[ok] & np.where(v[ok] == 0, 0x80, 0xFF) | (codes[ok] & 0x80))


def test_int4_minus_zero_exact_in_e4m3():
    d = np.arange(-15, 16, dtype=np.float32)
    assert np.array_equal(O.e4m3_decode(O.e4m3_encode(d)), d)


@pytest.mark.parametrize("i", [0, 1, 2])
def test_act_quant_bytes_match_reference(i):
    f = _load("act_quant.npz")
    q, s = O.act_quant(f[f"x{i}"])
    assert np.array_equal(q, f[f"q{i}"])


def test_pack_unpack_roundtrip():
    rng = np.random.default_rng(3)
    c = rng.integers(0, 16, (24, 64)).astype(np.uint8)
    assert np.array_equal(O.unpack_int4(O.pack_int4(c)), c)
    z = rng.integers(0, 16, (24, 5)).astype(np.uint8)
    assert np.array_equal(O.unpack_zeros(O.pack_zeros(z), 24), z)


@pytest.mark.parametrize("name", ["cfg0", "m1_g32_sym", "tail_17x48", "tail_100x80", "g128_sym",
                                  "g64_asym"])
def test_dense_oracle_matches_reference(name):
    d = _load("dense.npz")
    seed, M, N, K, g, asym = (int(v) for v in d[name + "_meta"])
    x, c, s, z = I.dense_case(seed, M, N, K, g, bool(asym))
    out = O.dense_gemm(x, O.pack_int4(c), s, O.pack_zeros(z) if asym else None)
    ref = d[name]
    # Same arithmetic; only the fp32 summation order may differ: at most 1 fp16 ulp, or a
    # 1e-6 * max|ref| absolute slack for outputs that are near-cancellations of large sums.
    ulp = np.spacing(np.abs(ref).astype(np.float16)).astype(np.float32)
    tol = np.maximum(ulp, 1e-6 * np.abs(ref.astype(np.float32)).max())
    assert np.all(np.abs(out.astype(np.float32) - ref.astype(np.float32)) <= tol)


@pytest.mark.parametrize("i", range(5))
def test_moe_align_matches_reference(i):
    f = _load("moe_align.npz")
    T, E, k, bm, ntp = (int(v) for v in f[f"meta{i}"])
    s, e, n = O.moe_align(f[f"ids{i}"], bm, E)
    assert n == ntp
    assert np.array_equal(s, f[f"sorted{i}"])
    assert np.array_equal(e, f[f"eids{i}"])


@pytest.mark.parametrize("name", ["a", "b", "c"])
def test_grouped_oracle_matches_reference(name):
    f = _load("moe_gemm.npz")
    seed, T, E, N, K, k, bm, g, asym = (int(v) for v in f[name + "_meta"])
    rng = np.random.default_rng(seed)
    x = rng.standard_normal((T, K), dtype=np.float32).astype(np.float16)
    codes, scales, zeros = I.expert_weights(rng, E, N, K, g, bool(asym))
    ids = np.stack([rng.permutation(E)[:k] for _ in range(T)]).astype(np.int32)
    s, e, n = O.moe_align(ids, bm, E)
    out = O.moe_gemm(x, O.pack_int4(codes), scales, O.pack_zeros(zeros) if asym else None,
                     s, e, n, k, bm)
    assert np.array_equal(out, f[name])


@pytest.mark.parametrize("name", ["small", "decode"])
def test_moe_layer_oracle_matches_reference(name):
    f = _load("moe_layer.npz")
    seed, T, E, H, Ii, k, g = (int(v) for v in f[name + "_meta"])
    c = I.moe_layer_case(seed, T, E, H, Ii, k, g)
    y = O.moe_layer(c["x"], O.pack_int4(c["c13"]), c["s13"], O.pack_zeros(c["z13"]),
                    O.pack_int4(c["c2"]), c["s2"], O.pack_zeros(c["z2"]), c["topk_ids"],
                    c["topk_weights"])
    np.testing.assert_allclose(y, f[name], rtol=0, atol=1e-6 * np.abs(f[name]).max())


def test_awq_conversion_matches_reference():
    f = _load("convert.npz")
    w, s, z = O.awq_to_op_layout(f["awq_qweight"], f["awq_scales"], f["awq_qzeros"])
    assert np.array_equal(w, f["op_w"]) and np.array_equal(s, f["op_s"])
    assert np.array_equal(z, f["op_z"])


def test_silu_and_mul_matches_reference():
    f = _load("convert.npz")
    assert np.array_equal(O.silu_and_mul(f["silu_in"]), f["silu_out"])
