"""GPU parity at the BASELINE configs' full sizes and on adversarial inputs.

* configs[2] prefill layer (4096 tokens, Zipf-biased routing over 256 experts + the shared
  expert as expert 256 with weight 1) through run_grouped_moe, the tile path;
* token counts that cross the composition's APPLY_CHUNK = 4096 boundary (4097, 8193);
* one expert owning >= 1024 rows, so it spans many 128-row tiles;
* decode-path GEMVs and the fused decode layer on activation rows that are all positive, hold
  one outlier channel at 60000, or look like post-SiLU rows;
* mxfp4 (E2M1) weights through mmq_fp8_gemm, against the oracle's E2M1 GEMM and the reference's
  own equivalence check (integer-valued E2M1 codes == int4 codes + 8, bit for bit);
* compressed-tensors and MoeWNA16 weights converted on the GPU and run through the layer.

The layer-sized checks use the plain-PyTorch fp32 reference (tests/torch_ref.py, pinned to the
numpy oracle by tests/test_torch_ref_cpu.py); the rest use the numpy oracle. The bar is the
north star's max-abs-rel <= 1e-2 (max |ours - ref| / max |ref|)."""
import os

import numpy as np
import pytest
import torch

import inputs as I
import torch_ref as R
import w4a8_oracle as O
from helpers import MAX_ABS_REL, max_abs_rel

pytestmark = pytest.mark.gpu
G = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")
H, INTER = 2048, 512


@pytest.fixture(scope="module")
def w4():
    assert torch.cuda.is_available(), "GPU tests need a CUDA device"
    import w4a8_fp8_wmma
    return w4a8_fp8_wmma


def cu(a):
    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


def rand_layer(seed, E, h=H, inter=INTER, asym=True):
    """Random op-layout weights on the GPU: uniform words = uniform 4-bit codes."""
    g = torch.Generator(device="cuda")
    g.manual_seed(seed)

    def words(*shape):
        return torch.randint(-2 ** 31, 2 ** 31 - 1, shape, dtype=torch.int32, device="cuda",
                             generator=g)

    def scales(*shape):
        return (torch.rand(shape, device="cuda", generator=g) * (2e-2 - 1e-3) + 1e-3).half()
    w13, s13 = words(E, 2 * inter, h // 8), scales(E, 2 * inter, h // 128)
    z13 = words(E, 2 * inter // 8, h // 128) if asym else None
    w2, s2 = words(E, h, inter // 8), scales(E, h, inter // 128)
    z2 = words(E, h // 8, inter // 128) if asym else None
    return w13, s13, z13, w2, s2, z2


def tokens(seed, T, E_routed, k, zipf, shared=True):
    rng = np.random.default_rng(seed)
    x = rng.standard_normal((T, H), dtype=np.float32).astype(np.float16)
    _, ids, w = I.routing(rng, T, E_routed, k, zipf_bias=zipf)
    if shared:
        ids = np.concatenate([ids, np.full((T, 1), E_routed, np.int32)], axis=1)
        w = np.concatenate([w, np.ones((T, 1), np.float32)], axis=1)
    return x, ids.astype(np.int32), w.astype(np.float32)


def run_layer(x, wts, ids, w, kernel="wmma"):
    from w4a8_fp8_wmma.moe_experts import run_grouped_moe
    w13, s13, z13, w2, s2, z2 = wts
    return run_grouped_moe(x, w13, w2, s13, s2, z13, z2, w, ids, kernel=kernel,
                           out_dtype=torch.float32)


def check_layer(x, wts, ids, w, kernel="wmma"):
    xd, idd, wd = cu(x), cu(ids), cu(w)
    y = run_layer(xd, wts, idd, wd, kernel)
    ref = R.moe_layer(xd, *wts, idd, wd)
    err = max_abs_rel(y.cpu().numpy(), ref.cpu().numpy())
    assert err <= MAX_ABS_REL, err
    return err


def test_torch_ref_act_quant_bit_exact_on_gpu(w4):
    """The reference's quantisation must be the oracle's on the GPU too (bytes and scales)."""
    rng = np.random.default_rng(90)
    x = (rng.standard_normal((512, 2048), dtype=np.float32) * 3).astype(np.float16)
    q, s = R.act_quant(cu(x))
    qr, sr = O.act_quant(x)
    assert np.array_equal(s.cpu().numpy().view(np.uint32), sr.view(np.uint32))
    assert np.array_equal(q.cpu().numpy().view(np.uint32), O.e4m3_decode(qr).view(np.uint32))
    qk, sk = w4.act_quant_fp8(cu(x))
    assert np.array_equal(qk.cpu().numpy(), qr)


# ------------------------------------------------------------ configs[2] and the tile path ---
def test_layer_configs2_prefill_zipf(w4):
    wts = rand_layer(2000, 257)
    x, ids, w = tokens(2, 4096, 256, 8, zipf=True)
    check_layer(x, wts, ids, w)


@pytest.mark.parametrize("T", [4097, 8193])
def test_layer_crosses_apply_chunk(w4, T):
    wts = rand_layer(2100 + T, 65)
    x, ids, w = tokens(T, T, 64, 8, zipf=True)
    check_layer(x, wts, ids, w)


def test_layer_hot_expert_many_tiles(w4):
    """Expert 5 is in every token's top-8: 2048 of its rows span 16 tiles of 128."""
    wts = rand_layer(2200, 33)
    x, ids, w = tokens(22, 2048, 32, 8, zipf=False)
    has5 = (ids[:, :8] == 5).any(axis=1)
    ids[~has5, 7] = 5
    check_layer(x, wts, ids, w)
    assert int((ids == 5).sum()) == 2048


def test_layer_decode_configs1(w4):
    wts = rand_layer(2300, 257)
    x, ids, w = tokens(1, 32, 256, 8, zipf=False)
    check_layer(x, wts, ids, w, kernel="wmma")


# ------------------------------------------------------------ adversarial activations --------
def adversarial(kind, T, K, seed, outlier=60000.0, const=3.0):
    rng = np.random.default_rng(seed)
    base = rng.standard_normal((T, K), dtype=np.float32)
    if kind == "positive":
        x = np.abs(base) + 0.5
    elif kind == "outlier":
        x = base.copy()
        x[:, 17] = outlier
        x[::2, 1000 % K] = -outlier
    elif kind == "post_silu":
        g = base * 3.0
        x = g / (1.0 + np.exp(-g))
    elif kind == "constant":
        x = np.full((T, K), const, np.float32)
    else:
        raise ValueError(kind)
    return x.astype(np.float16)


KINDS = ["positive", "outlier", "post_silu", "constant"]


@pytest.mark.parametrize("kind", KINDS)
@pytest.mark.parametrize("M,K,N", [(16, 2048, 1024), (4, 512, 2048)])
def test_dense_gemv_adversarial(w4, kind, M, K, N):
    _, codes, scales, zeros = I.dense_case(50, M, N, K, 128, True)
    x = adversarial(kind, M, K, 51)
    ref = O.dense_gemm(x, O.pack_int4(codes), scales, O.pack_zeros(zeros)).astype(np.float32)
    for kern in ("decode_gemv", "prefill_wmma"):
        out = w4.mmq_fp8_gemm(cu(x), cu(O.pack_int4(codes)), cu(scales), kernel=kern,
                              w_zeros=cu(O.pack_zeros(zeros))).cpu().numpy()
        assert max_abs_rel(out, ref) <= MAX_ABS_REL, (kern, max_abs_rel(out, ref))


@pytest.mark.parametrize("kind", KINDS)
def test_grouped_gemv_adversarial(w4, kind):
    T, E, k, N, K, bm = 32, 64, 8, 1024, 2048, 8
    rng = np.random.default_rng(60)
    codes, scales, zeros = I.expert_weights(rng, E, N, K, 128, True)
    ids = np.stack([rng.permutation(E)[:k] for _ in range(T)]).astype(np.int32)
    x = adversarial(kind, T, K, 61)
    s, e, n = O.moe_align(ids, bm, E)
    out = w4.mmq_fp8_moe_gemm(cu(x), cu(O.pack_int4(codes)), cu(scales), cu(s), cu(e),
                              cu(np.array([n], np.int32)), k, bm, kernel="gemv",
                              w_zeros=cu(O.pack_zeros(zeros))).cpu().numpy()
    ref = O.moe_gemm(x, O.pack_int4(codes), scales, O.pack_zeros(zeros), s, e, n, k, bm)
    valid = s < T * k
    assert max_abs_rel(out[valid], ref[valid].astype(np.float32)) <= MAX_ABS_REL


@pytest.mark.parametrize("kind", KINDS)
def test_fused_decode_layer_adversarial(w4, kind):
    """The whole decode layer (M <= 96: the fused decode op). Outliers of 200 sigma and
    constant rows of 0.05 keep the fp16 intermediates finite: at 60000 the reference's own
    fp16 gate/up product overflows to inf (the single-GEMM tests above cover 60000)."""
    wts = rand_layer(2400, 257)
    _, ids, w = tokens(3, 32, 256, 8, zipf=False)
    x = adversarial(kind, 32, H, 62, outlier=200.0, const=0.05)
    xd, idd, wd = cu(x), cu(ids), cu(w)
    assert torch.isfinite(R.moe_layer(xd, *wts, idd, wd)).all()
    check_layer(x, wts, ids, w, kernel="wmma")


# ------------------------------------------------------------ mxfp4 (E2M1) -----------------
@pytest.mark.parametrize("kernel", ["reference_scalar", "prefill_wmma", "prefill_wmma_ashuffle",
                                    "decode_gemv"])
def test_e2m1_dense_vs_oracle(w4, kernel):
    f = np.load(os.path.join(G, "formats.npz"))
    w, s = f["mx_op_w"][0], f["mx_op_s"][0]
    for M in (1, 16, 64):
        x = np.resize(f["mx_x"], (M, f["mx_x"].shape[1])).astype(np.float16)
        out = w4.mmq_fp8_gemm(cu(x), cu(w), cu(s), kernel=kernel,
                              weight_is_e2m1=True).cpu().numpy()
        ref = O.dense_gemm_e2m1(x, w, s).astype(np.float32)
        assert max_abs_rel(out, ref) <= MAX_ABS_REL


@pytest.mark.parametrize("kernel", ["reference_scalar", "prefill_wmma", "decode_gemv"])
def test_e2m1_integer_codes_equal_int4(w4, kernel):
    """The reference's bit-exact equivalence (mxfp4/test_mxfp4_kernel_gpu.py:45-61)."""
    rng = np.random.default_rng(70)
    int_codes = np.array([0, 2, 4, 5, 6, 7, 10, 12, 13, 14, 15])
    codes = int_codes[rng.integers(0, len(int_codes), (128, 512))].astype(np.uint8)
    c4 = (O.E2M1_VALUES[codes] + 8).astype(np.uint8)
    s = rng.uniform(0.25, 0.75, (128, 16)).astype(np.float16)
    for M in (4, 16):
        x = (rng.standard_normal((M, 512), dtype=np.float32) * 0.5).astype(np.float16)
        a = w4.mmq_fp8_gemm(cu(x), cu(O.pack_int4(codes)), cu(s), kernel=kernel,
                            weight_is_e2m1=True)
        b = w4.mmq_fp8_gemm(cu(x), cu(O.pack_int4(c4)), cu(s), kernel="reference_scalar")
        assert torch.equal(a.view(torch.int16), b.view(torch.int16))


# ------------------------------------------------------------ checkpoint formats on GPU -----
def test_ct_and_wna16_layers_on_gpu(w4):
    from w4a8_fp8_wmma.moe_experts import ct_moe_to_op_layout, wna16_moe_to_op_layout
    rng = np.random.default_rng(80)
    E, T, k, h, inter = 8, 12, 2, 256, 128
    # compressed-tensors (E, K/8, N) natural order, symmetric uint4b8
    q13 = rng.integers(-2 ** 31, 2 ** 31 - 1, (E, h // 8, 2 * inter), dtype=np.int64).astype(np.int32)
    q2 = rng.integers(-2 ** 31, 2 ** 31 - 1, (E, inter // 8, h), dtype=np.int64).astype(np.int32)
    s13 = rng.uniform(1e-3, 2e-2, (E, h // 128, 2 * inter)).astype(np.float16)
    s2 = rng.uniform(1e-3, 2e-2, (E, inter // 128, h)).astype(np.float16)
    w13, ss13 = ct_moe_to_op_layout(cu(q13), cu(s13))
    w2, ss2 = ct_moe_to_op_layout(cu(q2), cu(s2))
    x, ids, w = tokens(81, T, E, k, zipf=False, shared=False)
    xh = np.resize(x, (T, h)).astype(np.float16)
    y = run_layer(cu(xh), (w13, ss13, None, w2, ss2, None), cu(ids), cu(w)).cpu().numpy()
    ref = O.moe_layer(xh, w13.cpu().numpy(), ss13.cpu().numpy(), None, w2.cpu().numpy(),
                      ss2.cpu().numpy(), None, ids, w)
    assert max_abs_rel(y, ref) <= MAX_ABS_REL
    # MoeWNA16 u8 storage with zero points
    u13 = rng.integers(0, 256, (E, 2 * inter, h // 2), dtype=np.int64).astype(np.uint8)
    z13 = rng.integers(0, 256, (E, inter, h // 128), dtype=np.int64).astype(np.uint8)
    u2 = rng.integers(0, 256, (E, h, inter // 2), dtype=np.int64).astype(np.uint8)
    z2 = rng.integers(0, 256, (E, h // 2, inter // 128), dtype=np.int64).astype(np.uint8)
    a13 = wna16_moe_to_op_layout(cu(u13), cu(np.swapaxes(s13, 1, 2).copy()), cu(z13))
    a2 = wna16_moe_to_op_layout(cu(u2), cu(np.swapaxes(s2, 1, 2).copy()), cu(z2))
    y = run_layer(cu(xh), (a13[0], a13[1], a13[2], a2[0], a2[1], a2[2]), cu(ids),
                  cu(w)).cpu().numpy()
    n = lambda t: t.cpu().numpy()  # noqa: E731
    ref = O.moe_layer(xh, n(a13[0]), n(a13[1]), n(a13[2]), n(a2[0]), n(a2[1]), n(a2[2]), ids, w)
    assert max_abs_rel(y, ref) <= MAX_ABS_REL
