"""GPU parity tests: every op against the CPU oracle (and the reference-generated golden
fixtures) on identical seeded inputs.

Bars (north star): activation-quant bytes and scales, int4 unpack / zero handling and the
routing sort order are bit-exact; GEMM outputs are within max-abs-rel 1e-2 (max |ours - ref| /
max |ref|) of the fp32-accumulated oracle, and also pass the reference's own rule
(mean-abs and per-element atol/rtol, test_correctness.py:146-158)."""
import os

import numpy as np
import pytest
import torch

import inputs as I
import w4a8_oracle as O
from helpers import MAX_ABS_REL, max_abs_rel, reference_tolerance_ok

pytestmark = pytest.mark.gpu
G = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")


@pytest.fixture(scope="module")
def w4():
    assert torch.cuda.is_available(), "GPU tests need a CUDA device"
    import w4a8_fp8_wmma
    return w4a8_fp8_wmma


def cu(a, dtype=None):
    t = torch.from_numpy(np.ascontiguousarray(a)).cuda()
    return t if dtype is None else t.to(dtype)


# ------------------------------------------------------------------ activation quant -------
@pytest.mark.parametrize("M,K,seed", [(16, 2048, 0), (4096, 2048, 1), (257, 512, 2), (3, 44, 3),
                                      (1, 8, 4), (64, 7168, 5)])
def test_act_quant_bit_exact(w4, M, K, seed):
    rng = np.random.default_rng(seed)
    x = (rng.standard_normal((M, K), dtype=np.float32) * 3).astype(np.float16)
    x[0, :] = 0
    if M > 2:
        x[1] *= np.float16(1e-4)
        x[2, 0] = np.float16(65504.0)
    q, s = w4.act_quant_fp8(cu(x))
    qr, sr = O.act_quant(x)
    assert np.array_equal(q.cpu().numpy(), qr)
    assert np.array_equal(s.cpu().numpy().view(np.uint32), sr.view(np.uint32))


@pytest.mark.parametrize("i", [0, 1, 2])
def test_act_quant_golden(w4, i):
    f = np.load(os.path.join(G, "act_quant.npz"))
    q, _ = w4.act_quant_fp8(cu(f[f"x{i}"]))
    assert np.array_equal(q.cpu().numpy(), f[f"q{i}"])


# ------------------------------------------------------------------ moe_align ---------------
def _check_align(w4, ids, bm, E, expert_map=None, n_local=None):
    s, e, n = w4.moe_align_block_size(cu(ids), bm, E, expert_map, n_local)
    torch.cuda.synchronize()
    flat = ids.reshape(-1)
    if expert_map is not None:
        m = expert_map.cpu().numpy()
        loc = np.where((flat >= 0) & (flat < E), m[np.clip(flat, 0, E - 1)], -1)
        rs, re, rn = _align_local(loc, bm, n_local, flat.size)
    else:
        rs, re, rn = O.moe_align(ids, bm, E)
    n = int(n.item())
    assert n == rn
    assert np.array_equal(s.cpu().numpy()[:n], rs)
    assert np.array_equal(e.cpu().numpy()[:n // bm], re)
    assert np.all(s.cpu().numpy()[n:] == flat.size)
    assert np.all(e.cpu().numpy()[n // bm:] == -1)


def _align_local(loc, bm, E, num_slots):
    s, e = [], []
    for x in range(E):
        slots = np.nonzero(loc == x)[0].tolist()
        npad = (len(slots) + bm - 1) // bm * bm
        s += slots + [num_slots] * (npad - len(slots))
        e += [x] * (npad // bm)
    return np.asarray(s, np.int32), np.asarray(e, np.int32), len(s)


@pytest.mark.parametrize("T,E,k,bm,seed", [(32, 256, 8, 8, 0), (4096, 256, 8, 64, 1),
                                           (1, 8, 2, 16, 2), (64, 8, 2, 16, 3),
                                           (32, 257, 9, 8, 4), (9000, 64, 8, 16, 5)])
def test_moe_align_bit_exact(w4, T, E, k, bm, seed):
    _check_align(w4, I.random_topk(seed, T, E, k), bm, E)


def test_moe_align_zipf_prefill(w4):
    _, ids, _ = I.routing(np.random.default_rng(7), 4096, 256, 8, zipf_bias=True)
    _check_align(w4, ids, 64, 256)


@pytest.mark.parametrize("i", range(5))
def test_moe_align_golden(w4, i):
    f = np.load(os.path.join(G, "moe_align.npz"))
    T, E, k, bm, ntp = (int(v) for v in f[f"meta{i}"])
    s, e, n = w4.moe_align_block_size(cu(f[f"ids{i}"]), bm, E)
    assert int(n.item()) == ntp
    assert np.array_equal(s.cpu().numpy()[:ntp], f[f"sorted{i}"])
    assert np.array_equal(e.cpu().numpy()[:ntp // bm], f[f"eids{i}"])


def test_moe_align_expert_map(w4):
    E, rank, world = 256, 1, 4
    ids = I.random_topk(11, 32, E, 8)
    m = np.full(E, -1, np.int32)
    m[rank * 64:(rank + 1) * 64] = np.arange(64)
    _check_align(w4, ids, 8, E, cu(m), 64)


# ------------------------------------------------------------------ dense GEMM --------------
def _dense(w4, x, codes, scales, zeros, kernel):
    zp = cu(O.pack_zeros(zeros)) if zeros is not None else None
    return w4.mmq_fp8_gemm(cu(x), cu(O.pack_int4(codes)), cu(scales), kernel=kernel,
                           w_zeros=zp).cpu().numpy()


@pytest.mark.parametrize("kernel", ["decode_gemv", "prefill_wmma", "prefill_wmma_ashuffle",
                                    "reference_scalar"])
@pytest.mark.parametrize("name", ["cfg0", "m1_g32_sym", "tail_17x48", "tail_100x80", "g128_sym",
                                  "g64_asym"])
def test_dense_golden(w4, name, kernel):
    f = np.load(os.path.join(G, "dense.npz"))
    seed, M, N, K, g, asym = (int(v) for v in f[name + "_meta"])
    x, c, s, z = I.dense_case(seed, M, N, K, g, bool(asym))
    out = _dense(w4, x, c, s, z, kernel)
    ref = f[name].astype(np.float32)
    assert max_abs_rel(out, ref) <= MAX_ABS_REL
    assert reference_tolerance_ok(out, ref)


@pytest.mark.parametrize("M", [1, 16, 128])
@pytest.mark.parametrize("K,N", [(2048, 4096), (4096, 2048), (2048, 512), (2048, 8192)])
def test_dense_sweep_vs_oracle(w4, M, K, N):
    x, c, s, z = I.dense_case(100 + M, M, N, K, 128, True)
    out = _dense(w4, x, c, s, z, "prefill_wmma_ashuffle")
    ref = O.dense_gemm(x, O.pack_int4(c), s, O.pack_zeros(z)).astype(np.float32)
    assert max_abs_rel(out, ref) <= MAX_ABS_REL
    if M <= 16:
        out2 = _dense(w4, x, c, s, z, "decode_gemv")
        assert max_abs_rel(out2, ref) <= MAX_ABS_REL


def _torch_fp32_dense(x, codes, scales, zeros):
    """fp32 torch reference on the GPU for large M: dequantised weights times quantised acts."""
    xq, xs = O.act_quant(x)
    g = codes.shape[1] // scales.shape[1]
    xf = cu(O.e4m3_decode(xq))
    w = cu(codes.astype(np.float32)) - cu(np.repeat(zeros, g, axis=1).astype(np.float32))
    w = w * cu(np.repeat(scales.astype(np.float32), g, axis=1))
    torch.backends.cuda.matmul.allow_tf32 = False
    return ((xf @ w.T) * cu(xs)[:, None]).cpu().numpy()


@pytest.mark.parametrize("M", [2048, 8192])
@pytest.mark.parametrize("K,N", [(2048, 4096), (2048, 512)])
def test_dense_large_m_vs_torch_fp32(w4, M, K, N):
    x, c, s, z = I.dense_case(200 + M, M, N, K, 128, True)
    out = _dense(w4, x, c, s, z, "prefill_wmma_ashuffle")
    ref = _torch_fp32_dense(x, c, s, z)
    assert max_abs_rel(out, ref) <= MAX_ABS_REL


# ------------------------------------------------------------------ grouped GEMM ------------
def _grouped_inputs(seed, T, E, N, K, k, g, asym):
    rng = np.random.default_rng(seed)
    x = rng.standard_normal((T, K), dtype=np.float32).astype(np.float16)
    codes, scales, zeros = I.expert_weights(rng, E, N, K, g, asym)
    ids = np.stack([rng.permutation(E)[:k] for _ in range(T)]).astype(np.int32)
    return x, codes, scales, zeros, ids


def _run_grouped(w4, x, codes, scales, zeros, ids, bm, E, k, kernel, op="gemm"):
    s, e, n = O.moe_align(ids, bm, E)
    args = (cu(x), cu(O.pack_int4(codes)), cu(scales), cu(s), cu(e), cu(np.array([n], np.int32)),
            k, bm)
    zp = cu(O.pack_zeros(zeros)) if zeros is not None else None
    if op == "gemm":
        out = w4.mmq_fp8_moe_gemm(*args, kernel=kernel, w_zeros=zp)
    else:
        out = torch.ops.w4a8_b200.moe_gemm1_silu(*args[:3], zp if zp is not None else torch.empty(0, dtype=torch.int32, device="cuda"),
                                                 *args[3:], {"scalar": 0, "wmma": 6, "gemv": 7}[kernel], False)
    return out.cpu().numpy(), s, e, n


@pytest.mark.parametrize("kernel", ["gemv", "wmma", "scalar"])
@pytest.mark.parametrize("name", ["a", "b", "c"])
def test_grouped_golden(w4, name, kernel):
    f = np.load(os.path.join(G, "moe_gemm.npz"))
    seed, T, E, N, K, k, bm, g, asym = (int(v) for v in f[name + "_meta"])
    if kernel == "wmma" and bm % 16:
        pytest.skip("wmma needs block_m % 16 == 0 (reference rule)")
    x, codes, scales, zeros, ids = _grouped_inputs(seed, T, E, N, K, k, g, bool(asym))
    out, s, e, n = _run_grouped(w4, x, codes, scales, zeros, ids, bm, E, k, kernel)
    valid = s < T * k
    ref = f[name].astype(np.float32)
    assert max_abs_rel(out[valid], ref[valid]) <= MAX_ABS_REL
    assert reference_tolerance_ok(out[valid], ref[valid], mean_rtol=0.02)
    assert np.all(out[~valid] == 0)


@pytest.mark.parametrize("kernel,bm", [("gemv", 8), ("wmma", 64), ("wmma", 16)])
@pytest.mark.parametrize("which", ["gate_up", "down"])
def test_grouped_qwen_decode_shapes(w4, kernel, bm, which):
    T, E, k = 32, 256, 8
    N, K = (1024, 2048) if which == "gate_up" else (2048, 512)
    x, codes, scales, zeros, ids = _grouped_inputs(300, T, E, N, K, k, 128, True)
    out, s, e, n = _run_grouped(w4, x, codes, scales, zeros, ids, bm, E, k, kernel)
    ref = O.moe_gemm(x, O.pack_int4(codes), scales, O.pack_zeros(zeros), s, e, n, k, bm)
    valid = s < T * k
    assert max_abs_rel(out[valid], ref[valid].astype(np.float32)) <= MAX_ABS_REL


@pytest.mark.parametrize("kernel,bm", [("gemv", 8), ("wmma", 64), ("scalar", 16)])
def test_fused_silu_bit_exact_vs_unfused(w4, kernel, bm):
    """Fused gemm1+silu equals the unfused GEMM followed by the reference silu_and_mul on the
    GPU output, bit for bit (test_moe_experts.py:283-315)."""
    T, E, k, I_, K = 48, 16, 4, 256, 512
    x, codes, scales, zeros, ids = _grouped_inputs(400, T, E, 2 * I_, K, k, 128, True)
    out1, s, e, n = _run_grouped(w4, x, codes, scales, zeros, ids, bm, E, k, kernel)
    fused, *_ = _run_grouped(w4, x, codes, scales, zeros, ids, bm, E, k, kernel, op="silu")
    o1 = torch.from_numpy(out1).cuda()
    g, u = o1[:, :I_].float(), o1[:, I_:]
    ref = ((g / (1.0 + torch.exp(-g))).to(torch.float16) * u).cpu().numpy()
    valid = s < T * k
    assert np.array_equal(fused[valid].view(np.uint16), ref[valid].view(np.uint16))


def test_scatter_and_gather_reduce_vs_oracle(w4):
    T, E, k, N, K, bm = 24, 16, 4, 256, 512, 8
    x, codes, scales, zeros, ids = _grouped_inputs(500, T, E, N, K, k, 128, True)
    rng = np.random.default_rng(501)
    tw = rng.random((T, k), dtype=np.float32)
    s, e, n = O.moe_align(ids, bm, E)
    P = len(s)
    buf = rng.standard_normal((P, K), dtype=np.float32).astype(np.float16)
    # reference: per padded row, down GEMM of buf (identity gather), weighted into its token
    ident = np.where(s < T * k, np.arange(P), P).astype(np.int32)
    out2 = O.moe_gemm(buf, O.pack_int4(codes), scales, O.pack_zeros(zeros), ident, e, n, 1, bm)
    ref = O.gather_reduce(out2, s, tw, n, k)
    output = torch.zeros((T, N), dtype=torch.float32, device="cuda")
    w4.mmq_fp8_moe_gemm_scatter(cu(buf), cu(O.pack_int4(codes)), cu(scales), cu(s), cu(e),
                                cu(np.array([n], np.int32)), cu(tw.reshape(-1)), output, k, bm,
                                kernel="gemv", w_zeros=cu(O.pack_zeros(zeros)))
    assert max_abs_rel(output.cpu().numpy(), ref) <= MAX_ABS_REL
    red = w4.mmq_fp8_moe_gather_reduce(cu(out2), cu(s), cu(tw.reshape(-1)),
                                       cu(np.array([n], np.int32)), k).cpu().numpy()
    assert np.array_equal(red, ref)


# ------------------------------------------------------------------ whole layer -------------
def _layer_weights(c):
    return (cu(O.pack_int4(c["c13"])), cu(O.pack_int4(c["c2"])), cu(c["s13"]), cu(c["s2"]),
            cu(O.pack_zeros(c["z13"])), cu(O.pack_zeros(c["z2"])))


@pytest.mark.parametrize("name", ["small", "decode"])
@pytest.mark.parametrize("kernel", ["wmma", "scalar"])
def test_moe_layer_golden(w4, name, kernel):
    from w4a8_fp8_wmma.moe_experts import run_grouped_moe
    f = np.load(os.path.join(G, "moe_layer.npz"))
    seed, T, E, H, Ii, k, g = (int(v) for v in f[name + "_meta"])
    c = I.moe_layer_case(seed, T, E, H, Ii, k, g)
    w1, w2, s1, s2, z1, z2 = _layer_weights(c)
    y = run_grouped_moe(cu(c["x"]), w1, w2, s1, s2, z1, z2, cu(c["topk_weights"]),
                        cu(c["topk_ids"]), kernel=kernel, out_dtype=torch.float32)
    assert max_abs_rel(y.cpu().numpy(), f[name]) <= MAX_ABS_REL


@pytest.mark.parametrize("T", [32, 200])
def test_moe_layer_qwen_shape_vs_oracle(w4, T):
    from w4a8_fp8_wmma.moe_experts import run_grouped_moe
    c = I.moe_layer_case(600 + T, T, 256, 2048, 512, 8, 128)
    w1, w2, s1, s2, z1, z2 = _layer_weights(c)
    y = run_grouped_moe(cu(c["x"]), w1, w2, s1, s2, z1, z2, cu(c["topk_weights"]),
                        cu(c["topk_ids"]), out_dtype=torch.float32)
    ref = O.moe_layer(c["x"], O.pack_int4(c["c13"]), c["s13"], O.pack_zeros(c["z13"]),
                      O.pack_int4(c["c2"]), c["s2"], O.pack_zeros(c["z2"]), c["topk_ids"],
                      c["topk_weights"])
    assert max_abs_rel(y.cpu().numpy(), ref) <= MAX_ABS_REL


def test_awq_converter_on_gpu(w4):
    from w4a8_fp8_wmma.moe_experts import awq_moe_to_op_layout
    f = np.load(os.path.join(G, "convert.npz"))
    w, s, z = awq_moe_to_op_layout(cu(f["awq_qweight"]), cu(f["awq_scales"]), cu(f["awq_qzeros"]))
    assert np.array_equal(w.cpu().numpy(), f["op_w"])
    assert np.array_equal(s.cpu().numpy(), f["op_s"])
    assert np.array_equal(z.cpu().numpy(), f["op_z"])


def test_silu_op_requires_wmma(w4):
    x = torch.zeros(2, 128, dtype=torch.float16, device="cuda")
    w = torch.zeros(2, 16, 16, dtype=torch.int32, device="cuda")
    s = torch.zeros(2, 16, 1, dtype=torch.float16, device="cuda")
    i32 = torch.zeros(16, dtype=torch.int32, device="cuda")
    with pytest.raises(RuntimeError, match="needs the 'wmma' kernel"):
        w4.mmq_fp8_moe_gemm1_silu(x, w, s, i32, i32[:2], i32[:1], 2, 8, kernel="gemv")


@pytest.mark.parametrize("T,E,asym", [(1, 64, True), (32, 257, True), (32, 64, False),
                                      (96, 64, True)])
def test_fused_decode_layer_vs_oracle(w4, T, E, asym):
    """torch.ops.w4a8_b200.moe_decode (the one-call decode layer) against the oracle layer."""
    c = I.moe_layer_case(700 + T + E, T, E, 2048, 512, 8, 128, asym=asym)
    z1 = cu(O.pack_zeros(c["z13"])) if asym else torch.empty(0, dtype=torch.int32, device="cuda")
    z2 = cu(O.pack_zeros(c["z2"])) if asym else torch.empty(0, dtype=torch.int32, device="cuda")
    y = torch.ops.w4a8_b200.moe_decode(cu(c["x"]), cu(O.pack_int4(c["c13"])), cu(c["s13"]), z1,
                                       cu(O.pack_int4(c["c2"])), cu(c["s2"]), z2,
                                       cu(c["topk_weights"]), cu(c["topk_ids"]))
    ref = O.moe_layer(c["x"], O.pack_int4(c["c13"]), c["s13"],
                      O.pack_zeros(c["z13"]) if asym else None, O.pack_int4(c["c2"]), c["s2"],
                      O.pack_zeros(c["z2"]) if asym else None, c["topk_ids"], c["topk_weights"])
    assert y.dtype == torch.float16
    assert max_abs_rel(y.float().cpu().numpy(), ref) <= MAX_ABS_REL


def test_expert_parallel_layer_world1_vs_oracle(w4):
    """ExpertParallelMoE on a one-rank NCCL group (dispatch -> local experts -> combine, plus a
    replicated shared expert) against the oracle layer with the shared expert as expert E."""
    import socket
    from datetime import timedelta

    import torch.distributed as dist
    from w4a8_fp8_wmma.ep import ExpertParallelMoE
    T, E, H, Ii, k = 16, 32, 2048, 512, 4
    c = I.moe_layer_case(900, T, E + 1, H, Ii, k, 128)
    # routed slots only over experts 0..E-1; expert E is the shared one
    rng = np.random.default_rng(901)
    ids = np.stack([rng.permutation(E)[:k] for _ in range(T)]).astype(np.int32)
    w = rng.random((T, k), dtype=np.float32)
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    dist.init_process_group("nccl", init_method=f"tcp://127.0.0.1:{port}", rank=0, world_size=1,
                            timeout=timedelta(seconds=60), device_id=torch.device("cuda", 0))
    try:
        p13, p2 = O.pack_int4(c["c13"]), O.pack_int4(c["c2"])
        z13, z2 = O.pack_zeros(c["z13"]), O.pack_zeros(c["z2"])
        wts = (cu(p13[:E]), cu(c["s13"][:E]), cu(z13[:E]), cu(p2[:E]), cu(c["s2"][:E]), cu(z2[:E]))
        shared = (cu(p13[E:]), cu(c["s13"][E:]), cu(z13[E:]), cu(p2[E:]), cu(c["s2"][E:]),
                  cu(z2[E:]))
        layer = ExpertParallelMoE(*wts, E, k, shared=shared)
        y = layer(cu(c["x"]), cu(ids), cu(w)).cpu().numpy()
    finally:
        dist.destroy_process_group()
    ids_full = np.concatenate([ids, np.full((T, 1), E, np.int32)], axis=1)
    w_full = np.concatenate([w, np.ones((T, 1), np.float32)], axis=1)
    ref = O.moe_layer(c["x"], p13, c["s13"], z13, p2, c["s2"], z2, ids_full, w_full)
    assert max_abs_rel(y, ref) <= MAX_ABS_REL


def test_silu_and_mul_exhaustive_fp16_gate(w4):
    """Every finite fp16 gate value (with a fixed up value of 1) through the library's SiLU
    matches fp16(g / (1 + exp(-g))) computed by torch in fp32 with an IEEE divide, bit for bit:
    the fused epilogue's fast quotient falls back to the exact divide at fp16 rounding
    boundaries."""
    bits = torch.arange(0, 65536, dtype=torch.int32).to(torch.int16).view(torch.float16)
    g = bits[torch.isfinite(bits)].cuda()
    for up in (1.0, -0.75):
        x = torch.stack([g, torch.full_like(g, up)], 1).contiguous()  # (M, 2): inter = 1
        out = w4.silu_and_mul(x)[:, 0]
        gf = g.float()
        ref = (gf / (1.0 + torch.exp(-gf))).to(torch.float16) * torch.tensor(up, dtype=torch.float16, device="cuda")
        assert torch.equal(out.view(torch.int16), ref.view(torch.int16))


def test_ep_pack_and_gather_kernels_vs_torch(w4):
    """ep_pack against plan_dispatch and the oracle's quantisation: row positions, local ids and
    weights are integer/copy work and must match exactly, the e4m3 bytes are the oracle's (in
    the GEMV byte order), and ep_gather equals the rank-order fp32 sum plus the shared row."""
    from w4a8_fp8_wmma.ep import plan_dispatch
    T, k, H, E, W = 24, 4, 512, 64, 4
    rng = np.random.default_rng(77)
    ids = np.stack([rng.permutation(E)[:k] for _ in range(T)]).astype(np.int32)
    ids[3, 1] = E + 5  # out of range: dropped
    x = rng.standard_normal((T, H), dtype=np.float32).astype(np.float16)
    w = rng.random((T, k), dtype=np.float32)
    rows, pos = torch.ops.w4a8_b200.ep_pack(cu(x), cu(ids), cu(w), E // W, W, E // W)
    has, pos_ref, local = plan_dispatch(cu(ids), E // W, W)
    assert torch.equal(pos.long(), pos_ref)
    G = H // 128
    r = rows.cpu().numpy()
    q, sc = O.act_quant(x)
    perm = np.array([0, 2, 4, 6, 1, 3, 5, 7])
    qg = q.reshape(T, H // 8, 8)[:, :, perm].reshape(T, H)
    loc = local.cpu().numpy()
    o = H + 4 * G + 4
    for d in range(W):
        for t in range(T):
            p = int(pos_ref[d, t])
            if p < 0:
                continue
            row = r[d * T + p]
            assert np.array_equal(row[:H], qg[t])
            assert row[H + 4 * G:o].view(np.float32)[0] == sc[t]
            assert np.array_equal(row[o:o + 4 * k].view(np.int32), loc[d, t].astype(np.int32))
            assert np.array_equal(row[o + 4 * k:o + 8 * k].view(np.float32),
                                  np.where(loc[d, t] >= 0, w[t], 0).astype(np.float32))
    own = r[W * T:]
    assert np.all(own[:, o:o + 4].view(np.int32)[:, 0] == E // W)
    back = torch.randn((W * T, H), device="cuda")
    sh = torch.randn((T, H), device="cuda")
    out = torch.ops.w4a8_b200.ep_gather(back, pos, sh)
    ref = torch.zeros((T, H), device="cuda")
    for d in range(W):
        sel = pos_ref[d] >= 0
        ref[sel] = ref[sel] + back[d * T + pos_ref[d][sel]]
    assert torch.equal(out, ref + sh)

def test_fused_decode_layer_skips_invalid_ids(w4):
    """Slots whose expert id is -1 or >= E contribute nothing (the reference's align skips
    them); a token with no valid slot gets a zero row."""
    T, E, k = 24, 64, 8
    c = I.moe_layer_case(808, T, E, 2048, 512, k, 128)
    ids = c["topk_ids"].copy()
    ids[3, 2] = -1
    ids[5, 0] = E
    ids[7, :] = -1
    w = c["topk_weights"].copy()
    y = torch.ops.w4a8_b200.moe_decode(cu(c["x"]), cu(O.pack_int4(c["c13"])), cu(c["s13"]),
                                       cu(O.pack_zeros(c["z13"])), cu(O.pack_int4(c["c2"])),
                                       cu(c["s2"]), cu(O.pack_zeros(c["z2"])), cu(w), cu(ids))
    keep = (ids >= 0) & (ids < E)
    ids_o = np.where(keep, ids, 0)
    w_o = np.where(keep, w, 0.0).astype(np.float32)
    ref = O.moe_layer(c["x"], O.pack_int4(c["c13"]), c["s13"], O.pack_zeros(c["z13"]),
                      O.pack_int4(c["c2"]), c["s2"], O.pack_zeros(c["z2"]), ids_o, w_o)
    yn = y.float().cpu().numpy()
    assert np.all(yn[7] == 0)
    assert max_abs_rel(yn, ref) <= MAX_ABS_REL


@pytest.mark.parametrize("gate_up,asym", [(True, True), (False, True), (True, False)])
def test_stream_pack_matches_layout_restatement(w4, gate_up, asym):
    """The load-time prepack kernel writes exactly the block layout the oracle restates."""
    rng = np.random.default_rng(830)
    E, N, K = 3, (256 if gate_up else 256), 1024
    w = rng.integers(-2 ** 31, 2 ** 31 - 1, (E, N, K // 8), dtype=np.int64).astype(np.int32)
    s = rng.uniform(1e-3, 2e-2, (E, N, K // 128)).astype(np.float16)
    z = rng.integers(-2 ** 31, 2 ** 31 - 1, (E, N // 8, K // 128), dtype=np.int64).astype(np.int32) if asym else None
    zt = cu(z) if asym else torch.empty(0, dtype=torch.int32, device="cuda")
    p = torch.ops.w4a8_b200.stream_pack(cu(w), cu(s), zt, gate_up).cpu().numpy()
    assert np.array_equal(p, O.stream_pack(w, s, z, gate_up))


@pytest.mark.parametrize("T,E,asym", [(1, 64, True), (32, 257, True), (32, 64, False), (96, 64, True)])
def test_packed_decode_layer_equals_unpacked(w4, T, E, asym):
    """moe_decode_packed on prepacked weights (the tensor-core GEMV) and the op-layout
    moe_decode (the mma.sync GEMV) both meet the bar against the oracle; they accumulate in a
    different order, so they agree to fp32/fp16 rounding, not bit for bit."""
    c = I.moe_layer_case(1700 + T + E, T, E, 2048, 512, 8, 128, asym=asym)
    z1 = cu(O.pack_zeros(c["z13"])) if asym else torch.empty(0, dtype=torch.int32, device="cuda")
    z2 = cu(O.pack_zeros(c["z2"])) if asym else torch.empty(0, dtype=torch.int32, device="cuda")
    w1, w2 = cu(O.pack_int4(c["c13"])), cu(O.pack_int4(c["c2"]))
    s1, s2 = cu(c["s13"]), cu(c["s2"])
    tw, ids = cu(c["topk_weights"]), cu(c["topk_ids"])
    y = torch.ops.w4a8_b200.moe_decode(cu(c["x"]), w1, s1, z1, w2, s2, z2, tw, ids)
    p13 = torch.ops.w4a8_b200.stream_pack(w1, s1, z1, True)
    p2 = torch.ops.w4a8_b200.stream_pack(w2, s2, z2, False)
    yp = torch.ops.w4a8_b200.moe_decode_packed(cu(c["x"]), p13, p2, E, 512, tw, ids)
    ref = O.moe_layer(c["x"], O.pack_int4(c["c13"]), c["s13"], O.pack_zeros(c["z13"]) if asym else None,
                      O.pack_int4(c["c2"]), c["s2"], O.pack_zeros(c["z2"]) if asym else None,
                      c["topk_ids"], c["topk_weights"])
    assert max_abs_rel(yp.float().cpu().numpy(), ref) <= MAX_ABS_REL
    assert max_abs_rel(y.float().cpu().numpy(), ref) <= MAX_ABS_REL
