"""Generate golden fixtures by running the REFERENCE's own oracle functions on CPU.

The reference (patcarter883/rdna4-vllm) keeps its oracles inside its test modules
(w4a8_fp8_wmma/test_correctness.py, test_moe_correctness.py, test_moe_experts.py) and its
layout converter in w4a8_fp8_wmma/w4a8_fp8_wmma/moe_experts.py. Those modules import the
compiled extension at top level, so a stub package is placed in sys.modules first; nothing of
the reference's device code runs. Inputs come from tests/golden/inputs.py (seeded numpy), so
only outputs are stored. Run from the repo root in a container that has the reference:

    python tests/golden/make_golden.py /path/to/reference

The fixtures (tests/golden/*.npz) are committed; the GPU box never needs the reference.
"""
from __future__ import annotations

import importlib.util
import os
import sys
import types

import numpy as np
import torch

sys.dont_write_bytecode = True
HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, HERE)
import inputs  # noqa: E402


def load_reference(ref_root: str):
    pkg_dir = os.path.join(ref_root, "w4a8_fp8_wmma")
    stub = types.ModuleType("w4a8_fp8_wmma")
    stub.__path__ = [os.path.join(pkg_dir, "w4a8_fp8_wmma")]
    sys.modules["w4a8_fp8_wmma"] = stub
    mods = {}
    for name in ("test_correctness", "test_moe_correctness", "test_moe_experts"):
        spec = importlib.util.spec_from_file_location(name, os.path.join(pkg_dir, name + ".py"))
        m = importlib.util.module_from_spec(spec)
        spec.loader.exec_module(m)
        mods[name] = m
    return mods


def t(a, dtype=None):
    x = torch.from_numpy(np.ascontiguousarray(a))
    return x if dtype is None else x.to(dtype)


def main(ref_root: str) -> None:
    torch.manual_seed(0)
    m = load_reference(ref_root)
    tc, tm, te = m["test_correctness"], m["test_moe_correctness"], m["test_moe_experts"]
    from w4a8_fp8_wmma.moe_experts import _awq_moe_to_op_layout  # reference converter

    # ---- 1. activation quant bytes: capture the reference oracle's own e4m3 round trip ----
    rec = []
    orig = tc.to_e4m3_roundtrip

    def spy(v):
        out = orig(v)
        rec.append(out)
        return out

    act = {}
    for i, (M, K, seed) in enumerate([(16, 2048, 0), (7, 48, 1), (33, 512, 2)]):
        x, codes, scales, zeros = inputs.dense_case(seed, M, 8, K, 16, asym=False)
        x[0] = 0  # all-zero row -> amax floor
        if M > 2:
            x[1] *= np.float16(1e-3)
            x[2] = np.float16(60000.0) * np.sign(x[2]).astype(np.float16)
        rec.clear()
        tc.to_e4m3_roundtrip = spy
        tc.reference_fp8_model(t(x), t(tc_pack(codes)), t(scales), group_size=16)
        tc.to_e4m3_roundtrip = orig
        xq = rec[1].to(torch.float8_e4m3fn).view(torch.uint8).numpy()
        act[f"x{i}"] = x
        act[f"q{i}"] = xq
    np.savez_compressed(os.path.join(HERE, "act_quant.npz"), **act)

    # ---- 2. dense GEMM (reference_fp8_model / _asym) ----
    dense = {}
    cases = [("cfg0", 0, 16, 2048, 2048, 128, True), ("m1_g32_sym", 11, 1, 512, 256, 32, False),
             ("tail_17x48", 12, 17, 48, 256, 32, True), ("tail_100x80", 13, 100, 80, 256, 32, True),
             ("g128_sym", 14, 64, 256, 256, 128, False), ("g64_asym", 15, 8, 128, 512, 64, True)]
    for name, seed, M, N, K, g, asym in cases:
        x, codes, scales, zeros = inputs.dense_case(seed, M, N, K, g, asym)
        wp = tc.pack_uint4_weights(t(codes, torch.int8))
        if asym:
            out = tc.reference_fp8_model_asym(t(x), wp, t(scales), t(zeros, torch.int8), g)
        else:
            out = tc.reference_fp8_model(t(x), wp, t(scales), g)
        dense[name] = out.numpy()
        dense[name + "_meta"] = np.array([seed, M, N, K, g, int(asym)])
    np.savez_compressed(os.path.join(HERE, "dense.npz"), **dense)

    # ---- 3. moe_align order (reference Python moe_align) ----
    align = {}
    for i, (T, E, k, bm, seed) in enumerate([(32, 256, 8, 8, 0), (64, 8, 2, 16, 1),
                                               (1, 8, 2, 16, 2), (4096 // 16, 256, 8, 64, 3)]):
        ids = inputs.random_topk(seed, T, E, k)
        sti, eids, ntp, _ = tm.moe_align(t(ids), bm, E)
        align[f"ids{i}"] = ids
        align[f"sorted{i}"] = sti.numpy()
        align[f"eids{i}"] = eids.numpy()
        align[f"meta{i}"] = np.array([T, E, k, bm, int(ntp.item())])
    # skewed (Zipf-biased routing) case
    rng = np.random.default_rng(4)
    _, ids, _ = inputs.routing(rng, 512, 256, 8, zipf_bias=True)
    sti, eids, ntp, _ = tm.moe_align(t(ids), 64, 256)
    align["ids4"], align["sorted4"], align["eids4"] = ids, sti.numpy(), eids.numpy()
    align["meta4"] = np.array([512, 256, 8, 64, int(ntp.item())])
    np.savez_compressed(os.path.join(HERE, "moe_align.npz"), **align)

    # ---- 4. grouped op (test_moe_correctness.reference) ----
    grouped = {}
    gcases = [("a", 21, 16, 8, 128, 256, 2, 16, 128, True), ("b", 22, 5, 4, 64, 128, 2, 8, 32, False),
              ("c", 23, 32, 16, 256, 512, 4, 16, 128, True)]
    for name, seed, T, E, N, K, k, bm, g, asym in gcases:
        rng = np.random.default_rng(seed)
        x = rng.standard_normal((T, K), dtype=np.float32).astype(np.float16)
        codes, scales, zeros = inputs.expert_weights(rng, E, N, K, g, asym)
        ids = np.stack([rng.permutation(E)[:k] for _ in range(T)]).astype(np.int32)
        sti, eids, ntp, _ = tm.moe_align(t(ids), bm, E)
        out = tm.reference(t(x), t(codes, torch.int8), t(scales),
                           t(zeros, torch.int8) if asym else None, sti, eids, ntp, k, bm, g)
        grouped[name] = out.numpy()
        grouped[name + "_meta"] = np.array([seed, T, E, N, K, k, bm, g, int(asym)])
    np.savez_compressed(os.path.join(HERE, "moe_gemm.npz"), **grouped)

    # ---- 5. whole MoE layer (test_moe_experts.fp8_ref_moe) ----
    layer = {}
    for name, seed, T, E, H, I, k, g in [("small", 31, 4, 8, 256, 128, 2, 128),
                                         ("decode", 32, 3, 16, 512, 256, 4, 128)]:
        c = inputs.moe_layer_case(seed, T, E, H, I, k, g)
        # fp8_ref_moe takes (E, K_in, N_out) nibbles and (E, G, N) scales / zeros.
        y = te.fp8_ref_moe(t(c["x"]), t(np.swapaxes(c["c13"], 1, 2).astype(np.int32)),
                           t(np.swapaxes(c["s13"], 1, 2)), t(np.swapaxes(c["z13"], 1, 2).astype(np.int32)),
                           t(np.swapaxes(c["c2"], 1, 2).astype(np.int32)), t(np.swapaxes(c["s2"], 1, 2)),
                           t(np.swapaxes(c["z2"], 1, 2).astype(np.int32)), t(c["topk_ids"]),
                           t(c["topk_weights"]), g)
        layer[name] = y.numpy()
        layer[name + "_meta"] = np.array([seed, T, E, H, I, k, g])
    np.savez_compressed(os.path.join(HERE, "moe_layer.npz"), **layer)

    # ---- 6. AWQ -> op layout conversion and SiLU-and-mul ----
    conv = {}
    rng = np.random.default_rng(41)
    E, K, N, g = 2, 256, 64, 32
    q = rng.integers(0, 16, (E, K, N)).astype(np.int32)
    z = rng.integers(0, 16, (E, K // g, N)).astype(np.int32)
    s = rng.uniform(1e-3, 2e-2, (E, K // g, N)).astype(np.float16)
    qw = te.awq_pack(t(q))
    qz = te.awq_pack_zeros(t(z))
    w_op, s_op, z_op = _awq_moe_to_op_layout(qw, t(s), qz, g)
    conv.update(awq_qweight=qw.numpy(), awq_qzeros=qz.numpy(), awq_scales=s,
                op_w=w_op.numpy(), op_s=s_op.numpy(), op_z=z_op.numpy())
    o1 = (rng.standard_normal((24, 64), dtype=np.float32) * 4).astype(np.float16)
    conv["silu_in"] = o1
    conv["silu_out"] = te.silu_and_mul_ref(t(o1)).numpy()
    np.savez_compressed(os.path.join(HERE, "convert.npz"), **conv)
    formats(ref_root)
    print("fixtures written to", HERE)


def formats(ref_root: str) -> None:
    """compressed-tensors GPTQ, MoeWNA16 and mxfp4 checkpoints -> op layout, through the
    reference's own converters (moe_experts.py:437 _ct_moe_to_op_layout, :473
    _wna16_moe_to_op_layout; mxfp4/convert.py convert_mxfp4_moe / convert_mxfp4_weight), plus
    the reference's mxfp4 dense oracle (mxfp4/test_mxfp4_kernel_gpu.py:64-71) run on CPU."""
    if "w4a8_fp8_wmma" not in sys.modules:
        load_reference(ref_root)
    from w4a8_fp8_wmma.moe_experts import _ct_moe_to_op_layout, _wna16_moe_to_op_layout
    spec = importlib.util.spec_from_file_location(
        "ref_mxfp4_convert", os.path.join(ref_root, "w4a8_fp8_wmma", "mxfp4", "convert.py"))
    mx = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mx)
    out = {}
    rng = np.random.default_rng(51)
    # compressed-tensors: (E, K/8, N) int32 natural nibble order along K, scales (E, K/g, N)
    E, K, N, g = 3, 256, 64, 32
    ct_q = rng.integers(-2 ** 31, 2 ** 31 - 1, (E, K // 8, N), dtype=np.int64).astype(np.int32)
    ct_s = rng.uniform(1e-3, 2e-2, (E, K // g, N)).astype(np.float16)
    w, s = _ct_moe_to_op_layout(t(ct_q), t(ct_s))
    out.update(ct_qweight=ct_q, ct_scales=ct_s, ct_op_w=w.numpy(), ct_op_s=s.numpy())
    # MoeWNA16: qweight (E, N, K/2) u8, scales (E, N, K/g), qzeros (E, N/2, K/g) u8
    wq = rng.integers(0, 256, (E, N, K // 2), dtype=np.int64).astype(np.uint8)
    ws = rng.uniform(1e-3, 2e-2, (E, N, K // g)).astype(np.float16)
    wz = rng.integers(0, 256, (E, N // 2, K // g), dtype=np.int64).astype(np.uint8)
    w, s, z = _wna16_moe_to_op_layout(t(wq), t(ws), t(wz))
    out.update(wna16_qweight=wq, wna16_scales=ws, wna16_qzeros=wz, wna16_op_w=w.numpy(),
               wna16_op_s=s.numpy(), wna16_op_z=z.numpy())
    # mxfp4: weight_packed (E, N, K/2) u8 E2M1 pairs, weight_scale (E, N, K/32) u8 E8M0
    mp = rng.integers(0, 256, (E, N, K // 2), dtype=np.int64).astype(np.uint8)
    ms = rng.integers(124, 131, (E, N, K // 32), dtype=np.int64).astype(np.uint8)
    conv = mx.convert_mxfp4_moe(t(mp), t(ms))
    out.update(mx_packed=mp, mx_scale=ms, mx_op_w=conv["w_packed"].numpy(),
               mx_op_s=conv["scales"].numpy())
    # the reference's mxfp4 dense oracle on one expert (reciprocal-multiply act quant)
    x = (rng.standard_normal((16, K), dtype=np.float32) * 0.5).astype(np.float16)
    c1 = mx.convert_mxfp4_weight(t(mp[0]), t(ms[0]))
    spec2 = importlib.util.spec_from_file_location(
        "ref_mxfp4_gpu_test",
        os.path.join(ref_root, "w4a8_fp8_wmma", "mxfp4", "test_mxfp4_kernel_gpu.py"))
    src = open(spec2.origin).read()
    fn_src = src[src.index("def fp8_dense_ref"):src.index("def run_oracle")]
    ns = {"torch": torch, "unpack_e2m1_nibbles": mx.unpack_e2m1_nibbles,
          "FP4_E2M1_LUT": mx.FP4_E2M1_LUT, "OCP_MX_BLOCK_SIZE": mx.OCP_MX_BLOCK_SIZE}
    exec(compile(fn_src, spec2.origin, "exec"), ns)  # the function alone (the module needs a GPU)
    ref = ns["fp8_dense_ref"](t(x), t(mp[0]), t(ms[0]), c1)
    out.update(mx_x=x, mx_dense_ref=ref.numpy())
    np.savez_compressed(os.path.join(HERE, "formats.npz"), **out)


def tc_pack(codes):
    """Pack like test_correctness.pack_uint4_weights (used only for the act-quant capture)."""
    c = codes.astype(np.int64)
    out = np.zeros((c.shape[0], c.shape[1] // 8), np.int64)
    for i in range(8):
        out |= (c[:, i::8] & 0xF) << (i * 4)
    return out.astype(np.uint32).view(np.int32)


if __name__ == "__main__":
    if len(sys.argv) < 2:
        sys.exit("usage: python tests/golden/make_golden.py <path to the reference checkout>")
    if len(sys.argv) > 2 and sys.argv[2] == "--formats-only":
        torch.manual_seed(0)
        formats(sys.argv[1])
    else:
        main(sys.argv[1])
