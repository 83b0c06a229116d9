"""bench.py — MoE-layer throughput of the B200 W4A8 library (driver contract).

Workload (the metric's config): one Qwen3.6-35B-A3B-shaped MoE layer at
decode — 32 tokens, hidden 2048, 256 routed experts (top-8 softmax routing from N(0,1)
router logits, renormalised) plus 1 shared expert, gate_up K=2048 -> 2x512, SiLU-and-mul,
down K=512 -> 2048, AWQ int4 g128 weights (codes U{0..15}, scales U[1e-3,2e-2], zeros
U{0..15}), fp16 activations N(0,1). The shared expert rides the same grouped kernels as
expert 256 with routing weight 1.0 on every token. `--workload prefill` runs configs[2]
(4096 tokens, Zipf-biased routing).

A step = one full layer forward (moe_align -> gate_up+SiLU -> down -> topk-weighted reduce)
replayed from a CUDA graph with the inputs resident in HBM. Routing (softmax/top-k) is
computed once outside the timed region. The touched expert weights (~270 MB at decode,
~420 MB at prefill) exceed the 126 MB L2, so no explicit flush is needed.

With --gpus N (torchrun, one rank per GPU) the layer runs expert-parallel: rank r owns experts
[r*256/N, (r+1)*256/N) and its own 32 (decode) tokens; tokens reach the owners through NCCL
all-to-all dispatch and come back through an all-to-all combine ("scaling": "weak").

`--impl reference` times the reference's CPU implementation of the path (the numpy
restatement of its torch oracle in oracle/w4a8_oracle.py) on the host cores.
"""
from __future__ import annotations

import argparse
import json
import os
import subprocess
import sys
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.join(ROOT, "rdna4-vllm_b200"))
sys.path.insert(0, os.path.join(ROOT, "tests", "golden"))

H, INTER, E_ROUTED, TOP_K, GROUP = 2048, 512, 256, 8, 128
EXPERT_BYTES = (2 * INTER * H // 2 + 2 * INTER * (H // GROUP) * 2 + (2 * INTER // 8) * (H // GROUP) * 4
                + H * INTER // 2 + H * (INTER // GROUP) * 2 + (H // 8) * (INTER // GROUP) * 4)
W13_BYTES = 2 * INTER * H // 2 + 2 * INTER * (H // GROUP) * 2 + (2 * INTER // 8) * (H // GROUP) * 4


def peaks():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        d = json.load(open(p))
        return d["hbm_gbs"], 2 * d["bf16_tflops"], "measured"
    return 6650.0, 2 * 1590.0, "fallback"


def workload_config(name: str):
    if name == "prefill":
        return dict(T=4096, zipf=True, seed=2)
    return dict(T=32, zipf=False, seed=1)


def metric_name(workload: str) -> str:
    return ("MoE-layer tokens/s (Qwen3.6-35B-A3B-shaped, decode T=32)" if workload == "decode"
            else "MoE-layer tokens/s (Qwen3.6-35B-A3B-shaped, prefill T=4096)")


def base_config(workload: str, world: int, layers: int = 1) -> dict:
    """The workload description both arms print (the driver compares the two dicts)."""
    cfg = workload_config(workload)
    return {"workload": f"configs[{1 if workload == 'decode' else 2}] MoE layer {workload}",
            "tokens_per_gpu": cfg["T"], "hidden": H, "inter": INTER, "experts": E_ROUTED,
            "shared_experts": 1, "top_k": TOP_K, "group": GROUP, "layers": layers,
            "routing": "softmax top-8 renormalised" + (" + Zipf(1.1) expert bias"
                                                       if cfg["zipf"] else ""),
            "parallelism": f"ep{world}" if world > 1 else "single",
            "l2": ("touched weights > 126 MB L2 (no flush)" if world == 1 else
                   "per-rank weights ~53-105 MB; inputs re-read each step")}


def host_info() -> dict:
    model = None
    try:
        for line in open("/proc/cpuinfo"):
            if line.startswith("model name"):
                model = line.split(":", 1)[1].strip()
                break
    except OSError:
        pass
    try:
        import torch
        tv = torch.__version__
    except Exception:  # noqa: BLE001
        tv = None
    return {"cpu_model": model, "host_threads": os.cpu_count(), "torch": tv,
            "numpy": np.__version__}


# ------------------------------------------------------------------------------------------
# clocks sampling (nvidia-smi during the timed region)
# ------------------------------------------------------------------------------------------
class ClockSampler:
    Q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
         "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
         "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int):
        self.gpu = gpu_index
        self.proc = None
        self.path = os.path.join("/tmp", f"w4a8_clocks_{os.getpid()}.csv")

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.gpu}", f"--query-gpu={self.Q}", "--format=csv,noheader,nounits",
                 "-lms", "100"], stdout=open(self.path, "w"), stderr=subprocess.DEVNULL)
        except (FileNotFoundError, OSError):
            self.proc = None
        time.sleep(0.3)
        return self

    def __exit__(self, *a):
        if self.proc is not None:
            self.proc.terminate()
            self.proc.wait(timeout=5)

    def summary(self):
        if self.proc is None or not os.path.exists(self.path):
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        sm, smax, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for line in open(self.path):
            f = [v.strip() for v in line.split(",")]
            if len(f) < 9:
                continue
            try:
                sm.append(float(f[1]))
                smax = float(f[2])
            except ValueError:
                continue
            for n, v in zip(names, f[5:9]):
                if v.lower() == "active":
                    reasons.add(n)
        return {"sm_mhz": float(np.median(sm)) if sm else None, "sm_max_mhz": smax,
                "reasons": sorted(reasons), "samples": len(sm)}


# ------------------------------------------------------------------------------------------
# synthetic layer
# ------------------------------------------------------------------------------------------
def make_layer(torch, dev, seed: int, E: int):
    """Per-expert AWQ-style weights generated on the device (uniform nibbles == uniform words)."""
    g = torch.Generator(device=dev)
    g.manual_seed(seed)
    def words(*shape):
        return torch.randint(-2 ** 31, 2 ** 31 - 1, shape, dtype=torch.int32, device=dev, generator=g)
    def scales(*shape):
        return (torch.rand(shape, device=dev, generator=g) * (2e-2 - 1e-3) + 1e-3).to(torch.float16)
    w13 = words(E, 2 * INTER, H // 8)
    s13 = scales(E, 2 * INTER, H // GROUP)
    z13 = words(E, 2 * INTER // 8, H // GROUP)
    w2 = words(E, H, INTER // 8)
    s2 = scales(E, H, INTER // GROUP)
    z2 = words(E, H // 8, INTER // GROUP)
    return w13, s13, z13, w2, s2, z2


def make_tokens(T: int, zipf: bool, seed: int):
    """Host-side seeded tokens and routing; the shared expert is slot TOP_K (id 256, w 1.0)."""
    import inputs as I
    rng = np.random.default_rng(seed)
    x = rng.standard_normal((T, H), dtype=np.float32).astype(np.float16)
    _, ids, w = I.routing(rng, T, E_ROUTED, TOP_K, zipf_bias=zipf)
    ids = np.concatenate([ids, np.full((T, 1), E_ROUTED, np.int32)], axis=1)
    w = np.concatenate([w, np.ones((T, 1), np.float32)], axis=1)
    return x, ids.astype(np.int32), w.astype(np.float32)


# ------------------------------------------------------------------------------------------
# the B200 arm
# ------------------------------------------------------------------------------------------
def run_ours(args):
    import torch
    import torch.distributed as dist
    import w4a8_fp8_wmma as w4  # noqa: F401  (loads the native libraries)
    from w4a8_fp8_wmma.moe_experts import run_grouped_moe

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        import datetime
        # a collective that one rank never joins ends the run in two minutes, not NCCL's ten
        dist.init_process_group("nccl", device_id=dev, timeout=datetime.timedelta(seconds=120))
    cfg = workload_config(args.workload)
    T = cfg["T"]
    E_total = E_ROUTED + 1
    x_np, ids_np, w_np = make_tokens(T, cfg["zipf"], cfg["seed"] * 1000 + rank)
    x = torch.from_numpy(x_np).to(dev)
    ids = torch.from_numpy(ids_np).to(dev)
    tw = torch.from_numpy(w_np).to(dev)
    holder = {}
    if world > 1:
        from w4a8_fp8_wmma.ep import ExpertParallelMoE
        E_loc = E_ROUTED // world
        wts = make_layer(torch, dev, 1000 + rank, E_loc)
        shared = make_layer(torch, dev, 999, 1)
        w13, s13, z13, w2, s2, z2 = wts
        layer = ExpertParallelMoE(w13, s13, z13, w2, s2, z2, E_ROUTED, TOP_K, shared=shared)
        ids_r = ids[:, :TOP_K].contiguous()
        tw_r = tw[:, :TOP_K].contiguous()
        recorded = {}

        def step_fn():
            holder["y"] = layer(x, ids_r, tw_r)
            recorded["rows"] = layer.last_recv
    else:
        layer = None
        w13, s13, z13, w2, s2, z2 = make_layer(torch, dev, 1000, E_total)

        def step_fn():
            holder["y"] = run_grouped_moe(x, w13, w2, s13, s2, z13, z2, tw, ids,
                                          global_num_experts=E_total, out_dtype=torch.float16)

    # One CUDA graph per step (NCCL collectives included); eager replay if capture fails.
    stream = torch.cuda.Stream()
    stream.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(stream):
        for _ in range(2):
            step_fn()
    torch.cuda.current_stream().wait_stream(stream)
    torch.cuda.synchronize()
    graph = None
    try:
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, stream=stream):
            step_fn()
        graph = g
    except Exception as exc:  # noqa: BLE001
        print(f"[bench] graph capture failed ({type(exc).__name__}: {exc}); timing eager steps",
              file=sys.stderr)
        torch.cuda.synchronize()
    run = graph.replay if graph is not None else step_fn
    for _ in range(args.warmup):
        run()
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    replay_stream = torch.cuda.current_stream()  # graph.replay() launches here
    with ClockSampler(local) as clk:
        torch.cuda.synchronize()
        start.record(replay_stream)
        for _ in range(args.steps):
            run()
        end.record(replay_stream)
        torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    ms = _max_over_ranks(torch, dist, world, dev, start.elapsed_time(end) / args.steps)
    tokens_per_s = T * world / (ms / 1e3)

    # HBM bytes of the layer on this rank (max over ranks for the report).
    if world > 1:
        rec_ids = payload_ids(torch, recorded["rows"])
        touched = int(torch.unique(rec_ids[rec_ids >= 0]).numel())  # routed + shared (local)
    else:
        touched = len(np.unique(ids_np))
    touched_bytes = touched * EXPERT_BYTES
    hbm, fp8_peak, src = peaks()
    layer_bytes = touched_bytes + T * H * 2 * 2 + T * (TOP_K + 1) * 8
    flops = 2.0 * T * (TOP_K + 1) * (H * 2 * INTER + INTER * H)
    dom = dominant_kernel(torch, args, world, dist, dev, x, ids, w13, s13, z13, E_total, T,
                          recorded if world > 1 else tw, layer if world > 1 else (w2, s2, z2))
    e2e = end_to_end(torch, dist, args, world, dev, x_np, ids_np, w_np, layer, run_grouped_moe,
                     (w13, s13, z13, w2, s2, z2), E_total)
    # every rank takes part in the EP report's collectives before the others leave
    ep = ep_report(torch, dist, world, rank, dev, layer, x, ids, tw, wts, shared) if world > 1 else None
    if rank != 0:
        _leave(dist, world)
    # config is the workload description both arms print, identical between them
    config = base_config(args.workload, world)
    layer_info = {
        "rank0_hbm_bytes_per_step": layer_bytes,
        "layer_hbm_gbs": round(layer_bytes / (ms / 1e3) / 1e9, 1),
        "layer_hbm_frac_of_measured": round(layer_bytes / (ms / 1e3) / 1e9 / hbm, 4),
        "layer_tflops": round(flops / (ms / 1e3) / 1e12, 2),
        "graph": "one CUDA graph per step" if graph is not None else "eager steps"}
    res = {
        "metric": metric_name(args.workload),
        "value": round(tokens_per_s, 1), "unit": "tokens/s", "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": round(ms, 5), "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "e4m3 x int4 -> fp32 (fp16 io)",
        "data": "synthetic (seeded; random-init weights of the layer's shapes)",
        "config": config,
        "layer": layer_info,
        "roofline": dom,
        "clocks": clk.summary(),
        "e2e": e2e,
        "gpu_launches": args.steps * launches_per_step(args.workload, world),
    }
    if ep is not None:
        res["ep"] = ep
    if world == 1 and args.workload == "decode" and not args.no_extras:
        res["prefill"] = prefill_record(torch, dev, (w13, s13, z13, w2, s2, z2), E_total, args)
        res["dense"] = dense_record(torch, dev, args)
    if world == 1 and not args.no_cpu_baseline:
        res["cpu_baseline"] = cpu_baseline(args.workload, budget_s=args.cpu_seconds)
    print(json.dumps(res), flush=True)
    if world > 1:
        _leave(dist, world)


def _leave(dist, world):
    """End an EP rank: a last barrier, then exit without the NCCL teardown (which has been
    seen to block after a failed graph capture)."""
    dist.barrier()
    sys.stdout.flush()
    sys.stderr.flush()
    os._exit(0)


def _max_over_ranks(torch, dist, world, dev, v):
    t = torch.tensor([float(v)], device=dev)
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def launches_per_step(workload: str, world: int) -> int:
    """Kernels of this library per step: decode = decode_prep, gate_up GEMV, down GEMV (3);
    prefill = align count + place, then per GEMM tc_quant_rows + w4_tc_kernel (2 x 2), inverse
    map + gather-reduce (8). EP: ep_pack, the three decode-layer kernels on the payload rows,
    ep_gather (5)."""
    if world > 1:
        return 5
    return 3 if workload == "decode" else 8


def _event_time(torch, fn, reps=20):
    for _ in range(3):
        fn()
    torch.cuda.synchronize()
    st = torch.cuda.current_stream()
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a.record(st)
    for _ in range(reps):
        fn()
    b.record(st)
    torch.cuda.synchronize()
    return a.elapsed_time(b) / reps


def _graph_rotation_time(torch, fn, n, reps=5):
    """Device time per call of fn: n calls (one rotation over the weight copies) captured in one
    CUDA graph and replayed, so host launch overhead is not in the number; eager calls if the
    capture fails. Returns (ms per call, "graph" | "eager")."""
    stream = torch.cuda.Stream()
    stream.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(stream):
        for _ in range(n):
            fn()
    torch.cuda.current_stream().wait_stream(stream)
    torch.cuda.synchronize()
    try:
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, stream=stream):
            for _ in range(n):
                fn()
    except Exception:  # noqa: BLE001
        torch.cuda.synchronize()
        return _event_time(torch, fn, reps=max(n, 20)), "eager"
    g.replay()
    torch.cuda.synchronize()
    st = torch.cuda.current_stream()
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a.record(st)
    for _ in range(reps):
        g.replay()
    b.record(st)
    torch.cuda.synchronize()
    return a.elapsed_time(b) / (reps * n), "graph"


def payload_ids(torch, rows):
    """Local expert ids (R, top_k) held in expert-parallel payload rows (w4a8_ep_pack layout)."""
    o = H + 4 * (H // GROUP) + 4
    return rows[:, o:o + 4 * TOP_K].contiguous().view(torch.int32)


def dominant_kernel(torch, args, world, dist, dev, x, ids, w13, s13, z13, E_total, T, recorded,
                    layer):
    """The step's dominant op on this rank, timed alone with CUDA events on the launching stream.

    decode: the whole decode layer op (routing sort + token quant, gate_up GEMV with SiLU, down
    GEMV with the slot-order reduce: three launches) on the prepacked weights, HBM-bound;
    algorithmic bytes = touched experts x 1,634,304 B (codes + scales + zeros of w13 and w2)
    + the fp16 activations read and written. At N > 1 the op is ep_moe_rows on this rank's
    received rows plus its shared-expert rows.
    prefill: the tcgen05 tile op (tc_quant_rows_kernel, which quantises into sorted order, +
    w4_tc_kernel with the fused SiLU epilogue), tensor-bound; algorithmic FLOPs = 2 * routed rows * 2*inter * hidden
    (padding rows not counted); peak = the dense e4m3 rate, twice the measured bf16 GEMM rate."""
    hbm, fp8_peak, src = peaks()
    import w4a8_fp8_wmma as w4
    prefill = args.workload == "prefill" and world == 1
    if prefill:
        s, e, n = w4.moe_align_block_size(ids, 128, E_total)

        def launch():
            return torch.ops.w4a8_b200.moe_gemm1_silu(x, w13, s13, z13, s, e, n, ids.size(1),
                                                      128, 6, False)
        ms = _max_over_ranks(torch, dist, world, dev, _event_time(torch, launch))
        rows = int(ids.numel())
        flops = 2.0 * rows * 2 * INTER * H
        ach = flops / (ms / 1e3) / 1e12
        return {"kernel": "gate_up tile op: tc_quant_rows_kernel + w4_tc_kernel (SiLU epilogue)",
                "bound": "tensor", "achieved": round(ach, 1), "peak": round(fp8_peak, 1),
                "unit": "TFLOP/s", "frac": round(ach / fp8_peak, 4),
                "peak_source": f"{src} (e4m3 dense = 2 x measured bf16)",
                "algorithmic_flops_per_launch": flops, "avg_launch_us": round(ms * 1e3, 2),
                "traffic": TC_KERNEL_TRAFFIC,
                "traffic_source": "profiles/w4_tc_kernel_prefill.md (dram read+write of the "
                                  "w4_tc_kernel launch, one ncu capture)"}
    if world > 1:
        rows = recorded["rows"]
        R = rows.size(0)
        pk = layer.pack

        def launch():
            return torch.ops.w4a8_b200.ep_moe_rows(rows, pk.p13, pk.p2, pk.E, H, INTER, TOP_K)
        rid = payload_ids(torch, rows)
        touched = int(torch.unique(rid[rid >= 0]).numel())
        act = R * H + R * H * 4
        kern = "ep_moe_rows: decode_prep + gate_up GEMV + down GEMV (payload rows)"
    else:
        from w4a8_fp8_wmma.moe_experts import decode_pack_for
        w2, s2, z2 = layer
        pk = decode_pack_for(w13, w2, s13, s2, z13, z2)

        def launch():
            return pk(x, recorded, ids)
        touched = int(torch.unique(ids).numel())
        act = 2 * T * H * 2
        kern = "moe_decode_packed: decode_prep + gate_up GEMV + down GEMV"
    ms = _max_over_ranks(torch, dist, world, dev, _event_time(torch, launch))
    bytes_ = touched * EXPERT_BYTES + act
    ach = bytes_ / (ms / 1e3) / 1e9
    return {"kernel": kern, "bound": "hbm", "achieved": round(ach, 1), "peak": hbm,
            "unit": "GB/s", "frac": round(ach / hbm, 4), "peak_source": src,
            "algorithmic_bytes_per_launch": bytes_, "avg_launch_us": round(ms * 1e3, 2),
            "traffic": DECODE_TRAFFIC if world == 1 else None,
            "traffic_source": DECODE_TRAFFIC_SRC if world == 1 else None}


def run_stack(args):
    """a 40-layer MoE stack, expert parallel over the ranks of this node (256
    experts split evenly, the shared expert replicated), independently seeded weights per layer.
    Decode: 256 tokens in total (256/N per rank) through all layers, one CUDA graph per step.
    Prefill: a separate 16384-token batch (16384/N per rank), eager (its exchange sizes rows on
    the host). Each layer is applied to the step's input (the stack's work and traffic per layer
    without a residual stream). Rank 0 prints one JSON line; time is the max over ranks.
    Prefill parity: layer 0 on each rank's tokens against the single-GPU composition with the
    all-gathered weights (max-abs-rel, max over ranks)."""
    import datetime
    import torch
    import torch.distributed as dist
    import w4a8_fp8_wmma as w4  # noqa: F401
    from w4a8_fp8_wmma.ep import ExpertParallelMoE
    from w4a8_fp8_wmma.moe_experts import run_grouped_moe
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    os.environ.setdefault("MASTER_ADDR", "127.0.0.1")
    os.environ.setdefault("MASTER_PORT", "29533")
    os.environ.setdefault("RANK", "0")
    os.environ.setdefault("WORLD_SIZE", "1")
    dist.init_process_group("nccl", device_id=dev, timeout=datetime.timedelta(seconds=120))
    L = args.layers
    E_loc = E_ROUTED // world
    layers = []
    for l in range(L):
        w13, s13, z13, w2, s2, z2 = make_layer(torch, dev, 100000 + 1000 * l + rank, E_loc)
        shared = make_layer(torch, dev, 900000 + l, 1)
        layers.append(ExpertParallelMoE(w13, s13, z13, w2, s2, z2, E_ROUTED, TOP_K,
                                        shared=shared))

    def tokens(T, zipf, seed):
        x_np, ids_np, w_np = make_tokens(T, zipf, seed)
        return (torch.from_numpy(x_np).to(dev), torch.from_numpy(ids_np[:, :TOP_K].copy()).to(dev),
                torch.from_numpy(w_np[:, :TOP_K].copy()).to(dev))

    Td, Tp = 256 // world, 16384 // world
    xd, idd, twd = tokens(Td, False, 7000 + rank)
    xp, idp, twp = tokens(Tp, True, 8000 + rank)
    hold = {}

    def dec_step():
        for lay in layers:
            hold["d"] = lay(xd, idd, twd)

    def pre_step():
        for lay in layers:
            hold["p"] = lay(xp, idp, twp)

    dist.barrier()
    from w4a8_fp8_wmma.moe_experts import GEMV_MAX_M
    if Td <= GEMV_MAX_M:
        ms_d, graphed = _graph_time(torch, dec_step, args.steps, args.warmup)
    else:  # above the decode split the exchange sizes rows on the host: eager steps
        ms_d, graphed = _event_time(torch, dec_step, reps=args.steps), False
    ms_d = _max_over_ranks(torch, dist, world, dev, ms_d)
    dist.barrier()
    ms_p = _max_over_ranks(torch, dist, world, dev,
                           _event_time(torch, pre_step, reps=max(1, min(args.steps, 3))))
    # prefill parity, layer 0
    lay = layers[0]
    y = lay(xp, idp, twp)
    full = []
    for t_loc, t_sh in zip(lay.weights, lay.shared):
        parts = [torch.empty_like(t_loc) for _ in range(world)]
        dist.all_gather(parts, t_loc.contiguous())
        full.append(torch.cat(parts + [t_sh], 0).contiguous())
    w13, s13, z13, w2, s2, z2 = full
    ids_all = torch.cat([idp, torch.full((Tp, 1), E_ROUTED, dtype=idp.dtype, device=dev)], 1)
    tw_all = torch.cat([twp, torch.ones((Tp, 1), dtype=twp.dtype, device=dev)], 1)
    ref = run_grouped_moe(xp, w13, w2, s13, s2, z13, z2, tw_all, ids_all,
                          global_num_experts=E_ROUTED + 1, out_dtype=torch.float32)
    err = float((y.float() - ref).abs().max() / ref.abs().max().clamp_min(1e-30))
    err = _max_over_ranks(torch, dist, world, dev, err)
    del full, ref
    if rank == 0:
        res = {"metric": "40-layer MoE stack tokens/s (configs[4], expert parallel)",
               "value": round(256 / (ms_d / 1e3), 1), "unit": "tokens/s", "n_gpus": world,
               "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms_d, 4),
               "higher_is_better": True, "scaling": "strong",
               "dtype": "e4m3 x int4 -> fp32 (fp16 io)",
               "data": "synthetic (seeded; independently seeded random-init weights per layer)",
               "config": {"workload": "configs[4] 40-layer MoE stack, decode 256 tokens",
                          "layers": L, "tokens_total": 256, "tokens_per_gpu": Td,
                          "experts": E_ROUTED, "experts_per_gpu": E_loc, "shared_experts": 1,
                          "top_k": TOP_K, "hidden": H, "inter": INTER,
                          "parallelism": f"ep{world}",
                          "graph": "one CUDA graph per step" if graphed else "eager steps",
                          "layer_input": "each layer applied to the step's input"},
               "prefill": {"tokens_total": 16384, "tokens_per_gpu": Tp, "routing": "Zipf(1.1)",
                           "ms_per_step": round(ms_p, 3),
                           "tokens_per_s": round(16384 / (ms_p / 1e3), 1), "timing": "eager",
                           "parity_layer0": {"max_abs_rel": err, "pass": err <= 1e-2,
                                             "vs": "single-GPU run_grouped_moe with the "
                                                   "all-gathered weights"}}}
        print(json.dumps(res), flush=True)
    _leave(dist, world)


def _graph_time(torch, fn, steps, warmup):
    """Capture fn in a CUDA graph (eager if capture fails) and time `steps` replays."""
    stream = torch.cuda.Stream()
    stream.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(stream):
        for _ in range(2):
            fn()
    torch.cuda.current_stream().wait_stream(stream)
    torch.cuda.synchronize()
    run = fn
    try:
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, stream=stream):
            fn()
        run = g.replay
    except Exception:  # noqa: BLE001
        torch.cuda.synchronize()
    for _ in range(warmup):
        run()
    torch.cuda.synchronize()
    st = torch.cuda.current_stream()
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a.record(st)
    for _ in range(steps):
        run()
    b.record(st)
    torch.cuda.synchronize()
    return a.elapsed_time(b) / steps, run is not fn


def prefill_record(torch, dev, wts, E_total, args):
    """configs[2] on the same layer weights: the whole prefill layer (graph replay) and its
    dominant op (gate_up tile op, tensor-bound), with the clocks seen while it ran."""
    from w4a8_fp8_wmma.moe_experts import run_grouped_moe
    import w4a8_fp8_wmma as w4
    cfg = workload_config("prefill")
    T = cfg["T"]
    x_np, ids_np, w_np = make_tokens(T, True, cfg["seed"] * 1000)
    x = torch.from_numpy(x_np).to(dev)
    ids = torch.from_numpy(ids_np).to(dev)
    tw = torch.from_numpy(w_np).to(dev)
    w13, s13, z13, w2, s2, z2 = wts
    hbm, fp8_peak, src = peaks()

    def step():
        run_grouped_moe(x, w13, w2, s13, s2, z13, z2, tw, ids, global_num_experts=E_total,
                        out_dtype=torch.float16)
    with ClockSampler(dev.index or 0) as clk:
        ms, graphed = _graph_time(torch, step, max(5, args.steps // 4), args.warmup)
        s_, e_, n_ = w4.moe_align_block_size(ids, 128, E_total)

        def op1():
            torch.ops.w4a8_b200.moe_gemm1_silu(x, w13, s13, z13, s_, e_, n_, ids.size(1), 128,
                                               6, False)
        ms1 = _event_time(torch, op1)
        ident = torch.arange(s_.numel(), dtype=torch.int32, device=dev)
        buf2 = torch.randn((s_.numel(), INTER), device=dev).half()

        def op2():
            torch.ops.w4a8_fp8_wmma.mmq_fp8_moe_gemm(buf2, w2, s2, z2, ident, e_, n_, 1, 128,
                                                     6, False)
        ms2 = _event_time(torch, op2)
    rows = int(ids.numel())
    f1 = 2.0 * rows * 2 * INTER * H
    f2 = 2.0 * rows * INTER * H
    layer_flops = f1 + f2
    return {
        "workload": "configs[2] MoE layer prefill (T=4096, Zipf-biased top-8 + shared)",
        "tokens_per_s": round(T / (ms / 1e3), 1), "ms_per_step": round(ms, 4),
        "graph": graphed,
        "layer_tflops": round(layer_flops / (ms / 1e3) / 1e12, 1),
        "layer_frac_of_e4m3_peak": round(layer_flops / (ms / 1e3) / 1e12 / fp8_peak, 4),
        "roofline": {"kernel": "gate_up tile op (tc_quant_rows_kernel + w4_tc_kernel, SiLU "
                               "epilogue)", "bound": "tensor",
                     "achieved": round(f1 / (ms1 / 1e3) / 1e12, 1), "peak": round(fp8_peak, 1),
                     "unit": "TFLOP/s", "frac": round(f1 / (ms1 / 1e3) / 1e12 / fp8_peak, 4),
                     "peak_source": f"{src} (e4m3 dense = 2 x measured bf16)",
                     "algorithmic_flops_per_launch": f1, "avg_launch_us": round(ms1 * 1e3, 2),
                     "traffic": TC_KERNEL_TRAFFIC},
        "down_op": {"kernel": "down tile op (tc_quant_rows_kernel + w4_tc_kernel)",
                    "avg_launch_us": round(ms2 * 1e3, 2),
                    "tflops": round(f2 / (ms2 / 1e3) / 1e12, 1),
                    "frac": round(f2 / (ms2 / 1e3) / 1e12 / fp8_peak, 4)},
        "clocks": clk.summary(),
    }


DENSE_SHAPES = [(2048, 4096), (4096, 2048), (2048, 512), (2048, 8192)]


def dense_record(torch, dev, args, Ms=(1, 16, 2048)):
    """configs[3] dense W4A8 GEMM cells on one GPU: each cell rotates over enough weight copies
    (>= 256 MB) that every launch reads its weights from HBM, not L2."""
    import w4a8_fp8_wmma as w4
    hbm, fp8_peak, src = peaks()
    g = torch.Generator(device=dev)
    g.manual_seed(31)
    cells = []
    for K, N in DENSE_SHAPES:
        wbytes = N * K // 2 + N * (K // GROUP) * 2 + (N // 8) * (K // GROUP) * 4
        copies = max(2, -(-256 * 2 ** 20 // wbytes))
        ws = [(torch.randint(-2 ** 31, 2 ** 31 - 1, (N, K // 8), dtype=torch.int32, device=dev,
                             generator=g),
               (torch.rand((N, K // GROUP), device=dev, generator=g) * 0.019 + 1e-3).half(),
               torch.randint(-2 ** 31, 2 ** 31 - 1, (N // 8, K // GROUP), dtype=torch.int32,
                             device=dev, generator=g)) for _ in range(copies)]
        for M in Ms:
            x = torch.randn((M, K), device=dev, generator=g).half()
            kern = 11 if M <= 16 else 10
            it = [0]

            def launch():
                w, s, z = ws[it[0] % copies]
                it[0] += 1
                torch.ops.w4a8_fp8_wmma.mmq_fp8_gemm(x, w, s, z, kern, False)
            ms, how = _graph_rotation_time(torch, launch, copies)
            byt = wbytes + M * K * 2 + M * N * 2
            fl = 2.0 * M * N * K
            cell = {"M": M, "K": K, "N": N, "us": round(ms * 1e3, 2),
                    "kernel": "decode_gemv (stream)" if kern == 11 else "tile (tcgen05)",
                    "hbm_gbs": round(byt / (ms / 1e3) / 1e9, 1),
                    "tflops": round(fl / (ms / 1e3) / 1e12, 2), "timing": how}
            if M <= 16:
                cell.update(bound="hbm", frac=round(byt / (ms / 1e3) / 1e9 / hbm, 4))
            else:
                cell.update(bound="tensor", frac=round(fl / (ms / 1e3) / 1e12 / fp8_peak, 4))
            cells.append(cell)
        del ws
        torch.cuda.empty_cache()
    return {"workload": "configs[3] dense W4A8 sweep (M in {1,16,2048}; weights rotated "
                        "over >= 256 MB of copies; one rotation per CUDA graph replay)", "peak_hbm_gbs": hbm,
            "peak_e4m3_tflops": round(fp8_peak, 1), "peak_source": src, "cells": cells}


def ep_report(torch, dist, world, rank, dev, layer, x, ids, tw, wts, shared):
    """Expert-parallel extras: the all-to-all times of one eager step (CUDA events around each
    collective, max over ranks) and the output check: every rank all-gathers the per-rank
    expert weights, runs the single-GPU layer on its own tokens with the full weight set (the
    shared expert as expert E) and compares it with the EP output (max-abs-rel)."""
    from w4a8_fp8_wmma.moe_experts import run_grouped_moe
    layer.profile_a2a = True
    torch.cuda.synchronize()
    dist.barrier()
    y = layer(x, ids[:, :TOP_K].contiguous(), tw[:, :TOP_K].contiguous())
    torch.cuda.synchronize()
    layer.profile_a2a = False
    a2a = [float(_max_over_ranks(torch, dist, world, dev, v)) for v in layer.last_a2a_ms]
    full = []
    for t_loc, t_sh in zip(wts, shared):
        parts = [torch.empty_like(t_loc) for _ in range(world)]
        dist.all_gather(parts, t_loc.contiguous())
        full.append(torch.cat(parts + [t_sh], 0).contiguous())
    w13, s13, z13, w2, s2, z2 = full
    ref = run_grouped_moe(x, w13, w2, s13, s2, z13, z2, tw, ids,
                          global_num_experts=E_ROUTED + 1, out_dtype=torch.float32)
    err = float((y.float() - ref).abs().max() / ref.abs().max().clamp_min(1e-30))
    err = _max_over_ranks(torch, dist, world, dev, err)
    del full
    torch.cuda.empty_cache()
    return {"a2a_us": [round(v * 1e3, 2) for v in a2a],
            "a2a_what": list(layer.a2a_names),
            "parity": {"max_abs_rel": err, "vs": "single-GPU run_grouped_moe with the "
                       "all-gathered weights on each rank's own tokens (max over ranks)",
                       "pass": err <= 1e-2}}


# dram__bytes_read.sum + dram__bytes_write.sum of the three decode-layer launches in the
# committed ncu launch list (profiles/decode_layer_launches.md); None until captured.
DECODE_TRAFFIC = 266110208
DECODE_TRAFFIC_SRC = "profiles/decode_layer_launches.md (dram read+write summed over the three launches)"
# The same for the prefill gate_up w4_tc_kernel launch (profiles/w4_tc_kernel_prefill.md).
TC_KERNEL_TRAFFIC = 305_600_512 + 45_892_096


def end_to_end(torch, dist, args, world, dev, x_np, ids_np, w_np, layer, run_grouped_moe,
               wts, E_total):
    """Same metric through the public API with host buffers: pinned host inputs are copied in,
    the layer runs (eager), the fp16 output is copied back, all inside the timed region."""
    x_h = torch.from_numpy(x_np).pin_memory()
    ids_h = torch.from_numpy(ids_np).pin_memory()
    w_h = torch.from_numpy(w_np).pin_memory()
    T = x_np.shape[0]
    out_h = torch.empty((T, H), dtype=torch.float16).pin_memory()
    w13, s13, z13, w2, s2, z2 = wts

    def once():
        x = x_h.to(dev, non_blocking=True)
        ids = ids_h.to(dev, non_blocking=True)
        tw = w_h.to(dev, non_blocking=True)
        if world > 1:
            y = layer(x, ids[:, :TOP_K].contiguous(), tw[:, :TOP_K].contiguous())
        else:
            y = run_grouped_moe(x, w13, w2, s13, s2, z13, z2, tw, ids,
                                global_num_experts=E_total, out_dtype=torch.float16)
        out_h.copy_(y, non_blocking=True)
    if world > 1:
        dist.barrier()
    ms = _max_over_ranks(torch, dist, world, dev, _event_time(torch, once, reps=args.steps))
    return {"value": round(T * world / (ms / 1e3), 1), "unit": "tokens/s",
            "h2d_bytes_per_step": int(x_h.numel() * 2 + ids_h.numel() * 4 + w_h.numel() * 4),
            "d2h_bytes_per_step": int(out_h.numel() * 2), "ms_per_step": round(ms, 4),
            "path": "w4a8_fp8_wmma.moe_experts.run_grouped_moe" if world == 1 else
                    "w4a8_fp8_wmma.ep.ExpertParallelMoE", "graph": "eager"}


# ------------------------------------------------------------------------------------------
# CPU baseline / reference arm: the reference's CPU algorithm (numpy oracle port)
# ------------------------------------------------------------------------------------------
def cpu_layer_sample(workload: str, budget_s: float):
    """Time the oracle MoE layer on a bounded sample; returns (tokens/s, sample text)."""
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import w4a8_oracle as O
    cfg = workload_config(workload)
    T = cfg["T"]
    x, ids, w = make_tokens(T, cfg["zipf"], cfg["seed"])
    rng = np.random.default_rng(5)
    used = np.unique(ids)
    # Only the experts the sample touches are materialised (host memory stays small).
    def rand_w(n, k):
        return rng.integers(-2 ** 31, 2 ** 31 - 1, (n, k), dtype=np.int64).astype(np.int32)
    E_total = E_ROUTED + 1
    w13 = np.zeros((E_total, 2 * INTER, H // 8), np.int32)
    w2 = np.zeros((E_total, H, INTER // 8), np.int32)
    s13 = np.zeros((E_total, 2 * INTER, H // GROUP), np.float16)
    s2 = np.zeros((E_total, H, INTER // GROUP), np.float16)
    z13 = np.zeros((E_total, 2 * INTER // 8, H // GROUP), np.int32)
    z2 = np.zeros((E_total, H // 8, INTER // GROUP), np.int32)
    for e in used:
        w13[e] = rand_w(2 * INTER, H // 8)
        w2[e] = rand_w(H, INTER // 8)
        s13[e] = rng.uniform(1e-3, 2e-2, (2 * INTER, H // GROUP))
        s2[e] = rng.uniform(1e-3, 2e-2, (H, INTER // GROUP))
        z13[e] = rand_w(2 * INTER // 8, H // GROUP)
        z2[e] = rand_w(H // 8, INTER // GROUP)
    # Bounded sample: a prefix of the tokens, grown until ~budget_s of CPU work.
    n = min(T, 32)
    t0 = time.perf_counter()
    O.moe_layer(x[:n], w13, s13, z13, w2, s2, z2, ids[:n], w[:n])
    dt = time.perf_counter() - t0
    reps = max(1, int(budget_s / max(dt, 1e-3)))
    reps = min(reps, 20)
    t0 = time.perf_counter()
    for _ in range(reps):
        O.moe_layer(x[:n], w13, s13, z13, w2, s2, z2, ids[:n], w[:n])
    dt = (time.perf_counter() - t0) / reps
    return n / dt, f"{n} of {T} tokens of the {workload} layer (top-8 + shared), {reps} timed reps"


def cpu_baseline(workload: str, budget_s: float = 10.0):
    n = _use_all_threads()
    v, sample = cpu_layer_sample(workload, budget_s)
    return {"value": round(v, 2), "unit": "tokens/s", "cores": n, "kind": "port",
            "sample": sample, "what": "numpy restatement of the reference's torch oracle "
            "(oracle/w4a8_oracle.py), pinned to fixtures from the reference's own run",
            **host_info()}


def _use_all_threads() -> int:
    """Let the oracle's BLAS use every host thread; returns the thread count set."""
    n = os.cpu_count() or 1
    try:
        import threadpoolctl
        threadpoolctl.threadpool_limits(n)
    except Exception:  # noqa: BLE001
        pass
    return n


def run_reference(args):
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    n_threads = _use_all_threads()
    for _ in range(args.warmup):
        cpu_layer_sample(args.workload, 0.0)
    vals = []
    for _ in range(args.steps):
        v, sample = cpu_layer_sample(args.workload, 0.0)
        vals.append(v)
    v = float(np.median(vals))
    cfg = workload_config(args.workload)
    res = {
        "impl": "reference",
        "metric": metric_name(args.workload),
        "value": round(v, 2), "unit": "tokens/s", "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
        "dtype": "e4m3 x int4 -> fp32 (fp16 io)", "data": "synthetic (seeded)",
        "config": base_config(args.workload, world),
        "cpu_baseline": {"value": round(v, 2), "unit": "tokens/s", "cores": n_threads,
                         "kind": "port", "sample": sample, **host_info()},
        "e2e": {"value": round(v, 2), "unit": "tokens/s", "h2d_bytes_per_step": 0,
                "d2h_bytes_per_step": 0},
        "note": "the reference's kernels are gfx1201 HIP and cannot run here; its CPU algorithm "
                "(the torch oracle of its tests) is restated in numpy (oracle/w4a8_oracle.py, "
                "a port pinned to fixtures from the reference's own run) and timed on the "
                "host cores",
    }
    print(json.dumps(res))


def profile_op(args):
    """Run only the dominant op (the gate_up launch the roofline times) `--steps` times on one
    GPU, for an ncu capture of w4_stream_kernel (decode) or w4_tc_kernel (prefill) on the same
    inputs as the bench, without the rest of the bench around it."""
    import torch
    import w4a8_fp8_wmma as w4
    dev = torch.device("cuda", 0)
    cfg = workload_config(args.workload)
    x_np, ids_np, _ = make_tokens(cfg["T"], cfg["zipf"], cfg["seed"] * 1000)
    x = torch.from_numpy(x_np).to(dev)
    ids = torch.from_numpy(ids_np).to(dev)
    w13, s13, z13, _, _, _ = make_layer(torch, dev, 1000, E_ROUTED + 1)
    block_m, kern = (128, 6) if args.workload == "prefill" else (8, 7)
    s, e, n = w4.moe_align_block_size(ids, block_m, E_ROUTED + 1)
    for _ in range(args.steps):
        torch.ops.w4a8_b200.moe_gemm1_silu(x, w13, s13, z13, s, e, n, ids.size(1), block_m,
                                           kern, False)
    torch.cuda.synchronize()
    print(f"profile-op {args.workload}: {args.steps} launches of the gate_up op", flush=True)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=50)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--workload", choices=["decode", "prefill", "stack"], default="decode",
                    help="stack: configs[4], the 40-layer expert-parallel stack (run_stack)")
    ap.add_argument("--layers", type=int, default=40, help="layers of the stack workload")
    ap.add_argument("--cpu-seconds", type=float, default=10.0)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-extras", action="store_true",
                    help="skip the prefill and dense sub-records of the default run")
    ap.add_argument("--profile-op", action="store_true",
                    help="only launch the gate_up op --steps times (for an ncu capture)")
    args = ap.parse_args()
    if args.warmup < 3:
        args.warmup = 3
    if args.profile_op:
        profile_op(args)
    elif args.impl == "reference" and args.workload == "stack":
        print(json.dumps({"impl": "reference", "unavailable": "the reference has no expert "
                          "parallelism; the stack workload has no reference arm"}), flush=True)
    elif args.impl == "reference":
        run_reference(args)
    elif args.workload == "stack":
        run_stack(args)
    else:
        run_ours(args)


if __name__ == "__main__":
    main()
