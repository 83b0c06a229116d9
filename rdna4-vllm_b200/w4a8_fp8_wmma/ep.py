"""Expert-parallel MoE layer: experts sharded across ranks, NCCL all-to-all dispatch/combine.

The reference has no expert parallelism (its `expert_map` is only forwarded to vLLM's align,
w4a8_fp8_wmma/w4a8_fp8_wmma/moe_experts.py:587-589); this module adds it around the same
per-rank layer. Rank r of W owns routed experts [r*E/W, (r+1)*E/W) and its own tokens:

  1. dispatch — every (token, slot) whose expert lives on rank d is copied into the send
     buffer's chunk d at a stable position (slot order); chunks have a fixed capacity of
     T*top_k rows, so the exchange needs no host synchronisation and is graph-capturable.
     One all_to_all_single moves the fp16 rows, a second one the local expert id of each row
     (-1 marks an empty row).
  2. compute — the received rows run through the grouped layer with top_k = 1 (their own
     local expert, weight 1), producing one fp16 down-projection row per received slot.
  3. combine — an all_to_all_single returns those rows to their source rank in send order;
     the source applies its routing weights with the gather-reduce op (slot order) and adds
     the replicated shared expert, if any.

On GPUs steps 1 and 3 are the library's ep_dispatch / ep_combine kernels (stable positions and
row copies in one launch; the slot-order reduce plus the shared-expert add in one launch), and
the shared expert joins the routed layer call as local expert E_loc. The collectives use
torch.distributed (NCCL on GPUs, gloo for the CPU tests). `expert_fn`
makes the compute step pluggable so the permutation logic is testable on CPU ranks.
"""
from __future__ import annotations

from typing import Callable

import torch
import torch.distributed as dist

ExpertFn = Callable[[torch.Tensor, torch.Tensor], torch.Tensor]


def plan_dispatch(topk_ids: torch.Tensor, experts_per_rank: int, world: int, capacity: int):
    """Positions of every (token, slot) in the fixed-capacity send buffer.

    Returns (dest (S,), pos (S,), row (S,)) with S = T*top_k: the destination rank, the stable
    rank of the slot among slots with that destination, and the send-buffer row
    dest*capacity + pos. Pure tensor ops (no host sync)."""
    ids = topk_ids.reshape(-1).to(torch.int64)
    dest = torch.div(ids, experts_per_rank, rounding_mode="floor").clamp_(0, world - 1)
    # one-hot by comparison (F.one_hot validates its input with a device sync)
    onehot = (dest[:, None] == torch.arange(world, device=ids.device)[None, :]).to(torch.int64)
    pos = (onehot.cumsum(0) - onehot).gather(1, dest[:, None]).squeeze(1)
    return dest, pos, dest * capacity + pos


class ExpertParallelMoE:
    """One MoE layer sharded by expert over the ranks of `group`."""

    def __init__(self, w13, s13, z13, w2, s2, z2, num_experts: int, top_k: int,
                 group=None, shared=None, expert_fn: ExpertFn | None = None):
        self.group = group
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        if num_experts % self.world:
            raise ValueError(f"{num_experts} experts do not split over {self.world} ranks")
        self.E = num_experts
        self.E_loc = num_experts // self.world
        if w13 is not None and w13.size(0) != self.E_loc:
            raise ValueError(f"rank {self.rank} holds {w13.size(0)} experts, expected {self.E_loc}")
        self.top_k = top_k
        self.w = (w13, s13, z13, w2, s2, z2)
        self.shared = shared  # (w13, s13, z13, w2, s2, z2) of one replicated shared expert
        self.expert_fn = expert_fn or self._gpu_experts
        # With the built-in GPU experts the shared expert rides the routed call as local expert
        # E_loc: its weights are appended once here, and the rank's own tokens join the received
        # rows with that id, so a step runs one layer call instead of two.
        self._fused_shared = expert_fn is None and shared is not None and w13 is not None
        if self._fused_shared:
            cat = []
            for i, (t_r, t_s) in enumerate(zip(self.w, shared)):
                if t_r is None or t_r.numel() == 0:
                    if not (t_s is None or t_s.numel() == 0):
                        raise ValueError("routed and shared experts disagree on zero points")
                    cat.append(t_r)
                else:
                    cat.append(torch.cat([t_r, t_s], 0).contiguous())
            self.w_all = tuple(cat)
        self._ntp = {}  # cached device scalars (no host->device copies inside graph capture)
        # profile_a2a: record CUDA events around each collective of the next eager step and
        # leave their durations (ms) in last_a2a_ms, in the order of a2a_names
        self.profile_a2a = False
        self.last_a2a_ms: list[float] = []
        self.a2a_names = ("dispatch rows", "dispatch ids", "combine rows")
        self._ev = []

    # ---- compute on received rows ------------------------------------------------------
    def _gpu_experts(self, rows: torch.Tensor, local_ids: torch.Tensor) -> torch.Tensor:
        w13, s13, z13, w2, s2, z2 = self.w
        ids = local_ids.view(-1, 1).to(torch.int32)
        valid = ids >= 0
        ids = torch.where(valid, ids, torch.full_like(ids, self.E_loc))  # out of range: skipped
        ones = valid.to(torch.float32)
        return torch.ops.w4a8_b200.moe_decode(rows, w13, s13, z13, w2, s2, z2, ones, ids)

    def _shared(self, x: torch.Tensor) -> torch.Tensor | None:
        if self.shared is None:
            return None
        w13, s13, z13, w2, s2, z2 = self.shared
        T = x.size(0)
        ids = torch.zeros((T, 1), dtype=torch.int32, device=x.device)
        ones = torch.ones((T, 1), dtype=torch.float32, device=x.device)
        return torch.ops.w4a8_b200.moe_decode(x, w13, s13, z13, w2, s2, z2, ones, ids)

    # ---- forward ------------------------------------------------------------------------
    def forward(self, x: torch.Tensor, topk_ids: torch.Tensor,
                topk_weights: torch.Tensor) -> torch.Tensor:
        """x (T, H) fp16 local tokens; topk_ids/weights (T, top_k) with GLOBAL expert ids.
        Returns (T, H) fp32: the routed experts' weighted sum plus the shared expert."""
        if x.is_cuda:
            return self._forward_cuda(x, topk_ids, topk_weights)
        T, H = x.shape
        k = topk_ids.size(1)
        W, C = self.world, T * k
        dev = x.device
        dest, pos, row = plan_dispatch(topk_ids, self.E_loc, W, C)
        slots = torch.arange(T * k, device=dev)
        send_x = torch.zeros((W * C, H), dtype=x.dtype, device=dev)
        send_x[row] = x[slots // k]
        send_id = torch.full((W * C,), -1, dtype=torch.int32, device=dev)
        send_id[row] = (topk_ids.reshape(-1).to(torch.int64) - dest * self.E_loc).to(torch.int32)
        recv_x = torch.empty_like(send_x)
        recv_id = torch.empty_like(send_id)
        dist.all_to_all_single(recv_x, send_x, group=self.group)
        dist.all_to_all_single(recv_id, send_id, group=self.group)
        y = self.expert_fn(recv_x, recv_id).to(x.dtype).contiguous()  # (W*C, H)
        back = torch.empty_like(y)
        dist.all_to_all_single(back, y, group=self.group)
        # row `row[s]` of `back` holds slot s
        tw = topk_weights.reshape(-1).to(torch.float32).contiguous()
        # CPU ranks (tests): slot-order weighted sum, as the GPU combine kernel computes it
        out = torch.zeros((T, H), dtype=torch.float32)
        for j in range(k):
            s = torch.arange(T) * k + j
            out += tw[s, None] * back[row[s]].to(torch.float32)
        sh = self._shared(x)
        if sh is not None:
            out = out + sh.to(torch.float32)
        return out

    def _const(self, name: str, n: int, value, dtype, dev) -> torch.Tensor:
        """Cached constant device tensors (no host->device copies inside graph capture)."""
        key = (name, n, dev)
        if key not in self._ntp:
            self._ntp[key] = torch.full((n,), value, dtype=dtype, device=dev)
        return self._ntp[key]

    def _forward_cuda(self, x, topk_ids, topk_weights):
        """GPU path: the dispatch and combine kernels around the NCCL all-to-alls; with the
        built-in experts one decode-layer call serves the received rows and, as local expert
        E_loc, the replicated shared expert on this rank's own tokens."""
        T, H = x.shape
        k = topk_ids.size(1)
        W, C = self.world, T * k
        dev = x.device
        send_x, send_id, slot_row = torch.ops.w4a8_b200.ep_dispatch(
            x.contiguous(), topk_ids.to(torch.int32).contiguous(), self.E_loc, W, C)
        recv_x = torch.empty_like(send_x)
        recv_id = torch.empty_like(send_id)
        self._a2a(recv_x, send_x)
        self._a2a(recv_id, send_id)
        self.last_recv = (recv_x, recv_id)  # for profiling tools: this step's received rows
        sh = None
        if self._fused_shared:
            w13, s13, z13, w2, s2, z2 = self.w_all
            rows = torch.cat([recv_x, x], 0)
            ids = torch.cat([recv_id, self._const("shared_id", T, self.E_loc, torch.int32, dev)])
            ones = self._const("ones", W * C + T, 1.0, torch.float32, dev)
            # id -1 (unclaimed row) is outside [0, E_loc + 1): the layer skips it
            y_all = torch.ops.w4a8_b200.moe_decode(rows, w13, s13, z13, w2, s2, z2,
                                                   ones.view(-1, 1), ids.view(-1, 1))
            y, sh = y_all[:W * C], y_all[W * C:]
        else:
            y = self.expert_fn(recv_x, recv_id).to(x.dtype).contiguous()  # (W*C, H)
            sh = self._shared(x)
        back = torch.empty_like(y)
        self._a2a(back, y)
        if self.profile_a2a:
            torch.cuda.synchronize()
            self.last_a2a_ms = [a.elapsed_time(b) for a, b in self._ev]
            self._ev = []
        tw = topk_weights.reshape(-1).to(torch.float32).contiguous()
        return torch.ops.w4a8_b200.ep_combine(back, slot_row, tw,
                                              None if sh is None else sh.contiguous(), k)

    def _a2a(self, out, inp):
        if not self.profile_a2a:
            dist.all_to_all_single(out, inp, group=self.group)
            return
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record()
        dist.all_to_all_single(out, inp, group=self.group)
        b.record()
        self._ev.append((a, b))

    __call__ = forward
