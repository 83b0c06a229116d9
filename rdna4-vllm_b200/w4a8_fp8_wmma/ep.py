"""Expert-parallel MoE layer: experts sharded across ranks, two all-to-alls per step.

The reference has no expert parallelism (its `expert_map` is only forwarded to vLLM's align,
w4a8_fp8_wmma/w4a8_fp8_wmma/moe_experts.py:587-589); this module adds it around the same layer.
Rank r of W owns routed experts [r*E/W, (r+1)*E/W) and its own T tokens.

  1. dispatch - every token goes once to every rank that owns one of its top_k experts, as one
     row carrying the token, its top_k *local* expert ids on that rank (-1 = slot elsewhere) and
     its routing weights. Rank d's rows fill chunk d of the send buffer in token order; a chunk
     holds up to T rows (capacity T), so the exchange is one fixed-size all_to_all with no host
     synchronisation (graph-capturable). On GPUs the row is the token's e4m3 operand (quantised
     once, torch.ops.w4a8_b200.ep_pack), so the owner's layer needs no re-quantisation.
  2. compute - the owner runs the layer on the received rows: for each row the slot-order
     weighted sum over its local experts (fp32). The replicated shared expert rides the same
     call on the rank's own tokens, as local expert E/W.
  3. combine - one all_to_all returns each row to its source; the source sums a token's rows
     over ranks in rank order (fp32) and adds its shared-expert row.

Prefill-size batches (T > GEMV_MAX_M tokens per rank, the same split as run_grouped_moe) send
fp16 rows with their local ids and weights instead, and the owner runs the reference
composition (run_grouped_moe: tile GEMMs) on the received rows, with slots owned elsewhere
mapped to a remote expert through expert_map; the shared expert runs on the rank's own tokens.

Every rank must pass the same token count T (the all_to_all chunk size); the first call with a
new T checks this across the group and raises on a mismatch. A caller whose ranks hold different
token counts passes `max_tokens`: each rank's batch is padded to it with empty rows.
`expert_fn` makes the compute step pluggable so the exchange logic is testable on CPU ranks.
"""
from __future__ import annotations

from typing import Callable

import torch
import torch.distributed as dist

# expert_fn(rows (R, H) fp16, local_ids (R, k) int32 (-1 = none), weights (R, k) fp32)
#   -> (R, H) fp32: per row, the weighted sum over its valid local slots
ExpertFn = Callable[[torch.Tensor, torch.Tensor, torch.Tensor], torch.Tensor]


def plan_dispatch(topk_ids: torch.Tensor, experts_per_rank: int, world: int):
    """Rows of the send buffer: returns (has (W, T) bool, pos (W, T) int64, local (W, T, k)).

    has[d, t]: token t has a slot on rank d (ids outside [0, W*experts_per_rank) are dropped);
    pos[d, t]: its row within chunk d (tokens in order), -1 when not sent;
    local[d, t, j]: the slot's expert id local to rank d, -1 when that slot is elsewhere.
    Pure tensor ops (no host sync)."""
    ids = topk_ids.to(torch.int64)
    E = experts_per_rank * world
    valid = (ids >= 0) & (ids < E)
    dest = torch.where(valid, torch.div(ids, experts_per_rank, rounding_mode="floor"), -1)
    ranks = torch.arange(world, device=ids.device).view(world, 1, 1)
    on = dest.unsqueeze(0) == ranks                      # (W, T, k)
    has = on.any(-1)                                     # (W, T)
    cum = has.to(torch.int64).cumsum(1) - 1
    pos = torch.where(has, cum, torch.full_like(cum, -1))
    local = torch.where(on, ids.unsqueeze(0) - ranks * experts_per_rank,
                        torch.full_like(on, -1, dtype=torch.int64))
    return has, pos, local


class ExpertParallelMoE:
    """One MoE layer sharded by expert over the ranks of `group`."""

    def __init__(self, w13, s13, z13, w2, s2, z2, num_experts: int, top_k: int,
                 group=None, shared=None, expert_fn: ExpertFn | None = None,
                 max_tokens: int | None = None):
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
        self.max_tokens = max_tokens
        self.expert_fn = expert_fn
        self.shared = shared  # (w13, s13, z13, w2, s2, z2) of one replicated shared expert
        self.weights = (w13, s13, z13, w2, s2, z2)
        self._checked_T: set[int] = set()
        self._remote_map = None
        self.pack = None
        if expert_fn is None and w13 is not None and w13.is_cuda:
            from .moe_experts import DecodePack
            wts = [w13, s13, z13, w2, s2, z2]
            if shared is not None:
                # the shared expert joins the routed ones as local expert E_loc
                cat = []
                for t_r, t_s in zip(wts, shared):
                    if t_r is None or t_r.numel() == 0:
                        if not (t_s is None or t_s.numel() == 0):
                            raise ValueError("routed and shared experts disagree on zero points")
                        cat.append(None)
                    else:
                        cat.append(torch.cat([t_r, t_s], 0).contiguous())
                wts = cat
            w1, s1, z1, w2_, s2_, z2_ = wts
            self.pack = DecodePack(w1, w2_, s1, s2_, z1, z2_)
        # profile_a2a: record CUDA events around each collective of the next eager step and
        # leave their durations (ms) in last_a2a_ms, in the order of a2a_names
        self.profile_a2a = False
        self.last_a2a_ms: list[float] = []
        self.a2a_names = ("dispatch", "combine")
        self._ev = []
        self.last_recv = None

    # ---- token count agreement ----------------------------------------------------------
    def _check_tokens(self, T: int, dev) -> None:
        if T in self._checked_T:
            return
        t = torch.tensor([T, -T], dtype=torch.int64, device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX, group=self.group)
        if int(t[0]) != T or int(-t[1]) != T:
            raise ValueError(
                f"rank {self.rank}: {T} tokens, but the ranks hold between {int(-t[1])} and "
                f"{int(t[0])}; every rank must pass the same T (or set max_tokens)")
        self._checked_T.add(T)

    def _pad(self, x, topk_ids, topk_weights):
        T = x.size(0)
        M = self.max_tokens
        if M is None:
            self._check_tokens(T, x.device)
            return x, topk_ids, topk_weights
        if T > M:
            raise ValueError(f"{T} tokens exceed max_tokens={M}")
        if T == M:
            return x, topk_ids, topk_weights
        pad = M - T
        x = torch.cat([x, x.new_zeros((pad, x.size(1)))])
        topk_ids = torch.cat([topk_ids, topk_ids.new_full((pad, topk_ids.size(1)), -1)])
        topk_weights = torch.cat([topk_weights, topk_weights.new_zeros((pad, topk_weights.size(1)))])
        return x, topk_ids, topk_weights

    def _a2a(self, out, inp):
        if not self.profile_a2a:
            dist.all_to_all_single(out, inp, group=self.group)
            return
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record()
        dist.all_to_all_single(out, inp, group=self.group)
        b.record()
        self._ev.append((a, b))

    # ---- forward ------------------------------------------------------------------------
    def forward(self, x: torch.Tensor, topk_ids: torch.Tensor,
                topk_weights: torch.Tensor) -> torch.Tensor:
        """x (T, H) fp16 local tokens; topk_ids/weights (T, top_k) with GLOBAL expert ids.
        Returns (T, H) fp32: the routed experts' weighted sum plus the shared expert."""
        T_in = x.size(0)
        x, topk_ids, topk_weights = self._pad(x, topk_ids, topk_weights)
        if x.is_cuda and self.expert_fn is None:
            if self.pack is None:
                raise RuntimeError("ExpertParallelMoE: no CUDA expert weights on this rank")
            from .moe_experts import GEMV_MAX_M
            if x.size(0) > GEMV_MAX_M:
                out = self._forward_generic(x, topk_ids, topk_weights, self._prefill_experts,
                                            self._prefill_shared)
            else:
                out = self._forward_cuda(x, topk_ids, topk_weights)
        else:
            out = self._forward_generic(x, topk_ids, topk_weights)
        return out[:T_in]

    def _prefill_experts(self, rows, local_ids, w):
        """The rank's routed experts on received fp16 rows: run_grouped_moe with slots owned
        elsewhere (-1) sent to a remote expert id E_loc that expert_map drops."""
        from .moe_experts import run_grouped_moe
        w13, s13, z13, w2, s2, z2 = self.weights
        if self._remote_map is None or self._remote_map.device != rows.device:
            m = torch.arange(self.E_loc + 1, dtype=torch.int32, device=rows.device)
            m[self.E_loc] = -1
            self._remote_map = m
        ids = torch.where(local_ids >= 0, local_ids,
                          torch.full_like(local_ids, self.E_loc)).to(torch.int32)
        return run_grouped_moe(rows.to(torch.float16), w13, w2, s13, s2, z13, z2, w, ids,
                               global_num_experts=self.E_loc + 1, expert_map=self._remote_map,
                               out_dtype=torch.float32)

    def _prefill_shared(self, x):
        from .moe_experts import run_grouped_moe
        w13, s13, z13, w2, s2, z2 = self.shared
        T = x.size(0)
        ids = torch.zeros((T, 1), dtype=torch.int32, device=x.device)
        ones = torch.ones((T, 1), dtype=torch.float32, device=x.device)
        return run_grouped_moe(x.to(torch.float16), w13, w2, s13, s2, z13, z2, ones, ids,
                               out_dtype=torch.float32)

    def _forward_generic(self, x, topk_ids, topk_weights, expert_fn=None, shared_fn=None):
        """The exchange in plain torch ops: CPU ranks and custom experts (expert_fn), and the
        prefill path on GPUs (expert_fn = the routed experts on received rows, shared_fn = the
        shared expert on the rank's own tokens)."""
        expert_fn = expert_fn or self.expert_fn
        if expert_fn is None:
            raise RuntimeError("ExpertParallelMoE: CPU rows need an expert_fn (the built-in "
                               "experts run on CUDA weights)")
        T, H = x.shape
        k = topk_ids.size(1)
        W = self.world
        has, pos, local = plan_dispatch(topk_ids, self.E_loc, W)
        send_x = torch.zeros((W, T, H), dtype=x.dtype, device=x.device)
        send_id = torch.full((W, T, k), -1, dtype=torch.int32, device=x.device)
        send_w = torch.zeros((W, T, k), dtype=torch.float32, device=x.device)
        d_idx, t_idx = torch.nonzero(has, as_tuple=True)
        p_idx = pos[d_idx, t_idx]
        send_x[d_idx, p_idx] = x[t_idx]
        send_id[d_idx, p_idx] = local[d_idx, t_idx].to(torch.int32)
        wl = torch.where(local >= 0, topk_weights.to(torch.float32).unsqueeze(0),
                         torch.zeros((), dtype=torch.float32, device=x.device))
        send_w[d_idx, p_idx] = wl[d_idx, t_idx]
        recv_x, recv_id, recv_w = (torch.empty_like(send_x), torch.empty_like(send_id),
                                   torch.empty_like(send_w))
        self._a2a(recv_x.view(W * T, H), send_x.view(W * T, H))
        dist.all_to_all_single(recv_id.view(W * T, k), send_id.view(W * T, k), group=self.group)
        dist.all_to_all_single(recv_w.view(W * T, k), send_w.view(W * T, k), group=self.group)
        y = expert_fn(recv_x.view(W * T, H), recv_id.view(W * T, k), recv_w.view(W * T, k))
        y = y.to(torch.float32).contiguous()
        back = torch.empty_like(y)
        self._a2a(back, y)
        back = back.view(W, T, H)
        out = torch.zeros((T, H), dtype=torch.float32, device=x.device)
        for d in range(W):  # rank order, as the GPU gather
            sel = has[d]
            out[sel] = out[sel] + back[d, pos[d][sel]]
        if self.shared is not None:
            if shared_fn is not None:
                out = out + shared_fn(x).float()
            else:
                ids = torch.zeros((T, 1), dtype=torch.int32, device=x.device)
                out = out + expert_fn(x, ids, torch.ones((T, 1), device=x.device)).float()
        self._finish_profile()
        return out

    def _forward_cuda(self, x, topk_ids, topk_weights):
        """GPU path: ep_pack -> all_to_all -> ep_moe_rows (routed + shared in one call) ->
        all_to_all -> ep_gather."""
        T, H = x.shape
        k = topk_ids.size(1)
        W = self.world
        shared_id = self.E_loc if self.shared is not None else -1
        rows, pos = torch.ops.w4a8_b200.ep_pack(
            x.contiguous(), topk_ids.to(torch.int32).contiguous(),
            topk_weights.to(torch.float32).contiguous(), self.E_loc, W, shared_id)
        recv = torch.empty_like(rows)
        if shared_id >= 0:
            recv[W * T:] = rows[W * T:]
        self._a2a(recv[:W * T], rows[:W * T])
        self.last_recv = recv
        R = (W + 1) * T if shared_id >= 0 else W * T
        y = torch.ops.w4a8_b200.ep_moe_rows(recv[:R], self.pack.p13, self.pack.p2, self.pack.E,
                                            H, self.pack.inter, k)
        back = torch.empty((W * T, H), dtype=torch.float32, device=x.device)
        self._a2a(back, y[:W * T])
        self._finish_profile()
        return torch.ops.w4a8_b200.ep_gather(back, pos, y[W * T:] if shared_id >= 0 else None)

    def _finish_profile(self):
        if self.profile_a2a and self._ev:
            torch.cuda.synchronize()
            self.last_a2a_ms = [a.elapsed_time(b) for a, b in self._ev]
        self._ev = []

    __call__ = forward
