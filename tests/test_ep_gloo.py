"""Expert-parallel dispatch/combine on CPU `gloo` ranks (world sizes 2 and 4), with an identity
"expert" so the permutation logic is checked exactly; plus host-side failure cases: a rank
that dies before the exchange, a rank holding the wrong expert shard, and ranks passing
different token counts raise instead of hanging or corrupting rows.
"""
import os
import socket
import traceback

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from w4a8_fp8_wmma.ep import ExpertParallelMoE, plan_dispatch


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _init(rank, world, port, timeout_s=20):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    from datetime import timedelta
    dist.init_process_group("gloo", rank=rank, world_size=world,
                            timeout=timedelta(seconds=timeout_s))


def _worker_identity(rank, world, port, q):
    try:
        _init(rank, world, port)
        ok_all, count_all = True, True
        for skew in (False, True):
            torch.manual_seed(100 + rank)
            T, H, E, k = 6, 16, 16, 3
            x = torch.randn(T, H).to(torch.float16)
            if skew:  # every slot routes to rank 0's experts
                ids = torch.stack([torch.randperm(E // world)[:k] for _ in range(T)]).to(torch.int32)
            else:
                ids = torch.stack([torch.randperm(E)[:k] for _ in range(T)]).to(torch.int32)
            w = torch.rand(T, k)
            seen = []

            def identity(rows, local_ids, wts):
                seen.append(int((local_ids >= 0).sum()))
                assert torch.all(local_ids < E // world)
                # every expert returns its input row: the row's result is its weight sum * row
                wsum = torch.where(local_ids >= 0, wts, torch.zeros_like(wts)).sum(1, keepdim=True)
                return wsum * rows.to(torch.float32)

            layer = ExpertParallelMoE(None, None, None, None, None, None, E, k, expert_fn=identity)
            out = layer(x, ids, w)
            ref = w.sum(1, keepdim=True) * x.to(torch.float32)
            ok_all &= bool(torch.allclose(out, ref, rtol=1e-3, atol=1e-3))
            # every slot is computed exactly once somewhere
            tot = torch.tensor([seen[0]])
            dist.all_reduce(tot)
            count_all &= int(tot.item()) == T * k * world
        q.put((rank, ok_all, count_all, None))
        dist.destroy_process_group()
    except Exception:
        q.put((rank, False, False, traceback.format_exc()))


def _spawn(fn, world, *args, reporters=None):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=fn, args=(r, world, port, q) + args) for r in range(world)]
    for p in procs:
        p.start()
    res = [q.get(timeout=120) for _ in range(reporters or world)]
    for p in procs:
        p.join(timeout=60)
    return sorted(res, key=lambda r: r[0])


@pytest.mark.parametrize("world", [2, 4])
def test_ep_dispatch_combine_identity(world):
    res = _spawn(_worker_identity, world)
    for rank, ok, count_ok, err in res:
        assert err is None, err
        assert ok and count_ok, (rank, ok, count_ok)


def test_plan_dispatch_rows_are_stable_and_dense():
    # E=8 over 2 ranks (4 each); token 2 has both slots on rank 0; id 9 is out of range
    ids = torch.tensor([[0, 5], [4, 9], [3, 2], [6, 7]], dtype=torch.int32)
    has, pos, local = plan_dispatch(ids, 4, 2)
    assert has.tolist() == [[True, False, True, False], [True, True, False, True]]
    assert pos.tolist() == [[0, -1, 1, -1], [0, 1, -1, 2]]
    assert local[0].tolist() == [[0, -1], [-1, -1], [3, 2], [-1, -1]]
    assert local[1].tolist() == [[-1, 1], [0, -1], [-1, -1], [2, 3]]


def _worker_dies(rank, world, port, q):
    try:
        _init(rank, world, port, timeout_s=10)
        if rank == 1:
            os._exit(0)  # leaves before the exchange without a word
        layer = ExpertParallelMoE(None, None, None, None, None, None, 4, 1,
                                  expert_fn=lambda r, i, w: r.float())
        try:
            layer(torch.zeros(2, 8, dtype=torch.float16), torch.tensor([[3], [2]], dtype=torch.int32),
                  torch.ones(2, 1))
            q.put((rank, False, False, "exchange with a dead peer returned"))
        except Exception:  # expected: connection closed or timeout
            q.put((rank, True, True, None))
    except Exception:
        q.put((rank, False, False, traceback.format_exc()))


def test_dead_peer_raises_instead_of_hanging():
    res = _spawn(_worker_dies, 2, reporters=1)  # only the surviving rank reports
    for rank, ok, _, err in res:
        assert err is None, err
        assert ok, rank


def _worker_bad_shard(rank, world, port, q):
    try:
        _init(rank, world, port)
        w13 = torch.zeros(3 if rank == 1 else 4, 8, 2, dtype=torch.int32)
        try:
            ExpertParallelMoE(w13, None, None, None, None, None, 8, 2)
            q.put((rank, rank == 0, True, None if rank == 0 else "bad shard accepted"))
        except ValueError:
            q.put((rank, rank == 1, True, None))
        dist.destroy_process_group()
    except Exception:
        q.put((rank, False, False, traceback.format_exc()))


def test_wrong_expert_shard_rejected():
    res = _spawn(_worker_bad_shard, 2)
    for rank, ok, _, err in res:
        assert err is None, err
        assert ok, rank


def _worker_unequal_T(rank, world, port, q):
    try:
        _init(rank, world, port)
        E, k, H = 8, 2, 16
        T = 4 if rank == 0 else 6
        x = torch.randn(T, H).to(torch.float16)
        ids = torch.stack([torch.randperm(E)[:k] for _ in range(T)]).to(torch.int32)
        w = torch.rand(T, k)

        def identity(rows, local_ids, wts):
            wsum = torch.where(local_ids >= 0, wts, torch.zeros_like(wts)).sum(1, keepdim=True)
            return wsum * rows.to(torch.float32)
        raised = False
        try:
            ExpertParallelMoE(None, None, None, None, None, None, E, k, expert_fn=identity)(x, ids, w)
        except ValueError:
            raised = True
        # with a common max_tokens the same batches exchange correctly
        layer = ExpertParallelMoE(None, None, None, None, None, None, E, k, expert_fn=identity,
                                  max_tokens=8)
        out = layer(x, ids, w)
        ok = out.shape == (T, H) and bool(torch.allclose(out, w.sum(1, keepdim=True) * x.float(),
                                                         rtol=1e-3, atol=1e-3))
        q.put((rank, raised, ok, None))
        dist.destroy_process_group()
    except Exception:
        q.put((rank, False, False, traceback.format_exc()))


def test_unequal_token_counts_raise_or_pad():
    res = _spawn(_worker_unequal_T, 2)
    for rank, raised, ok, err in res:
        assert err is None, err
        assert raised, f"rank {rank}: unequal T was accepted"
        assert ok, f"rank {rank}: max_tokens padding gave a wrong result"


def _fake_grouped_moe(x, w1, w2, w1_s, w2_s, w1_zp, w2_zp, topk_weights, topk_ids,
                      kernel="wmma", global_num_experts=None, expert_map=None,
                      apply_router_weight_on_input=False, out_dtype=None):
    """A stand-in for run_grouped_moe with the same id semantics: local expert e scales its
    row by w1[e] (a scalar per expert here); ids that expert_map sends to -1 contribute
    nothing."""
    ids = topk_ids.long()
    loc = expert_map.long()[ids] if expert_map is not None else ids
    valid = loc >= 0
    f = torch.where(valid, w1.float()[loc.clamp_min(0)], torch.zeros((), dtype=torch.float32))
    y = (topk_weights.float() * f).sum(1, keepdim=True) * x.float()
    return y.to(out_dtype or x.dtype)


def _worker_prefill_map(rank, world, port, q):
    try:
        _init(rank, world, port)
        import w4a8_fp8_wmma.moe_experts as me
        me.run_grouped_moe = _fake_grouped_moe
        torch.manual_seed(7 + rank)
        T, H, E, k = 9, 16, 16, 4
        E_loc = E // world
        x = torch.randn(T, H).to(torch.float16)
        ids = torch.stack([torch.randperm(E)[:k] for _ in range(T)]).to(torch.int32)
        w = torch.rand(T, k)
        # "weights": expert e (global) scales by 1 + e; the shared expert by 100
        w1 = (1.0 + torch.arange(rank * E_loc, (rank + 1) * E_loc)).float()
        shared = (torch.tensor([100.0]),) * 6
        layer = ExpertParallelMoE(w1, w1, w1, w1, w1, w1, E, k, shared=shared)
        out = layer._forward_generic(x, ids, w, layer._prefill_experts, layer._prefill_shared)
        ref = ((w * (1.0 + ids.float())).sum(1, keepdim=True) + 100.0) * x.float()
        q.put((rank, bool(torch.allclose(out, ref, rtol=1e-3, atol=1e-2)), None))
    except Exception:  # noqa: BLE001
        q.put((rank, False, traceback.format_exc()))
    finally:
        if dist.is_initialized():
            dist.destroy_process_group()


@pytest.mark.parametrize("world", [2, 4])
def test_prefill_path_maps_remote_slots_and_adds_shared(world):
    """The GPU prefill path's exchange and id mapping on CPU ranks: each rank runs the
    composition (a stand-in here) on received rows with slots owned elsewhere mapped to a
    remote expert, and the shared expert on its own tokens."""
    res = _spawn(_worker_prefill_map, world)
    for r, ok, err in res:
        assert ok, err
