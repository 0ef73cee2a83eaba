"""Expert-parallel dispatch/combine (llapis_b200/ep.py) on CPU: world_size-2 gloo groups, with
host functions standing in for the GPU router and expert kernels. Checks that every row reaches
exactly the ranks owning its experts, that each rank computes only its own experts, and that the
combined output equals the single-process result."""
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from llapis_b200.ep import EPMoE, dispatch_plan, local_experts, owner

E, K, D, T_LOCAL = 8, 3, 16, 7


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _route(x, w_r, bias):
    logits = x @ w_r.T + bias
    p = torch.softmax(logits, dim=-1)
    top = torch.topk(p, K, dim=-1)
    w = top.values / top.values.sum(dim=-1, keepdim=True)
    return top.indices.to(torch.int32), w.to(torch.float32)


def _expert(e, x):
    return torch.tanh(x * (e + 1) / 7.0)


def _dense(x, ids, w):
    out = torch.zeros_like(x)
    for j in range(K):
        out += w[:, j:j + 1] * torch.stack([_expert(int(ids[t, j]), x[t]) for t in range(x.shape[0])])
    return out


def _worker(rank, world, port, skew):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        g = torch.Generator().manual_seed(5)
        w_r = torch.randn((E, D), generator=g)
        x_all = torch.randn((world * T_LOCAL, D), generator=g)
        # skew: route everything to rank 0's experts (rank 1 receives no rows)
        bias = torch.where(torch.arange(E) < E // world, 0.0, -1e4) if skew else torch.zeros(E)
        x = x_all[rank * T_LOCAL:(rank + 1) * T_LOCAL]
        mine = set(local_experts(rank, E, world).tolist())
        seen = []

        def experts_fn(rows, ids, w):
            assert all(int(e) in mine for e in ids.reshape(-1).tolist() if e >= 0), "row routed to a foreign expert"
            # fixed-size blocks: each source sends T_LOCAL rows, its present rows first, then absent ones
            assert rows.shape[0] == world * T_LOCAL
            has = (ids >= 0).any(dim=1).reshape(world, T_LOCAL)
            for blk in has:
                n = int(blk.sum())
                assert bool(blk[:n].all()) and not bool(blk[n:].any()), "present rows must lead their block"
            seen.append(int(has.sum()))
            out = torch.zeros_like(rows)
            for j in range(K):
                for r in range(rows.shape[0]):
                    if ids[r, j] >= 0:
                        out[r] += w[r, j] * _expert(int(ids[r, j]), rows[r])
            return out

        ep = EPMoE(E, K, lambda xx: _route(xx, w_r, bias), experts_fn)
        out = ep(x)
        ids, w = _route(x, w_r, bias)
        want = _dense(x, ids, w)
        torch.testing.assert_close(out, want, rtol=1e-5, atol=1e-6)
        if skew and rank == 1:
            assert seen == [0], "rank 1 owns no routed expert and must receive only absent rows"
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("skew", [False, True])
def test_ep_dispatch_combine_world2(skew):
    mp.spawn(_worker, args=(2, _free_port(), skew), nprocs=2, join=True)


def test_dispatch_plan_dedups_per_rank():
    ids = torch.tensor([[0, 1, 5], [4, 6, 7], [2, 3, 1]], dtype=torch.int32)   # E=8, world=2: 0-3 | 4-7
    r_idx, t_idx, counts, sent_ids = dispatch_plan(ids, 8, 2)
    assert counts.tolist() == [2, 2]                     # token 1 has no rank-0 expert, token 2 no rank-1
    assert list(zip(r_idx.tolist(), t_idx.tolist())) == [(0, 0), (0, 2), (1, 0), (1, 1)]
    assert sent_ids.tolist() == [[0, 1, -1], [2, 3, 1], [-1, -1, 5], [4, 6, 7]]
    assert owner(torch.tensor([0, 3, 4, 7]), 8, 2).tolist() == [0, 0, 1, 1]


def _norm_rows(v, w, scale=1.0, eps=1e-6):
    s = 1.0 / torch.sqrt(torch.mean(v.double() ** 2, dim=1, keepdim=True) + eps)
    return (v * s.float() * scale) * w


def _norm_worker(rank, world, port):
    """The Gemma-4 block around the expert-parallel layer: norms on the source rank before the
    dispatch (router and expert inputs) and after the combine (output norm)."""
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        g = torch.Generator().manual_seed(9)
        w_r = torch.randn((E, D), generator=g)
        pre, rsc, post = (1 + 0.1 * torch.randn(D, generator=g) for _ in range(3))
        x_all = torch.randn((world * T_LOCAL, D), generator=g) * 3
        x = x_all[rank * T_LOCAL:(rank + 1) * T_LOCAL]

        def experts_fn(rows, ids, w):
            out = torch.zeros_like(rows)
            for j in range(K):
                for r in range(rows.shape[0]):
                    if ids[r, j] >= 0:
                        out[r] += w[r, j] * _expert(int(ids[r, j]), rows[r])
            return out

        ep = EPMoE(E, K, lambda xx: _route(xx, w_r, torch.zeros(E)), experts_fn,
                   norm_in=lambda v: (_norm_rows(v, rsc, D ** -0.5), _norm_rows(v, pre)),
                   norm_out=lambda v: _norm_rows(v, post))
        out = ep(x)
        ids, w = _route(_norm_rows(x, rsc, D ** -0.5), w_r, torch.zeros(E))
        want = _norm_rows(_dense(_norm_rows(x, pre), ids, w), post)
        torch.testing.assert_close(out, want, rtol=1e-5, atol=1e-5)
    finally:
        dist.destroy_process_group()


def test_ep_block_norms_world2():
    mp.spawn(_norm_worker, args=(2, _free_port()), nprocs=2, join=True)


def _leave_worker(rank, world, port, announce, q):
    """Rank 1 takes one step and leaves between steps (announced, or silently); rank 0's next step
    must fail with RankFailure on the host, before any collective, within the heartbeat deadline."""
    import time
    from datetime import timedelta

    from llapis_b200.ep import Heartbeat, RankFailure
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timedelta(seconds=60))
    g = torch.Generator().manual_seed(5)
    w_r = torch.randn((E, D), generator=g)
    x = torch.randn((T_LOCAL, D), generator=g)
    hb = Heartbeat(dist.distributed_c10d._get_default_store(), rank, world, deadline_s=2.0)
    ep = EPMoE(E, K, lambda xx: _route(xx, w_r, torch.zeros(E)), lambda rows, ids, w: torch.zeros_like(rows),
               heartbeat=hb)
    ep(x)
    if rank == 1:
        if announce:
            hb.leave()
        q.put(("rank1", "left"))
        q.close()
        q.join_thread()   # the message is flushed before the process leaves
        os._exit(0)       # between steps: none of its collectives in flight
    t0 = time.monotonic()
    try:
        ep(x)
        q.put(("rank0", "no failure raised"))
    except RankFailure as e:
        q.put(("rank0", f"ok {time.monotonic() - t0:.2f} {e}"))
    q.close()
    q.join_thread()
    os._exit(0)       # the departed peer never joins a teardown


@pytest.mark.parametrize("announce", [True, False])
def test_ep_departed_rank_detected_on_host(announce):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_leave_worker, args=(r, 2, port, announce, q)) for r in range(2)]
    for p in procs:
        p.start()
    msgs = dict(q.get(timeout=120) for _ in range(2))
    for p in procs:
        p.join(timeout=60)
    status = msgs["rank0"]
    assert status.startswith("ok"), status
    elapsed = float(status.split()[1])
    assert elapsed < (1.0 if announce else 10.0), status
    assert ("left" in status) if announce else ("did not reach step 1" in status), status


def _hb_worker(rank, world, port, q):
    """Five heartbeats on both ranks: every step's records exist while it runs, and each rank
    deletes its records older than two steps (the store does not grow with the step count)."""
    from datetime import timedelta

    from llapis_b200.ep import Heartbeat
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timedelta(seconds=60))
    store = dist.distributed_c10d._get_default_store()
    hb = Heartbeat(store, rank, world, deadline_s=10.0, prefix="hbtest")
    for step in range(5):
        hb.beat(step)
    dist.barrier()
    kept = [s for s in range(5) if store.check([f"hbtest/s{s}/r{rank}"])]
    q.put((rank, kept))
    q.close()
    q.join_thread()
    dist.destroy_process_group()


def test_heartbeat_keeps_the_store_bounded():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_hb_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = dict(q.get(timeout=120) for _ in range(2))
    for p in procs:
        p.join(timeout=60)
    assert res[0] == [3, 4] and res[1] == [3, 4], res
