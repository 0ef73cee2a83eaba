"""Expert-parallel MoE layer over torch.distributed (one process per GPU, NCCL over NVLink).

Expert e lives on rank floor(e * G / E) (contiguous blocks); every rank holds the router and a
shard of the batch. One forward:

  1. route the local tokens (replicated router: moeb_layer_route);
  2. dispatch: for every (token, rank) pair with at least one of the token's top-k experts on that
     rank, send the token's row once, with its k expert ids (-1 where the expert lives elsewhere)
     and routing weights -- one all-to-all of fixed-size blocks;
  3. each rank runs the expert half on what it received (moeb_layer_forward_routed), which sums
     its own experts' weighted outputs per row in slot order;
  4. combine: all-to-all-v of those partial rows back to their source rank, which adds them in
     rank order.

This mirrors the reference's single-GPU arithmetic except for the final order of additions: the
reference adds all k weighted outputs in slot order, here the slot-ordered partial sums of each
rank are added in rank order (a difference of float rounding only).

The data path is collectives of fixed size (rows out, with a small message of their ids and
weights, and partial rows back): each rank sends every rank a block of T rows, its own rows first
and absent rows (ids all -1) after them, so no split sizes cross to the host and a step needs no
host synchronisation. The
bookkeeping (which rows go where) is a handful of device-side index operations.
"""
from __future__ import annotations

import numpy as np
import torch
import torch.distributed as dist


def owner(e: torch.Tensor, n_expert: int, world: int) -> torch.Tensor:
    """Rank holding expert e: contiguous blocks of n_expert / world experts."""
    return (e * world) // n_expert


def local_experts(rank: int, n_expert: int, world: int) -> np.ndarray:
    e = np.arange(n_expert)
    return e[(e * world) // n_expert == rank].astype(np.int32)


def _a2a(out: torch.Tensor, inp: torch.Tensor, out_splits, in_splits, group):
    dist.all_to_all_single(out, inp, out_splits, in_splits, group=group)
    return out


def presence(ids: torch.Tensor, n_expert: int, world: int):
    """[world, T] bool: whether token t has at least one of its top-k experts on rank r, and the
    per-rank counts (device tensors: no host synchronisation)."""
    T, k = ids.shape
    dest = owner(ids.long(), n_expert, world)                                  # [T, k]
    present = torch.zeros((world, T), dtype=torch.bool, device=ids.device)
    present[dest.t().reshape(-1), torch.arange(T, device=ids.device).repeat(k)] = True
    return dest, present, present.sum(dim=1)


def dispatch_plan(ids: torch.Tensor, n_expert: int, world: int, n_sent: int | None = None):
    """For local routing ids [T, k]: the (rank, token) pairs to send, rank-major then token order,
    the per-rank counts, and each sent row's ids with experts of other ranks masked to -1. With
    n_sent (the total, already known on the host) the compaction needs no host synchronisation."""
    dest, present, counts = presence(ids, n_expert, world)
    if n_sent is None:
        r_idx, t_idx = present.nonzero(as_tuple=True)                          # rank-major, tokens ascending
    else:
        nz = torch.nonzero_static(present, size=n_sent)
        r_idx, t_idx = nz[:, 0], nz[:, 1]
    sent_ids = torch.where(dest[t_idx] == r_idx[:, None], ids[t_idx], torch.full_like(ids[t_idx], -1))
    return r_idx, t_idx, counts, sent_ids


class EPMoE:
    """One layer's expert-parallel forward for this rank.

    route_fn(x) -> (ids [T, k] i32, w [T, k] f32) and experts_fn(rows, ids, w) -> partial rows are
    the local compute; by default they are a MoELayer's route / forward_routed (sm_100a kernels).
    Tests on CPU pass host functions instead, over a gloo group."""

    def __init__(self, n_expert: int, top_k: int, route_fn, experts_fn, group=None):
        self.E, self.k = n_expert, top_k
        self.route_fn, self.experts_fn = route_fn, experts_fn
        self.group = group
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        self.timing = {}

    @classmethod
    def from_layer(cls, layer, group=None):
        return cls(layer.host.n_expert, layer.host.top_k, lambda x: layer.route(x)[1:],
                   lambda rows, ids, w: layer.forward_routed(rows, ids, w), group)

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        G, d, k, dev = self.world, x.shape[1], self.k, x.device
        T = x.shape[0]
        ids, w = self.route_fn(x)
        dest, present, _ = presence(ids, self.E, G)                        # [T, k], [G, T]
        # Fixed-capacity messages: each rank gets a block of T rows (its rows first, in token order,
        # then absent rows with every id -1), so the exchange needs no split sizes on the host and
        # the step runs without any host synchronisation.
        pos = torch.cumsum(present.to(torch.int32), dim=1) - 1             # slot of token t in rank r's block
        base = torch.arange(G, device=dev, dtype=torch.int64)[:, None] * T
        dump = G * T                                                       # one spare row takes the absent pairs
        idx = torch.where(present, base + pos.long(), torch.full_like(base + pos.long(), dump)).reshape(-1)
        mine = dest.t()[:, :, None] == torch.arange(G, device=dev)[None, None, :]   # [k, T, G]
        mine = mine.permute(2, 1, 0)                                                 # [G, T, k]
        sids = torch.where(mine, ids[None].expand(G, T, k), torch.full((G, T, k), -1, dtype=ids.dtype, device=dev))
        sw = torch.where(mine, w[None].expand(G, T, k), torch.zeros((G, T, k), dtype=w.dtype, device=dev))
        # rows: gathered straight into the send buffer through the inverse of idx (absent rows repeat
        # token 0; their ids are all -1, so nothing reads them); ids and weights: a small second message
        inv = torch.zeros(G * T + 1, dtype=torch.int64, device=dev)
        inv.index_put_((idx,), torch.arange(T, device=dev).repeat(G))
        sent_x = x.index_select(0, inv[:G * T])
        meta = torch.empty((G * T + 1, 2 * k), dtype=torch.float32, device=dev)
        meta[:G * T, :k] = torch.full((), -1, dtype=torch.int32, device=dev).view(torch.float32)   # absent ids
        meta.index_put_((idx,), torch.cat([sids.to(torch.int32).view(torch.float32), sw.float()], dim=2).reshape(G * T, 2 * k))
        recv_x = torch.empty((G * T, d), dtype=x.dtype, device=dev)
        recv_meta = torch.empty((G * T, 2 * k), dtype=torch.float32, device=dev)
        _a2a(recv_x, sent_x, None, None, self.group)
        _a2a(recv_meta, meta[:G * T], None, None, self.group)
        recv_ids = recv_meta[:, :k].contiguous().view(torch.int32)
        recv_w = recv_meta[:, k:].contiguous()
        # the local experts' weighted sums per received row (absent rows give zeros)
        partial = self.experts_fn(recv_x, recv_ids, recv_w)
        back = torch.empty((G * T, d), dtype=x.dtype, device=dev)
        _a2a(back, partial.contiguous(), None, None, self.group)
        # combine in rank order
        out = torch.zeros_like(x)
        for r in range(G):
            got = back[(r * T + pos[r].clamp(min=0)).long()]
            out += torch.where(present[r][:, None], got, torch.zeros_like(got))
        return out

    __call__ = forward
