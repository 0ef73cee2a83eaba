"""Expert-parallel MoE layer over torch.distributed (one process per GPU, NCCL over NVLink).

Expert e lives on rank floor(e * G / E) (contiguous blocks); every rank holds the router and a
shard of the batch. One forward:

  1. route the local tokens (replicated router: moeb_layer_route);
  2. dispatch: for every (token, rank) pair with at least one of the token's top-k experts on that
     rank, send the token's row once, with its k expert ids (-1 where the expert lives elsewhere)
     and routing weights -- all-to-all-v of the counts, then of rows, ids and weights;
  3. each rank runs the expert half on what it received (moeb_layer_forward_routed), which sums
     its own experts' weighted outputs per row in slot order;
  4. combine: all-to-all-v of those partial rows back to their source rank, which adds them in
     rank order.

This mirrors the reference's single-GPU arithmetic except for the final order of additions: the
reference adds all k weighted outputs in slot order, here the slot-ordered partial sums of each
rank are added in rank order (a difference of float rounding only).

The data path is three collectives (counts, rows with their ids and weights out, partials back)
with one host synchronisation (the split sizes); the bookkeeping between them (which rows go where)
is a handful of device-side index operations.
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
        ids, w = self.route_fn(x)
        _, _, counts = presence(ids, self.E, G)
        # counts, then the one host synchronisation of the step: both sides' split sizes
        recv_counts = torch.empty_like(counts)
        _a2a(recv_counts, counts, None, None, self.group)
        both = torch.stack([counts, recv_counts]).tolist()
        in_splits, out_splits = both[0], both[1]
        n_recv = int(sum(out_splits))
        r_idx, t_idx, _, sent_ids = dispatch_plan(ids, self.E, G, n_sent=int(sum(in_splits)))
        sent_w = torch.where(sent_ids >= 0, w[t_idx], torch.zeros_like(w[t_idx]))
        # one message per row: the f32 row, its k ids (bit-cast) and its k weights
        sent = torch.cat([x[t_idx].float(), sent_ids.to(torch.int32).view(torch.float32), sent_w.float()], dim=1)
        recv = torch.empty((n_recv, d + 2 * k), dtype=torch.float32, device=dev)
        _a2a(recv, sent.contiguous(), out_splits, in_splits, self.group)
        recv_x = recv[:, :d].to(x.dtype).contiguous()
        recv_ids = recv[:, d:d + k].contiguous().view(torch.int32)
        recv_w = recv[:, d + k:].contiguous()
        # the local experts' weighted sums per received row
        partial = self.experts_fn(recv_x, recv_ids, recv_w) if n_recv else torch.empty((0, d), dtype=x.dtype,
                                                                                          device=dev)
        back = torch.empty((int(sum(in_splits)), d), dtype=x.dtype, device=dev)
        _a2a(back, partial.contiguous(), in_splits, out_splits, self.group)
        # combine in rank order (the sent rows are rank-major)
        out = torch.zeros_like(x)
        start = 0
        for r in range(G):
            n = in_splits[r]
            if n:
                out.index_add_(0, t_idx[start:start + n], back[start:start + n])
            start += n
        return out

    __call__ = forward
