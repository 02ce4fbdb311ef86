"""Expert parallelism for the routed-expert layer (one process per GPU, torch.distributed over NCCL).

The reference runs one GPU (tensor-parallel 1, docker/entrypoint.sh:135-140) and keeps experts in host
RAM; here the experts are HBM-resident and sharded instead: global expert e lives on rank
e // (E / world). One layer step for this rank's T tokens:

  1. dispatch plan: the distinct destination ranks of each token's top-k routes; (token, rank) pairs in
     rank-major order (a token routed to several experts of one rank is sent once)
  2. counts all-to-all (int64 [world]), then the payload all-to-all of the pairs' hidden rows (bf16/fp16)
     and their route metadata (local expert id or -1, routing weight) -- NCCL over NVLink
  3. the received rows run through the local layer (apply_exl3_fused_moe with local ids), which already
     applies the routing weights and sums over the row's local experts -> fp32 partial per row
  4. reverse all-to-all of the fp32 partials, then out[token] += partial, in rank order
With world == 1 the call is the plain single-GPU layer (no collective).

`EPMoE` takes the local expert computation as a function so the dispatch/combine bookkeeping can be
tested on CPU ranks (gloo) with a stand-in expert.
"""
from __future__ import annotations

from typing import Callable

import torch
import torch.distributed as dist


class EPMoE:
    def __init__(self, expert_fn: Callable, num_global_experts: int, group=None):
        """expert_fn(x_rows [R, H], local_ids [R, k] int64 (-1 = none), weights [R, k] fp32) -> fp32 [R, H],
        the weighted sum of the row's local experts."""
        self.expert_fn = expert_fn
        self.E = int(num_global_experts)
        self.group = group
        self.world = dist.get_world_size(group) if dist.is_initialized() else 1
        self.rank = dist.get_rank(group) if dist.is_initialized() else 0
        if self.E % self.world:
            raise ValueError(f"{self.E} experts do not shard evenly over {self.world} ranks")
        self.E_loc = self.E // self.world
        self.stats = {"sent_rows": 0, "recv_rows": 0, "a2a_bytes_out": 0, "a2a_bytes_back": 0}

    @property
    def expert_range(self):
        return self.rank * self.E_loc, (self.rank + 1) * self.E_loc

    def plan(self, ids: torch.Tensor):
        """(token index, destination rank) pairs in rank-major order and per-rank counts."""
        T, k = ids.shape
        valid = (ids >= 0) & (ids < self.E)
        dest = torch.where(valid, ids // self.E_loc, torch.full_like(ids, -1))
        mask = torch.zeros(T, self.world, dtype=torch.bool, device=ids.device)
        rows = torch.arange(T, device=ids.device).unsqueeze(1).expand(T, k)
        mask[rows[valid], dest[valid]] = True
        pairs = mask.t().nonzero()            # [S, 2] = (rank, token), rank-major, tokens ascending
        counts = mask.sum(0)                  # [world]
        return pairs[:, 1].contiguous(), pairs[:, 0].contiguous(), counts, dest

    def __call__(self, x2d: torch.Tensor, ids: torch.Tensor, weights: torch.Tensor) -> torch.Tensor:
        T, H = x2d.shape
        ids = ids.reshape(T, -1).to(torch.int64)
        weights = weights.reshape(T, ids.shape[1]).to(torch.float32)
        if self.world == 1:
            return self.expert_fn(x2d, torch.where((ids >= 0) & (ids < self.E), ids, torch.full_like(ids, -1)), weights)
        if 0 < T <= self.slot_capacity:
            return self._fixed_slots(x2d, ids, weights)
        return self._compact(x2d, ids, weights)

    # Fixed-slot dispatch for small batches: every rank pads its batch to the same `slot_capacity`
    # tokens (all ranks must use the same value, e.g. the largest decode batch a serving engine
    # captures) and every token gets a slot in every destination's block, so all split sizes are
    # equal and known: no host synchronisation (CUDA-graph capturable). The padding costs
    # slot_capacity * world rows of traffic, negligible at decode batch sizes. 0 = always compact.
    slot_capacity = 0

    def _fixed_slots(self, x2d, ids, weights):
        T0, H = x2d.shape
        k = ids.shape[1]
        T = self.slot_capacity
        if T0 < T:  # pad with tokens that have no route
            x2d = torch.cat([x2d, torch.zeros((T - T0, H), dtype=x2d.dtype, device=x2d.device)])
            ids = torch.cat([ids, torch.full((T - T0, k), -1, dtype=ids.dtype, device=ids.device)])
            weights = torch.cat([weights, torch.zeros((T - T0, k), dtype=weights.dtype, device=weights.device)])
        valid = (ids >= 0) & (ids < self.E)
        dest = torch.where(valid, ids // self.E_loc, torch.full_like(ids, -1))
        ranks = torch.arange(self.world, device=ids.device).view(self.world, 1, 1)
        own = dest.unsqueeze(0) == ranks                                   # [world, T, k]
        local = torch.where(own, ids.unsqueeze(0) - ranks * self.E_loc, torch.full_like(own, -1, dtype=torch.int64))
        meta = torch.cat([local.to(torch.int32), weights.unsqueeze(0).expand(self.world, T, k).view(torch.int32)], 2)
        send = x2d.unsqueeze(0).expand(self.world, T, H).contiguous()
        recv = torch.empty_like(send)
        recv_meta = torch.empty_like(meta)
        dist.all_to_all_single(recv.view(self.world * T, H), send.view(self.world * T, H), group=self.group)
        dist.all_to_all_single(recv_meta.view(self.world * T, 2 * k), meta.contiguous().view(self.world * T, 2 * k),
                               group=self.group)
        rm = recv_meta.view(self.world * T, 2 * k)
        part = self.expert_fn(recv.view(self.world * T, H), rm[:, :k].to(torch.int64),
                              rm[:, k:].contiguous().view(torch.float32))
        back = torch.empty((self.world, T, H), dtype=torch.float32, device=x2d.device)
        dist.all_to_all_single(back.view(self.world * T, H), part.contiguous(), group=self.group)
        self.stats["sent_rows"] += self.world * T
        self.stats["recv_rows"] += self.world * T
        self.stats["a2a_bytes_out"] += int(send.numel() * send.element_size() + meta.numel() * 4)
        self.stats["a2a_bytes_back"] += int(back.numel() * 4)
        return back.sum(0)[:T0]

    def _compact(self, x2d, ids, weights):
        T, H = x2d.shape
        tok, dst, counts, dest = self.plan(ids)
        k = ids.shape[1]
        # routes (not rows) per destination: the receiver sizes its local forward by them
        routes = torch.bincount(dest[dest >= 0], minlength=self.world)[: self.world]
        counts = torch.stack([counts, routes], 1).reshape(-1)           # [world * 2]
        # metadata of each sent row: local expert ids of the routes owned by the destination (-1 otherwise)
        r_ids = ids[tok]
        own = dest[tok] == dst.unsqueeze(1)
        local = torch.where(own, r_ids - dst.unsqueeze(1) * self.E_loc, torch.full_like(r_ids, -1))
        meta = torch.cat([local.to(torch.int32), weights[tok].view(torch.int32)], 1).contiguous()   # [S, 2k]
        send = x2d[tok].contiguous()
        # counts exchange, then the host-visible split sizes
        recv_counts = torch.empty_like(counts)
        dist.all_to_all_single(recv_counts, counts.contiguous(), group=self.group)
        both = torch.stack([counts, recv_counts]).tolist()              # one host sync
        sc, rc = both[0][0::2], both[1][0::2]
        recv_routes = int(sum(both[1][1::2]))
        R = int(sum(rc))
        recv = torch.empty((R, H), dtype=x2d.dtype, device=x2d.device)
        recv_meta = torch.empty((R, 2 * k), dtype=torch.int32, device=x2d.device)
        dist.all_to_all_single(recv, send, rc, sc, group=self.group)
        dist.all_to_all_single(recv_meta, meta, rc, sc, group=self.group)
        part = self.expert_fn(recv, recv_meta[:, :k].to(torch.int64), recv_meta[:, k:].contiguous().view(torch.float32),
                              max_routes=recv_routes)
        back = torch.empty((send.shape[0], H), dtype=torch.float32, device=x2d.device)
        dist.all_to_all_single(back, part.contiguous(), sc, rc, group=self.group)
        out = torch.zeros((T, H), dtype=torch.float32, device=x2d.device)
        out.index_add_(0, tok, back)
        self.stats["sent_rows"] += int(send.shape[0])
        self.stats["recv_rows"] += R
        self.stats["a2a_bytes_out"] += int(send.numel() * send.element_size() + meta.numel() * 4)
        self.stats["a2a_bytes_back"] += int(back.numel() * 4)
        return out


def local_layer_fn(layer, limit: float | None = 10.0, fat_threshold: int | None = None):
    """expert_fn running this rank's experts through the B200 kernels (apply_exl3_fused_moe)."""
    from .exl3 import apply_exl3_fused_moe

    def fn(x, local_ids, w, max_routes=0):
        if x.shape[0] == 0:
            return torch.zeros((0, x.shape[1]), dtype=torch.float32, device=x.device)
        return apply_exl3_fused_moe(x, local_ids, w, layer, None, None, limit, fat_threshold=fat_threshold,
                                    max_routes=max_routes)

    return fn
