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

import ctypes as C
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


class EPPeerMoE:
    """Expert parallelism over NVLink peer memory, no collective library on the data path.

    Each rank holds `layer` = its shard of E/world experts (global expert e on rank e // (E/world)).
    Construction is collective over `group` (every rank must construct with the same arguments): the
    ranks allocate one shared device buffer each, exchange CUDA IPC handles over the process group
    (host side only) and map each other's buffers. A call runs one layer step for this rank's
    T <= tokens_cap tokens: the row transform pulls each routed token row from its rank (peer loads)
    and the down pass's epilogue stores each expert output row into its token owner's receive slot
    (peer stores), ordered by step stamps in the shared buffers (bounded device waits; `read_status()`
    reports an expired wait); the combine then sums the rank's own slots. Every rank must call once per step, in the same order. No host synchronisation:
    steps of equal parity can be captured in one CUDA graph.
    """

    def __init__(self, layer, num_global_experts: int, tokens_cap: int, topk: int, group=None,
                 limit: float | None = 10.0, fat_threshold: int | None = None, wait_limit_us: int = 0):
        """wait_limit_us bounds each device-side wait for the peers' step stamps (0 = 2 s); a wait that
        runs out makes the step give up with status 1 (read_status())."""
        from . import _lib, exl3
        self.layer = layer
        self.world = dist.get_world_size(group) if dist.is_initialized() else 1
        self.rank = dist.get_rank(group) if dist.is_initialized() else 0
        if self.world > _lib.MAX_PEERS:
            raise ValueError(f"world {self.world} > {_lib.MAX_PEERS} peer ranks")
        e_here = layer._exl3_num_experts
        if num_global_experts % self.world or e_here != num_global_experts // self.world:
            raise ValueError(f"layer holds {e_here} experts; expected {num_global_experts} / {self.world}")
        self.E, self.tokens_cap, self.topk, self.group = int(num_global_experts), int(tokens_cap), int(topk), group
        self.limit = 0.0 if limit is None else float(limit)
        self.fat = exl3.FAT_EXPERT_THRESHOLD if fat_threshold is None else int(fat_threshold)
        self.device = layer.device
        self.step = 0
        L = _lib.load()
        self._L = L
        g = _lib.EpPeerGroup()
        g.rank, g.world, g.num_global_experts, g.tokens_cap = self.rank, self.world, self.E, self.tokens_cap
        g.wait_limit_us = int(wait_limit_us)
        self._g = g
        # sizes only depend on the arguments, so every rank computes the same layout
        for d in range(self.world):
            g.bases[d] = 1
        nbytes = C.c_size_t()
        with torch.cuda.device(self.device):
            _lib.check(L.dsv41_ep_peer_buffer_size(C.byref(g), C.byref(layer._c), self.topk, self.fat,
                                                   C.byref(nbytes)), "ep_peer_buffer_size")
            base = C.c_void_p()
            handle = (C.c_uint8 * _lib.IPC_HANDLE_BYTES)()
            _lib.check(L.dsv41_ep_peer_alloc(nbytes.value, C.byref(base), handle), "ep_peer_alloc")
        self.nbytes = nbytes.value
        self._own = base.value
        handles = [None] * self.world
        if self.world > 1:
            dist.all_gather_object(handles, bytes(handle), group=group)
        else:
            handles[0] = bytes(handle)
        self._opened = []
        with torch.cuda.device(self.device):
            for d in range(self.world):
                if d == self.rank:
                    g.bases[d] = self._own
                    continue
                h = (C.c_uint8 * _lib.IPC_HANDLE_BYTES).from_buffer_copy(handles[d])
                pb = C.c_void_p()
                _lib.check(L.dsv41_ep_peer_open(h, C.byref(pb)), f"ep_peer_open(rank {d})")
                g.bases[d] = pb.value
                self._opened.append(pb.value)
        if self.world > 1:
            dist.barrier(group=group)   # every buffer is mapped before any rank signals into it
        self.stats = {"steps": 0}

    def __call__(self, x2d: torch.Tensor, ids: torch.Tensor, weights: torch.Tensor, layer=None) -> torch.Tensor:
        """One step; `layer` optionally replaces the local shard for this call (another layer of the same
        shape, e.g. the next layer of a stack sharing these buffers)."""
        from . import _lib, exl3
        layer = self.layer if layer is None else layer
        if layer._exl3_num_experts != self.layer._exl3_num_experts or layer.w13_suh.shape != self.layer.w13_suh.shape \
                or layer.w13_svh.shape != self.layer.w13_svh.shape:
            raise ValueError("layer shape differs from the one the buffers were sized for")
        T, H = x2d.shape
        if T > self.tokens_cap:
            raise ValueError(f"{T} tokens > tokens_cap {self.tokens_cap}")
        ids = ids.reshape(T, -1)
        if ids.shape[1] != self.topk:
            raise ValueError(f"topk {ids.shape[1]} != {self.topk}")
        ids = ids.to(torch.int64).contiguous()
        weights = weights.reshape(T, self.topk).to(torch.float32).contiguous()
        x2d = x2d.contiguous()
        out = torch.empty((T, H), dtype=torch.float32, device=x2d.device)
        stream = torch.cuda.current_stream(x2d.device)
        with torch.cuda.device(x2d.device):
            _lib.check(self._L.dsv41_ep_peer_forward(
                C.byref(layer._c), C.byref(self._g), self.step & 0xFFFFFFFF, x2d.data_ptr(),
                exl3._DTYPES[x2d.dtype], T, ids.data_ptr(), weights.data_ptr(), self.topk, self.limit, self.fat,
                out.data_ptr(), C.c_void_p(stream.cuda_stream)), "ep_peer_forward")
        self.step += 1
        self.stats["steps"] += 1
        return out

    def read_status(self) -> int:
        """Synchronise; 0 = ok, 1 = a bounded device wait (peer stamp or pipeline) ran out."""
        st = C.c_int32()
        stream = torch.cuda.current_stream(self.device)
        with torch.cuda.device(self.device):
            from . import _lib
            _lib.check(self._L.dsv41_ep_peer_read_status(C.byref(self._g), C.byref(self.layer._c), self.topk, self.fat,
                                                         C.c_void_p(stream.cuda_stream), C.byref(st)),
                       "ep_peer_read_status")
        return st.value

    def close(self) -> None:
        """Collective: unmap the peers' buffers and free this rank's once every rank is done."""
        if self._own is None:
            return
        from . import _lib
        torch.cuda.synchronize(self.device)
        if self.world > 1:
            dist.barrier(group=self.group)
        with torch.cuda.device(self.device):
            for pb in self._opened:
                _lib.check(self._L.dsv41_ep_peer_close(C.c_void_p(pb)), "ep_peer_close")
            if self.world > 1:
                dist.barrier(group=self.group)
            _lib.check(self._L.dsv41_ep_peer_free(C.c_void_p(self._own)), "ep_peer_free")
        self._opened, self._own = [], None
