"""Busy-expert GEMM entry, mirroring the reference's runtime/dma_gemm.py:5-26 `run_batch`.

The reference stages a batch of host-resident experts into VRAM slots and sends the experts of that
batch with more than `cap` rows through apply_exl3_batched_fat (reconstruct + FP16 GEMM,
patches/vllm-exl3-host-dma.patch:182-201), accumulating into `out`. Here every expert is resident
in HBM, so the staging slots are unnecessary: the same experts' rows run through
libdsv41_b200.so's dsv41_expert_gemm and are accumulated into `out` the same way.

`D` keeps the reference's shape: D["batches"][batch] = (first, last) into D["h13"].cold (expert
ids); D["layer"] is the Exl3MoELayer holding the weights (it replaces the reference's `inners` +
staging tensors, which are accepted and unused).
"""
from __future__ import annotations

import ctypes as C

import torch

from . import _lib
from .exl3 import _DTYPES, _stream_ptr


def expert_gemm(layer, x: torch.Tensor, experts, counts, token_sorted: torch.Tensor, weight_sorted: torch.Tensor,
                out: torch.Tensor, limit: float | None = None) -> None:
    """out[token] += weight * expert_e(x[token]) for the rows of each listed expert.
    counts: per-expert row counts (host list/tensor, length E) of the caller's expert-sorted rows."""
    L = _lib.load()
    dev = layer.device
    E = layer._exl3_num_experts
    cnt = torch.zeros(E + 1, dtype=torch.int64)
    c = torch.as_tensor(counts, dtype=torch.int64).reshape(-1)[:E].cpu()
    cnt[: c.numel()] = c
    off = torch.zeros(E + 1, dtype=torch.int64)
    off[1:] = torch.cumsum(cnt[:E], 0)
    total = int(off[E] + cnt[E])
    ex = torch.as_tensor(list(experts), dtype=torch.int32).to(dev)
    cnt_d, off_d = cnt.to(dev), off.to(dev)
    ts = token_sorted.to(device=dev, dtype=torch.int32).contiguous()
    wsrt = weight_sorted.to(device=dev, dtype=torch.float32).contiguous()
    xx = x.contiguous()
    n = C.c_size_t()
    _lib.check(L.dsv41_expert_gemm_workspace_size(total, ex.numel(), layer._exl3_hidden_size,
                                                  layer._exl3_intermediate_local, C.byref(n)), "expert_gemm_workspace_size")
    ws = torch.zeros(n.value, dtype=torch.uint8, device=dev)
    lim = float(limit) if (limit is not None and limit > 0) else 0.0
    with torch.cuda.device(dev):
        rc = L.dsv41_expert_gemm(C.byref(layer._c), xx.data_ptr(), _DTYPES[xx.dtype], xx.shape[0], ex.data_ptr(),
                                 ex.numel(), cnt_d.data_ptr(), off_d.data_ptr(), ts.data_ptr(), wsrt.data_ptr(), total,
                                 lim, out.data_ptr(), ws.data_ptr(), ws.numel(),
                                 _stream_ptr(torch.cuda.current_stream(dev)))
    _lib.check(rc, "dsv41_expert_gemm")


def run_batch(D, st, batch, inners, counts, cap, x, token_sorted, weight_sorted, limit, out, apply_fat=None,
              use_kernel=True):
    """runtime/dma_gemm.py:5-26: the busy (> cap rows) experts of batch `batch` accumulate into out."""
    first, last = D["batches"][batch]
    h13 = D["h13"]
    cold = h13.cold if hasattr(h13, "cold") else h13["cold"]
    experts = list(cold[first:last])
    cnt = torch.as_tensor(counts).reshape(-1).tolist()
    busy = [e for e in experts if cnt[e] > cap]
    if not busy:
        return
    expert_gemm(D["layer"], x, busy, cnt, token_sorted, weight_sorted, out, limit)
