"""vLLM / vllm_exl3 plugin glue: route the engine's routed-expert MoE through the B200 kernels.

The reference plugs its CPU expert tier into vllm_exl3 by module attribute replacement
(ct/ct_vllm.py:446-456, `install(X)` with X = vllm_exl3.exl3): it swaps X.apply_exl3_fused_moe
(the function Exl3MoEMethod.apply reaches through apply_exl3_experts, patches/vllm-exl3-host-dma.patch
:496-505) and wraps X.Exl3MoEMethod.process_weights_after_loading to register every layer once its
weights are loaded. `install` here does the same two things with this package's drop-in:

  X.apply_exl3_fused_moe                    -> exl3.apply_exl3_fused_moe (same signature and
                                               return: contiguous fp32 [T, H])
  Exl3MoEMethod.process_weights_after_loading -> the original, then the layer's B200 view (pointer
                                               tables + C descriptor, exl3.as_layer) built once

The call allocates nothing after its workspace exists and never synchronises the host, so vLLM's
own CUDA-graph capture of decode steps records it; `reserve_workspace` sizes the workspace of the
capture stream up front. `DecodeGraphs` captures the layer call alone for a set of batch sizes
(the decode-call graph of a serving engine without whole-model capture).
"""
from __future__ import annotations

import importlib

import torch

from . import exl3

_ATTR = "_dsv41_b200_original"


def install(X=None, *, fat_threshold: int | None = None) -> None:
    """Patch the vllm_exl3 module `X` (default: import vllm_exl3.exl3). Idempotent; `uninstall` undoes it.
    fat_threshold overrides VLLM_EXL3_FAT_THRESHOLD for the busy-expert GEMM path."""
    if X is None:
        X = importlib.import_module("vllm_exl3.exl3")
    if getattr(X, _ATTR, None) is not None:
        return
    orig = {"fused": X.apply_exl3_fused_moe}
    method = getattr(X, "Exl3MoEMethod", None)
    if method is not None and hasattr(method, "process_weights_after_loading"):
        orig["pwal"] = method.process_weights_after_loading

        def process_weights_after_loading(self, layer, _o=orig["pwal"]):
            _o(self, layer)
            exl3.as_layer(layer)   # build the B200 view once, outside any graph capture

        method.process_weights_after_loading = process_weights_after_loading

    def apply_exl3_fused_moe(x2d, ids, weights, layer, inners=None, expert_map=None, limit=None):
        return exl3.apply_exl3_fused_moe(x2d, ids, weights, layer, inners, expert_map, limit,
                                         fat_threshold=fat_threshold)

    apply_exl3_fused_moe.__doc__ = exl3.apply_exl3_fused_moe.__doc__
    X.apply_exl3_fused_moe = apply_exl3_fused_moe
    setattr(X, _ATTR, orig)


def uninstall(X=None) -> None:
    if X is None:
        X = importlib.import_module("vllm_exl3.exl3")
    orig = getattr(X, _ATTR, None)
    if orig is None:
        return
    X.apply_exl3_fused_moe = orig["fused"]
    if "pwal" in orig:
        X.Exl3MoEMethod.process_weights_after_loading = orig["pwal"]
    setattr(X, _ATTR, None)


def reserve_workspace(max_tokens: int, topk: int, layer, stream: torch.cuda.Stream | None = None,
                      fat_threshold: int | None = None) -> None:
    """Allocate the workspace that calls of up to max_tokens tokens on `stream` (default: current) use,
    so a later CUDA-graph capture on that stream allocates nothing."""
    lay = exl3.as_layer(layer)
    stream = stream or torch.cuda.current_stream(lay.device)
    exl3._workspace(lay.device, exl3.workspace_bytes(max_tokens, topk, lay, fat_threshold), stream)


class DecodeGraphs:
    """CUDA graphs of one layer's decode call for fixed batch sizes.

    For every size T in `sizes` the call is captured once over static input/output buffers on a private
    stream. A call with t tokens replays the smallest captured T >= t after copying the inputs in; the
    t..T padding rows carry no route (ids -1), so they cost nothing and their outputs are not returned.
    Each replay writes the same static output buffer: the returned view is valid until the next call.
    """

    def __init__(self, layer, hidden_dtype=torch.bfloat16, sizes=(1, 2, 4, 8, 16, 32, 64), topk: int = 8,
                 limit: float | None = 10.0, fat_threshold: int | None = None):
        self.layer = exl3.as_layer(layer)
        self.topk, self.limit, self.fat = topk, limit, fat_threshold
        dev, H = self.layer.device, self.layer._exl3_hidden_size
        self.sizes = sorted(set(int(s) for s in sizes))
        self.stream = torch.cuda.Stream(dev)
        self.bufs, self.graphs = {}, {}
        self.stream.wait_stream(torch.cuda.current_stream(dev))
        with torch.cuda.device(dev), torch.cuda.stream(self.stream):
            reserve_workspace(self.sizes[-1], topk, self.layer, self.stream, fat_threshold)
            for T in reversed(self.sizes):
                x = torch.zeros(T, H, dtype=hidden_dtype, device=dev)
                ids = torch.full((T, topk), -1, dtype=torch.int64, device=dev)
                w = torch.zeros(T, topk, dtype=torch.float32, device=dev)
                out = torch.empty(T, H, dtype=torch.float32, device=dev)
                self._call(x, ids, w, out)   # eager once on this stream (nothing left to allocate)
                g = torch.cuda.CUDAGraph()
                with torch.cuda.graph(g, stream=self.stream):
                    self._call(x, ids, w, out)
                self.bufs[T] = (x, ids, w, out)
                self.graphs[T] = g
        torch.cuda.current_stream(dev).wait_stream(self.stream)

    def _call(self, x, ids, w, out):
        exl3.apply_exl3_fused_moe(x, ids, w, self.layer, None, None, self.limit, fat_threshold=self.fat, out=out)

    def __call__(self, x2d: torch.Tensor, ids: torch.Tensor, weights: torch.Tensor) -> torch.Tensor:
        t = x2d.shape[0]
        T = next((s for s in self.sizes if s >= t), None)
        if T is None:
            return exl3.apply_exl3_fused_moe(x2d, ids, weights, self.layer, None, None, self.limit,
                                             fat_threshold=self.fat)
        x, sid, sw, out = self.bufs[T]
        x[:t].copy_(x2d)
        sid[:t].copy_(ids.reshape(t, -1))
        sw[:t].copy_(weights.reshape(t, -1))
        if t < T:
            sid[t:].fill_(-1)
        self.graphs[T].replay()
        return out[:t]

    def close(self) -> None:
        self.graphs.clear()
        self.bufs.clear()
