"""The reference's CPU-tier expert call, served by the B200 kernels.

Mirrors the module API of kernels/cpu_avx2/ft_tier_ext.cpp (pybind names and argument meaning,
:235-248): tier_init / tier_add_layer / tier_forward / tier_set_mode / tier_set_band /
tier_set_limit / tier_stats / tier_start / tier_stop. In the reference those run the AVX2 expert
kernels on pinned host cores behind a GPU<->host mailbox; here every expert is resident in HBM and
tier_forward runs the same expert math on the GPU through libdsv41_b200.so (no CPU fallback).

Differences, by design:
* tier_add_layer's `ptrs` [E, 3] are device addresses of each expert's gate/up/down trellis
  (HBM), not host addresses; the scale tensors may be on the host or the device.
* `mode` (0 AFFINE, 1 EXACT, 2 I16, -1 auto in the reference, ft_core.h:937) is accepted and
  recorded; the GPU always decodes weights exactly (the reference's EXACT rounding points).
* The mailbox tensors of tier_init (ctrl, hx, picks, hout) are kept for API compatibility but
  unused: no host worker exists (tier_start only marks the tier started).
"""
from __future__ import annotations

import torch

from . import exl3

_T = None


class _Tier:
    def __init__(self, mode, H, I, nlayers, keep):
        self.mode, self.H, self.I = int(mode), int(H), int(I)
        self.layers = [None] * int(nlayers)
        self.keep = list(keep)
        self.limit = 0.0
        self.band = 0
        self.running = False
        self.stats = {"jobs": 0, "experts": 0, "tokens": 0, "empty": 0}
        self.device = torch.device("cuda", torch.cuda.current_device())


def tier_init(threads, cpus, ctrl, hx, picks, hout, mode, H, I, nlayers, swz) -> None:
    """ft_tier_ext.cpp:36-53. threads/cpus/swz are accepted for compatibility (no host pool)."""
    global _T
    if _T is not None:
        raise RuntimeError("tier already initialised")
    _T = _Tier(mode, H, I, nlayers, (ctrl, hx, picks, hout))


def tier_add_layer(li, ptrs, suh_g, svh_g, suh_u, svh_u, suh_d, svh_d) -> None:
    """ft_tier_ext.cpp:56-101: ptrs int64 [E, 3] (gate, up, down trellis device addresses),
    scales fp16 [E, H] / [E, I] (gate/up suh [E,H], svh [E,I]; down suh [E,I], svh [E,H])."""
    if _T is None:
        raise RuntimeError("init first")
    E = int(ptrs.shape[0])
    H, I = _T.H, _T.I
    dev = _T.device
    for t in (suh_g, svh_g, suh_u, svh_u, suh_d, svh_d):
        if t.dtype != torch.float16 or t.shape[0] != E:
            raise ValueError("scales: fp16 [E, .]")
    if suh_g.shape[1] != H or svh_g.shape[1] != I or suh_d.shape[1] != I or svh_d.shape[1] != H:
        raise ValueError("scale shapes")
    p = ptrs.to(device=dev, dtype=torch.int64)
    tabs = {"gate_trellis": p[:, 0].contiguous(), "up_trellis": p[:, 1].contiguous(),
            "down_trellis": p[:, 2].contiguous()}
    w13_suh = torch.stack([suh_g, suh_u], 1).to(dev).contiguous()
    w13_svh = torch.stack([svh_g, svh_u], 1).to(dev).contiguous()
    layer = exl3.Exl3MoELayer.from_pointer_tables(tabs, w13_suh, w13_svh, suh_d.to(dev).contiguous(),
                                                 svh_d.to(dev).contiguous())
    _T.layers[int(li)] = layer


def tier_forward(li, x, sel, w, mode) -> torch.Tensor:
    """ft_tier_ext.cpp:177-191: x fp32 [m, H] (fp16-valued), sel int32 [m, k] (-1 = none),
    w fp32 [m, k] -> fp32 [m, H] on x's device."""
    if _T is None or _T.layers[int(li)] is None:
        raise RuntimeError("tier_forward: layer not added")
    layer = _T.layers[int(li)]
    dev = layer.device
    xd = x.to(device=dev, dtype=torch.float32).contiguous()
    out = exl3.apply_exl3_fused_moe(xd, sel.to(device=dev, dtype=torch.int64), w.to(device=dev, dtype=torch.float32),
                                    layer, None, None, _T.limit if _T.limit > 0 else None)
    _T.stats["jobs"] += 1
    _T.stats["tokens"] += int(x.shape[0])
    _T.stats["experts"] += int((sel >= 0).sum())
    return out.to(x.device) if x.device != dev else out


def tier_set_mode(mode) -> None:
    if _T is not None:
        _T.mode = int(mode)


def tier_set_band(band) -> None:
    if _T is not None:
        _T.band = int(band)


def tier_set_limit(limit) -> None:
    """B004 SwiGLU clamp (ft_tier_ext.cpp:225); 0 = off."""
    if _T is not None:
        _T.limit = float(limit)


def tier_stats() -> list:
    """[jobs, experts, tokens, empty, busy_ns, swz_bytes] (ft_tier_ext.cpp:227-231)."""
    if _T is None:
        return []
    s = _T.stats
    return [s["jobs"], s["experts"], s["tokens"], s["empty"], 0, 0]


def tier_start(cpu0=0) -> None:
    if _T is None or _T.running:
        raise RuntimeError("init first / already running")
    _T.running = True


def tier_stop() -> None:
    global _T
    _T = None
