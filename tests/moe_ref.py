"""Helpers that run the CPU oracle on exactly the tensors a GPU layer holds (test infrastructure)."""
import numpy as np
import torch


def layer_numpy_scales(layer):
    return tuple(t.detach().cpu().numpy() for t in (layer.w13_suh, layer.w13_svh, layer.w2_suh, layer.w2_svh))


def oracle_out(oracle, layer, x, ids, w, limit=0.0, expert_map=None, per_route=False):
    """Oracle MoE output for a GPU Exl3MoELayer (copies only the routed experts' words back)."""
    E = layer._exl3_num_experts
    ids_np = ids.detach().cpu().numpy().astype(np.int64)
    emap = None if expert_map is None else expert_map.detach().cpu().numpy().astype(np.int32)
    used = set()
    for i in ids_np.reshape(-1).tolist():
        if emap is not None:
            if 0 <= i < len(emap) and 0 <= emap[i] < E:
                used.add(int(emap[i]))
        elif 0 <= i < E:
            used.add(int(i))
    gate, up, down = [None] * E, [None] * E, [None] * E
    for e in sorted(used):
        gate[e] = layer.w13_trellis[e, 0].cpu().numpy()
        up[e] = layer.w13_trellis[e, 1].cpu().numpy()
        down[e] = layer.w2_trellis[e].cpu().numpy()
    s13, v13, s2, v2 = layer_numpy_scales(layer)
    xf = x.detach().to(torch.float16).float().cpu().numpy()
    wn = None if w is None else w.detach().float().cpu().numpy()
    prev = oracle.bits
    oracle.set_bits(getattr(layer, "bits", 3))
    try:
        return oracle.moe_layer(xf, ids_np, wn, gate, up, down, s13, v13, s2, v2, limit=limit, expert_map=emap,
                                per_route=per_route)
    finally:
        oracle.set_bits(prev)
