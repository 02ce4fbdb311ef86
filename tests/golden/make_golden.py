"""Generate the golden vectors in tests/golden/ from the REFERENCE's own compiled code.

Runs only where the reference tree has been built into oracle/_ref/ (a machine with the reference checkout):
  * oracle/_ref/libref_shim.so      kernels/cpu_avx2/ft_core.h compiled unchanged (oracle/Makefile)
  * oracle/_ref/tier_*/ft_tier_host  kernels/cpu_avx2/ft_tier_ext.cpp (oracle/build_ref_tier.py)
Inputs come from dsv41_flash_offload_b200.synth (seeded, counter-based), so tests regenerate them
bit-identically and compare the plain-C oracle (and the GPU kernels) against these outputs.

usage: python tests/golden/make_golden.py
"""
from __future__ import annotations

import hashlib
import os
import sys

import numpy as np

ROOT = os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
sys.path.insert(0, ROOT)

from dsv41_flash_offload_b200 import synth  # noqa: E402
from oracle.oracle import RefShim, load_ref_tier  # noqa: E402

OUT = os.path.dirname(os.path.abspath(__file__))
LIMIT = 10.0  # SWIGLU_LIMIT_DEFAULT (patches/vllm-exl3-host-dma.patch:5), deployed clamp


def f16(a):
    return np.asarray(a, np.float32).astype(np.float16).astype(np.float32)


def format_fixtures(ref: RefShim):
    table = ref.weight_table().view(np.uint16)
    digest = hashlib.sha256(table.tobytes()).hexdigest()
    rng = np.random.default_rng(123)
    sample_idx = rng.choice(65536, 4096, replace=False).astype(np.int64)
    # one small matrix decoded by the reference
    k, n = 64, 128
    tr = synth.trellis_np(11, 99, 0, (k // 16) * (n // 16) * 48).reshape(k // 16, n // 16, 48)
    W = ref.dense_weights(tr, k, n).astype(np.float16)
    states = np.stack([ref.states(tr.reshape(-1, 48)[i]) for i in range(4)])
    # transforms and act
    xs = f16(synth.normal(5, 1, 16 * 128).reshape(16, 128))
    suh = np.where(synth.hash_u32(5, 2, 0, 16 * 128) & np.uint64(1), 1.0, -1.0).astype(np.float16).reshape(16, 128)
    prep = np.stack([ref.prep_block(xs[i], suh[i]) for i in range(16)])
    ys = (synth.normal(5, 3, 16 * 128) * 40).astype(np.float32).reshape(16, 128)
    svh = ((0.5 + synth.uniform01(5, 4, 0, 16 * 128)) / 64).astype(np.float16).reshape(16, 128)
    outb = np.stack([ref.out_block(ys[i], svh[i]) for i in range(16)])
    g = (synth.normal(5, 5, 4096) * 6).astype(np.float32)
    u = (synth.normal(5, 6, 4096) * 6).astype(np.float32)
    act10 = np.array([ref.act(a, b, 10.0) for a, b in zip(g, u)], np.float32)
    act0 = np.array([ref.act(a, b, 0.0) for a, b in zip(g, u)], np.float32)
    np.savez_compressed(os.path.join(OUT, "format.npz"), table_sha256=np.array(digest), sample_idx=sample_idx,
                        sample_bits=table[sample_idx], decode_trellis=tr, decode_W=W, states=states,
                        prep_x=xs, prep_suh=suh, prep_out=prep, outb_y=ys, outb_svh=svh, outb_out=outb,
                        act_g=g, act_u=u, act_10=act10, act_0=act0)
    print("format.npz: table", digest[:16])


def expert_fixture(ref: RefShim):
    H, I, e, seed = 256, 2048, 3, 0
    gate, up, down = synth.expert_trellis_np(seed, H, I, e)
    s13, v13, s2, v2 = synth.scales_np(seed, e + 1, H, I)
    x = f16(synth.hidden_np(seed, 2, H))
    args = (gate, up, down, s13[e, 0], v13[e, 0], s13[e, 1], v13[e, 1], s2[e], v2[e])
    y10 = np.stack([ref.expert(*args, x[i], 10.0) for i in range(2)])
    y0 = np.stack([ref.expert(*args, x[i], 0.0) for i in range(2)])
    np.savez_compressed(os.path.join(OUT, "expert_small.npz"), H=H, I=I, e=e, seed=seed, y_limit10=y10, y_limit0=y0)
    print("expert_small.npz")


def layer_c0_fixture(ref: RefShim):
    """4 tokens, H 4096, E 384, I 2048, top-8 softmax(N(0,1)), seed 0."""
    T, H, I, E, k, seed = 4, 4096, 2048, 384, 8, 0
    x = f16(synth.hidden_np(seed, T, H))
    ids, w = synth.routing_np(seed, T, E, k)
    s13, v13, s2, v2 = synth.scales_np(seed, E, H, I)
    used = sorted(set(ids.reshape(-1).tolist()))
    tr = {e: synth.expert_trellis_np(seed, H, I, e) for e in used}
    yr = np.zeros((T * k, H), np.float32)
    for t in range(T):
        for j in range(k):
            e = int(ids[t, j])
            gate, up, down = tr[e]
            yr[t * k + j] = ref.expert(gate, up, down, s13[e, 0], v13[e, 0], s13[e, 1], v13[e, 1], s2[e], v2[e],
                                       x[t], LIMIT)
    out = np.zeros((T, H), np.float32)
    for t in range(T):
        for j in range(k):
            out[t] += np.float32(w[t, j]) * yr[t * k + j]
    # the reference's AVX2 CPU tier on the same inputs (tier_forward, modes EXACT and auto)
    import torch

    Hx = load_ref_tier("v3")
    Hx.tier_init(1, [0], torch.zeros(16, dtype=torch.int64), torch.zeros(64 * H, dtype=torch.half),
                 torch.zeros(64 * 24, dtype=torch.int32), torch.zeros(64 * H), -1, H, I, 1, 0)
    Hx.tier_set_limit(LIMIT)
    pad = 4096 // 2
    keep = []
    dummy = torch.zeros((H // 16) * (I // 16) * 48 + pad, dtype=torch.int16)
    ptrs = torch.zeros(E, 3, dtype=torch.int64)
    for e in range(E):
        for m in range(3):
            if e in tr:
                buf = torch.zeros(tr[e][m].size + pad, dtype=torch.int16)
                buf[: tr[e][m].size] = torch.from_numpy(np.ascontiguousarray(tr[e][m]).reshape(-1))
                keep.append(buf)
                ptrs[e, m] = buf.data_ptr()
            else:
                ptrs[e, m] = dummy.data_ptr()
    sc = lambda a: torch.from_numpy(np.ascontiguousarray(a))
    Hx.tier_add_layer(0, ptrs, sc(s13[:, 0]), sc(v13[:, 0]), sc(s13[:, 1]), sc(v13[:, 1]), sc(s2), sc(v2))
    xt = torch.from_numpy(x)
    sel = torch.from_numpy(ids.astype(np.int32))
    wt = torch.from_numpy(w)
    tier_exact = Hx.tier_forward(0, xt, sel, wt, 1).numpy()
    tier_auto = Hx.tier_forward(0, xt, sel, wt, -1).numpy()
    Hx.tier_stop()
    np.savez_compressed(os.path.join(OUT, "layer_c0.npz"), T=T, H=H, I=I, E=E, k=k, seed=seed, limit=LIMIT,
                        ids=ids, weights=w, out_ref=out, tier_exact=tier_exact,
                        tier_auto=tier_auto)
    cos = float((tier_exact * out).sum() / np.sqrt((tier_exact ** 2).sum() * (out ** 2).sum()))
    print("layer_c0.npz: |out| max", float(np.abs(out).max()), "tier EXACT vs ref cos", cos,
          "max abs", float(np.abs(tier_exact - out).max()))


def permute_fixture():
    """The routing prep of apply_exl3_fused_moe (patches/vllm-exl3-host-dma.patch:204-226, 300-312),
    run as the reference's own torch ops: local ids with the n_exp sentinel, scatter_add counts,
    expert-sorted order (stable)."""
    import torch

    cases = {}
    rng = np.random.default_rng(7)
    specs = [(4, 8, 384, None), (64, 8, 384, None), (1, 8, 16, None), (300, 6, 64, "map"), (2048, 8, 384, "bad")]
    for ci, (T, k, E, kind) in enumerate(specs):
        ids = rng.integers(0, E, (T, k)).astype(np.int64)
        emap = None
        if kind == "bad":
            ids[rng.random((T, k)) < 0.05] = -1
            ids[rng.random((T, k)) < 0.05] = E + 3
        if kind == "map":
            G = 2 * E
            ids = rng.integers(0, G, (T, k)).astype(np.int64)
            emap = np.full(G, -1, np.int32)
            emap[E // 2: E // 2 + E] = np.arange(E, dtype=np.int32)
        ti = torch.from_numpy(ids)
        if emap is not None:
            m = torch.from_numpy(emap).long()
            local = torch.where((ti >= 0) & (ti < len(emap)), m[ti.clamp(0, len(emap) - 1)], torch.full_like(ti, -1))
            local = torch.where(local < 0, torch.full_like(local, E), local)
        else:
            local = torch.where((ti >= 0) & (ti < E), ti, torch.full_like(ti, E))
        local = local.reshape(-1)
        flat_token = torch.arange(T).repeat_interleave(k)
        count = torch.zeros(E + 1, dtype=torch.long).scatter_add_(0, local, torch.ones_like(local))
        order = torch.argsort(local, stable=True)
        cases[f"c{ci}_ids"] = ids
        cases[f"c{ci}_E"] = np.array(E)
        cases[f"c{ci}_map"] = emap if emap is not None else np.zeros(0, np.int32)
        cases[f"c{ci}_counts"] = count.numpy()
        cases[f"c{ci}_order"] = order.numpy().astype(np.int32)
        cases[f"c{ci}_token_sorted"] = flat_token[order].numpy().astype(np.int32)
    cases["n"] = np.array(len(specs))
    np.savez_compressed(os.path.join(OUT, "permute.npz"), **cases)
    print("permute.npz")


def main():
    ref = RefShim()
    format_fixtures(ref)
    expert_fixture(ref)
    permute_fixture()
    layer_c0_fixture(ref)


if __name__ == "__main__":
    main()
