#!/usr/bin/env python
"""Benchmark of the B200 routed-expert MoE layer (BASELINE.json metric:
"MoE-layer tok/s (decode B=64, prefill 16k) @1/2/4/8 B200; % HBM/tensor peak").

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

One step = one MoE-layer forward (E 384, H 4096, I 2048, top-8, EXL3 3.0-bpw trellis words, SwiGLU
clamp 10) over one batch: the headline workload is BASELINE configs[1]'s decode batch of 64 tokens
with uniform top-8 routing (all 384 experts HBM-resident). Synthetic seeded inputs stand in for real
weights (no checkpoint): uniform random trellis words, +-1 suh, U(0.5,1.5)/64 svh, N(0,1) bf16
hidden states, softmax(N(0,1)) top-8 routing. Layers and routing batches are cycled so every step
streams ~2.7 GB of distinct routed experts' words at N=1 (inputs far larger than the 126 MB L2).

value   = tokens of all ranks / max-over-ranks device time of K steps (inputs resident in HBM)
e2e     = the same through apply_exl3_fused_moe with pinned host inputs: H2D of x/ids/weights and
          D2H of the fp32 output inside each timed step
roofline= the dominant kernel (decode-GEMV gate/up pass): algorithmic bytes (distinct routed
          experts' gate+up trellis and scales, activations in, down-input out) / its average
          duration from CUDA events on its own stream inside the timed region, against the
          measured HBM copy bandwidth (MEASURED_PEAKS.json)
sweep   = (N=1) decode T = 1/8/32/64 through the same call, timed as eager calls and as replays of
          CUDA graphs of those calls (graph_*: the serving form, without the host's per-call work)
cpu_baseline / --impl reference = the reference's own AVX2 CPU expert tier
          (kernels/cpu_avx2/ft_tier_ext.cpp tier_forward, built into oracle/_ref) on the same
          decode batches, all host cores, rank 0 only.
N > 1 (torchrun, one rank per GPU) runs the expert-parallel layer: each rank holds E/N experts and
its own 64-token batch (weak scaling); the dispatch/combine exchange is done by peer loads inside the
layer kernels (--ep peer, default) or by fixed-slot NCCL all-to-all (--ep nccl), no host sync. The same
line then carries `ep_parity` (the first batch through the peer and NCCL paths vs the single-GPU
layer of all experts on every rank; the run exits 3 if either is outside the parity bar), and `ep40` /
`prefill_ep`: BASELINE configs[3] (40-layer stack, 256-token decode batch) and configs[4] (131,072
tokens x 8 layers, Zipf(1.5); compact NCCL all-to-all, or the peer path with --prefill-exchange peer)
measured in the same process (strong scaling; --no-stack skips them).
--workload ep40 / prefill-ep run configs[3] / configs[4] alone as the line.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import tempfile
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

E, H, I, TOPK = 384, 4096, 2048, 8
LIMIT = 10.0
METRIC = "MoE-layer tok/s (decode B=64, prefill 16k) @1/2/4/8 B200; % HBM/tensor peak"
GEMV_PROFILE = "gemv_decode_T64.txt"   # ncu summary of the decode-GEMV at the headline workload
TILE_BYTES_PER_MATRIX = (H // 16) * (I // 16) * 96          # 3,145,728
EXPERT_BYTES = 3 * TILE_BYTES_PER_MATRIX + (2 * H + 2 * I + I + H) * 2   # 9,474,048 (3 weight matrices + suh/svh)


def claim_stdout():
    """Route everything written to file descriptor 1 (NCCL prints its version banner there with printf)
    to stderr, and return a writer for the saved stdout so the result line is the only thing on it."""
    sys.stdout.flush()
    saved = os.dup(1)
    os.dup2(2, 1)
    out = os.fdopen(saved, "w", buffering=1)

    def emit(obj):
        out.write(json.dumps(obj) + "\n")
        out.flush()
    return emit


EMIT = None   # set by main(): writes one JSON line to the real stdout


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=400)
    ap.add_argument("--warmup", type=int, default=10)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--tokens", type=int, default=64)
    ap.add_argument("--layers", type=int, default=4, help="layers cycled per step (defeats L2 reuse)")
    ap.add_argument("--batches", type=int, default=8)
    ap.add_argument("--no-sweep", action="store_true")
    ap.add_argument("--no-prefill", action="store_true")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--cpu-seconds", type=float, default=12.0)
    ap.add_argument("--no-stack", action="store_true",
                    help="N > 1: skip the configs[3] / configs[4] stack measurements that follow the decode line")
    ap.add_argument("--workload", choices=["decode", "prefill", "ep40", "prefill-ep"], default="decode",
                    help="decode: BASELINE configs[1] (default); prefill: configs[2] alone (one 16k-token Zipf(1.1) "
                         "batch, GEMM tensor roofline); ep40: configs[3] 40-layer stack, 256-token decode batch; "
                         "prefill-ep: configs[4] 131,072 tokens x 8 layers, Zipf(1.5)")
    ap.add_argument("--ep", choices=["peer", "nccl"], default="peer",
                    help="N > 1 decode exchange (one layer and the configs[3] stack): peer = token rows read from "
                         "peers' memory by the row transform and expert outputs stored into the token owners' memory "
                         "by the down pass (EPPeerMoE); nccl = fixed-slot NCCL all-to-all (EPMoE)")
    ap.add_argument("--prefill-exchange", choices=["nccl", "peer"], default="nccl",
                    help="N > 1 configs[4] stack exchange: nccl = compact NCCL all-to-all (EPMoE); peer = EPPeerMoE")
    ap.add_argument("--prefill-tokens", type=int, default=16384, help="--workload prefill: tokens per batch")
    ap.add_argument("--experts", type=int, default=E,
                    help="--workload prefill: experts in the layer (fewer = a smaller case for profiling)")
    return ap.parse_args()


# ------------------------------------------------------------------------------------------
# environment helpers
# ------------------------------------------------------------------------------------------
def measured_peaks():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        d = json.load(open(p))
        return float(d["hbm_gbs"]), float(d["bf16_tflops"]), float(d.get("bf16_tflops_sustained", d["bf16_tflops"])), \
            "MEASURED_PEAKS.json"
    return 6650.0, 1590.0, 1400.0, "fallback (6.65 TB/s, 1.59 PFLOP/s)"


class ClockSampler:
    """nvidia-smi clocks / throttle reasons sampled every 50 ms while running."""

    Q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,clocks_event_reasons.hw_slowdown,"
         "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,"
         "clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_id: str):
        self.f = tempfile.NamedTemporaryFile("w+", suffix=".csv", delete=False)
        try:
            self.p = subprocess.Popen(["nvidia-smi", f"--query-gpu={self.Q}", "--format=csv,noheader,nounits",
                                       "-lms", "50", "-i", gpu_id], stdout=self.f, stderr=subprocess.DEVNULL)
        except OSError:
            self.p = None

    def stop(self):
        if self.p is not None:
            self.p.terminate()
            try:
                self.p.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.p.kill()
        self.f.flush()
        rows = []
        for line in open(self.f.name):
            parts = [x.strip() for x in line.split(",")]
            if len(parts) >= 9:
                try:
                    rows.append(dict(sm=float(parts[1]), smax=float(parts[2]), power=float(parts[3]),
                                     hw=parts[5], hwt=parts[6], swt=parts[7], swp=parts[8]))
                except ValueError:
                    pass
        os.unlink(self.f.name)
        if not rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["no samples"], "samples": 0}
        load = [r for r in rows if r["power"] > 250.0] or rows
        reasons = sorted({name for r in load for name, key in (("hw_slowdown", "hw"), ("hw_thermal_slowdown", "hwt"),
                                                               ("sw_thermal_slowdown", "swt"), ("sw_power_cap", "swp"))
                          if r[key].lower().startswith("active")})
        return {"sm_mhz": statistics.median(r["sm"] for r in load), "sm_max_mhz": max(r["smax"] for r in rows),
                "reasons": reasons, "samples": len(rows), "samples_under_load": len(load),
                "power_w_max": max(r["power"] for r in rows)}


# ------------------------------------------------------------------------------------------
# workload
# ------------------------------------------------------------------------------------------
def make_batches(T, n, seed0, kind="uniform", zipf_s=1.1, num_experts=E):
    from dsv41_flash_offload_b200 import synth
    out = []
    for b in range(n):
        x = synth.hidden_np(seed0 + b, T, H)
        ids, w = synth.routing_np(seed0 + b, T, num_experts, TOPK, kind=kind, zipf_s=zipf_s)
        out.append((x, ids, w))
    return out


def to_device(batches, dev):
    import torch
    return [(torch.from_numpy(x).to(dev, torch.bfloat16), torch.from_numpy(ids).to(dev), torch.from_numpy(w).to(dev))
            for x, ids, w in batches]


def launches_per_step(T, fat):
    from dsv41_flash_offload_b200 import _lib  # noqa: F401
    N = T * TOPK
    perm = 1 if N <= 8192 else 3
    # permute, prep, 2 decode-GEMV passes, combine (+ GEMM plan and 2 tcgen05 GEMM passes when some expert
    # can exceed the busy threshold: the library skips them when T * topk <= fat)
    return perm + 1 + 2 + 1 + (3 if fat >= 0 and N > fat else 0)


def time_steps(fn, K, W, dist_on):
    """W untimed + K timed calls; device time by CUDA events on the current stream, max over ranks."""
    import torch
    for i in range(W):
        fn(i)
    torch.cuda.synchronize()
    if dist_on:
        torch.distributed.barrier()
    torch.cuda.synchronize()
    s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    s.record()
    for i in range(K):
        fn(W + i)
    e.record()
    torch.cuda.synchronize()
    ms = s.elapsed_time(e)
    if dist_on:
        t = torch.tensor([ms], device="cuda")
        torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX)
        ms = float(t.item())
        torch.distributed.barrier()
    return ms


def stage_times(fn, K, W):
    """Average per-stage device times (ms) over K calls recorded by the library's stage events."""
    import ctypes as C
    import torch
    from dsv41_flash_offload_b200 import _lib
    L = _lib.load()
    for i in range(W):
        fn(i)
    torch.cuda.synchronize()
    _lib.check(L.dsv41_set_stage_timing(1), "set_stage_timing")
    K = min(K, 256)
    for i in range(K):
        fn(W + i)
    buf = (C.c_float * (K * _lib.N_STAGES))()
    n = C.c_int32()
    _lib.check(L.dsv41_read_stage_times(buf, K, C.byref(n)), "read_stage_times")
    _lib.check(L.dsv41_set_stage_timing(0), "set_stage_timing")
    vals = list(buf)[: n.value * _lib.N_STAGES]
    return {name: sum(vals[c * _lib.N_STAGES + s] for c in range(n.value)) / max(n.value, 1)
            for s, name in enumerate(_lib.STAGE_NAMES)}


# compressed bytes one routed expert streams through the decode-GEMV (gate, up, down trellis and the
# w13_svh, w2_suh, w2_svh scales it reads; w13_suh is read by the row transform)
GEMV_EXPERT_BYTES = 3 * TILE_BYTES_PER_MATRIX + (2 * I + I + H) * 2
# activation bytes per routed row: xt_g, xt_u read; the down input written and read back; y written
GEMV_ROW_BYTES = 2 * H * 2 + I * 2 + I * 2 + H * 2


def gemv_bytes(ids, T):
    """Algorithmic bytes of one decode-GEMV launch (gate/up and down passes in one kernel): every distinct
    routed expert's words and scales once, and each routed row's activations."""
    import numpy as np
    d = len(np.unique(ids))
    return d * GEMV_EXPERT_BYTES + T * TOPK * GEMV_ROW_BYTES, d


def gemv_bytes_ep(ids_all, lo, hi):
    """gemv_bytes for the local forward of the rank owning experts [lo, hi) under expert parallelism:
    the distinct routed experts in its range and the routes it serves, over all ranks' tokens."""
    import numpy as np
    cat = np.concatenate([i.reshape(-1) for i in ids_all])
    mine = cat[(cat >= lo) & (cat < hi)]
    return len(np.unique(mine)) * GEMV_EXPERT_BYTES + mine.size * GEMV_ROW_BYTES, len(np.unique(mine))


def layer_bytes(ids, T):
    import numpy as np
    d = len(np.unique(ids))
    return d * EXPERT_BYTES + T * H * 2 + T * H * 4 + T * TOPK * 12


def traffic_ratio_from_profile():
    """DRAM bytes / algorithmic bytes of the decode-GEMV launch captured with ncu (committed summary), or
    None. Traffic per launch of this run = ratio x its algorithmic bytes per launch (the capture is the
    same kernel and shape; the bytes scale with the distinct experts a batch routes to)."""
    p = os.path.join(ROOT, "profiles", GEMV_PROFILE)
    if not os.path.exists(p):
        return None
    for line in open(p):
        if line.startswith("traffic_over_algorithmic:"):
            try:
                return float(line.split(":")[1].split()[0])
            except ValueError:
                return None
    return None


# ------------------------------------------------------------------------------------------
# reference CPU tier (cpu_baseline and the --impl reference arm)
# ------------------------------------------------------------------------------------------
def reference_cpu_tier(layer, batches, seconds, T):
    """tokens/s of the reference's AVX2 expert tier (tier_forward, mode -1 = its deployed auto mode)
    over the decode batches, all host cores."""
    import numpy as np
    import torch
    from oracle.oracle import load_ref_tier, ref_tier_path
    path = ref_tier_path()
    mod = load_ref_tier()
    ncpu = os.cpu_count() or 1
    pad = 2048  # int16 words: the AVX2 decoder reads up to 8 bytes past the last tile
    w13 = torch.empty(layer.w13_trellis.numel() + pad, dtype=torch.int16)
    w13[: layer.w13_trellis.numel()].copy_(layer.w13_trellis.reshape(-1))
    w2 = torch.empty(layer.w2_trellis.numel() + pad, dtype=torch.int16)
    w2[: layer.w2_trellis.numel()].copy_(layer.w2_trellis.reshape(-1))
    g13 = layer.w13_trellis[0].numel()
    g = layer.w13_trellis[0, 0].numel()
    g2 = layer.w2_trellis[0].numel()
    ptrs = torch.zeros(E, 3, dtype=torch.int64)
    for e in range(E):
        ptrs[e, 0] = w13.data_ptr() + 2 * (e * g13)
        ptrs[e, 1] = w13.data_ptr() + 2 * (e * g13 + g)
        ptrs[e, 2] = w2.data_ptr() + 2 * (e * g2)
    mod.tier_init(ncpu, list(range(ncpu)), torch.zeros(16, dtype=torch.int64), torch.zeros(64 * H, dtype=torch.half),
                  torch.zeros(64 * 24, dtype=torch.int32), torch.zeros(64 * H), -1, H, I, 1, 0)
    mod.tier_set_limit(LIMIT)
    cpu = lambda t: t.detach().cpu().contiguous()
    mod.tier_add_layer(0, ptrs, cpu(layer.w13_suh[:, 0]), cpu(layer.w13_svh[:, 0]), cpu(layer.w13_suh[:, 1]),
                       cpu(layer.w13_svh[:, 1]), cpu(layer.w2_suh), cpu(layer.w2_svh))
    host = [(torch.from_numpy(x.astype(np.float16).astype(np.float32)), torch.from_numpy(ids.astype(np.int32)),
             torch.from_numpy(w)) for x, ids, w in batches]
    def timed(mode, secs):
        mod.tier_forward(0, *host[0], mode)  # warm-up (page-in)
        calls, t0 = 0, time.perf_counter()
        per = []
        while True:
            x, sel, w = host[calls % len(host)]
            t1 = time.perf_counter()
            mod.tier_forward(0, x, sel, w, mode)
            per.append(time.perf_counter() - t1)
            calls += 1
            if time.perf_counter() - t0 >= secs and calls >= 3:
                break
        return calls, time.perf_counter() - t0, statistics.median(per)

    calls, total, med = timed(-1, seconds)
    # EXACT mode (per-weight fp16 decode, the mode the GPU kernels match), a shorter sample
    e_calls, e_total, e_med = timed(1, max(2.0, seconds / 3))
    mod.tier_stop()
    build = f"{os.path.basename(os.path.dirname(path))} build of kernels/cpu_avx2/ft_tier_ext.cpp"
    return {"value": round(T * calls / total, 2), "unit": "tok/s", "cores": ncpu, "kind": "reference",
            "cpu_model": cpu_model(),
            "sample": f"{calls} tier_forward calls (decode batches of {T} tokens x top-{TOPK}, mode -1 auto, "
                      f"clamp {LIMIT}) in {total:.1f} s; median {med * 1e3:.1f} ms/call; {build}",
            "exact_mode": {"value": round(T * e_calls / e_total, 2), "unit": "tok/s", "mode": 1,
                           "sample": f"{e_calls} tier_forward calls, mode 1 (EXACT), in {e_total:.1f} s; "
                                     f"median {e_med * 1e3:.1f} ms/call"}}


def cpu_model():
    """The host CPU's model name (first 'model name' line of /proc/cpuinfo) and its logical CPU count."""
    name = "unknown"
    try:
        for line in open("/proc/cpuinfo"):
            if line.startswith("model name"):
                name = line.split(":", 1)[1].strip()
                break
    except OSError:
        pass
    return f"{name} ({os.cpu_count()} logical CPUs)"


def prefill_measure(layers, dev, Tp, fat, tf_burst, tf_sus, peak_src, dist_on, n=6, num_experts=E, warm=3):
    """one Tp-token prefill batch (Zipf(1.1) top-8) through the layers in turn; the
    tensor roofline covers the two GEMM kernels (busy-expert rows only)."""
    import numpy as np
    import torch
    from dsv41_flash_offload_b200 import exl3
    hp = make_batches(Tp, 1, 3000, kind="zipf", zipf_s=1.1, num_experts=num_experts)
    bp = to_device(hp, dev)
    op = torch.empty(Tp, H, dtype=torch.float32, device=dev)

    def pstep(i):
        x, ids, w = bp[0]
        exl3.apply_exl3_fused_moe(x, ids, w, layers[i % len(layers)], None, None, LIMIT, out=op)

    pms = time_steps(pstep, n, warm, dist_on)
    pst = stage_times(pstep, 4, 1)
    flops = 2.0 * Tp * TOPK * 3 * H * I
    cnt = np.bincount(hp[0][1].reshape(-1), minlength=num_experts)
    busy_rows = int(cnt[cnt > fat].sum()) if fat >= 0 else 0
    gemm_ms = pst["gemm_gateup"] + pst["gemm_down"]
    gemm_tf = 2.0 * busy_rows * 3 * H * I / (gemm_ms / 1e3) / 1e12 if gemm_ms > 0 and busy_rows else 0.0
    return {"workload": f"prefill T={Tp}, Zipf(1.1) top-{TOPK} over {num_experts} experts"
                        + (" (BASELINE configs[2])" if Tp == 16384 and num_experts == E else ""),
            "tok_s": round(Tp * n / (pms / 1e3), 1), "ms_per_step": round(pms / n, 3),
            "layer_tflops": round(flops / (pms / n / 1e3) / 1e12, 1),
            "layer_frac_of_bf16_peak": round(flops / (pms / n / 1e3) / 1e12 / tf_burst, 4),
            "experts_over_32_rows": int((cnt > 32).sum()), "busy_rows": busy_rows,
            "max_rows": int(cnt.max()),
            "path": "decode-GEMV row groups" if fat < 0 else
                    f"tcgen05 GEMM for experts > {fat} rows, decode-GEMV for the rest",
            "roofline": {"bound": "tensor", "kernel": "exl3_gemm_kernel<0>+<1> (decode-to-smem tcgen05)",
                         "achieved": round(gemm_tf, 1), "peak": tf_burst, "unit": "TFLOP/s",
                         "frac": round(gemm_tf / tf_burst, 4), "peak_sustained": tf_sus,
                         "peak_source": f"{peak_src} bf16_tflops (cuBLAS bf16 GEMM, burst)"},
            "stage_ms": {k: round(v, 3) for k, v in pst.items()}}


def run_prefill_workload(a, world, rank, dev, dist_on, tf_burst, tf_sus, peak_src):
    """BASELINE configs[2] on its own (one GPU; other ranks run the same as replicas and only rank 0
    prints): --prefill-tokens tokens through --layers layers of --experts experts."""
    import torch
    from dsv41_flash_offload_b200 import exl3
    layers = [exl3.Exl3MoELayer.synthetic(a.experts, H, I, seed=0, layer=l, device=dev) for l in range(a.layers)]
    fat = exl3.FAT_EXPERT_THRESHOLD
    sampler = ClockSampler(gpu_uuid(dev) or str(dev.index))
    pf = prefill_measure(layers, dev, a.prefill_tokens, fat, tf_burst, tf_sus, peak_src, dist_on,
                         n=max(a.steps, 1), num_experts=a.experts, warm=max(a.warmup, 3))
    clocks = sampler.stop()
    line = {"metric": METRIC, "value": round(world * pf["tok_s"], 1), "unit": "tok/s", "n_gpus": world,
            "steps": max(a.steps, 1), "warmup": max(a.warmup, 3), "ms_per_step": pf["ms_per_step"], "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None,
            "dtype": "f16 (fp16 operands, fp32 accumulate; EXL3 3-bit weights decoded exactly)",
            "data": "synthetic (seeded random EXL3 trellis words; N(0,1) bf16 hidden; Zipf(1.1) top-8 routing)",
            "config": {"workload": pf["workload"], "layers_cycled": a.layers,
                       "parallelism": f"{world} independent replica(s)" if world > 1 else "single GPU",
                       "l2": "inputs larger than L2 (each step streams every busy expert's words and ~1 GB of rows)"},
            "roofline": pf["roofline"], "prefill": pf, "clocks": clocks}
    if rank == 0:
        EMIT(line)
    if dist_on:
        torch.distributed.barrier()
        torch.distributed.destroy_process_group()


# ------------------------------------------------------------------------------------------
def run_stack_workload(a, kind, world, rank, local, dev, dist_on, hbm, tf_burst, peak_src):
    """BASELINE configs[3] (ep40) or configs[4] (prefill-ep) as the run's own line (--workload)."""
    import torch
    uuid = gpu_uuid(dev)
    sampler = ClockSampler(uuid or str(local))
    line = stack_measure(a, kind, world, rank, dev, dist_on, hbm)
    line["clocks"] = sampler.stop()
    if rank == 0:
        EMIT(line)
    if dist_on:
        torch.distributed.barrier()
        torch.distributed.destroy_process_group()


def gpu_uuid(dev):
    import torch
    try:
        return "GPU-" + str(torch.cuda.get_device_properties(dev).uuid).replace("GPU-", "")
    except Exception:
        return None


def stack_measure(a, kind, world, rank, dev, dist_on, hbm):
    """BASELINE configs[3] (ep40) and configs[4] (prefill-ep): a stack of MoE layers, experts sharded
    E/world per rank (expert parallel) -- world 1 runs the same stack on one GPU. Total tokens are fixed
    (strong scaling) and split evenly over the ranks; the next layer's input is the residual
    x + moe(x). Returns the measurement as a bench line (every rank takes the same collective steps)."""
    import numpy as np
    import torch
    from dsv41_flash_offload_b200 import exl3, synth
    from dsv41_flash_offload_b200.ep import EPMoE, EPPeerMoE, local_layer_fn

    n_layers, total, zipf = (40, 256, None) if kind == "ep40" else (8, 131072, 1.5)
    T = total // world
    e_loc = E // world
    lo, hi = rank * e_loc, (rank + 1) * e_loc
    layers = [exl3.Exl3MoELayer.synthetic(E, H, I, seed=0, layer=l, device=dev,
                                          expert_range=(lo, hi) if world > 1 else None) for l in range(n_layers)]
    # decode stack: peer-memory exchange (--ep; one set of shared buffers for all layers); prefill stack:
    # --prefill-exchange, NCCL all-to-all with compact (deduplicated) dispatch by default. Measured at N=2
    # (131,072 tokens, 8 layers): NCCL 376.6 ms per step, peer 395.5 ms -- the peer path moves every route's
    # token row (4.2M routes served per rank) where the compact dispatch sends each token once per rank (1.05M)
    exchange = a.ep if kind == "ep40" else a.prefill_exchange
    peer = EPPeerMoE(layers[0], E, T, TOPK, limit=LIMIT) if world > 1 and exchange == "peer" else None
    eps = [] if peer is not None else [EPMoE(local_layer_fn(lay, LIMIT), E) for lay in layers]
    if kind == "ep40":
        for ep in eps:
            ep.slot_capacity = T  # decode batches: fixed-slot dispatch, no host synchronisation
    g = torch.Generator(device=dev).manual_seed(7000 + rank)
    x0 = torch.randn(T, H, generator=g, device=dev).to(torch.bfloat16)

    def route_np(r, l):
        return synth.routing_np(9000 + 100 * r + l, T, E, TOPK, kind="zipf" if zipf else "uniform", zipf_s=zipf or 1.1)

    routes_np = [route_np(rank, l) for l in range(n_layers)]
    routes = [(torch.from_numpy(ids).to(dev), torch.from_numpy(w).to(dev)) for ids, w in routes_np]

    def step(i):
        x = x0
        for l in range(n_layers):
            ids, w = routes[l]
            y = peer(x, ids, w, layer=layers[l]) if peer is not None else eps[l](x, ids, w)
            x = (x.float() + y).to(torch.bfloat16)
        return x

    steps, warm = (max(1, min(a.steps, 10)) if kind == "ep40" else max(1, min(a.steps, 3))), 3
    ms = time_steps(step, steps, warm, dist_on)
    for e in eps:
        e.stats = {k: 0 for k in e.stats}
    st = stage_times(step, 1, 0)  # one step, per-stage times averaged over its layers' local forwards
    local_ms = sum(st.values()) * n_layers
    if peer is not None:   # the exchange waits sit inside the permute and combine stages
        local_ms -= (st.get("permute", 0.0) + st.get("combine", 0.0)) * n_layers
    recv = sum(e.stats["recv_rows"] for e in eps)
    a2a = sum(e.stats["a2a_bytes_out"] + e.stats["a2a_bytes_back"] for e in eps)
    # every rank's routing of every layer is regenerated here from its seed (no collective needed): the
    # routes each rank serves and the gate/up decode-GEMV bytes of this rank's local forwards
    if kind == "ep40":
        all_ids = [[route_np(r, l)[0] for r in range(world)] for l in range(n_layers)]
        gu = [gemv_bytes_ep(all_ids[l], lo, hi)[0] for l in range(n_layers)]
        gemv_ms = st["gemv"] + st["gemv_down"]
        gemv_frac = statistics.mean(gu) / (gemv_ms / 1e3) / 1e9 / hbm if gemv_ms > 0 else None
    else:
        gemv_frac = None
    if peer is not None:
        # routes each rank serves (summed over all ranks' tokens and all layers) and the bytes this rank
        # moves: token rows of the routes it serves + expert outputs of its own valid routes (each rank
        # counts where its own routes go; one all-gather of the counts)
        mine = np.zeros(world)
        own = 0
        for ids_l, _ in routes_np:
            v = ids_l.reshape(-1)
            v = v[(v >= 0) & (v < E)]
            mine += np.bincount(v // e_loc, minlength=world)[:world]
            own += int(v.size)
        cnt = torch.tensor(mine, dtype=torch.float64, device=dev)
        cnts = [torch.zeros_like(cnt) for _ in range(world)]
        torch.distributed.all_gather(cnts, cnt)
        recv = float(sum(float(c[rank]) for c in cnts))
        a2a = (recv + own) * H * 2
        peer.close()
    t = torch.tensor([recv, a2a, local_ms], dtype=torch.float64, device=dev)
    allv = [torch.zeros_like(t) for _ in range(world)]
    if dist_on:
        torch.distributed.all_gather(allv, t)
    else:
        allv = [t]
    rows = [float(v[0]) for v in allv]
    value = total * steps / (ms / 1e3)
    line = {"metric": METRIC, "value": round(value, 1), "unit": "tok/s", "n_gpus": world, "steps": steps,
            "warmup": warm, "ms_per_step": round(ms / steps, 3), "higher_is_better": True, "scaling": "strong",
            "vs_baseline": None, "dtype": "f16 (fp16 operands, fp32 accumulate; EXL3 3-bit weights decoded exactly)",
            "data": "synthetic (seeded random EXL3 trellis words; N(0,1) bf16 hidden; routing "
                    + ("Zipf(1.5)" if zipf else "softmax(N(0,1))") + " top-8)",
            "config": {"workload": (f"BASELINE configs[3]: {n_layers}-layer MoE stack E={E} H={H} I={I} top-{TOPK}, "
                                    f"decode batch {total} tokens" if kind == "ep40" else
                                    f"BASELINE configs[4]: {total} tokens through {n_layers} MoE layers, Zipf(1.5) "
                                    "routing"),
                       "parallelism": (f"expert parallel over {world} GPU(s), {e_loc} experts each, {T} tokens per "
                                       "GPU, " + ("dispatch/combine by peer loads inside the layer kernels (no NCCL)"
                                                  if peer is not None else "NCCL all-to-all dispatch/combine"))
                                      if world > 1 else "single GPU",
                       "l2": "inputs larger than L2 (every step streams the routed experts of all layers)"},
            "layer_tok_s": round(value * n_layers, 1),
            "ep": {"exchange": "peer memory" if peer is not None else "NCCL all-to-all",
                   ("routes_served_per_gpu_per_step" if peer is not None else "rows_per_gpu_per_step"):
                       [round(r, 1) for r in rows],
                   "max_over_mean_rows": round(max(rows) / max(statistics.mean(rows), 1e-9), 3),
                   ("peer_bytes_per_step" if peer is not None else "a2a_bytes_per_step"):
                       [round(float(v[1])) for v in allv],
                   "local_moe_ms_per_step": [round(float(v[2]), 3) for v in allv],
                   "a2a_and_dispatch_share": round(max(0.0, 1.0 - max(float(v[2]) for v in allv) / (ms / steps)), 4)}}
    if gemv_frac is not None:
        line["ep"]["gemv_hbm_frac_rank0_layers"] = round(gemv_frac, 4)
    del layers, eps, routes
    torch.cuda.synchronize()
    torch.cuda.empty_cache()
    return line


def main():
    global EMIT
    a = parse()
    EMIT = claim_stdout()
    import torch

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    dist_on = world > 1
    if dist_on:
        import datetime
        torch.cuda.set_device(local)
        torch.distributed.init_process_group("nccl", timeout=datetime.timedelta(seconds=300),
                                             device_id=torch.device("cuda", local))
    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    T = a.tokens
    hbm, tf_burst, tf_sus, peak_src = measured_peaks()

    if a.impl == "reference":
        if rank != 0:
            if dist_on:
                torch.distributed.destroy_process_group()
            return
        from dsv41_flash_offload_b200.exl3 import Exl3MoELayer
        try:
            layer = Exl3MoELayer.synthetic(E, H, I, seed=0, layer=0, device=dev)
            batches = make_batches(T, a.batches, 1000)
            cb = reference_cpu_tier(layer, batches, max(a.cpu_seconds, 5.0), T)
        except FileNotFoundError as exc:
            EMIT({"impl": "reference", "unavailable": f"reference CPU tier not built: {exc}"})
            return
        EMIT({"metric": METRIC, "value": cb["value"], "unit": "tok/s", "n_gpus": a.gpus, "steps": a.steps,
                          "warmup": a.warmup, "ms_per_step": round(1e3 * T / cb["value"], 4), "higher_is_better": True,
                          "scaling": "weak", "vs_baseline": None, "dtype": "f32", "impl": "reference",
                          "data": "synthetic (seeded random EXL3 trellis words; N(0,1) hidden; softmax top-8 routing)",
                          "config": {"workload": f"decode T={T}: one MoE layer E={E} H={H} I={I} top-{TOPK}, uniform "
                                                 f"routing, reference AVX2 CPU tier on host cores"},
                          "cpu_baseline": cb, "e2e": {"value": cb["value"], "unit": "tok/s", "h2d_bytes_per_step": 0,
                                                      "d2h_bytes_per_step": 0}})
        if dist_on:
            torch.distributed.destroy_process_group()
        return

    if a.workload == "prefill":
        return run_prefill_workload(a, world, rank, dev, dist_on, tf_burst, tf_sus, peak_src)
    if a.workload != "decode":
        return run_stack_workload(a, a.workload, world, rank, local, dev, dist_on, hbm, tf_burst, peak_src)

    from dsv41_flash_offload_b200 import exl3
    from dsv41_flash_offload_b200.ep import EPMoE, EPPeerMoE, local_layer_fn
    e_loc = E // world
    lo, hi = rank * e_loc, (rank + 1) * e_loc
    # N > 1: expert parallelism -- this rank holds experts [lo, hi) of every layer and its own tokens
    layers = [exl3.Exl3MoELayer.synthetic(E, H, I, seed=0, layer=l, device=dev,
                                          expert_range=(lo, hi) if world > 1 else None) for l in range(a.layers)]
    peer = EPPeerMoE(layers[0], E, T, TOPK, limit=LIMIT) if world > 1 and a.ep == "peer" else None
    eps = [EPMoE(local_layer_fn(lay, LIMIT), E) for lay in layers] if world > 1 and peer is None else None
    for ep in eps or []:
        ep.slot_capacity = T  # every rank runs T-token decode batches: fixed-slot dispatch
    all_batches = [make_batches(T, a.batches, 1000 + 100 * r) for r in range(world)]
    host_batches = all_batches[rank]
    batches = to_device(host_batches, dev)
    out = torch.empty(T, H, dtype=torch.float32, device=dev)
    fat = exl3.FAT_EXPERT_THRESHOLD

    def forward(i, x, ids, w, o):
        if peer is not None:
            o.copy_(peer(x, ids, w, layer=layers[i % len(layers)]))
        elif eps is None:
            exl3.apply_exl3_fused_moe(x, ids, w, layers[i % len(layers)], None, None, LIMIT, out=o)
        else:
            o.copy_(eps[i % len(eps)](x, ids, w))

    def step(i):
        x, ids, w = batches[i % len(batches)]
        forward(i, x, ids, w, out)

    uuid = gpu_uuid(dev)
    # clocks are sampled from the first timed step through the end-to-end timed steps (two timed
    # regions of K steps and the stage-timing pass between them): short steps at large N leave too
    # few 50 ms samples inside one region alone
    sampler = ClockSampler(uuid or str(local))
    ms = time_steps(step, a.steps, a.warmup, dist_on)
    value = world * T * a.steps / (ms / 1e3)

    # dominant kernel: per-stage events over the same steps
    st = stage_times(step, a.steps, 2)
    if world == 1:
        gb = [gemv_bytes(ids, T) for _, ids, _ in host_batches]
        lb = [layer_bytes(ids, T) for _, ids, _ in host_batches]
    else:
        # what this rank's local forward streams: the distinct experts of [lo, hi) routed by any rank's
        # tokens in that step, and the (token, rank) rows it receives
        gb, lb = [], []
        for b in range(a.batches):
            ids_all = [all_batches[r][b][1] for r in range(world)]
            gb.append(gemv_bytes_ep(ids_all, lo, hi))
            rows = sum(int(((i >= lo) & (i < hi)).any(axis=1).sum()) for i in ids_all)
            lb.append(gb[-1][1] * EXPERT_BYTES + rows * H * 6 + rows * TOPK * 12)
    if eps is not None:
        for e in eps:
            e.stats = {k: 0 for k in e.stats}
    bytes_gu = statistics.mean(b for b, _ in gb)
    distinct = statistics.mean(d for _, d in gb)
    gemv_ms = st["gemv"] + st["gemv_down"]   # one launch with split 1 (gemv_down is then empty)
    achieved = bytes_gu / (gemv_ms / 1e3) / 1e9
    layer_gbs = statistics.mean(lb) / (ms / a.steps / 1e3) / 1e9
    ratio = traffic_ratio_from_profile() if world == 1 else None  # the committed capture is the N=1 workload
    traffic = round(ratio * bytes_gu) if ratio else None

    # end to end through the public API with pinned host buffers
    hb = [(torch.from_numpy(x).to(torch.bfloat16).pin_memory(), torch.from_numpy(ids).pin_memory(),
           torch.from_numpy(w).pin_memory()) for x, ids, w in host_batches]
    dx, dids, dw = (torch.empty_like(t, device=dev) for t in hb[0])
    out_host = torch.empty(T, H, dtype=torch.float32).pin_memory()

    def e2e_step(i):
        x, ids, w = hb[i % len(hb)]
        dx.copy_(x, non_blocking=True)
        dids.copy_(ids, non_blocking=True)
        dw.copy_(w, non_blocking=True)
        forward(i, dx, dids, dw, out)
        out_host.copy_(out, non_blocking=True)

    e2e_ms = time_steps(e2e_step, a.steps, a.warmup, dist_on)
    clocks = sampler.stop()
    clocks["window"] = "timed steps, stage-timing pass and end-to-end timed steps"
    e2e_val = world * T * a.steps / (e2e_ms / 1e3)
    h2d = hb[0][0].numel() * 2 + hb[0][1].numel() * 8 + hb[0][2].numel() * 4

    line = {
        "metric": METRIC, "value": round(value, 1), "unit": "tok/s", "n_gpus": world, "steps": a.steps,
        "warmup": a.warmup, "ms_per_step": round(ms / a.steps, 5), "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "f16 (fp16 operands, fp32 accumulate; EXL3 3-bit weights decoded exactly)",
        "data": "synthetic (seeded random EXL3 trellis words, +-1 suh, U(0.5,1.5)/64 svh; N(0,1) bf16 hidden; "
                "softmax(N(0,1)) top-8 routing)",
        "config": {"workload": f"decode T={T}: one MoE layer E={E} H={H} I={I} top-{TOPK} SwiGLU clamp {LIMIT}, "
                               f"uniform routing, all experts HBM-resident (BASELINE configs[1])",
                   "layers_cycled": a.layers, "routing_batches": a.batches,
                   "l2": "inputs larger than L2: each step streams the distinct routed experts' words "
                         f"(~{statistics.mean(lb) / 1e9:.2f} GB), layers and batches cycled",
                   "parallelism": (f"expert parallel over {world} GPUs ({e_loc} experts each, {T} tokens per GPU), "
                                   "NCCL all-to-all dispatch/combine") if world > 1 else "single GPU",
                   "fat_threshold": fat},
        "roofline": {"bound": "hbm", "kernel": "exl3_gemv_kernel (decode-GEMV: gate/up + SwiGLU + down, one launch)",
                     "achieved": round(achieved, 1), "peak": hbm, "unit": "GB/s", "frac": round(achieved / hbm, 4),
                     "traffic": traffic, "traffic_source": f"profiles/{GEMV_PROFILE} DRAM/algorithmic "
                     f"ratio {ratio} x bytes_per_launch" if ratio else None,
                     "peak_source": f"{peak_src} hbm_gbs (copy bandwidth)",
                     "bytes_per_launch": round(bytes_gu), "distinct_experts_per_step": round(distinct, 1),
                     "avg_launch_ms": round(gemv_ms, 5)},
        "layer_hbm": {"achieved_gbs": round(layer_gbs, 1), "frac": round(layer_gbs / hbm, 4),
                      "bytes_per_step": round(statistics.mean(lb))},
        "stage_ms": {k: round(v, 5) for k, v in st.items()},
        "e2e": {"value": round(e2e_val, 1), "unit": "tok/s", "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": T * H * 4},
        "gpu_launches": a.steps * (launches_per_step(world * T, fat) + 4 if peer is not None else launches_per_step(T, fat)),
        "clocks": clocks,
    }
    if peer is not None:
        # bytes pulled over NVLink per step by this rank: the token rows of the routes it serves (row
        # transform) and the expert outputs of its own valid routes (combine)
        pulled = []
        for b in range(a.batches):
            ids_all = [all_batches[r][b][1] for r in range(world)]
            rows = sum(int(((i >= lo) & (i < hi)).sum()) for i in ids_all)
            own = int(((ids_all[rank] >= 0) & (ids_all[rank] < E)).sum())
            pulled.append((rows + own) * H * 2)
        exch = st.get("permute", 0.0) + st.get("combine", 0.0)
        line["ep"] = {"mode": "peer memory (EPPeerMoE): rows pulled by the row transform, outputs by the combine",
                      "experts_per_gpu": e_loc, "peer_bytes_per_step": round(statistics.mean(pulled)),
                      "step_ms": round(ms / a.steps, 5),
                      "exchange_stages_ms": {"publish_gather_permute": round(st.get("permute", 0.0), 5),
                                             "combine_pull": round(st.get("combine", 0.0), 5)},
                      "exchange_and_permute_share": round(min(1.0, exch / (ms / a.steps)), 4)}
        line["config"]["parallelism"] = (f"expert parallel over {world} GPUs ({e_loc} experts each, {T} tokens per "
                                         "GPU), dispatch/combine by peer loads inside the layer kernels (no NCCL)")
    if eps is not None:
        calls = a.warmup + a.steps  # the e2e pass, counted since the stats were reset
        sent = sum(e.stats["sent_rows"] for e in eps) / calls
        a2a = sum(e.stats["a2a_bytes_out"] + e.stats["a2a_bytes_back"] for e in eps) / calls
        local_ms = sum(v for v in st.values())
        line["ep"] = {"experts_per_gpu": e_loc, "rows_sent_per_step": round(sent, 1),
                      "a2a_bytes_per_step": round(a2a), "local_moe_ms": round(local_ms, 5),
                      "step_ms": round(ms / a.steps, 5),
                      "a2a_and_dispatch_share": round(max(0.0, 1.0 - local_ms / (ms / a.steps)), 4)}

    parity_ok = True
    if world > 1:
        line["ep_parity"] = ep_parity_check(peer, layers, batches, dev, world, T)
        parity_ok = line["ep_parity"]["ok"]
        if peer is not None:
            peer.close()
        if not a.no_stack:
            # BASELINE configs[3] and configs[4] in the same run (strong scaling); the decode layers go first
            del layers, eps, peer, forward, step, e2e_step
            torch.cuda.synchronize()
            torch.cuda.empty_cache()
            for key, kind in (("ep40", "ep40"), ("prefill_ep", "prefill-ep")):
                sl = stack_measure(a, kind, world, rank, dev, dist_on, hbm)
                line[key] = {"workload": sl["config"]["workload"], "parallelism": sl["config"]["parallelism"],
                             "tok_s": sl["value"], "ms_per_step": sl["ms_per_step"], "steps": sl["steps"],
                             "warmup": sl["warmup"], "scaling": "strong", "layer_tok_s": sl["layer_tok_s"],
                             "ep": sl["ep"]}

    if not a.no_sweep and world == 1:
        sweep = {}
        for Ts in (1, 8, 32, 64):
            hbs = make_batches(Ts, 4, 2000 + Ts)
            bs = to_device(hbs, dev)
            o2 = torch.empty(Ts, H, dtype=torch.float32, device=dev)

            def sstep(i, bs=bs, o2=o2):
                x, ids, w = bs[i % len(bs)]
                exl3.apply_exl3_fused_moe(x, ids, w, layers[i % len(layers)], None, None, LIMIT, out=o2)

            n = 100
            sms = time_steps(sstep, n, 5, dist_on)
            sst = stage_times(sstep, 64, 2)
            # the same calls replayed from CUDA graphs (the serving form: vLLM captures its decode steps),
            # i.e. without the host's per-call work between the launches
            gstream = torch.cuda.Stream(dev)
            gstream.wait_stream(torch.cuda.current_stream(dev))
            graphs = []
            with torch.cuda.stream(gstream):
                for b in range(len(bs)):
                    sstep(b)   # eager once on this stream: sizes its workspace before the capture
                    g = torch.cuda.CUDAGraph()
                    with torch.cuda.graph(g, stream=gstream):
                        sstep(b)
                    graphs.append(g)
            torch.cuda.current_stream(dev).wait_stream(gstream)
            gms = time_steps(lambda i, gs=graphs: gs[i % len(gs)].replay(), n, 5, dist_on)
            del graphs
            lbs = statistics.mean(layer_bytes(ids, Ts) for _, ids, _ in hbs)
            gbs = statistics.mean(gemv_bytes(ids, Ts)[0] for _, ids, _ in hbs)
            sweep[str(Ts)] = {"tok_s": round(world * Ts * n / (sms / 1e3), 1), "ms_per_step": round(sms / n, 5),
                              "graph_tok_s": round(world * Ts * n / (gms / 1e3), 1),
                              "graph_ms_per_step": round(gms / n, 5),
                              "layer_hbm_frac": round(lbs / (sms / n / 1e3) / 1e9 / hbm, 4),
                              "gemv_hbm_frac": round(gbs / ((sst["gemv"] + sst["gemv_down"]) / 1e3) / 1e9 / hbm, 4)}
        line["sweep"] = sweep

    if not a.no_prefill and world == 1:
        line["prefill"] = prefill_measure(layers, dev, 16384, fat, tf_burst, tf_sus, peak_src, dist_on)

    if rank == 0 and world == 1 and not a.no_cpu_baseline:
        try:
            line["cpu_baseline"] = reference_cpu_tier(layers[0], host_batches, a.cpu_seconds, T)
        except FileNotFoundError as exc:
            line["cpu_baseline"] = {"value": None, "unavailable": str(exc)}

    if rank == 0:
        EMIT(line)
    if dist_on:
        torch.distributed.barrier()
        torch.distributed.destroy_process_group()
    if not parity_ok:
        sys.stderr.write(f"expert-parallel output outside the parity bar: {line.get('ep_parity')}\n")
        sys.exit(3)


def ep_parity_check(peer, layers, batches, dev, world, T):
    """Expert-parallel output of this run's first routing batch (layer 0) through the peer-memory path
    (when it is the one timed) and through the NCCL fixed-slot path, against the single-GPU layer of all
    E experts -- the layer the GPU tests pin to the oracle -- on every rank. Max-abs and cosine are
    reduced over the ranks (max / min). Bar: max-abs 2e-2, cosine 0.9999."""
    import torch
    from dsv41_flash_offload_b200 import exl3
    from dsv41_flash_offload_b200.ep import EPMoE, local_layer_fn
    full = exl3.Exl3MoELayer.synthetic(E, H, I, seed=0, layer=0, device=dev)
    x, ids, w = batches[0]
    ref = exl3.apply_exl3_fused_moe(x, ids, w, full, None, None, LIMIT)
    nccl = EPMoE(local_layer_fn(layers[0], LIMIT), E)
    nccl.slot_capacity = T
    outs = {"nccl_fixed_slots": nccl(x, ids, w)}
    if peer is not None:
        outs["peer_memory"] = peer(x, ids, w, layer=layers[0])
    res = {}
    for name, out in sorted(outs.items()):
        d = (out - ref).abs().max().double()
        r, o = ref.double().reshape(-1), out.double().reshape(-1)
        cos = (r @ o) / torch.sqrt(torch.clamp((r @ r) * (o @ o), min=1e-300))
        v = torch.stack([d, -cos]).reshape(2)
        torch.distributed.all_reduce(v, op=torch.distributed.ReduceOp.MAX)
        res[name] = {"max_abs": float(v[0]), "cos": round(-float(v[1]), 8)}
    st = torch.tensor([exl3.read_status(device=dev) + (peer.read_status() if peer is not None else 0)],
                      device=dev)
    torch.distributed.all_reduce(st, op=torch.distributed.ReduceOp.MAX)
    ok = all(r["max_abs"] <= 2e-2 and r["cos"] >= 0.9999 for r in res.values()) and int(st.item()) == 0
    del full, ref, outs
    torch.cuda.empty_cache()
    return {**res, "tokens": world * T, "reference": "single-GPU layer of all 384 experts (oracle-pinned)",
            "tolerance": {"max_abs": 2e-2, "cos": 0.9999}, "status": int(st.item()), "ok": ok}


if __name__ == "__main__":
    main()
