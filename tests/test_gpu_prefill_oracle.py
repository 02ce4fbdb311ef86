"""BASELINE configs[2] and configs[4] batches through apply_exl3_fused_moe, checked against the oracle.

one prefill chunk of 16,384 tokens, Zipf(1.1) top-8 over E=384 (H 4096, I 2048) -- the
bench's own batch (seed 3000). configs[4]: one of its layers, 131,072 tokens with Zipf(1.5) routing
(seed 9000). Both run whole, with the deployed busy-expert threshold of 32 rows
(docker/entrypoint.sh:69 of the reference), so every pass of the tcgen05 GEMM plan runs exactly as in
the benchmark: the hottest expert's dozens of row passes, two-pass experts, ~100-row experts, and the
decode-GEMV experts at or under the threshold.

The CPU oracle cannot recompute 130k-1M routes (50 MFLOP each) in a test, so the check samples routes:
the routing ids stay as generated (the GPU's work lists are unchanged), and the routing weights are
replaced by 1 on one sampled route per sampled token and 0 elsewhere. Each sampled token's output row
then equals that route's expert output, which the oracle computes for exactly those rows
(kernels/cpu_avx2/ft_core.h:994-1011 restated in oracle/exl3_oracle.c). Samples include the first and
last row of every chosen expert and the rows on both sides of each GEMM pass boundary (256 rows per
gate/up pass, 512 per down pass)."""
from concurrent.futures import ThreadPoolExecutor

import numpy as np
import pytest
import torch

from conftest import assert_close_layer
from dsv41_flash_offload_b200 import exl3, synth

pytestmark = pytest.mark.gpu
DEV = "cuda:0"
E, H, I, K = 384, 4096, 2048, 8
LIMIT = 10.0
FAT = 32


@pytest.fixture(scope="module")
def layer_full():
    return exl3.Exl3MoELayer.synthetic(E, H, I, seed=0, device=DEV)


def _sample_positions(n, want):
    """Row positions (in expert-sorted order) to check for an expert with n rows: first/last, both sides
    of every 256- and 512-row pass boundary, and evenly spaced rows, at most `want` in all."""
    pos = {0, n - 1}
    for b in range(256, n, 256):
        pos.update((b - 1, b))
    pos = sorted(p for p in pos if 0 <= p < n)
    if len(pos) > want:   # keep the ends and spread the rest over the boundaries
        keep = np.linspace(0, len(pos) - 1, want).round().astype(int)
        pos = [pos[i] for i in sorted(set(keep.tolist()))]
    extra = want - len(pos)
    if extra > 0:
        pos = sorted(set(pos) | set(np.linspace(0, n - 1, extra + 2).round().astype(int).tolist()))
    return pos


def _choose_experts(counts):
    """The hottest expert, a two-pass expert (257-512 rows), four ~100-row experts and two experts at or
    under the busy threshold (decode-GEMV path), where the batch has them."""
    order = np.argsort(-counts, kind="stable")
    chosen = [(int(order[0]), 48)]
    two = [e for e in order if 257 <= counts[e] <= 512]
    if two:
        chosen.append((int(two[0]), 16))
    hundred = sorted((e for e in order if 64 <= counts[e] <= 160), key=lambda e: abs(int(counts[e]) - 100))
    chosen += [(int(e), 6) for e in hundred[:4]]
    small = [e for e in order[::-1] if 0 < counts[e] <= FAT]
    chosen += [(int(e), 3) for e in small[:2]]
    return chosen


def _check_sampled_routes(oracle, layer, T, seed, zipf_s, want_kinds):
    x_np = synth.hidden_np(seed, T, H)
    ids_np, _ = synth.routing_np(seed, T, E, K, kind="zipf", zipf_s=zipf_s)
    counts = np.bincount(ids_np.reshape(-1), minlength=E)
    chosen = _choose_experts(counts)
    kinds = {"hot": counts[chosen[0][0]] > 2048, "two_pass": any(257 <= counts[e] <= 512 for e, _ in chosen),
             "gemv": any(counts[e] <= FAT for e, _ in chosen)}
    for k in want_kinds:
        assert kinds[k], f"batch lacks a {k} expert: {kinds}"
    flat = ids_np.reshape(-1)
    sel_w = np.zeros((T, K), np.float32)
    used = np.zeros(T, bool)
    picks = {}   # expert -> token list (sorted-row order)
    for e, want in chosen:
        routes = np.flatnonzero(flat == e)             # flat route order = the expert's sorted-row order
        toks = []
        for p in _sample_positions(len(routes), want):
            t, j = divmod(int(routes[p]), K)
            if used[t]:
                continue
            used[t] = True
            sel_w[t, j] = 1.0
            toks.append(t)
        picks[e] = toks
    x = torch.from_numpy(x_np).to(DEV, torch.bfloat16)
    ids = torch.from_numpy(ids_np).to(DEV)
    w = torch.from_numpy(sel_w).to(DEV)
    ws = torch.empty(exl3.workspace_bytes(T, K, layer, fat_threshold=FAT), dtype=torch.uint8, device=DEV)
    out = exl3.apply_exl3_fused_moe(x, ids, w, layer, None, None, LIMIT, fat_threshold=FAT, workspace=ws)
    assert exl3.read_status(workspace=ws) == 0
    del ws
    xf = x.half().float().cpu().numpy()
    scales = [t.cpu().numpy() for t in (layer.w13_suh, layer.w13_svh, layer.w2_suh, layer.w2_svh)]

    def ref_rows(e, toks):
        s13, v13, s2, v2 = (s[e] for s in scales)
        return oracle.expert(layer.w13_trellis[e, 0].cpu().numpy(), layer.w13_trellis[e, 1].cpu().numpy(),
                             layer.w2_trellis[e].cpu().numpy(), s13[0], v13[0], s13[1], v13[1], s2, v2,
                             xf[toks], LIMIT)

    jobs = [(e, toks[i:i + 4]) for e, toks in picks.items() for i in range(0, len(toks), 4)]
    with ThreadPoolExecutor(max_workers=16) as ex:
        refs = list(ex.map(lambda a: ref_rows(*a), jobs))
    got = out.cpu().numpy()
    n = 0
    for (e, toks), ref in zip(jobs, refs):
        assert_close_layer(got[toks], ref, f"expert {e} ({counts[e]} rows), tokens {toks}")
        n += len(toks)
    assert n >= 60, n
    return {int(e): int(counts[e]) for e, _ in chosen}


def test_configs2_prefill_16k_zipf11_sampled_routes_vs_oracle(oracle, layer_full):
    """16,384 tokens, Zipf(1.1) -- the batch bench.py times (hottest expert ~14k rows)."""
    chosen = _check_sampled_routes(oracle, layer_full, 16384, 3000, 1.1, ("hot", "two_pass", "gemv"))
    assert max(chosen.values()) > 8192


def test_configs4_layer_131k_zipf15_sampled_routes_vs_oracle(oracle, layer_full):
    """configs[4]'s layer batch on one GPU: 131,072 tokens, Zipf(1.5) (hottest expert ~128k rows)."""
    chosen = _check_sampled_routes(oracle, layer_full, 131072, 9000, 1.5, ("hot", "two_pass"))
    assert max(chosen.values()) > 65536
    torch.cuda.empty_cache()
