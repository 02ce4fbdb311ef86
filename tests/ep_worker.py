"""Worker for tests/test_gpu_ep.py (launched with torchrun, one rank per GPU, NCCL).

Each rank holds its shard E/world of a synthetic BASELINE-shape layer and routes its own 64 tokens over
all global experts; the expert-parallel output (NCCL all-to-all dispatch/combine) must match the
single-GPU layer (every rank also builds the full layer) within the parity bar; then the same for
the peer-memory path (EPPeerMoE: token rows read from peers, expert outputs stored into the token
owners' memory, no collective), at decode and at prefill sizes; last,
a rank that skips one step makes the other ranks' exchange waits run out (status 1, bounded at 50 ms)."""
import datetime
import os
import sys
import time

import numpy as np
import torch
import torch.distributed as dist

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, ROOT)
sys.path.insert(0, os.path.join(ROOT, "tests"))

from conftest import assert_close_layer  # noqa: E402
from dsv41_flash_offload_b200 import exl3, synth  # noqa: E402
from dsv41_flash_offload_b200.ep import EPMoE, EPPeerMoE, local_layer_fn  # noqa: E402

E, H, I, K, T = 384, 4096, 2048, 8, 64
TB = 1536   # tokens per rank of the prefill-sized peer steps (world * TB * K > 8192 gathered routes)


def main():
    local = int(os.environ["LOCAL_RANK"])
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=dev)
    rank, world = dist.get_rank(), dist.get_world_size()
    e_loc = E // world
    shard = exl3.Exl3MoELayer.synthetic(E, H, I, seed=0, device=dev, expert_range=(rank * e_loc, (rank + 1) * e_loc))
    full = exl3.Exl3MoELayer.synthetic(E, H, I, seed=0, device=dev)
    ep = EPMoE(local_layer_fn(shard, 10.0), E)
    for case in range(6):
        ep.slot_capacity = 96 if case >= 3 else 0   # compact dispatch, then fixed slots
        case %= 3
        seed = 500 + 10 * case + rank
        x = torch.from_numpy(synth.hidden_np(seed, T, H)).to(dev, torch.bfloat16)
        kind = "zipf" if case == 2 else "uniform"
        ids_np, w_np = synth.routing_np(seed, T, E, K, kind=kind, zipf_s=1.5)
        ids, w = torch.from_numpy(ids_np).to(dev), torch.from_numpy(w_np).to(dev)
        if case == 1:
            ids[0, :] = -1
            ids[1, 3] = E + 1
        out = ep(x, ids, w)
        ref = exl3.apply_exl3_fused_moe(x, ids, w, full, None, None, 10.0)
        torch.cuda.synchronize()
        assert_close_layer(out.cpu().numpy(), ref.cpu().numpy(), f"rank {rank} case {case}")
    assert exl3.read_status(device=dev) == 0
    # peer-memory expert parallelism (no collective on the data path): three steps cover both
    # buffer parities; rank 1 runs fewer tokens than the capacity; invalid ids and empty rows
    peer = EPPeerMoE(shard, E, tokens_cap=T, topk=K, limit=10.0)
    for case in range(3):
        seed = 700 + 10 * case + rank
        Tc = T if (rank == 0 or case != 1) else 40
        x = torch.from_numpy(synth.hidden_np(seed, Tc, H)).to(dev, torch.bfloat16)
        ids_np, w_np = synth.routing_np(seed, Tc, E, K, kind="zipf" if case == 2 else "uniform", zipf_s=1.5)
        ids, w = torch.from_numpy(ids_np).to(dev), torch.from_numpy(w_np).to(dev)
        if case == 1:
            ids[0, :] = -1
            ids[2, 5] = E + 3
        out = peer(x, ids, w)
        ref = exl3.apply_exl3_fused_moe(x, ids, w, full, None, None, 10.0)
        torch.cuda.synchronize()
        assert_close_layer(out.cpu().numpy(), ref.cpu().numpy(), f"peer rank {rank} case {case}")
    assert peer.read_status() == 0
    peer.close()
    # prefill-sized steps: more gathered routes than the single-CTA permutation takes (separate gather
    # launch + multi-CTA permutation) and busy experts on the tcgen05 GEMM, whose down epilogue stores the
    # output rows into the token owners' receive slots
    big = EPPeerMoE(shard, E, tokens_cap=TB, topk=K, limit=10.0)
    for case in range(2):
        seed = 800 + 10 * case + rank
        x = torch.from_numpy(synth.hidden_np(seed, TB, H)).to(dev, torch.bfloat16)
        ids_np, w_np = synth.routing_np(seed, TB, E, K, kind="zipf", zipf_s=1.1 if case == 0 else 1.5)
        ids, w = torch.from_numpy(ids_np).to(dev), torch.from_numpy(w_np).to(dev)
        out = big(x, ids, w)
        ref = exl3.apply_exl3_fused_moe(x, ids, w, full, None, None, 10.0)
        torch.cuda.synchronize()
        assert_close_layer(out.cpu().numpy(), ref.cpu().numpy(), f"peer prefill rank {rank} case {case}")
    assert big.read_status() == 0
    big.close()
    expired = wait_expiry(shard, full, dev, rank, world)
    dist.barrier()
    print(f"rank {rank}/{world} ok: sent {ep.stats['sent_rows']} rows, received {ep.stats['recv_rows']}; "
          f"peer steps {peer.stats['steps']}; {expired}", flush=True)
    dist.destroy_process_group()


def wait_expiry(shard, full, dev, rank, world):
    """A peer that stays alive but skips a step: the exchange waits of the ranks that did run it give up
    after the group's 50 ms wait limit with status 1 (the reference counts the same event for its
    combine wait, ct/ft_tier_cu_v.cu:116-120) and the context stays usable. The failure is made on the
    host: rank world-1 does not call the step. Every wait in the step is bounded, and no rank leaves
    while one of its kernels is in flight."""
    peer = EPPeerMoE(shard, E, tokens_cap=16, topk=K, limit=10.0, wait_limit_us=50000)
    x = torch.from_numpy(synth.hidden_np(900 + rank, 16, H)).to(dev, torch.bfloat16)
    ids_np, w_np = synth.routing_np(900 + rank, 16, E, K)
    ids, w = torch.from_numpy(ids_np).to(dev), torch.from_numpy(w_np).to(dev)
    ref = exl3.apply_exl3_fused_moe(x, ids, w, full, None, None, 10.0)
    out = peer(x, ids, w)                                    # step 0: every rank takes part
    assert peer.read_status() == 0
    assert_close_layer(out.cpu().numpy(), ref.cpu().numpy(), f"rank {rank} before the skipped step")
    dist.barrier()
    skipper = world - 1
    msg = "skipped step 1"
    if rank != skipper:
        torch.cuda.synchronize()
        t0 = time.perf_counter()
        out = peer(x, ids, w)                                # step 1: rank `skipper` never arrives
        status = peer.read_status()
        dt = time.perf_counter() - t0
        assert status == 1, status
        assert 0.05 <= dt < 1.5, dt                          # the 50 ms limit, not the 2 s default
        assert float(out.abs().max()) == 0.0                 # the gave-up step returns an empty result
        again = exl3.apply_exl3_fused_moe(x, ids, w, full, None, None, 10.0)
        assert torch.equal(again, ref)                       # the context is still usable
        msg = f"exchange wait expired after {dt * 1e3:.0f} ms with status 1"
    dist.barrier()
    peer.close()
    return msg


if __name__ == "__main__":
    main()
