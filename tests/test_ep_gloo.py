"""Expert-parallel dispatch/combine bookkeeping on CPU ranks (gloo, world size 2 and 4).

Each rank owns E/world experts; a stand-in expert e multiplies its row by (e + 1), so the combined
output has a closed form: out[t] = sum_j w[t, j] * (ids[t, j] + 1) * x[t] over valid routes. Covers
tokens routed several times to one rank (sent once), invalid ids, tokens with no valid route and ranks
that receive no rows."""
import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from dsv41_flash_offload_b200.ep import EPMoE

E, H, K = 16, 8, 4


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _inputs(rank, case):
    g = torch.Generator().manual_seed(100 * case + rank)
    T = 13 + rank
    ids = torch.randint(0, E, (T, K), generator=g)
    if case == 1:
        ids[0] = torch.tensor([-1, E, E + 7, -5])       # no valid route
        ids[1] = torch.tensor([3, 3, 2, 1])              # several routes to one rank
    if case == 2:
        ids = torch.randint(0, E // 4, (T, K), generator=g)   # every route to rank 0's experts
    w = torch.rand(T, K, generator=g)
    x = torch.randn(T, H, generator=g)
    return x, ids, w


def _reference(x, ids, w):
    valid = (ids >= 0) & (ids < E)
    scale = torch.where(valid, w * (ids + 1).float(), torch.zeros_like(w)).sum(1, keepdim=True)
    return scale * x


def _worker(rank, world, port, case, q, fixed_slots):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        e_loc = E // world

        def expert_fn(xr, local_ids, wr, max_routes=0):
            if max_routes:
                assert int((local_ids >= 0).sum()) == max_routes
            glob = torch.where(local_ids >= 0, local_ids + rank * e_loc, torch.full_like(local_ids, -1))
            assert bool(((local_ids >= -1) & (local_ids < e_loc)).all())
            scale = torch.where(glob >= 0, wr * (glob + 1).float(), torch.zeros_like(wr)).sum(1, keepdim=True)
            return scale * xr

        ep = EPMoE(expert_fn, E)
        ep.slot_capacity = 16 if fixed_slots else 0   # both dispatch modes (T = 13 + rank <= 16)
        x, ids, w = _inputs(rank, case)
        out = ep(x, ids, w)
        err = float((out - _reference(x, ids, w)).abs().max())
        q.put((rank, err, ep.stats["sent_rows"], ep.stats["recv_rows"]))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("fixed_slots", [False, True])
@pytest.mark.parametrize("world,case", [(2, 0), (2, 1), (2, 2), (4, 0), (4, 2)])
def test_ep_dispatch_combine_gloo(world, case, fixed_slots):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, case, q, fixed_slots)) for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=120)
    assert all(p.exitcode == 0 for p in procs), [p.exitcode for p in procs]
    res = [q.get(timeout=10) for _ in range(world)]
    for rank, err, sent, recv in res:
        assert err < 1e-5, (rank, err)
    assert sum(r[2] for r in res) == sum(r[3] for r in res)  # every sent row was received once
