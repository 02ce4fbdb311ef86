"""GPU parity of the building-block kernels, through the C ABI: trellis decode (bit-exact),
routing permutation (bit-exact vs the reference's routing prep), weighted combine."""
import numpy as np
import pytest
import torch

from conftest import golden
from dsv41_flash_offload_b200 import exl3, synth

pytestmark = pytest.mark.gpu
DEV = "cuda:0"


def test_decode_dense_matches_reference_fixture():
    g = golden("format.npz")
    tr = torch.from_numpy(g["decode_trellis"]).to(DEV)
    W = exl3.decode_dense(tr, 64, 128).cpu().numpy()
    assert np.array_equal(W.view(np.uint16), g["decode_W"].view(np.uint16))


def test_decode_dense_all_states_bit_exact(oracle):
    # 65536 tiles x 256 symbols: every 16-bit state appears (P(miss) ~ 65536 e^-256)
    k = n = 4096
    tr = torch.empty((k // 16, n // 16, 48), dtype=torch.int16, device=DEV)
    synth.fill_trellis_torch(tr, 21, 77)
    W = exl3.decode_dense(tr, k, n).cpu().numpy()
    ref = oracle.decode_matrix(tr.cpu().numpy(), k, n)
    assert np.array_equal(W.view(np.uint16), ref.view(np.uint16))


def test_decode_dense_rectangular_and_gate_layout(oracle):
    k, n = 256, 2048
    tr = torch.empty((k // 16, n // 16, 48), dtype=torch.int16, device=DEV)
    synth.fill_trellis_torch(tr, 5, 3)
    W = exl3.decode_dense(tr, k, n).cpu().numpy()
    assert np.array_equal(W.view(np.uint16), oracle.decode_matrix(tr.cpu().numpy(), k, n).view(np.uint16))


def _check_perm(r, ref, N):
    for key in ("counts", "offsets"):
        assert np.array_equal(r[key].cpu().numpy(), ref[key]), key
    for key in ("token_sorted", "route_sorted", "route_pos"):
        assert np.array_equal(r[key].cpu().numpy()[:N], ref[key][:N]), key
    assert np.array_equal(r["weight_sorted"].cpu().numpy()[:N], ref["weight_sorted"][:N])


def test_permute_matches_reference_prep_fixture():
    g = golden("permute.npz")
    for ci in range(int(g["n"])):
        ids = g[f"c{ci}_ids"]
        E = int(g[f"c{ci}_E"])
        emap = g[f"c{ci}_map"]
        m = torch.from_numpy(emap).to(DEV) if emap.size else None
        r = exl3.permute(torch.from_numpy(ids).to(DEV), None, E, m)
        assert np.array_equal(r["counts"].cpu().numpy(), g[f"c{ci}_counts"])
        assert np.array_equal(r["route_sorted"].cpu().numpy(), g[f"c{ci}_order"])
        assert np.array_equal(r["token_sorted"].cpu().numpy(), g[f"c{ci}_token_sorted"])


@pytest.mark.parametrize("T,E,kind", [(0, 384, "uniform"), (1, 384, "uniform"), (64, 384, "uniform"),
                                      (1024, 384, "zipf"), (16384, 384, "zipf"), (9000, 1000, "uniform"),
                                      (3000, 7, "uniform")])
def test_permute_vs_oracle(oracle, T, E, kind):
    k = 8 if E >= 8 else 4
    if T:
        ids, w = synth.routing_np(T, T, E, k, kind=kind, zipf_s=1.1)
        rng = np.random.default_rng(T)
        bad = rng.random(ids.shape) < 0.02
        ids[bad] = rng.choice([-1, E, E + 100], bad.sum())
    else:
        ids, w = np.zeros((0, k), np.int64), np.zeros((0, k), np.float32)
    ref = oracle.permute(ids, w, E)
    r = exl3.permute(torch.from_numpy(ids).to(DEV), torch.from_numpy(w).to(DEV), E)
    _check_perm(r, ref, T * k)


def test_permute_expert_map_vs_oracle(oracle):
    T, k, E, G = 700, 8, 96, 384
    ids, w = synth.routing_np(9, T, G, k)
    emap = np.full(G, -1, np.int32)
    emap[96:192] = np.arange(E, dtype=np.int32)
    ref = oracle.permute(ids, w, E, emap)
    r = exl3.permute(torch.from_numpy(ids).to(DEV), torch.from_numpy(w).to(DEV), E, torch.from_numpy(emap).to(DEV))
    _check_perm(r, ref, T * k)


def test_combine_matches_numpy():
    T, k, H, rows = 37, 8, 512, 250
    rng = np.random.default_rng(0)
    y = rng.standard_normal((rows, H)).astype(np.float16)
    pos = rng.integers(-1, rows, (T, k)).astype(np.int32)
    w = rng.random((T, k)).astype(np.float32)
    out = exl3.combine(torch.from_numpy(y).to(DEV), torch.from_numpy(pos).to(DEV), torch.from_numpy(w).to(DEV))
    ref = np.zeros((T, H), np.float64)
    for t in range(T):
        for j in range(k):
            if pos[t, j] >= 0:
                ref[t] += float(w[t, j]) * y[pos[t, j]].astype(np.float64)
    np.testing.assert_allclose(out.cpu().numpy(), ref, rtol=1e-5, atol=1e-5)


def test_bounded_wait_gives_up_with_status_and_context_survives():
    """Failure detection without a fault: a device wait that nothing completes must give up after its
    limit, leave status 1 for the host, and leave the context usable (a decode afterwards is exact)."""
    import time
    torch.cuda.synchronize()
    t0 = time.perf_counter()
    assert exl3.wait_selftest(limit_us=20000, device=DEV) == 1
    assert time.perf_counter() - t0 >= 0.02
    assert exl3.wait_selftest(limit_us=1000, device=DEV) == 1       # status was cleared and set again
    g = golden("format.npz")
    W = exl3.decode_dense(torch.from_numpy(g["decode_trellis"]).to(DEV), 64, 128).cpu().numpy()
    assert np.array_equal(W.view(np.uint16), g["decode_W"].view(np.uint16))
