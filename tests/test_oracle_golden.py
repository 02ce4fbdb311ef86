"""The plain-C oracle pinned against golden vectors produced by the reference's own compiled code
(tests/golden/make_golden.py), and -- where the reference build exists locally -- directly against it."""
import hashlib

import numpy as np
import pytest

from conftest import assert_close_layer, golden
from dsv41_flash_offload_b200 import synth


def test_weight_table_digest(oracle):
    g = golden("format.npz")
    table = oracle.weight_table()
    assert hashlib.sha256(table.tobytes()).hexdigest() == str(g["table_sha256"])
    assert np.array_equal(table[g["sample_idx"]], g["sample_bits"])


def test_perm_is_fragment_layout(oracle):
    # stream symbol 8t+q of a tile sits at (k, n) of mma B fragment lane t, element q
    for i in range(256):
        t, q = divmod(i, 8)
        r = (t % 4) * 2 + (0, 1, 8, 9)[q % 4]
        c = t // 4 + (8 if q >= 4 else 0)
        assert oracle.L.orc_perm(i) == r * 16 + c


def test_decode_matrix_matches_reference(oracle):
    g = golden("format.npz")
    tr = g["decode_trellis"]
    W = oracle.decode_matrix(tr, 64, 128)
    assert np.array_equal(W.view(np.uint16), g["decode_W"].view(np.uint16))
    for i in range(4):
        assert np.array_equal(oracle.states(tr.reshape(-1, 48)[i]), g["states"][i])


def test_transforms_and_act_match_reference(oracle):
    g = golden("format.npz")
    for i in range(16):
        assert np.array_equal(oracle.prep_block(g["prep_x"][i], g["prep_suh"][i]), g["prep_out"][i])
        assert np.array_equal(oracle.out_block(g["outb_y"][i], g["outb_svh"][i]), g["outb_out"][i])
    a10 = np.array([oracle.act(a, b, 10.0) for a, b in zip(g["act_g"], g["act_u"])], np.float32)
    a0 = np.array([oracle.act(a, b, 0.0) for a, b in zip(g["act_g"], g["act_u"])], np.float32)
    # the reference uses std::exp; allow 1 ulp of fp32 on the activation itself
    np.testing.assert_allclose(a10, g["act_10"], rtol=3e-7, atol=0)
    np.testing.assert_allclose(a0, g["act_0"], rtol=3e-7, atol=0)


def test_expert_matches_reference(oracle):
    g = golden("expert_small.npz")
    H, I, e, seed = int(g["H"]), int(g["I"]), int(g["e"]), int(g["seed"])
    gate, up, down = synth.expert_trellis_np(seed, H, I, e)
    s13, v13, s2, v2 = synth.scales_np(seed, e + 1, H, I)
    x = synth.hidden_np(seed, 2, H).astype(np.float16).astype(np.float32)
    args = (gate, up, down, s13[e, 0], v13[e, 0], s13[e, 1], v13[e, 1], s2[e], v2[e], x)
    np.testing.assert_array_equal(oracle.expert(*args, limit=10.0), g["y_limit10"])
    np.testing.assert_array_equal(oracle.expert(*args, limit=0.0), g["y_limit0"])


def test_permute_matches_reference_prep(oracle):
    g = golden("permute.npz")
    for ci in range(int(g["n"])):
        ids = g[f"c{ci}_ids"]
        E = int(g[f"c{ci}_E"])
        emap = g[f"c{ci}_map"]
        r = oracle.permute(ids, None, E, emap if emap.size else None)
        assert np.array_equal(r["counts"], g[f"c{ci}_counts"])
        assert np.array_equal(r["route_sorted"], g[f"c{ci}_order"])
        assert np.array_equal(r["token_sorted"], g[f"c{ci}_token_sorted"])
        # route_pos inverts the order for valid routes
        n_valid = int(r["offsets"][E])
        pos = r["route_pos"]
        assert np.array_equal(pos[r["route_sorted"][:n_valid]], np.arange(n_valid))
        assert (pos[r["route_sorted"][n_valid:]] == -1).all()


def test_layer_c0_matches_reference(oracle):
    """BASELINE config 0 (4 tokens, H 4096, E 384, I 2048, top-8), seed 0."""
    g = golden("layer_c0.npz")
    T, H, I, E, k, seed = (int(g[n]) for n in ("T", "H", "I", "E", "k", "seed"))
    x = synth.hidden_np(seed, T, H).astype(np.float16).astype(np.float32)
    ids, w = synth.routing_np(seed, T, E, k)
    assert np.array_equal(ids, g["ids"]) and np.array_equal(w, g["weights"])
    s13, v13, s2, v2 = synth.scales_np(seed, E, H, I)
    gate, up, down = [None] * E, [None] * E, [None] * E
    for e in sorted(set(ids.reshape(-1).tolist())):
        gate[e], up[e], down[e] = synth.expert_trellis_np(seed, H, I, e)
    out = oracle.moe_layer(x, ids, w, gate, up, down, s13, v13, s2, v2, limit=float(g["limit"]))
    np.testing.assert_allclose(out, g["out_ref"], rtol=0, atol=2e-6)
    # the reference's own AVX2 tier (EXACT mode) agrees within the parity bar too
    assert_close_layer(g["tier_exact"], g["out_ref"], "reference AVX2 tier EXACT")


def test_oracle_against_local_reference_build(oracle):
    """Direct pin where oracle/_ref was built from the reference tree (machines with the reference checkout)."""
    from oracle.oracle import RefShim
    if not RefShim.available():
        pytest.skip("oracle/_ref not built here")
    ref = RefShim()
    assert np.array_equal(oracle.weight_table(), ref.weight_table().view(np.uint16))
    rng = np.random.default_rng(1)
    for _ in range(64):
        tile = rng.integers(0, 65536, 48, dtype=np.uint16)
        assert np.array_equal(oracle.states(tile), ref.states(tile))


def test_router_oracle_matches_vllm_golden():
    """The numpy router restatement reproduces vLLM's own routing (golden vectors from its torch
    grouped_topk: softmax top-k, sigmoid + correction bias with groups, grouped max, grouped softmax)."""
    from oracle.router import router_topk
    g = golden("router.npz")
    names = sorted(set(k.split("__")[0] for k in g.files))
    assert len(names) == 4
    for n in names:
        T, E, k, sig, renorm, ng, tg, wb, scale = g[n + "__cfg"]
        ids, w = router_topk(g[n + "__logits"], int(k), "sigmoid" if sig else "softmax", bool(renorm), int(ng),
                             int(tg), g[n + "__bias"] if wb else None, float(scale))
        for a, wa, b, wbv in zip(ids, w, g[n + "__ids"], g[n + "__w"]):
            assert set(a.tolist()) == set(b.tolist()), n
            ref = dict(zip(b.tolist(), wbv.tolist()))
            assert max(abs(x - ref[i]) for i, x in zip(a.tolist(), wa.tolist())) < 1e-6, n
