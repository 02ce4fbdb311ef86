"""GPU parity of the full routed-expert layer (the apply_exl3_fused_moe drop-in) against the oracle
and the reference's golden outputs, plus the tier_forward / run_batch mirrors, determinism and
CUDA-graph capture. Bar: max-abs <= 2e-2 and cosine >= 0.9999."""
import numpy as np
import pytest
import torch

from conftest import assert_close_layer, golden
from dsv41_flash_offload_b200 import dma_gemm, exl3, synth, tier
from moe_ref import oracle_out

pytestmark = pytest.mark.gpu
DEV = "cuda:0"
LIMIT = 10.0


@pytest.fixture(scope="module")
def layer_full():
    """BASELINE shape: E 384, H 4096, I 2048 (3.6 GB of trellis words, seed 0)."""
    return exl3.Exl3MoELayer.synthetic(384, 4096, 2048, seed=0, device=DEV)


@pytest.fixture(scope="module")
def layer_small():
    return exl3.Exl3MoELayer.synthetic(16, 512, 256, seed=3, device=DEV)


def _inputs(seed, T, H, E, k=8, kind="uniform", zipf_s=1.1):
    x = torch.from_numpy(synth.hidden_np(seed, T, H)).to(DEV, torch.bfloat16)
    ids, w = synth.routing_np(seed, T, E, k, kind=kind, zipf_s=zipf_s)
    return x, torch.from_numpy(ids).to(DEV), torch.from_numpy(w).to(DEV)


def test_layer_c0_matches_reference_golden(layer_full):
    """BASELINE config 0 inputs on the GPU vs the reference's own outputs (ft_core.h ref_expert,
    and its AVX2 tier in EXACT mode)."""
    g = golden("layer_c0.npz")
    T, H, E, k, seed = (int(g[n]) for n in ("T", "H", "E", "k", "seed"))
    x, ids, w = _inputs(seed, T, H, E, k)
    assert np.array_equal(ids.cpu().numpy(), g["ids"])
    out = exl3.apply_exl3_fused_moe(x, ids, w, layer_full, None, None, float(g["limit"]))
    got = out.cpu().numpy()
    assert_close_layer(got, g["out_ref"], "GPU vs reference ref_expert")
    assert_close_layer(got, g["tier_exact"], "GPU vs reference AVX2 tier")
    assert exl3.read_status(device=DEV) == 0


@pytest.mark.parametrize("T", [1, 8, 32, 64])
def test_decode_sweep_vs_oracle(oracle, layer_full, T):
    x, ids, w = _inputs(100 + T, T, 4096, 384)
    out = exl3.apply_exl3_fused_moe(x, ids, w, layer_full, None, None, LIMIT)
    ref = oracle_out(oracle, layer_full, x, ids, w, LIMIT)
    assert_close_layer(out.cpu().numpy(), ref, f"decode T={T}")


def test_small_layer_edge_cases_vs_oracle(oracle, layer_small):
    """Duplicate experts per token, invalid ids (-1, >= E), zero weights, no clamp."""
    T, H, E, k = 37, 512, 16, 6
    x, ids, w = _inputs(7, T, H, E, k)
    ids[0, :] = 3                       # one token routed 6x to the same expert
    ids[1, 2] = -1
    ids[2, 0] = E + 5
    ids[3, :] = -1                      # token with no valid route -> zeros
    w[4, 1] = 0.0
    out = exl3.apply_exl3_fused_moe(x, ids, w, layer_small, None, None, None)
    ref = oracle_out(oracle, layer_small, x, ids, w, 0.0)
    assert_close_layer(out.cpu().numpy(), ref, "small layer")
    assert float(out[3].abs().max()) == 0.0


def test_expert_map_vs_oracle(oracle, layer_small):
    T, H, k, G = 20, 512, 8, 64
    x = torch.from_numpy(synth.hidden_np(8, T, H)).to(DEV, torch.bfloat16)
    ids_np, w_np = synth.routing_np(8, T, G, k)
    emap = torch.full((G,), -1, dtype=torch.int32)
    emap[16:32] = torch.arange(16, dtype=torch.int32)
    ids, w = torch.from_numpy(ids_np).to(DEV), torch.from_numpy(w_np).to(DEV)
    out = exl3.apply_exl3_fused_moe(x, ids, w, layer_small, None, emap.to(DEV), LIMIT)
    ref = oracle_out(oracle, layer_small, x, ids, w, LIMIT, expert_map=emap)
    assert_close_layer(out.cpu().numpy(), ref, "expert_map")


def test_many_rows_per_expert_vs_oracle(oracle, layer_small):
    """Rows beyond one 16-row group per expert (groups loop) on the GEMV path."""
    T, H, E, k = 300, 512, 16, 4
    x, ids, w = _inputs(11, T, H, E, k, kind="zipf", zipf_s=1.5)
    out = exl3.apply_exl3_fused_moe(x, ids, w, layer_small, None, None, LIMIT, fat_threshold=-1)
    ref = oracle_out(oracle, layer_small, x, ids, w, LIMIT)
    assert_close_layer(out.cpu().numpy(), ref, "many rows")


def test_gemm_path_small_vs_oracle(oracle, layer_small):
    """Busy experts (> 32 rows) through the decode-to-smem tcgen05 GEMM, several M tiles each."""
    T, H, E, k = 300, 512, 16, 4
    x, ids, w = _inputs(41, T, H, E, k, kind="zipf", zipf_s=1.5)
    counts = torch.bincount(ids.reshape(-1), minlength=E)
    assert int((counts > 32).sum()) >= 4 and int(counts.max()) > 256
    out = exl3.apply_exl3_fused_moe(x, ids, w, layer_small, None, None, LIMIT, fat_threshold=32)
    assert exl3.read_status(device=DEV) == 0
    ref = oracle_out(oracle, layer_small, x, ids, w, LIMIT)
    assert_close_layer(out.cpu().numpy(), ref, "gemm small")


def test_gemm_path_full_shape_vs_oracle(oracle, layer_full):
    """BASELINE layer shape, four busy experts with 160 rows each (two M tiles, one pass)."""
    T, k = 160, 4
    experts = torch.tensor([5, 77, 200, 383])
    g = torch.Generator().manual_seed(0)
    ids = torch.stack([experts[torch.randperm(4, generator=g)] for _ in range(T)]).to(DEV)
    w = torch.softmax(torch.randn(T, k, generator=g), 1).to(DEV)
    x = torch.from_numpy(synth.hidden_np(42, T, 4096)).to(DEV, torch.bfloat16)
    out = exl3.apply_exl3_fused_moe(x, ids, w, layer_full, None, None, LIMIT, fat_threshold=32)
    assert exl3.read_status(device=DEV) == 0
    ref = oracle_out(oracle, layer_full, x, ids, w, LIMIT)
    assert_close_layer(out.cpu().numpy(), ref, "gemm full shape")


@pytest.fixture(scope="module")
def layer_real():
    """The model's real expert shape, H 5120 and I 2304 (64 experts to bound memory)."""
    return exl3.Exl3MoELayer.synthetic(64, 5120, 2304, seed=11, device=DEV)


def test_real_shape_top6_vs_oracle(oracle, layer_real):
    """H 5120 / I 2304 / top-6: a decode batch (GEMV) and four busy experts of 40 rows (GEMM)."""
    x, ids, w = _inputs(300, 16, 5120, 64, 6)
    out = exl3.apply_exl3_fused_moe(x, ids, w, layer_real, None, None, LIMIT)
    assert_close_layer(out.cpu().numpy(), oracle_out(oracle, layer_real, x, ids, w, LIMIT), "real shape decode")
    T = 40
    g = torch.Generator().manual_seed(1)
    experts = torch.tensor([0, 9, 33, 63])
    ids = torch.stack([experts[torch.randperm(4, generator=g)] for _ in range(T)]).to(DEV)
    w = torch.softmax(torch.randn(T, 4, generator=g), 1).to(DEV)
    x = torch.from_numpy(synth.hidden_np(301, T, 5120)).to(DEV, torch.bfloat16)
    out = exl3.apply_exl3_fused_moe(x, ids, w, layer_real, None, None, LIMIT, fat_threshold=32)
    assert exl3.read_status(device=DEV) == 0
    assert_close_layer(out.cpu().numpy(), oracle_out(oracle, layer_real, x, ids, w, LIMIT), "real shape gemm")


def test_gemm_matches_gemv_on_prefill(layer_full):
    """Prefill chunk (2048 tokens, Zipf 1.1): tensor-core path for busy experts vs all-GEMV."""
    x, ids, w = _inputs(43, 2048, 4096, 384, kind="zipf", zipf_s=1.1)
    a = exl3.apply_exl3_fused_moe(x, ids, w, layer_full, None, None, LIMIT, fat_threshold=32)
    b = exl3.apply_exl3_fused_moe(x, ids, w, layer_full, None, None, LIMIT, fat_threshold=-1)
    assert exl3.read_status(device=DEV) == 0
    assert_close_layer(a.cpu().numpy(), b.cpu().numpy(), "gemm vs gemv")


def test_max_routes_bound(layer_small):
    """Row buffers sized by a caller bound on valid routes (expert-parallel receivers): an exact bound
    gives the same output; a bound that is too small drops the call (zeros) and sets status 3."""
    T, H, E, k = 40, 512, 16, 4
    x, ids, w = _inputs(51, T, H, E, k)
    ids[(torch.arange(T * k, device=DEV).reshape(T, k) % 3) == 0] = -1
    nvalid = int((ids >= 0).sum())
    ref = exl3.apply_exl3_fused_moe(x, ids, w, layer_small, None, None, LIMIT)
    a = exl3.apply_exl3_fused_moe(x, ids, w, layer_small, None, None, LIMIT, max_routes=nvalid)
    assert torch.equal(a, ref)
    assert exl3.read_status(device=DEV) == 0
    b = exl3.apply_exl3_fused_moe(x, ids, w, layer_small, None, None, LIMIT, max_routes=nvalid - 1)
    assert float(b.abs().max()) == 0.0
    assert exl3.read_status(device=DEV) == 3
    assert exl3.read_status(device=DEV) == 0


def test_input_dtypes_agree(layer_small):
    T, H, E = 9, 512, 16
    x, ids, w = _inputs(12, T, H, E, 4)
    outs = [exl3.apply_exl3_fused_moe(x.to(dt), ids, w, layer_small, None, None, LIMIT)
            for dt in (torch.bfloat16, torch.float16, torch.float32)]
    assert torch.equal(outs[0], outs[1]) and torch.equal(outs[0], outs[2])


def test_deterministic_and_split_invariant(layer_full):
    x, ids, w = _inputs(5, 4, 4096, 384)
    a = exl3.apply_exl3_fused_moe(x, ids, w, layer_full, None, None, LIMIT)
    b = exl3.apply_exl3_fused_moe(x, ids, w, layer_full, None, None, LIMIT)
    assert torch.equal(a, b)
    for s in (1, 2, 4, 8):
        c = exl3.apply_exl3_fused_moe(x, ids, w, layer_full, None, None, LIMIT, split_k=s)
        assert_close_layer(c.cpu().numpy(), a.cpu().numpy(), f"split {s}")


def test_cuda_graph_capture_replay(layer_full):
    T = 16
    x, ids, w = _inputs(21, T, 4096, 384)
    sx, sid, sw = x.clone(), ids.clone(), w.clone()
    out = torch.empty(T, 4096, dtype=torch.float32, device=DEV)
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        exl3.apply_exl3_fused_moe(sx, sid, sw, layer_full, None, None, LIMIT, out=out)  # eager: sizes workspace
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, stream=s):
            exl3.apply_exl3_fused_moe(sx, sid, sw, layer_full, None, None, LIMIT, out=out)
    torch.cuda.current_stream().wait_stream(s)
    for seed in (22, 23):
        x2, ids2, w2 = _inputs(seed, T, 4096, 384)
        sx.copy_(x2); sid.copy_(ids2); sw.copy_(w2)
        g.replay()
        torch.cuda.synchronize()
        ref = exl3.apply_exl3_fused_moe(x2, ids2, w2, layer_full, None, None, LIMIT)
        assert torch.equal(out, ref)
    del g


def test_tier_forward_mirror(layer_full):
    """tier_init/tier_add_layer/tier_forward (ft_tier_ext.cpp API) on the GPU vs the golden
    output of the reference's own AVX2 tier."""
    g = golden("layer_c0.npz")
    E, H, I = 384, 4096, 2048
    tier.tier_stop()
    tier.tier_init(1, [0], None, None, None, None, -1, H, I, 1, 0)
    tier.tier_set_limit(float(g["limit"]))
    ptrs = torch.stack([layer_full._exl3_ptrs[k] for k in ("gate_trellis", "up_trellis", "down_trellis")], 1).cpu()
    tier.tier_add_layer(0, ptrs, layer_full.w13_suh[:, 0].cpu(), layer_full.w13_svh[:, 0].cpu(),
                        layer_full.w13_suh[:, 1].cpu(), layer_full.w13_svh[:, 1].cpu(), layer_full.w2_suh.cpu(),
                        layer_full.w2_svh.cpu())
    x = torch.from_numpy(synth.hidden_np(0, 4, H)).to(torch.float16).float()
    out = tier.tier_forward(0, x, torch.from_numpy(g["ids"].astype(np.int32)), torch.from_numpy(g["weights"]), -1)
    assert out.device.type == "cpu"
    assert_close_layer(out.numpy(), g["tier_exact"], "tier_forward mirror")
    assert tier.tier_stats()[0] == 1
    tier.tier_stop()


def test_run_batch_mirror_vs_oracle(oracle, layer_small):
    """runtime/dma_gemm.py run_batch semantics: busy experts (> cap rows) of a batch accumulate."""
    T, H, E, k, cap = 200, 512, 16, 4, 32
    x, ids, w = _inputs(31, T, H, E, k, kind="zipf", zipf_s=1.1)
    flat = ids.reshape(-1)
    order = torch.argsort(flat, stable=True)
    counts = torch.bincount(flat, minlength=E).cpu()
    token_sorted = (torch.arange(T, device=DEV).repeat_interleave(k))[order]
    weight_sorted = w.reshape(-1)[order]
    out = torch.zeros(T, H, dtype=torch.float32, device=DEV)
    D = {"batches": [(0, 8), (8, 16)], "h13": {"cold": list(range(E))}, "layer": layer_small}
    for b in range(2):
        dma_gemm.run_batch(D, None, b, None, counts, cap, x.half(), token_sorted, weight_sorted, LIMIT, out)
    busy = [e for e in range(E) if int(counts[e]) > cap]
    assert busy, "test needs busy experts"
    wb = w.clone()
    keep = torch.zeros_like(ids, dtype=torch.bool)
    for e in busy:
        keep |= ids == e
    wb[~keep] = 0.0
    ref = oracle_out(oracle, layer_small, x, ids, wb, LIMIT)
    assert_close_layer(out.cpu().numpy(), ref, "run_batch")


def test_vllm_plugin_and_decode_graphs(layer_small):
    """The installed module function on a vLLM-style layer (parameters only) equals the direct call;
    DecodeGraphs replays are bit-identical to eager calls for batch sizes on and between the captured ones."""
    import types
    from dsv41_flash_offload_b200 import vllm_plugin
    X = types.ModuleType("fake_vllm_exl3")
    X.apply_exl3_fused_moe = lambda *a, **k: None
    vllm_plugin.install(X)
    vl = types.SimpleNamespace(**{n: torch.nn.Parameter(getattr(layer_small, n), requires_grad=False)
                                  for n in ("w13_trellis", "w2_trellis", "w13_suh", "w13_svh", "w2_suh", "w2_svh")})
    x, ids, w = _inputs(51, 9, 512, 16, 6)
    got = X.apply_exl3_fused_moe(x, ids, w, vl, None, None, LIMIT)
    ref = exl3.apply_exl3_fused_moe(x, ids, w, layer_small, None, None, LIMIT)
    assert torch.equal(got, ref)
    dg = vllm_plugin.DecodeGraphs(layer_small, sizes=(1, 4, 16), topk=6, limit=LIMIT)
    for t, seed in ((1, 52), (3, 53), (16, 54), (11, 55)):
        x, ids, w = _inputs(seed, t, 512, 16, 6)
        out = dg(x, ids, w)
        assert torch.equal(out, exl3.apply_exl3_fused_moe(x, ids, w, layer_small, None, None, LIMIT)), t
    dg.close()


def test_gemm_many_rows_per_expert_vs_oracle(oracle):
    """Busy experts with many row passes (over 768 rows each), and more than 48 of them, vs oracle."""
    lay = exl3.Exl3MoELayer.synthetic(16, 512, 256, seed=8, device=DEV)
    x, ids, w = _inputs(71, 1000, 512, 16, 4, kind="zipf", zipf_s=2.0)
    counts = torch.bincount(ids.reshape(-1), minlength=16)
    assert int(counts.max()) > 768
    out = exl3.apply_exl3_fused_moe(x, ids, w, lay, None, None, LIMIT, fat_threshold=32)
    assert exl3.read_status(device=DEV) == 0
    assert_close_layer(out.cpu().numpy(), oracle_out(oracle, lay, x, ids, w, LIMIT), "many passes")
    lay2 = exl3.Exl3MoELayer.synthetic(64, 256, 256, seed=9, device=DEV)
    x, ids, w = _inputs(72, 8000, 256, 64, 8)
    assert int((torch.bincount(ids.reshape(-1), minlength=64) > 768).sum()) > 48
    out = exl3.apply_exl3_fused_moe(x, ids, w, lay2, None, None, LIMIT, fat_threshold=32)
    assert exl3.read_status(device=DEV) == 0
    assert_close_layer(out.cpu().numpy(), oracle_out(oracle, lay2, x, ids, w, LIMIT), "many busy experts")
