"""GPU router top-k (dsv41_router_topk / dsv41_moe_forward_logits) against vLLM's own routing
(golden vectors) and the numpy restatement (oracle/router.py): ids exact, weights to 1e-5."""
import numpy as np
import pytest
import torch

from conftest import golden
from dsv41_flash_offload_b200 import exl3, synth
from oracle.router import router_topk

pytestmark = pytest.mark.gpu
DEV = "cuda:0"


def test_router_matches_vllm_golden():
    g = golden("router.npz")
    for n in sorted(set(k.split("__")[0] for k in g.files)):
        T, E, k, sig, renorm, ng, tg, wb, scale = g[n + "__cfg"]
        bias = torch.from_numpy(g[n + "__bias"]).to(DEV) if wb else None
        ids, w = exl3.route_topk(torch.from_numpy(g[n + "__logits"]).to(DEV), int(k),
                                 scoring="sigmoid" if sig else "softmax", renormalize=bool(renorm),
                                 num_expert_group=int(ng), topk_group=int(tg), correction_bias=bias,
                                 routed_scaling_factor=float(scale))
        ids, w = ids.cpu().numpy(), w.cpu().numpy()
        for a, wa, b, wbv in zip(ids, w, g[n + "__ids"], g[n + "__w"]):
            assert set(a.tolist()) == set(b.tolist()), n
            ref = dict(zip(b.tolist(), wbv.tolist()))
            assert max(abs(x - ref[i]) for i, x in zip(a.tolist(), wa.tolist())) < 1e-5, n


@pytest.mark.parametrize("E,k,scoring,ng,tg,bias,renorm,scale,dtype", [
    (384, 8, "softmax", 0, 0, False, True, 1.0, torch.float32),
    (384, 8, "softmax", 0, 0, False, True, 1.0, torch.bfloat16),
    (1024, 32, "softmax", 0, 0, False, False, 1.0, torch.float16),
    (256, 8, "sigmoid", 8, 4, True, True, 2.5, torch.float32),
    (384, 6, "sigmoid", 32, 5, True, True, 1.0, torch.bfloat16),
    (64, 4, "sigmoid", 0, 0, False, False, 1.0, torch.float32),
    (7, 3, "softmax", 0, 0, False, True, 1.0, torch.float32),
])
def test_router_vs_oracle(E, k, scoring, ng, tg, bias, renorm, scale, dtype):
    T = 300
    g = torch.Generator().manual_seed(E * 31 + k)
    logits = torch.randn(T, E, generator=g).to(dtype)
    b = (torch.rand(E, generator=g) * 0.2 - 0.1) if bias else None
    ids, w = exl3.route_topk(logits.to(DEV), k, scoring=scoring, renormalize=renorm, num_expert_group=ng,
                             topk_group=tg, correction_bias=b.to(DEV) if b is not None else None,
                             routed_scaling_factor=scale)
    rids, rw = router_topk(logits.float().numpy(), k, scoring, renorm, ng, tg, b.numpy() if b is not None else None,
                           scale)
    assert np.array_equal(ids.cpu().numpy(), rids)
    np.testing.assert_allclose(w.cpu().numpy(), rw, rtol=1e-5, atol=1e-6)


def test_forward_logits_equals_router_then_layer():
    layer = exl3.Exl3MoELayer.synthetic(16, 512, 256, seed=3, device=DEV)
    T = 40
    x = torch.from_numpy(synth.hidden_np(61, T, 512)).to(DEV, torch.bfloat16)
    logits = torch.randn(T, 16, generator=torch.Generator().manual_seed(62)).to(DEV)
    out, (ids, w) = exl3.apply_exl3_fused_moe_logits(x, logits, layer, 6, 10.0, return_routes=True)
    rids, rw = exl3.route_topk(logits, 6)
    assert torch.equal(ids, rids) and torch.equal(w, rw)
    ref = exl3.apply_exl3_fused_moe(x, rids, rw, layer, None, None, 10.0)
    assert torch.equal(out, ref)
    out2 = exl3.apply_exl3_fused_moe_logits(x, logits, layer, 6, 10.0)
    assert torch.equal(out2, ref)
    assert exl3.read_status(device=DEV) == 0


def test_router_argument_errors():
    logits = torch.randn(4, 2048, device=DEV)
    with pytest.raises(Exception, match="1..1024"):
        exl3.route_topk(logits, 8)
    with pytest.raises(Exception, match="num_expert_group"):
        exl3.route_topk(torch.randn(4, 384, device=DEV), 8, num_expert_group=7, topk_group=2)
