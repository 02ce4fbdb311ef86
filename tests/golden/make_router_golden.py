"""Golden router fixtures from vLLM's own torch implementation of the routing rule (vLLM 0.22 in this
build image: vllm.model_executor.layers.fused_moe.router.grouped_topk_router.grouped_topk, CPU path).
vLLM is the reference's router (third-party, not vendored). Writes tests/golden/router.npz.

    python tests/golden/make_router_golden.py     (needs the vllm package; not run by the tests)
"""
import os

os.environ.setdefault("TORCHDYNAMO_DISABLE", "1")   # vLLM wraps grouped_topk in torch.compile; run it eagerly

import numpy as np
import torch

from vllm.model_executor.layers.fused_moe.router.grouped_topk_router import grouped_topk

HERE = os.path.dirname(os.path.abspath(__file__))
# name: (T, E, k, scoring, renormalize, n_group, topk_group, with_bias, scale)
CASES = {
    "softmax_e384_k8": (64, 384, 8, "softmax", True, 1, 1, False, 1.0),       # BASELINE synthetic routing
    "sigmoid_bias_grouped": (48, 256, 8, "sigmoid", True, 8, 4, True, 2.5),   # DeepSeek-V3-style noaux_tc
    "sigmoid_grouped_max": (40, 384, 6, "sigmoid", False, 8, 3, False, 1.0),
    "softmax_grouped": (33, 128, 8, "softmax", True, 4, 2, False, 1.0),
}


def main():
    out = {}
    for name, (T, E, k, scoring, renorm, ng, tg, with_bias, scale) in CASES.items():
        g = torch.Generator().manual_seed(hash(name) % (2 ** 31))
        logits = torch.randn(T, E, generator=g, dtype=torch.float32)
        bias = (torch.rand(E, generator=g) * 0.2 - 0.1) if with_bias else None
        w, ids = grouped_topk(torch.zeros(T, 8), logits, k, renorm, num_expert_group=ng, topk_group=tg,
                              scoring_func=scoring, routed_scaling_factor=scale, e_score_correction_bias=bias)
        # vLLM leaves the order of the k ids unspecified: the tests compare them as sets
        ids = ids.long()
        out[f"{name}__logits"] = logits.numpy()
        out[f"{name}__ids"] = ids.numpy()
        out[f"{name}__w"] = w.numpy()
        out[f"{name}__bias"] = bias.numpy() if bias is not None else np.zeros(0, np.float32)
        out[f"{name}__cfg"] = np.array([T, E, k, scoring == "sigmoid", renorm, ng, tg, with_bias, scale], np.float64)
    np.savez_compressed(os.path.join(HERE, "router.npz"), **out)
    print("wrote", len(CASES), "cases")


if __name__ == "__main__":
    main()
