"""TEST INFRASTRUCTURE ONLY -- numpy restatement of the router top-k rule (the checker for
csrc/router.cu; the product path never imports it).

The reference takes topk_ids/topk_weights from vLLM's FusedMoE router (third-party, not vendored:
vLLM 0.13 as deployed, docker/entrypoint.sh; the rule is unchanged in vLLM 0.22, the version in this
image: model_executor/layers/fused_moe/router/grouped_topk_router.py grouped_topk and the softmax
top-k of fused_topk_router.py). Restated from that published algorithm:

  scores    = softmax(logits) over all experts, or sigmoid(logits)          (fp32)
  selection = scores + correction_bias (if given), else scores
  if n_group > 1: group score = sum of the 2 largest selection values in the group (with a bias),
                  else the group's largest; the topk_group best groups compete, others are excluded
  ids       = indices of the k largest selection values among competing experts
  weights   = scores[ids]; / sum(weights) if renormalize; * routed_scaling_factor

Pinned against vLLM's own implementation by tests/golden/router.npz (make_router_golden.py).
Ties between equal values go to the lower index here (torch.topk leaves them unspecified; the
golden inputs have none).
"""
from __future__ import annotations

import numpy as np


def router_topk(logits: np.ndarray, k: int, scoring: str = "softmax", renormalize: bool = True,
                n_group: int = 0, topk_group: int = 0, bias: np.ndarray | None = None,
                scale: float = 1.0) -> tuple[np.ndarray, np.ndarray]:
    lg = np.asarray(logits, np.float32)
    T, E = lg.shape
    if scoring == "softmax":
        m = lg.max(axis=1, keepdims=True)
        ex = np.exp(lg - m, dtype=np.float32)
        scores = (ex / ex.sum(axis=1, keepdims=True, dtype=np.float32)).astype(np.float32)
    elif scoring == "sigmoid":
        scores = (1.0 / (1.0 + np.exp(-lg, dtype=np.float32))).astype(np.float32)
    else:
        raise ValueError(scoring)
    sel = scores + bias.astype(np.float32)[None, :] if bias is not None else scores.copy()
    if n_group > 1:
        g = sel.reshape(T, n_group, E // n_group)
        if bias is not None:
            top2 = -np.sort(-g, axis=2)[:, :, :2]
            gscore = top2.sum(axis=2, dtype=np.float32)
        else:
            gscore = g.max(axis=2)
        order = np.lexsort((np.broadcast_to(np.arange(n_group), gscore.shape), -gscore), axis=1)
        keep = np.zeros((T, n_group), bool)
        np.put_along_axis(keep, order[:, :topk_group], True, axis=1)
        sel = np.where(np.repeat(keep, E // n_group, axis=1), sel, -np.inf).astype(np.float32)
    # k largest, lower index first on ties: sort by (-value, index)
    idx = np.broadcast_to(np.arange(E), sel.shape)
    order = np.lexsort((idx, -sel), axis=1)
    ids = order[:, :k].astype(np.int64)
    w = np.take_along_axis(scores, ids, axis=1).astype(np.float32)
    if renormalize:
        w = (w / w.sum(axis=1, keepdims=True, dtype=np.float32)).astype(np.float32)
    return ids, (w * np.float32(scale)).astype(np.float32)
