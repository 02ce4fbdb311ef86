"""Seeded synthetic inputs for the routed-expert MoE layer (the reference publishes no dataset for
this path; BASELINE's configs describe random inputs, restated here).

Everything is derived from a counter-based 32-bit hash (the "lowbias32" integer finaliser) of
(seed, stream, index), so any slice of any tensor can be regenerated independently and the same
bits come out of numpy on the host and torch on the device:

* trellis words: uniform 16-bit, in vllm_exl3's stacked layout
  w13_trellis [E, 2, H/16, I/16, 48] int16 (gate = 0, up = 1), w2_trellis [E, I/16, H/16, 48];
* w13_suh / w2_suh: random +-1 fp16 Hadamard sign vectors;
* w13_svh / w2_svh: fp16 U(0.5, 1.5) / sqrt(4096) channel scales;
* hidden states: N(0, 1) (Box-Muller in float64) rounded to bf16;
* routing: softmax(N(0,1) logits [T, E]) top-k ("uniform"), or Zipf(s) expert popularity drawn per
  token by Gumbel-top-k over log p_zipf ("zipf"); weights = softmax over the selected k scores.
"""
from __future__ import annotations

import math

import numpy as np

M32 = 0xFFFFFFFF
STREAM_W13, STREAM_W2, STREAM_SUH13, STREAM_SVH13, STREAM_SUH2, STREAM_SVH2 = range(6)
STREAM_X, STREAM_ROUTE, STREAM_ZIPF_RANK = 6, 7, 8


def _lowbias32_np(x: np.ndarray) -> np.ndarray:
    x = x.astype(np.uint64) & M32
    x ^= x >> np.uint64(16)
    x = (x * np.uint64(0x7FEB352D)) & M32
    x ^= x >> np.uint64(15)
    x = (x * np.uint64(0x846CA68B)) & M32
    x ^= x >> np.uint64(16)
    return x


def stream_key(seed: int, stream: int, layer: int = 0) -> int:
    k = (seed * 0x9E3779B1 + stream * 0x85EBCA77 + layer * 0xC2B2AE3D + 0x27D4EB2F) & M32
    return int(_lowbias32_np(np.array([k], np.uint64))[0])


def hash_u32(seed: int, stream: int, start: int, count: int, layer: int = 0) -> np.ndarray:
    key = stream_key(seed, stream, layer)
    idx = (np.arange(start, start + count, dtype=np.uint64) + np.uint64(key)) & M32
    return _lowbias32_np(_lowbias32_np(idx) ^ np.uint64(key))


def uniform01(seed, stream, start, count, layer=0) -> np.ndarray:
    """Uniform in (0, 1) from the top 24 bits (never 0)."""
    return ((hash_u32(seed, stream, start, count, layer) >> np.uint64(8)).astype(np.float64) + 0.5) / 16777216.0


def normal(seed, stream, count, layer=0) -> np.ndarray:
    n2 = (count + 1) // 2
    u1 = uniform01(seed, stream, 0, n2, layer)
    u2 = uniform01(seed, stream, n2, n2, layer)
    r = np.sqrt(-2.0 * np.log(u1))
    z = np.concatenate([r * np.cos(2 * math.pi * u2), r * np.sin(2 * math.pi * u2)])
    return z[:count]


# ------------------------------------------------------------------------------------------
# weights
# ------------------------------------------------------------------------------------------
def tiles_per_matrix(H: int, I: int) -> int:
    return (H // 16) * (I // 16)


def trellis_np(seed: int, stream: int, start_word: int, count: int, layer: int = 0) -> np.ndarray:
    """`count` int16 words of the stacked tensor `stream` starting at flat word index `start_word`."""
    return (hash_u32(seed, stream, start_word, count, layer) & np.uint64(0xFFFF)).astype(np.uint16).view(np.int16)


def expert_trellis_np(seed: int, H: int, I: int, e: int, layer: int = 0, bits: int = 3):
    """(gate, up, down) int16 arrays of expert e in [k/16, n/16, 16*bits] layout."""
    tw = 16 * bits
    G = tiles_per_matrix(H, I) * tw
    gate = trellis_np(seed, STREAM_W13, (2 * e + 0) * G, G, layer).reshape(H // 16, I // 16, tw)
    up = trellis_np(seed, STREAM_W13, (2 * e + 1) * G, G, layer).reshape(H // 16, I // 16, tw)
    down = trellis_np(seed, STREAM_W2, e * G, G, layer).reshape(I // 16, H // 16, tw)
    return gate, up, down


def scales_np(seed: int, E: int, H: int, I: int, layer: int = 0):
    """w13_suh [E,2,H], w13_svh [E,2,I], w2_suh [E,I], w2_svh [E,H] as float16."""
    def signs(stream, n):
        b = hash_u32(seed, stream, 0, n, layer) & np.uint64(1)
        return np.where(b == 1, 1.0, -1.0).astype(np.float16)

    def svh(stream, n):
        return ((0.5 + uniform01(seed, stream, 0, n, layer)) / math.sqrt(4096.0)).astype(np.float16)

    return (signs(STREAM_SUH13, E * 2 * H).reshape(E, 2, H), svh(STREAM_SVH13, E * 2 * I).reshape(E, 2, I),
            signs(STREAM_SUH2, E * I).reshape(E, I), svh(STREAM_SVH2, E * H).reshape(E, H))


# ------------------------------------------------------------------------------------------
# activations and routing
# ------------------------------------------------------------------------------------------
def bf16_round(x: np.ndarray) -> np.ndarray:
    """float -> nearest bf16 (ties to even), returned as float32."""
    b = np.ascontiguousarray(x, np.float32).view(np.uint32).astype(np.uint64)
    r = (b + np.uint64(0x7FFF) + ((b >> np.uint64(16)) & np.uint64(1))) & np.uint64(0xFFFF0000)
    return r.astype(np.uint32).view(np.float32)


def hidden_np(seed: int, T: int, H: int, layer: int = 0) -> np.ndarray:
    """bf16-valued N(0,1) hidden states [T, H] as float32."""
    return bf16_round(normal(seed, STREAM_X, T * H, layer).astype(np.float32)).reshape(T, H)


def _softmax_rows(v: np.ndarray) -> np.ndarray:
    v = v - v.max(axis=1, keepdims=True)
    e = np.exp(v)
    return e / e.sum(axis=1, keepdims=True)


def routing_np(seed: int, T: int, E: int, topk: int, kind: str = "uniform", zipf_s: float = 1.1,
               layer: int = 0):
    """(ids int64 [T, topk], weights float32 [T, topk])."""
    if kind == "uniform":
        scores = normal(seed, STREAM_ROUTE, T * E, layer).reshape(T, E)
    elif kind == "zipf":
        rank = np.argsort(hash_u32(seed, STREAM_ZIPF_RANK, 0, E, layer), kind="stable")
        logp = -zipf_s * np.log(np.arange(1, E + 1, dtype=np.float64))
        logp_e = np.empty(E)
        logp_e[rank] = logp
        u = uniform01(seed, STREAM_ROUTE, 0, T * E, layer).reshape(T, E)
        scores = logp_e[None, :] - np.log(-np.log(u))
    else:
        raise ValueError(kind)
    ids = np.argsort(-scores, axis=1, kind="stable")[:, :topk]
    sel = np.take_along_axis(scores, ids, axis=1)
    w = _softmax_rows(sel).astype(np.float32)
    return ids.astype(np.int64), w


# ------------------------------------------------------------------------------------------
# torch (device) generation of the trellis: identical bits to trellis_np
# ------------------------------------------------------------------------------------------
def _mul32_t(x, c: int):
    # exact (x * c) mod 2^32 in int64 without overflow
    return ((x & 0xFFFF) * c + (((x >> 16) * (c & 0xFFFF)) << 16)) & M32


def _lowbias32_t(x):
    x = x & M32
    x = x ^ (x >> 16)
    x = _mul32_t(x, 0x7FEB352D)
    x = x ^ (x >> 15)
    x = _mul32_t(x, 0x846CA68B)
    x = x ^ (x >> 16)
    return x


def fill_trellis_torch(out, seed: int, stream: int, start_word: int = 0, layer: int = 0,
                       chunk: int = 1 << 24) -> None:
    """Fill an int16 tensor (any device) with words [start_word, start_word + numel) of `stream`."""
    import torch

    flat = out.view(-1)
    key = stream_key(seed, stream, layer)
    n = flat.numel()
    for s in range(0, n, chunk):
        cnt = min(chunk, n - s)
        idx = (torch.arange(start_word + s, start_word + s + cnt, device=flat.device, dtype=torch.int64) + key) & M32
        h = _lowbias32_t(_lowbias32_t(idx) ^ key)
        v = h & 0xFFFF
        flat[s:s + cnt] = torch.where(v >= 0x8000, v - 0x10000, v).to(torch.int16)
