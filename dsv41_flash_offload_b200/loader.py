"""EXL3 checkpoint loader for the routed experts: safetensors shards -> one HBM-resident layer.

Checkpoint convention (the reference's packs, patches/vllm-exl3-host-dma.patch:569-577 and
pack/prepare_pack.py:16-64): tensors named `[model.]layers.{L}.ffn.experts.{e}.{w}.{suffix}` with
w = w1 (gate), w3 (up), w2 (down) and suffix = trellis (int16 [K/16, N/16, 16*bits]), suh (fp16
[K]), svh (fp16 [N]) and the codebook markers mcg / mul1; shards listed by
model.safetensors.index.json (or a single model.safetensors); config.json's quantization_config
gives bits, codebook and per-layer `layer_bits` overrides.

`load_moe_layer` stacks one layer's experts (or an expert-parallel shard of them) into vllm_exl3's
layout (w13_trellis [E, 2, H/16, I/16, 48], w2_trellis [E, I/16, H/16, 48], w13_suh [E, 2, H], ...,
patch:633-684) on the device, ready for apply_exl3_fused_moe. The mul1 codebook at 2, 3 or 4 bits
per weight is accepted (what the kernels decode); other layers raise NotImplementedError. The safetensors format
is parsed here directly (8-byte little-endian header length, JSON header, raw little-endian data),
so nothing beyond numpy and torch is needed; `write_safetensors` is the matching writer.
"""
from __future__ import annotations

import json
import os
import re
import struct

import numpy as np
import torch

MUL1 = 0x83DCD12D
_DTYPES = {"I16": np.int16, "U16": np.uint16, "F16": np.float16, "I32": np.int32, "U32": np.uint32,
           "F32": np.float32, "I64": np.int64, "U8": np.uint8, "I8": np.int8, "F64": np.float64}
_NAMES = {np.dtype(v): k for k, v in _DTYPES.items()}
_EXPERT = re.compile(r"^(?P<prefix>.*?)layers\.(?P<layer>\d+)\.ffn\.experts\.(?P<e>\d+)\.(?P<w>w[123])\.(?P<s>\w+)$")


def read_header(path: str) -> tuple[dict, int]:
    """({name: {"dtype", "shape", "data_offsets"}}, byte offset of the data section)."""
    with open(path, "rb") as f:
        n = struct.unpack("<Q", f.read(8))[0]
        if n > 1 << 28:
            raise ValueError(f"{path}: implausible safetensors header length {n}")
        hdr = json.loads(f.read(n))
    hdr.pop("__metadata__", None)
    return hdr, 8 + n


def write_safetensors(path: str, tensors: dict, metadata: dict | None = None) -> None:
    """Write numpy arrays (C order, little-endian dtypes of _DTYPES) as one safetensors file."""
    hdr, off, blobs = {}, 0, []
    for name, a in tensors.items():
        a = np.ascontiguousarray(a)
        if a.dtype not in _NAMES:
            raise TypeError(f"{name}: unsupported dtype {a.dtype}")
        b = a.tobytes()
        hdr[name] = {"dtype": _NAMES[a.dtype], "shape": list(a.shape), "data_offsets": [off, off + len(b)]}
        off += len(b)
        blobs.append(b)
    if metadata:
        hdr["__metadata__"] = {str(k): str(v) for k, v in metadata.items()}
    h = json.dumps(hdr, separators=(",", ":")).encode()
    h += b" " * (-len(h) % 8)
    with open(path, "wb") as f:
        f.write(struct.pack("<Q", len(h)))
        f.write(h)
        for b in blobs:
            f.write(b)


class Checkpoint:
    """Read access to a safetensors checkpoint directory (or a single .safetensors file)."""

    def __init__(self, path: str):
        self.root = path if os.path.isdir(path) else os.path.dirname(path)
        if os.path.isdir(path):
            idx = os.path.join(path, "model.safetensors.index.json")
            if os.path.exists(idx):
                wm = json.load(open(idx))["weight_map"]
                files = sorted(set(wm.values()))
            else:
                files = sorted(f for f in os.listdir(path) if f.endswith(".safetensors"))
        else:
            files = [os.path.basename(path)]
        self.files = {}
        self.where = {}
        for fn in files:
            full = os.path.join(self.root, fn)
            hdr, start = read_header(full)
            self.files[fn] = (full, hdr, start)
            for name in hdr:
                self.where[name] = fn
        cfg = os.path.join(self.root, "config.json")
        self.config = json.load(open(cfg)) if os.path.exists(cfg) else {}
        self._mmaps = {}

    def names(self):
        return self.where.keys()

    def has(self, name: str) -> bool:
        return name in self.where

    def tensor(self, name: str) -> np.ndarray:
        """Zero-copy (memory-mapped) view of one tensor."""
        fn = self.where[name]
        full, hdr, start = self.files[fn]
        m = self._mmaps.get(fn)
        if m is None:
            m = self._mmaps[fn] = np.memmap(full, dtype=np.uint8, mode="r")
        ent = hdr[name]
        a, b = ent["data_offsets"]
        return m[start + a:start + b].view(_DTYPES[ent["dtype"]]).reshape(ent["shape"])

    def quantization(self) -> dict:
        return self.config.get("quantization_config", {}) or {}

    def layer_bits(self, layer: int) -> int:
        q = self.quantization()
        return int((q.get("layer_bits") or {}).get(str(layer), q.get("bits", 3)))

    def expert_ids(self, layer: int) -> tuple[str, list[int]]:
        """(name prefix, sorted expert ids) of `layer`'s routed experts."""
        found, prefix = set(), None
        for n in self.where:
            m = _EXPERT.match(n)
            if m and int(m["layer"]) == layer:
                found.add(int(m["e"]))
                prefix = m["prefix"]
        if not found:
            raise KeyError(f"no routed experts of layer {layer} in {self.root}")
        return prefix, sorted(found)


def _check_codebook(ck: Checkpoint, key: str) -> None:
    if ck.has(key + ".mcg") and np.any(ck.tensor(key + ".mcg") != 0):
        raise NotImplementedError(f"{key}: mcg codebook (the kernels decode the mul1 codebook)")
    if ck.has(key + ".mul1"):
        m = np.asarray(ck.tensor(key + ".mul1")).reshape(-1)
        if m.size == 1 and m.dtype.kind in "iu" and (int(m[0]) & 0xFFFFFFFF) not in (0, MUL1):
            raise NotImplementedError(f"{key}: mul1 multiplier {int(m[0]) & 0xFFFFFFFF:#x} != {MUL1:#x}")


def load_moe_layer(path_or_ckpt, layer: int, device="cuda", expert_range: tuple | None = None):
    """The routed experts of `layer` as an Exl3MoELayer on `device` (experts [lo, hi) of
    expert_range for an expert-parallel shard, local ids 0..hi-lo-1)."""
    from .exl3 import Exl3MoELayer
    ck = path_or_ckpt if isinstance(path_or_ckpt, Checkpoint) else Checkpoint(path_or_ckpt)
    q = ck.quantization()
    if q.get("codebook", "mul1") != "mul1":
        raise NotImplementedError(f"codebook {q.get('codebook')!r}: the kernels decode the mul1 codebook")
    bits = ck.layer_bits(layer)
    if bits not in (2, 3, 4):
        raise NotImplementedError(f"layer {layer} is {bits}-bit; the kernels decode 2, 3 or 4 bits per weight")
    prefix, ids = ck.expert_ids(layer)
    E = ids[-1] + 1
    if ids != list(range(E)):
        raise KeyError(f"layer {layer}: experts {sorted(set(range(E)) - set(ids))} missing")
    lo, hi = expert_range if expert_range is not None else (0, E)
    if not (0 <= lo < hi <= E):
        raise ValueError(f"expert_range {expert_range} outside 0..{E}")
    base = lambda e, w: f"{prefix}layers.{layer}.ffn.experts.{e}.{w}"
    t1 = ck.tensor(base(0, "w1") + ".trellis")
    Ht, It, kw = t1.shape
    if kw != 16 * bits or t1.dtype != np.int16:
        raise ValueError(f"w1 trellis of layer {layer} is {t1.dtype} {t1.shape}; expected int16 "
                         f"[H/16, I/16, {16 * bits}] at {bits} bits")
    H, I = Ht * 16, It * 16
    n = hi - lo
    dev = torch.device(device)
    w13 = torch.empty((n, 2, Ht, It, kw), dtype=torch.int16, device=dev)
    w2 = torch.empty((n, It, Ht, kw), dtype=torch.int16, device=dev)
    suh13 = torch.empty((n, 2, H), dtype=torch.float16, device=dev)
    svh13 = torch.empty((n, 2, I), dtype=torch.float16, device=dev)
    suh2 = torch.empty((n, I), dtype=torch.float16, device=dev)
    svh2 = torch.empty((n, H), dtype=torch.float16, device=dev)

    def put(dst, name, shape, dtype):
        a = ck.tensor(name)
        if tuple(a.shape) != shape or a.dtype != dtype:
            raise ValueError(f"{name}: {a.dtype} {tuple(a.shape)}; expected {np.dtype(dtype)} {shape}")
        dst.copy_(torch.from_numpy(np.array(a)))   # host copy of the read-only map, then to the device

    for j, e in enumerate(range(lo, hi)):
        for w, m in (("w1", 0), ("w3", 1)):
            key = base(e, w)
            _check_codebook(ck, key)
            put(w13[j, m], key + ".trellis", (Ht, It, kw), np.int16)
            put(suh13[j, m], key + ".suh", (H,), np.float16)
            put(svh13[j, m], key + ".svh", (I,), np.float16)
        key = base(e, "w2")
        _check_codebook(ck, key)
        put(w2[j], key + ".trellis", (It, Ht, kw), np.int16)
        put(suh2[j], key + ".suh", (I,), np.float16)
        put(svh2[j], key + ".svh", (H,), np.float16)
    return Exl3MoELayer(w13, w2, suh13, svh13, suh2, svh2)
