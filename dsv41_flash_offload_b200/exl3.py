"""Drop-in for the vllm_exl3 fused-MoE op on B200.

`apply_exl3_fused_moe(x2d, ids, weights, layer, inners, expert_map, limit)` has the signature and
contract of the reference's op (patches/vllm-exl3-host-dma.patch:203-449, wrapped by
ct/ct_vllm.py:181-225 `_fused`): x2d [T, H] bf16/fp16/fp32 (cast to fp16 inside), ids [T, k] int
(negative or >= E = skipped), weights [T, k] fp32; returns a contiguous fp32 [T, H] tensor. All
work runs on the current CUDA stream through libdsv41_b200.so; nothing synchronises the host, so
the call can be captured in a CUDA graph once its workspace exists.

`Exl3MoELayer` holds one layer's experts in vllm_exl3's Exl3MoEMethod layout
(patch:633-684): w13_trellis [E, 2, H/16, I/16, 48] int16 (gate = 0, up = 1),
w2_trellis [E, I/16, H/16, 48], w13_suh [E, 2, H], w13_svh [E, 2, I], w2_suh [E, I],
w2_svh [E, H] fp16, plus the device pointer tables `_exl3_ptrs` the fused kernel reads
(patch:66-69). All experts are resident in HBM.
"""
from __future__ import annotations

import ctypes as C
import os
import threading

import torch

from . import _lib
from . import synth

SWIGLU_LIMIT_DEFAULT = 10.0       # patch:5
TEMP_ROWS_FUSED = 2048            # patch:6 (rows per expert the reference's fused kernel covers)


def _env_int(name: str, default: int) -> int:
    try:
        return int(os.environ.get(name, default))
    except (TypeError, ValueError):
        return default


# experts with more rows than this go to the tensor-core grouped GEMM (VLLM_EXL3_FAT_THRESHOLD,
# patch:146; 32 deployed by the reference's entrypoint, docker/entrypoint.sh:69). -1 keeps every
# expert on the decode GEMV.
FAT_EXPERT_THRESHOLD = _env_int("VLLM_EXL3_FAT_THRESHOLD", 32)

def _rows2d(t: torch.Tensor, T: int) -> torch.Tensor:
    """[T, k] view of a routing tensor given as [T, k] or flat [T*k] (also for T == 0)."""
    if t.dim() == 2 and t.shape[0] == T:
        return t
    k = t.shape[-1] if t.dim() >= 2 else (t.numel() // T if T else 0)
    return t.reshape(T, k)


_DTYPES = {torch.float16: _lib.DTYPE_F16, torch.bfloat16: _lib.DTYPE_BF16, torch.float32: _lib.DTYPE_F32}


class Exl3MoELayer:
    """One MoE layer's routed experts, HBM-resident, in the vllm_exl3 stacked layout."""

    def __init__(self, w13_trellis: torch.Tensor, w2_trellis: torch.Tensor, w13_suh: torch.Tensor,
                 w13_svh: torch.Tensor, w2_suh: torch.Tensor, w2_svh: torch.Tensor, ptrs: dict | None = None):
        E, two, ht, it, kw = w13_trellis.shape
        if two != 2 or kw not in (32, 48, 64):
            raise ValueError("w13_trellis must be [E, 2, H/16, I/16, 16*bits] with bits 2, 3 or 4")
        if tuple(w2_trellis.shape) != (E, it, ht, kw):
            raise ValueError(f"w2_trellis must be [E, I/16, H/16, {kw}]")
        self.bits = kw // 16
        H, I = ht * 16, it * 16
        for name, t, shape in (("w13_suh", w13_suh, (E, 2, H)), ("w13_svh", w13_svh, (E, 2, I)),
                               ("w2_suh", w2_suh, (E, I)), ("w2_svh", w2_svh, (E, H))):
            if tuple(t.shape) != shape or t.dtype != torch.float16 or not t.is_contiguous():
                raise ValueError(f"{name} must be contiguous fp16 {shape}")
        if w13_trellis.dtype != torch.int16 or w2_trellis.dtype != torch.int16:
            raise ValueError("trellis tensors must be int16")
        self.w13_trellis, self.w2_trellis = w13_trellis, w2_trellis
        self.w13_suh, self.w13_svh, self.w2_suh, self.w2_svh = w13_suh, w13_svh, w2_suh, w2_svh
        self._exl3_num_experts, self._exl3_hidden_size, self._exl3_intermediate_local = E, H, I
        dev = w13_suh.device
        if ptrs is None:
            if not (w13_trellis.is_contiguous() and w2_trellis.is_contiguous()):
                raise ValueError("trellis tensors must be contiguous (or pass pointer tables)")
            g0 = w13_trellis.data_ptr()
            d0 = w2_trellis.data_ptr()
            s13 = w13_trellis.stride(0) * 2
            ar = torch.arange(E, dtype=torch.int64)
            ptrs = {"gate_trellis": (g0 + ar * s13).to(dev), "up_trellis": (g0 + w13_trellis.stride(1) * 2 + ar * s13).to(dev),
                    "down_trellis": (d0 + ar * w2_trellis.stride(0) * 2).to(dev)}
        self._exl3_ptrs = ptrs
        self._c = _lib.MoeLayer(E, H, I, self.bits, ptrs["gate_trellis"].data_ptr(), ptrs["up_trellis"].data_ptr(),
                                ptrs["down_trellis"].data_ptr(), w13_suh.data_ptr(), w13_svh.data_ptr(),
                                w2_suh.data_ptr(), w2_svh.data_ptr())

    @classmethod
    def from_pointer_tables(cls, ptrs: dict, w13_suh: torch.Tensor, w13_svh: torch.Tensor, w2_suh: torch.Tensor,
                            w2_svh: torch.Tensor, bits: int = 3) -> "Exl3MoELayer":
        """Layer over expert trellis that live anywhere in device memory: ptrs holds device int64
        [E] address tables 'gate_trellis', 'up_trellis', 'down_trellis' (patch:66-69); the caller keeps
        the trellis storage alive. Addresses must be 16-byte aligned."""
        E, _, H = w13_suh.shape
        I = w13_svh.shape[2]
        self = cls.__new__(cls)
        for name, t, shape in (("w13_suh", w13_suh, (E, 2, H)), ("w13_svh", w13_svh, (E, 2, I)),
                               ("w2_suh", w2_suh, (E, I)), ("w2_svh", w2_svh, (E, H))):
            if tuple(t.shape) != shape or t.dtype != torch.float16 or not t.is_contiguous():
                raise ValueError(f"{name} must be contiguous fp16 {shape}")
        for k in ("gate_trellis", "up_trellis", "down_trellis"):
            t = ptrs[k]
            if t.dtype != torch.int64 or t.numel() != E or t.device != w13_suh.device:
                raise ValueError(f"ptrs[{k}] must be int64 [E] on the scales' device")
            if bool(((t % 16) != 0).any()):
                raise ValueError(f"ptrs[{k}] has an address that is not 16-byte aligned")
        if bits not in (2, 3, 4):
            raise ValueError(f"bits {bits} (2, 3 or 4)")
        self.bits = bits
        self.w13_trellis = self.w2_trellis = None
        self.w13_suh, self.w13_svh, self.w2_suh, self.w2_svh = w13_suh, w13_svh, w2_suh, w2_svh
        self._exl3_num_experts, self._exl3_hidden_size, self._exl3_intermediate_local = E, H, I
        self._exl3_ptrs = {k: ptrs[k].contiguous() for k in ("gate_trellis", "up_trellis", "down_trellis")}
        p = self._exl3_ptrs
        self._c = _lib.MoeLayer(E, H, I, self.bits, p["gate_trellis"].data_ptr(), p["up_trellis"].data_ptr(),
                                p["down_trellis"].data_ptr(), w13_suh.data_ptr(), w13_svh.data_ptr(),
                                w2_suh.data_ptr(), w2_svh.data_ptr())
        return self

    @property
    def device(self):
        return self.w13_suh.device

    @classmethod
    def synthetic(cls, num_experts: int, hidden: int, intermediate: int, seed: int = 0, layer: int = 0,
                  device="cuda", expert_range: tuple | None = None, bits: int = 3) -> "Exl3MoELayer":
        """Random EXL3 layer (BASELINE's synthetic weights; `bits` per weight, 3 by default),
        generated on the device. expert_range=(lo, hi) builds only experts lo..hi-1 of the
        num_experts-expert layer (an expert-parallel shard), bit-identical to those experts of
        the full layer."""
        E, H, I = num_experts, hidden, intermediate
        lo, hi = expert_range if expert_range is not None else (0, E)
        n = hi - lo
        dev = torch.device(device)
        w13 = torch.empty((n, 2, H // 16, I // 16, 16 * bits), dtype=torch.int16, device=dev)
        w2 = torch.empty((n, I // 16, H // 16, 16 * bits), dtype=torch.int16, device=dev)
        per13, per2 = w13[0].numel() if n else 0, w2[0].numel() if n else 0
        synth.fill_trellis_torch(w13, seed, synth.STREAM_W13, lo * per13, layer)
        synth.fill_trellis_torch(w2, seed, synth.STREAM_W2, lo * per2, layer)
        s13, v13, s2, v2 = (torch.from_numpy(a[lo:hi].copy()).to(dev) for a in synth.scales_np(seed, E, H, I, layer))
        return cls(w13, w2, s13.contiguous(), v13.contiguous(), s2.contiguous(), v2.contiguous())

    def expert_bytes(self) -> int:
        """Compressed bytes one expert streams per forward (three trellis matrices + fp16 scales)."""
        H, I = self._exl3_hidden_size, self._exl3_intermediate_local
        return 3 * (H // 16) * (I // 16) * 32 * self.bits + (2 * H + 2 * I + I + H) * 2


def as_layer(layer) -> Exl3MoELayer:
    """The Exl3MoELayer for `layer`: itself, or -- for a vLLM FusedMoE layer set up by vllm_exl3's
    Exl3MoEMethod (w13_trellis/w2_trellis/w13_suh/w13_svh/w2_suh/w2_svh parameters, patch:633-684) --
    a view of its tensors, built once and cached on the layer as `_dsv41`."""
    if isinstance(layer, Exl3MoELayer):
        return layer
    cached = getattr(layer, "_dsv41", None)
    if cached is not None:
        return cached
    t = lambda name: getattr(layer, name).data if hasattr(getattr(layer, name), "data") else getattr(layer, name)
    view = Exl3MoELayer(t("w13_trellis"), t("w2_trellis"), t("w13_suh").contiguous(), t("w13_svh").contiguous(),
                        t("w2_suh").contiguous(), t("w2_svh").contiguous())
    layer._dsv41 = view
    return view


# --------------------------------------------------------------------------------------------
# workspaces: one grow-only device buffer per (device, stream); callers that overlap calls on
# several streams get one each. Graph capture needs the buffer to exist before capture.
# --------------------------------------------------------------------------------------------
_ws_lock = threading.Lock()
_ws: dict = {}


def _workspace(device: torch.device, nbytes: int, stream: torch.cuda.Stream) -> torch.Tensor:
    key = (device.index, stream.cuda_stream)
    with _ws_lock:
        buf = _ws.get(key)
        if buf is None or buf.numel() < nbytes:
            if torch.cuda.is_current_stream_capturing():
                raise RuntimeError("dsv41: workspace must be allocated before CUDA-graph capture (run once eagerly)")
            buf = torch.zeros(max(nbytes, 1 << 20), dtype=torch.uint8, device=device)
            _ws[key] = buf
        return buf


def workspace_bytes(T: int, topk: int, layer: Exl3MoELayer, fat_threshold: int | None = None, split_k: int = 0) -> int:
    fat = FAT_EXPERT_THRESHOLD if fat_threshold is None else fat_threshold
    opt = _lib.MoeOptions(fat, 0.0, None, 0, split_k)
    n = C.c_size_t()
    L = _lib.load()
    _lib.check(L.dsv41_moe_workspace_size(T, topk, layer._exl3_num_experts, layer._exl3_hidden_size,
                                          layer._exl3_intermediate_local, C.byref(opt), C.byref(n)), "workspace_size")
    return n.value


def _stream_ptr(s: torch.cuda.Stream):
    return C.c_void_p(s.cuda_stream)


def apply_exl3_fused_moe(x2d: torch.Tensor, ids: torch.Tensor, weights: torch.Tensor, layer: Exl3MoELayer,
                         inners=None, expert_map: torch.Tensor | None = None, limit: float | None = None,
                         *, fat_threshold: int | None = None, split_k: int = 0, max_routes: int = 0,
                         out: torch.Tensor | None = None, workspace: torch.Tensor | None = None) -> torch.Tensor:
    """Routed-expert MoE forward; returns fp32 [T, H] (see module docstring). `inners` is accepted for
    signature compatibility and unused (the experts come from `layer`)."""
    L = _lib.load()
    layer = as_layer(layer)
    if x2d.dim() != 2:
        raise ValueError("x2d must be [T, H]")
    T, H = x2d.shape
    if H != layer._exl3_hidden_size:
        raise ValueError(f"hidden size {H} != layer's {layer._exl3_hidden_size}")
    dev = layer.device
    if x2d.device != dev or not x2d.is_cuda:
        raise ValueError("x2d must live on the layer's CUDA device")
    if x2d.dtype not in _DTYPES:
        raise TypeError(f"unsupported activation dtype {x2d.dtype}")
    x2d = x2d.contiguous()
    ids = _rows2d(ids, T).to(device=dev, dtype=torch.int64).contiguous()
    topk = ids.shape[1]
    weights = weights.reshape(T, topk).to(device=dev, dtype=torch.float32).contiguous()
    if out is None:
        out = torch.empty((T, H), dtype=torch.float32, device=dev)
    elif out.shape != (T, H) or out.dtype != torch.float32 or not out.is_contiguous() or out.device != dev:
        raise ValueError("out must be a contiguous fp32 [T, H] tensor on the layer's device")
    fat = FAT_EXPERT_THRESHOLD if fat_threshold is None else int(fat_threshold)
    lim = float(limit) if (limit is not None and limit > 0) else 0.0
    emap = None
    if expert_map is not None:
        emap = expert_map.to(device=dev, dtype=torch.int32).contiguous()
    opt = _lib.MoeOptions(fat, lim, emap.data_ptr() if emap is not None else None,
                          emap.numel() if emap is not None else 0, split_k, int(max_routes))
    stream = torch.cuda.current_stream(dev)
    nbytes = C.c_size_t()
    _lib.check(L.dsv41_moe_workspace_size(T, topk, layer._exl3_num_experts, H, layer._exl3_intermediate_local,
                                          C.byref(opt), C.byref(nbytes)), "workspace_size")
    ws = workspace if workspace is not None else _workspace(dev, nbytes.value, stream)
    if ws.numel() < nbytes.value:
        raise ValueError(f"workspace of {ws.numel()} bytes < {nbytes.value}")
    with torch.cuda.device(dev):
        rc = L.dsv41_moe_forward(C.byref(layer._c), x2d.data_ptr(), _DTYPES[x2d.dtype], T, ids.data_ptr(),
                                 weights.data_ptr(), topk, C.byref(opt), out.data_ptr(), ws.data_ptr(), ws.numel(),
                                 _stream_ptr(stream))
    _lib.check(rc, "dsv41_moe_forward")
    return out


_SCORING = {"softmax": 0, "sigmoid": 1}


def _router_opts(scoring, renormalize, num_expert_group, topk_group, correction_bias, routed_scaling_factor, dev):
    if scoring not in _SCORING:
        raise ValueError(f"scoring must be one of {sorted(_SCORING)}")
    bias = None
    if correction_bias is not None:
        bias = correction_bias.to(device=dev, dtype=torch.float32).contiguous()
    opt = _lib.RouterOptions(_SCORING[scoring], int(bool(renormalize)), int(num_expert_group or 0), int(topk_group or 0),
                             bias.data_ptr() if bias is not None else None, float(routed_scaling_factor))
    return opt, bias


def route_topk(logits: torch.Tensor, topk: int, *, scoring: str = "softmax", renormalize: bool = True,
               num_expert_group: int = 0, topk_group: int = 0, correction_bias: torch.Tensor | None = None,
               routed_scaling_factor: float = 1.0) -> tuple[torch.Tensor, torch.Tensor]:
    """Router top-k on the GPU (vLLM's routing rule, see dsv41_router_topk): gating logits [T, E]
    (fp16/bf16/fp32) -> (ids int64 [T, topk], weights fp32 [T, topk]), ids in descending order of
    their selection value."""
    L = _lib.load()
    if logits.dim() != 2 or not logits.is_cuda or logits.dtype not in _DTYPES:
        raise ValueError("logits must be a CUDA [T, E] fp16/bf16/fp32 tensor")
    logits = logits.contiguous()
    T, E = logits.shape
    dev = logits.device
    opt, bias = _router_opts(scoring, renormalize, num_expert_group, topk_group, correction_bias,
                             routed_scaling_factor, dev)
    ids = torch.empty((T, topk), dtype=torch.int64, device=dev)
    w = torch.empty((T, topk), dtype=torch.float32, device=dev)
    with torch.cuda.device(dev):
        _lib.check(L.dsv41_router_topk(logits.data_ptr(), _DTYPES[logits.dtype], T, E, topk, C.byref(opt),
                                       ids.data_ptr(), w.data_ptr(), _stream_ptr(torch.cuda.current_stream(dev))),
                   "dsv41_router_topk")
    return ids, w


def apply_exl3_fused_moe_logits(x2d: torch.Tensor, logits: torch.Tensor, layer: Exl3MoELayer, topk: int,
                                limit: float | None = None, *, scoring: str = "softmax", renormalize: bool = True,
                                num_expert_group: int = 0, topk_group: int = 0,
                                correction_bias: torch.Tensor | None = None, routed_scaling_factor: float = 1.0,
                                fat_threshold: int | None = None, return_routes: bool = False):
    """Router top-k and the routed-expert layer in one C-ABI call (dsv41_moe_forward_logits): the ids
    and weights go from the router kernel to the permute kernel without leaving the workspace.
    Returns fp32 [T, H] (and (ids, weights) when return_routes)."""
    L = _lib.load()
    layer = as_layer(layer)
    T, H = x2d.shape
    dev = layer.device
    if logits.shape != (T, layer._exl3_num_experts) or logits.dtype not in _DTYPES or x2d.dtype not in _DTYPES:
        raise ValueError("logits must be [T, E] fp16/bf16/fp32 and x2d fp16/bf16/fp32")
    x2d, logits = x2d.contiguous(), logits.to(dev).contiguous()
    ropt, bias = _router_opts(scoring, renormalize, num_expert_group, topk_group, correction_bias,
                              routed_scaling_factor, dev)
    fat = FAT_EXPERT_THRESHOLD if fat_threshold is None else int(fat_threshold)
    lim = float(limit) if (limit is not None and limit > 0) else 0.0
    opt = _lib.MoeOptions(fat, lim, None, 0, 0, 0)
    out = torch.empty((T, H), dtype=torch.float32, device=dev)
    ids = torch.empty((T, topk), dtype=torch.int64, device=dev) if return_routes else None
    w = torch.empty((T, topk), dtype=torch.float32, device=dev) if return_routes else None
    stream = torch.cuda.current_stream(dev)
    nbytes = C.c_size_t()
    _lib.check(L.dsv41_moe_workspace_size(T, topk, layer._exl3_num_experts, H, layer._exl3_intermediate_local,
                                          C.byref(opt), C.byref(nbytes)), "workspace_size")
    ws = _workspace(dev, nbytes.value, stream)
    with torch.cuda.device(dev):
        _lib.check(L.dsv41_moe_forward_logits(C.byref(layer._c), x2d.data_ptr(), _DTYPES[x2d.dtype], T,
                                              logits.data_ptr(), _DTYPES[logits.dtype], C.byref(ropt), topk,
                                              C.byref(opt), out.data_ptr(), ids.data_ptr() if ids is not None else None,
                                              w.data_ptr() if w is not None else None, ws.data_ptr(), ws.numel(),
                                              _stream_ptr(stream)), "dsv41_moe_forward_logits")
    return (out, (ids, w)) if return_routes else out


def apply_exl3_experts(x: torch.Tensor, topk_ids: torch.Tensor, topk_weights: torch.Tensor, layer: Exl3MoELayer,
                       expert_map: torch.Tensor | None = None, limit: float | None = SWIGLU_LIMIT_DEFAULT,
                       **kw) -> torch.Tensor:
    """apply_exl3_experts (patch:496-505): flatten leading dims, run the fused op, restore shape."""
    shape = x.shape
    x2d = x.reshape(-1, shape[-1])
    T = x2d.shape[0]
    out = apply_exl3_fused_moe(x2d, _rows2d(topk_ids, T), _rows2d(topk_weights, T), layer, None, expert_map,
                               limit, **kw)
    return out.view(*shape[:-1], shape[-1])


def read_status(workspace: torch.Tensor | None = None, device=None) -> int:
    """Synchronise and return (then clear) the device status word of a workspace: 0 = ok,
    1 = a bounded device-side wait ran out (results of that call are invalid), 3 = more valid routes
    than max_routes (that call's output is zero)."""
    L = _lib.load()
    if workspace is None:
        dev = torch.device(device) if device is not None else torch.device("cuda", torch.cuda.current_device())
        stream = torch.cuda.current_stream(dev)
        workspace = _ws.get((dev.index, stream.cuda_stream))
        if workspace is None:
            return 0
    st = C.c_int32()
    with torch.cuda.device(workspace.device):
        _lib.check(L.dsv41_read_status(workspace.data_ptr(), _stream_ptr(torch.cuda.current_stream(workspace.device)),
                                       C.byref(st)), "read_status")
    return st.value


def wait_selftest(limit_us: int = 20000, device=None) -> int:
    """Failure-detection self test: one device wait that can never complete runs through the bounded
    wait of the pipeline kernels with a `limit_us` limit; returns the status word it left (1 when the
    wait gave up as designed). The context stays usable afterwards."""
    L = _lib.load()
    dev = torch.device(device) if device is not None else torch.device("cuda", torch.cuda.current_device())
    ws = torch.zeros(256, dtype=torch.uint8, device=dev)
    with torch.cuda.device(dev):
        _lib.check(L.dsv41_wait_selftest(ws.data_ptr(), int(limit_us), _stream_ptr(torch.cuda.current_stream(dev))),
                   "wait_selftest")
    return read_status(ws)


# --------------------------------------------------------------------------------------------
# lower-level entry points
# --------------------------------------------------------------------------------------------
def permute(ids: torch.Tensor, weights: torch.Tensor | None, num_experts: int, expert_map: torch.Tensor | None = None):
    """Routing permutation on the device (bit-exact, stable). Returns dict of tensors:
    counts/offsets int64 [E+1], token_sorted/route_sorted int32 [N], weight_sorted fp32 [N],
    route_pos int32 [N] (-1 = skipped route)."""
    L = _lib.load()
    dev = ids.device
    T = ids.shape[0]
    ids = _rows2d(ids, T).to(torch.int64).contiguous()
    k = ids.shape[1]
    N = T * k
    w = None if weights is None else weights.reshape(T, k).to(torch.float32).contiguous()
    emap = None if expert_map is None else expert_map.to(device=dev, dtype=torch.int32).contiguous()
    E = num_experts
    o = dict(counts=torch.empty(E + 1, dtype=torch.int64, device=dev),
             offsets=torch.empty(E + 1, dtype=torch.int64, device=dev),
             token_sorted=torch.empty(max(N, 1), dtype=torch.int32, device=dev),
             weight_sorted=torch.empty(max(N, 1), dtype=torch.float32, device=dev),
             route_sorted=torch.empty(max(N, 1), dtype=torch.int32, device=dev),
             route_pos=torch.empty(max(N, 1), dtype=torch.int32, device=dev))
    ws = torch.empty(L.dsv41_permute_workspace_size(T, k, E), dtype=torch.uint8, device=dev)
    stream = torch.cuda.current_stream(dev)
    with torch.cuda.device(dev):
        rc = L.dsv41_permute(ids.data_ptr(), None if w is None else w.data_ptr(), T, k, E,
                             None if emap is None else emap.data_ptr(), 0 if emap is None else emap.numel(),
                             o["counts"].data_ptr(), o["offsets"].data_ptr(), o["token_sorted"].data_ptr(),
                             o["weight_sorted"].data_ptr(), o["route_sorted"].data_ptr(), o["route_pos"].data_ptr(),
                             ws.data_ptr(), ws.numel(), _stream_ptr(stream))
    _lib.check(rc, "dsv41_permute")
    for key in ("token_sorted", "weight_sorted", "route_sorted", "route_pos"):
        o[key] = o[key][:N]
    return o


def combine(y: torch.Tensor, route_pos: torch.Tensor, weights: torch.Tensor, out: torch.Tensor | None = None,
            accumulate: bool = False) -> torch.Tensor:
    """out[t] = sum_j weights[t, j] * y[route_pos[t, j]] (fp32), y [rows, H] fp16."""
    L = _lib.load()
    T, k = weights.shape
    H = y.shape[1]
    if out is None:
        out = torch.empty((T, H), dtype=torch.float32, device=y.device)
    rp = route_pos.to(torch.int32).contiguous()
    w = weights.to(torch.float32).contiguous()
    with torch.cuda.device(y.device):
        rc = L.dsv41_combine(y.contiguous().data_ptr(), rp.data_ptr(), w.data_ptr(), T, k, H, int(accumulate),
                             out.data_ptr(), _stream_ptr(torch.cuda.current_stream(y.device)))
    _lib.check(rc, "dsv41_combine")
    return out


def decode_dense(trellis: torch.Tensor, k: int, n: int, bits: int | None = None) -> torch.Tensor:
    """Dense fp16 W [k, n] of one trellis matrix [k/16, n/16, 16*bits] (bit-exact reconstruct);
    bits (2, 3 or 4) defaults to what the trellis size implies."""
    L = _lib.load()
    t = trellis.contiguous()
    tiles = (k // 16) * (n // 16)
    if bits is None:
        bits = t.numel() // (16 * tiles) if tiles else 3
    if bits not in (2, 3, 4) or t.numel() != tiles * 16 * bits:
        raise ValueError("trellis size does not match k x n at 2, 3 or 4 bits per weight")
    w = torch.empty((k, n), dtype=torch.float16, device=t.device)
    with torch.cuda.device(t.device):
        rc = L.dsv41_decode_dense_bits(t.data_ptr(), k, n, bits, w.data_ptr(),
                                       _stream_ptr(torch.cuda.current_stream(t.device)))
    _lib.check(rc, "dsv41_decode_dense_bits")
    return w
