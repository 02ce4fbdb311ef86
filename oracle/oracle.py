"""TEST INFRASTRUCTURE ONLY -- ctypes access to the CPU checker.

`Oracle` wraps liboracle.so, the plain-C restatement of the reference's EXL3 mul1 expert path
(exl3_oracle.c). `RefShim` wraps oracle/_ref/libref_shim.so, the reference's own
kernels/cpu_avx2/ft_core.h compiled unchanged (built only where the reference tree exists).
`load_ref_tier()` imports the reference's CPU tier host (kernels/cpu_avx2/ft_tier_ext.cpp) built
by build_ref_tier.py -- the timed CPU baseline.

Only tests/, __graft_entry__.smoke() and bench.py's cpu_baseline / reference legs use this module,
as the checker or as the reference arm; the product path never imports it.
"""
from __future__ import annotations

import ctypes as C
import importlib.util
import os
import subprocess

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
REF_DIR = os.path.join(HERE, "_ref")

_f32p = np.ctypeslib.ndpointer(np.float32, flags="C")
_u16p = np.ctypeslib.ndpointer(np.uint16, flags="C")
_i64p = np.ctypeslib.ndpointer(np.int64, flags="C")
_i32p = np.ctypeslib.ndpointer(np.int32, flags="C")


def build(ref: bool = False) -> None:
    """Compile liboracle.so (and, with ref=True and the reference tree present, _ref/)."""
    targets = ["all"] + (["ref"] if ref else [])
    subprocess.run(["make", "-s", "-C", HERE] + targets, check=True)


def _ptr_array(arrs):
    a = (C.c_void_p * len(arrs))()
    for i, x in enumerate(arrs):
        a[i] = None if x is None else x.ctypes.data
    return a


class Oracle:
    def __init__(self, path: str | None = None):
        path = path or os.path.join(HERE, "liboracle.so")
        if not os.path.exists(path):
            build()
        L = C.CDLL(path)
        L.orc_h2f.restype = C.c_float
        L.orc_h2f.argtypes = [C.c_uint16]
        L.orc_set_bits.argtypes = [C.c_int]
        L.orc_get_bits.restype = C.c_int
        L.orc_f2h.restype = C.c_uint16
        L.orc_f2h.argtypes = [C.c_float]
        L.orc_perm.restype = C.c_int
        L.orc_perm.argtypes = [C.c_int]
        L.orc_state.restype = C.c_uint16
        L.orc_state.argtypes = [_u16p, C.c_int]
        L.orc_bytesum.restype = C.c_int
        L.orc_bytesum.argtypes = [C.c_uint16]
        L.orc_weight_bits.restype = C.c_uint16
        L.orc_weight_bits.argtypes = [C.c_uint16]
        L.orc_decode_matrix.argtypes = [_u16p, C.c_int, C.c_int, _u16p]
        L.orc_prep_block.argtypes = [_f32p, _u16p, _f32p]
        L.orc_out_block.argtypes = [_f32p, _u16p]
        L.orc_act.restype = C.c_float
        L.orc_act.argtypes = [C.c_float, C.c_float, C.c_float]
        L.orc_linear.argtypes = [_u16p, _u16p, _u16p, C.c_int, C.c_int, C.c_int, _f32p, _f32p]
        L.orc_expert.argtypes = [_u16p] * 3 + [_u16p] * 6 + [C.c_int] * 3 + [_f32p, C.c_float, _f32p]
        L.orc_permute.argtypes = [_i64p, C.c_void_p, C.c_int, C.c_int, C.c_int, C.c_void_p, C.c_int,
                                  _i64p, _i64p, _i32p, _f32p, _i32p, _i32p]
        common = [C.c_void_p, C.c_int, C.c_int, C.c_int, C.c_void_p]
        L.orc_moe_layer.argtypes = common + [C.c_void_p, C.c_int, C.c_int, C.c_void_p, C.c_int] + \
            [C.c_void_p] * 7 + [C.c_float, C.c_int, C.c_void_p]
        L.orc_moe_routes.argtypes = common + [C.c_int, C.c_int, C.c_void_p, C.c_int] + \
            [C.c_void_p] * 7 + [C.c_float, C.c_int, C.c_void_p]
        self.L = L

    def set_bits(self, bits: int) -> None:
        """Bits per weight K of the trellis tiles (2, 3 or 4) for every following call."""
        self.L.orc_set_bits(int(bits))

    @property
    def bits(self) -> int:
        return self.L.orc_get_bits()

    # --- format -------------------------------------------------------------------------
    def weight_table(self) -> np.ndarray:
        """fp16 bits of the decoded weight for every 16-bit state (65536 entries)."""
        return np.array([self.L.orc_weight_bits(s) for s in range(65536)], dtype=np.uint16)

    def decode_matrix(self, trellis: np.ndarray, k: int, n: int) -> np.ndarray:
        tr = np.ascontiguousarray(trellis).view(np.uint16).reshape(-1)
        W = np.empty((k, n), dtype=np.uint16)
        self.L.orc_decode_matrix(tr, k, n, W)
        return W.view(np.float16)

    def states(self, tile: np.ndarray) -> np.ndarray:
        t = np.ascontiguousarray(tile).view(np.uint16).reshape(-1)
        return np.array([self.L.orc_state(t, i) for i in range(256)], dtype=np.uint16)

    def prep_block(self, x, suh):
        xt = np.empty(128, np.float32)
        self.L.orc_prep_block(np.ascontiguousarray(x, np.float32), np.ascontiguousarray(suh).view(np.uint16), xt)
        return xt

    def out_block(self, y, svh):
        y = np.array(y, dtype=np.float32)
        self.L.orc_out_block(y, np.ascontiguousarray(svh).view(np.uint16))
        return y

    def act(self, g, u, limit):
        return self.L.orc_act(g, u, limit)

    def expert(self, gate, up, down, suh_g, svh_g, suh_u, svh_u, suh_d, svh_d, x, limit=0.0):
        x = np.ascontiguousarray(x, np.float32)
        m, H = x.shape
        I = svh_g.shape[-1]
        y = np.empty((m, H), np.float32)
        u16 = lambda a: np.ascontiguousarray(a).view(np.uint16).reshape(-1)
        self.L.orc_expert(u16(gate), u16(up), u16(down), u16(suh_g), u16(svh_g), u16(suh_u), u16(svh_u),
                          u16(suh_d), u16(svh_d), H, I, m, x, float(limit), y)
        return y

    # --- routing ------------------------------------------------------------------------
    def permute(self, ids: np.ndarray, weights: np.ndarray | None, E: int, expert_map=None):
        ids = np.ascontiguousarray(ids, np.int64)
        T, k = ids.shape
        n = T * k
        counts = np.empty(E + 1, np.int64)
        offsets = np.empty(E + 1, np.int64)
        ts = np.empty(max(n, 1), np.int32)
        ws = np.empty(max(n, 1), np.float32)
        rs = np.empty(max(n, 1), np.int32)
        rp = np.empty(max(n, 1), np.int32)
        w = None if weights is None else np.ascontiguousarray(weights, np.float32)
        mp = None if expert_map is None else np.ascontiguousarray(expert_map, np.int32)
        self.L.orc_permute(ids.reshape(-1), None if w is None else w.ctypes.data, T, k, E,
                           None if mp is None else mp.ctypes.data, 0 if mp is None else len(mp),
                           counts, offsets, ts, ws, rs, rp)
        return dict(counts=counts, offsets=offsets, token_sorted=ts[:n], weight_sorted=ws[:n],
                    route_sorted=rs[:n], route_pos=rp[:n])

    # --- layer --------------------------------------------------------------------------
    def moe_layer(self, x, ids, weights, gate, up, down, w13_suh, w13_svh, w2_suh, w2_svh,
                  limit=0.0, expert_map=None, nthreads=None, per_route=False):
        """x [T,H] fp16-valued float32; gate/up/down: list over experts of uint16/int16 arrays
        (None for experts that are never routed); scales as numpy float16 stacked tensors."""
        x = np.ascontiguousarray(x, np.float32)
        ids = np.ascontiguousarray(ids, np.int64)
        T, H = x.shape
        k = ids.shape[1]
        E = len(gate)
        I = w13_svh.shape[-1]
        keep = [np.ascontiguousarray(a).view(np.uint16) if a is not None else None for a in (*gate, *up, *down)]
        g, u, d = _ptr_array(keep[:E]), _ptr_array(keep[E:2 * E]), _ptr_array(keep[2 * E:])
        sc = [np.ascontiguousarray(a).view(np.uint16) for a in (w13_suh, w13_svh, w2_suh, w2_svh)]
        mp = None if expert_map is None else np.ascontiguousarray(expert_map, np.int32)
        nthreads = nthreads or os.cpu_count() or 1
        args_map = (None if mp is None else mp.ctypes.data, 0 if mp is None else len(mp))
        if per_route:
            y = np.empty((T * k, H), np.float32)
            self.L.orc_moe_routes(x.ctypes.data, T, H, I, ids.ctypes.data, k, E, *args_map,
                                  g, u, d, *[s.ctypes.data for s in sc], float(limit), int(nthreads), y.ctypes.data)
            return y
        w = np.ascontiguousarray(weights, np.float32)
        out = np.empty((T, H), np.float32)
        self.L.orc_moe_layer(x.ctypes.data, T, H, I, ids.ctypes.data, w.ctypes.data, k, E, *args_map,
                             g, u, d, *[s.ctypes.data for s in sc], float(limit), int(nthreads), out.ctypes.data)
        return out


class RefShim:
    """The reference's own ft_core.h (compiled unchanged by oracle/Makefile `ref`)."""

    def __init__(self, path: str | None = None):
        path = path or os.path.join(REF_DIR, "libref_shim.so")
        L = C.CDLL(path)
        L.refshim_init()
        L.refshim_state.restype = C.c_uint16
        L.refshim_state.argtypes = [_u16p, C.c_int]
        L.refshim_bytesum.restype = C.c_int
        L.refshim_bytesum.argtypes = [C.c_uint16]
        L.refshim_weight.restype = C.c_float
        L.refshim_weight.argtypes = [C.c_uint16]
        L.refshim_perm.restype = C.c_int
        L.refshim_perm.argtypes = [C.c_int]
        L.refshim_dense_weights.argtypes = [C.c_void_p, C.c_int, C.c_int, _f32p]
        L.refshim_prep_block.argtypes = [_f32p, _u16p, _f32p]
        L.refshim_out_block.argtypes = [_f32p, _u16p]
        L.refshim_act.restype = C.c_float
        L.refshim_act.argtypes = [C.c_float, C.c_float, C.c_float]
        L.refshim_ref_expert.restype = C.c_int
        L.refshim_ref_expert.argtypes = [C.c_void_p] * 3 + [_u16p] * 6 + [C.c_int, C.c_int, _f32p, C.c_float, _f32p]
        self.L = L

    @staticmethod
    def available(path: str | None = None) -> bool:
        return os.path.exists(path or os.path.join(REF_DIR, "libref_shim.so"))

    def weight_table(self) -> np.ndarray:
        return np.array([self.L.refshim_weight(s) for s in range(65536)], dtype=np.float32).astype(np.float16)

    def states(self, tile):
        t = np.ascontiguousarray(tile).view(np.uint16).reshape(-1)
        return np.array([self.L.refshim_state(t, i) for i in range(256)], dtype=np.uint16)

    def dense_weights(self, trellis, k, n):
        # the reference's AVX2 decoder over-reads past a tile store; pad every buffer we hand it
        tr = np.zeros(trellis.size + 4096, np.uint16)
        tr[: trellis.size] = np.ascontiguousarray(trellis).view(np.uint16).reshape(-1)
        W = np.empty((k, n), np.float32)
        self.L.refshim_dense_weights(tr.ctypes.data, k, n, W)
        return W

    def prep_block(self, x, suh):
        xt = np.empty(128, np.float32)
        self.L.refshim_prep_block(np.ascontiguousarray(x, np.float32), np.ascontiguousarray(suh).view(np.uint16), xt)
        return xt

    def out_block(self, y, svh):
        y = np.array(y, dtype=np.float32)
        self.L.refshim_out_block(y, np.ascontiguousarray(svh).view(np.uint16))
        return y

    def act(self, g, u, limit):
        return self.L.refshim_act(g, u, limit)

    def expert(self, gate, up, down, suh_g, svh_g, suh_u, svh_u, suh_d, svh_d, x, limit=0.0):
        x = np.ascontiguousarray(x, np.float32).reshape(-1)
        H = x.size
        I = svh_g.size
        pads = []
        for a in (gate, up, down):
            p = np.zeros(a.size + 4096, np.uint16)
            p[: a.size] = np.ascontiguousarray(a).view(np.uint16).reshape(-1)
            pads.append(p)
        y = np.empty(H, np.float32)
        u16 = lambda a: np.ascontiguousarray(a).view(np.uint16).reshape(-1)
        rc = self.L.refshim_ref_expert(*[p.ctypes.data for p in pads], u16(suh_g), u16(svh_g), u16(suh_u),
                                       u16(svh_u), u16(suh_d), u16(svh_d), H, I, x, float(limit), y)
        if rc != 0:
            raise ValueError("reference ref_expert supports I == 2048 only")
        return y


def ref_tier_path(variant: str = "auto") -> str | None:
    """Path of the prebuilt reference CPU tier (ft_tier_host*.so) for this host's ISA."""
    if variant == "auto":
        flags = ""
        try:
            with open("/proc/cpuinfo") as f:
                for line in f:
                    if line.startswith("flags"):
                        flags = line
                        break
        except OSError:
            pass
        v4 = all(f" {x}" in flags for x in ("avx512f", "avx512bw", "avx512dq", "avx512vl", "avx512cd"))
        order = ["v4", "v3"] if v4 else ["v3"]
    else:
        order = [variant]
    for v in order:
        d = os.path.join(REF_DIR, f"tier_{v}")
        if os.path.isdir(d):
            for fn in sorted(os.listdir(d)):
                if fn.startswith("ft_tier_host") and fn.endswith(".so"):
                    return os.path.join(d, fn)
    return None


def load_ref_tier(variant: str = "auto"):
    """Import the reference's CPU tier torch extension (kernels/cpu_avx2/ft_tier_ext.cpp)."""
    import torch  # noqa: F401  (the extension links against libtorch)
    path = ref_tier_path(variant)
    if path is None:
        raise FileNotFoundError("oracle/_ref/tier_*/ft_tier_host*.so not built (oracle/build_ref_tier.py)")
    name = os.path.basename(path).split(".")[0]  # torch may have suffixed the module name (_v1)
    spec = importlib.util.spec_from_file_location(name, path)
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod
