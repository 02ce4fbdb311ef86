"""ctypes binding of libdsv41_b200.so (the C ABI declared in include/dsv41_b200.h).

The library is built in-tree by dsv41_flash_offload_b200/build.py. There is no fallback: if the
library is missing or fails to load, every entry point raises.
"""
from __future__ import annotations

import ctypes as C
import os
import threading

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "libdsv41_b200.so")

DTYPE_F16, DTYPE_BF16, DTYPE_F32 = 0, 1, 2
OK, E_INVALID, E_CUDA, E_WORKSPACE = 0, -1, -2, -3

# exported symbols, in include/dsv41_b200.h order
SYMBOLS = (
    "dsv41_last_error", "dsv41_abi_version", "dsv41_build_info", "dsv41_moe_workspace_size",
    "dsv41_moe_forward", "dsv41_moe_forward_noalloc", "dsv41_moe_noalloc_read_status",
    "dsv41_permute_workspace_size", "dsv41_permute", "dsv41_combine",
    "dsv41_decode_dense", "dsv41_decode_dense_bits", "dsv41_expert_gemm", "dsv41_expert_gemm_workspace_size",
    "dsv41_read_status", "dsv41_wait_selftest",
    "dsv41_router_topk", "dsv41_moe_forward_logits",
    "dsv41_ep_peer_buffer_size", "dsv41_ep_peer_alloc", "dsv41_ep_peer_open", "dsv41_ep_peer_close", "dsv41_ep_peer_free",
    "dsv41_ep_peer_forward", "dsv41_ep_peer_read_status",
    "dsv41_set_stage_timing", "dsv41_read_stage_times",
)
ABI_VERSION = 2
MAX_PEERS = 8
IPC_HANDLE_BYTES = 64
N_STAGES = 7
# "gemv": the decode-GEMV launch (gate/up and down together when split-K is 1; "gemv_down" is then empty)
STAGE_NAMES = ("permute", "prep", "gemv", "gemm_gateup", "gemv_down", "gemm_down", "combine")


class MoeLayer(C.Structure):
    _fields_ = [("num_experts", C.c_int32), ("hidden", C.c_int32), ("intermediate", C.c_int32),
                ("bits", C.c_int32), ("gate_ptrs", C.c_void_p), ("up_ptrs", C.c_void_p),
                ("down_ptrs", C.c_void_p), ("w13_suh", C.c_void_p), ("w13_svh", C.c_void_p),
                ("w2_suh", C.c_void_p), ("w2_svh", C.c_void_p)]


class MoeOptions(C.Structure):
    _fields_ = [("fat_threshold", C.c_int32), ("limit", C.c_float), ("expert_map", C.c_void_p),
                ("map_len", C.c_int32), ("split_k", C.c_int32), ("max_routes", C.c_int32)]


class RouterOptions(C.Structure):
    _fields_ = [("scoring", C.c_int32), ("renormalize", C.c_int32), ("num_expert_group", C.c_int32),
                ("topk_group", C.c_int32), ("correction_bias", C.c_void_p), ("routed_scaling_factor", C.c_float)]


class EpPeerGroup(C.Structure):
    _fields_ = [("rank", C.c_int32), ("world", C.c_int32), ("num_global_experts", C.c_int32),
                ("tokens_cap", C.c_int32), ("bases", C.c_void_p * MAX_PEERS), ("wait_limit_us", C.c_int32)]


class Dsv41Error(RuntimeError):
    pass


_lock = threading.Lock()
_lib = None


def load(path: str | None = None):
    """Load (once) and return the library handle; raises if it is missing."""
    global _lib
    with _lock:
        if _lib is not None:
            return _lib
        p = path or os.environ.get("DSV41_B200_LIB", LIB_PATH)
        if not os.path.exists(p):
            raise Dsv41Error(f"{p} not built: run `python -m dsv41_flash_offload_b200.build` (no CPU fallback)")
        L = C.CDLL(p)
        vp, i32, i64p = C.c_void_p, C.c_int32, C.c_void_p
        L.dsv41_last_error.restype = C.c_char_p
        L.dsv41_last_error.argtypes = []
        L.dsv41_abi_version.restype = C.c_int
        L.dsv41_build_info.restype = C.c_char_p
        L.dsv41_moe_workspace_size.restype = C.c_int
        L.dsv41_moe_workspace_size.argtypes = [i32, i32, i32, i32, i32, C.POINTER(MoeOptions), C.POINTER(C.c_size_t)]
        L.dsv41_moe_forward.restype = C.c_int
        L.dsv41_moe_forward.argtypes = [C.POINTER(MoeLayer), vp, i32, i32, i64p, vp, i32, C.POINTER(MoeOptions), vp,
                                        vp, C.c_size_t, vp]
        L.dsv41_moe_forward_noalloc.restype = C.c_int
        L.dsv41_moe_forward_noalloc.argtypes = [C.POINTER(MoeLayer), vp, i32, i32, i64p, vp, i32, C.POINTER(MoeOptions),
                                                vp, vp]
        L.dsv41_moe_noalloc_read_status.restype = C.c_int
        L.dsv41_moe_noalloc_read_status.argtypes = [vp, C.POINTER(C.c_int32)]
        L.dsv41_permute_workspace_size.restype = C.c_size_t
        L.dsv41_permute_workspace_size.argtypes = [i32, i32, i32]
        L.dsv41_permute.restype = C.c_int
        L.dsv41_permute.argtypes = [i64p, vp, i32, i32, i32, vp, i32, vp, vp, vp, vp, vp, vp, vp, C.c_size_t, vp]
        L.dsv41_combine.restype = C.c_int
        L.dsv41_combine.argtypes = [vp, vp, vp, i32, i32, i32, i32, vp, vp]
        L.dsv41_decode_dense.restype = C.c_int
        L.dsv41_decode_dense.argtypes = [vp, i32, i32, vp, vp]
        L.dsv41_decode_dense_bits.restype = C.c_int
        L.dsv41_decode_dense_bits.argtypes = [vp, i32, i32, i32, vp, vp]
        L.dsv41_expert_gemm.restype = C.c_int
        L.dsv41_expert_gemm.argtypes = [C.POINTER(MoeLayer), vp, i32, i32, vp, i32, vp, vp, vp, vp, i32, C.c_float, vp,
                                        vp, C.c_size_t, vp]
        L.dsv41_expert_gemm_workspace_size.restype = C.c_int
        L.dsv41_expert_gemm_workspace_size.argtypes = [i32, i32, i32, i32, C.POINTER(C.c_size_t)]
        L.dsv41_read_status.restype = C.c_int
        L.dsv41_read_status.argtypes = [vp, vp, C.POINTER(C.c_int32)]
        L.dsv41_wait_selftest.restype = C.c_int
        L.dsv41_wait_selftest.argtypes = [vp, C.c_uint32, vp]
        rp = C.POINTER(RouterOptions)
        L.dsv41_router_topk.restype = C.c_int
        L.dsv41_router_topk.argtypes = [vp, i32, i32, i32, i32, rp, i64p, vp, vp]
        L.dsv41_moe_forward_logits.restype = C.c_int
        L.dsv41_moe_forward_logits.argtypes = [C.POINTER(MoeLayer), vp, i32, i32, vp, i32, rp, i32,
                                               C.POINTER(MoeOptions), vp, vp, vp, vp, C.c_size_t, vp]
        gp = C.POINTER(EpPeerGroup)
        L.dsv41_ep_peer_buffer_size.restype = C.c_int
        L.dsv41_ep_peer_buffer_size.argtypes = [gp, C.POINTER(MoeLayer), i32, i32, C.POINTER(C.c_size_t)]
        L.dsv41_ep_peer_alloc.restype = C.c_int
        L.dsv41_ep_peer_alloc.argtypes = [C.c_size_t, C.POINTER(C.c_void_p), vp]
        L.dsv41_ep_peer_open.restype = C.c_int
        L.dsv41_ep_peer_open.argtypes = [vp, C.POINTER(C.c_void_p)]
        L.dsv41_ep_peer_close.restype = C.c_int
        L.dsv41_ep_peer_close.argtypes = [vp]
        L.dsv41_ep_peer_free.restype = C.c_int
        L.dsv41_ep_peer_free.argtypes = [vp]
        L.dsv41_ep_peer_forward.restype = C.c_int
        L.dsv41_ep_peer_forward.argtypes = [C.POINTER(MoeLayer), gp, C.c_uint32, vp, i32, i32, i64p, vp, i32,
                                            C.c_float, i32, vp, vp]
        L.dsv41_ep_peer_read_status.restype = C.c_int
        L.dsv41_ep_peer_read_status.argtypes = [gp, C.POINTER(MoeLayer), i32, i32, vp, C.POINTER(C.c_int32)]
        L.dsv41_set_stage_timing.restype = C.c_int
        L.dsv41_set_stage_timing.argtypes = [i32]
        L.dsv41_read_stage_times.restype = C.c_int
        L.dsv41_read_stage_times.argtypes = [C.POINTER(C.c_float), i32, C.POINTER(C.c_int32)]
        if L.dsv41_abi_version() != ABI_VERSION:
            raise Dsv41Error("libdsv41_b200.so ABI version mismatch")
        _lib = L
        return L


def check(rc: int, what: str) -> None:
    if rc != OK:
        msg = load().dsv41_last_error().decode(errors="replace")
        raise Dsv41Error(f"{what} failed ({rc}): {msg}")
