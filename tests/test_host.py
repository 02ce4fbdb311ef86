"""CPU-only tests: synthetic generator consistency, a restatement of the GPU's register decode
checked against the oracle, the C ABI (loads, exports every declared symbol, rejects bad input
without touching a GPU), and host-side argument validation."""
import ctypes as C
import os
import re

import numpy as np
import pytest
import torch

from conftest import ROOT
from dsv41_flash_offload_b200 import _lib, synth


def test_synth_torch_matches_numpy():
    n = 10000
    ref = synth.trellis_np(3, synth.STREAM_W13, 12345, n, layer=2)
    t = torch.empty(n, dtype=torch.int16)
    synth.fill_trellis_torch(t, 3, synth.STREAM_W13, 12345, layer=2, chunk=4096)
    assert np.array_equal(t.numpy(), ref)


def test_synth_routing_shapes():
    ids, w = synth.routing_np(0, 16, 384, 8)
    assert ids.shape == (16, 8) and w.shape == (16, 8)
    assert all(len(set(r)) == 8 for r in ids.tolist())
    np.testing.assert_allclose(w.sum(1), 1.0, rtol=1e-6)
    zi, zw = synth.routing_np(0, 4096, 384, 8, kind="zipf", zipf_s=1.5)
    counts = np.bincount(zi.reshape(-1), minlength=384)
    top = np.sort(counts)[::-1][:38].sum() / counts.sum()
    # heavily skewed: Zipf(1.5) popularity with 8 distinct draws per token puts ~80% of the
    # assignments on the top 10% of experts (the realised share is reported by the bench)
    assert 0.5 < top < 0.95


def _lane_setup(t):
    start = (24 * t - 13 + 768) % 768
    a, o = start >> 5, start & 31
    if o < 16:
        return a, (a + 1) % 24, 16, 32 - o
    return a, (a + 1) % 24, 0, 48 - o


def _funnel_r(lo, hi, s):
    return ((hi << 32 | lo) >> (s & 31)) & 0xFFFFFFFF


def test_register_decode_restatement_matches_oracle(oracle):
    """The exact integer steps of decode_lane() (csrc/common.cuh), in Python, for every lane of
    random tiles: window words, pre-shift, funnel shifts -> states equal the oracle's."""
    rng = np.random.default_rng(0)
    for _ in range(40):
        tile = rng.integers(0, 65536, 48, dtype=np.uint16)
        words = [int(tile[2 * i]) | int(tile[2 * i + 1]) << 16 for i in range(24)]
        ref = oracle.states(tile)
        for t in range(32):
            whi_i, wlo_i, pre, base = _lane_setup(t)
            whi, wlo = words[whi_i], words[wlo_i]
            lo = _funnel_r(wlo, whi, pre)
            hi = whi >> pre
            for j in range(8):
                assert _funnel_r(lo, hi, base - 3 * j) & 0xFFFF == ref[8 * t + j]


def _funnel_l(lo, hi, s):
    return (((hi << 32 | lo) << (s & 31)) >> 32) & 0xFFFFFFFF


def test_uniform_window_decode_restatement_matches_oracle(oracle):
    """decode_lane_u() (csrc/common.cuh): lane t's 64-bit window = 8 stream bytes from byte 3t-4,
    assembled from 3 words with two left funnel shifts by 8*(b0%4); state j = bits [29-3j, 45-3j):
    states 0-4 straddle (hi, lo) and come from a right funnel shift, 5-7 lie in lo (state 7 is
    bytes 1-2 of lo, which one byte permute extracts)."""
    rng = np.random.default_rng(2)
    for _ in range(40):
        tile = rng.integers(0, 65536, 48, dtype=np.uint16)
        words = [int(tile[2 * i]) | int(tile[2 * i + 1]) << 16 for i in range(24)]
        ref = oracle.states(tile)
        for t in range(32):
            b0 = (3 * t - 4) % 96
            q, r8 = b0 // 4, 8 * (b0 % 4)
            w0, w1, w2 = words[q], words[(q + 1) % 24], words[(q + 2) % 24]
            hi = _funnel_l(w1, w0, r8)
            lo = _funnel_l(w2, w1, r8)
            for j in range(5):
                assert _funnel_r(lo, hi, 29 - 3 * j) & 0xFFFF == ref[8 * t + j]
            for j in range(5, 7):
                assert (lo >> (29 - 3 * j)) & 0xFFFF == ref[8 * t + j]
            assert ((lo >> 8) & 0xFF) | (((lo >> 16) & 0xFF) << 8) == ref[8 * t + 7]


def test_half_fma_decode_matches_oracle_for_all_states(oracle):
    """(0x6400 | bytesum) as fp16 = 1024 + s exactly; one fp16 rounding of (1024+s)*KINV + KBIAS
    (what HFMA2 computes) equals the oracle's decoded weight for all 65536 states."""
    table = oracle.weight_table()
    st = np.arange(65536, dtype=np.uint64)
    x = (st * np.uint64(0x83DCD12D)) & np.uint64(0xFFFFFFFF)
    s = sum(((x >> np.uint64(8 * b)) & np.uint64(0xFF)) for b in range(4)).astype(np.int64)
    code = (0x6400 + s).astype(np.uint16).view(np.float16).astype(np.float64)
    assert np.array_equal(code, 1024.0 + s)
    kinv = np.array([0x1EEE], np.uint16).view(np.float16).astype(np.float64)[0]
    kbias = np.array([0xC931], np.uint16).view(np.float16).astype(np.float64)[0]
    w = (code * kinv + kbias).astype(np.float16)  # exact in float64, then a single rounding
    assert np.array_equal(w.view(np.uint16), table)


def _declared_functions():
    hdr = open(os.path.join(ROOT, "include", "dsv41_b200.h")).read()
    hdr = re.sub(r"/\*.*?\*/", "", hdr, flags=re.S)
    return sorted(set(re.findall(r"\b(dsv41_[a-z0-9_]+)\s*\(", hdr)))


def test_capi_library_exports_every_declared_symbol():
    L = _lib.load()
    declared = _declared_functions()
    assert set(declared) == set(_lib.SYMBOLS)
    for name in declared:
        assert hasattr(L, name), name
    assert L.dsv41_abi_version() == _lib.ABI_VERSION == 2
    assert b"sm_100a" in L.dsv41_build_info()


def test_capi_rejects_bad_arguments_without_gpu():
    L = _lib.load()
    n = C.c_size_t()
    rc = L.dsv41_moe_workspace_size(4, 8, 384, 4000, 2048, None, C.byref(n))
    assert rc == _lib.E_INVALID and b"H=4000" in L.dsv41_last_error()
    rc = L.dsv41_decode_dense(None, 15, 16, None, None)
    assert rc == _lib.E_INVALID and b"multiples of 16" in L.dsv41_last_error()
    rc = L.dsv41_moe_forward(None, None, 0, 1, None, None, 8, None, None, None, 0, None)
    assert rc == _lib.E_INVALID and b"layer is NULL" in L.dsv41_last_error()
    layer = _lib.MoeLayer(384, 4096, 2048, 0, 0, 0, 0, 0, 0, 0, 0)
    rc = L.dsv41_moe_forward(C.byref(layer), None, 0, 1, None, None, 8, None, None, None, 0, None)
    assert rc == _lib.E_INVALID and b"NULL tensor" in L.dsv41_last_error()
    rc = L.dsv41_permute(None, None, 4, 8, 0, None, 0, None, None, None, None, None, None, None, 0, None)
    assert rc == _lib.E_INVALID


def test_capi_rejects_misaligned_buffers_without_gpu():
    # the pointers are never dereferenced: the argument checks run before any device work
    L = _lib.load()
    fake = 1 << 20
    layer = _lib.MoeLayer(384, 4096, 2048, 0, *([fake] * 7))
    ids = (C.c_int64 * 8)()
    w = (C.c_float * 8)()

    def fwd(x, out, ws):
        return L.dsv41_moe_forward(C.byref(layer), C.c_void_p(x), 0, 1, ids, w, 8, None, C.c_void_p(out),
                                   C.c_void_p(ws), 1 << 30, None)

    assert fwd(fake + 8, fake, fake) == _lib.E_INVALID and b"16-byte aligned" in L.dsv41_last_error()
    assert fwd(fake, fake + 4, fake) == _lib.E_INVALID and b"out must be 16-byte" in L.dsv41_last_error()
    assert fwd(fake, fake, fake + 16) == _lib.E_INVALID and b"256-byte aligned" in L.dsv41_last_error()
    rc = L.dsv41_combine(C.c_void_p(fake + 2), C.c_void_p(fake), C.c_void_p(fake), 1, 8, 4096, 0, C.c_void_p(fake), None)
    assert rc == _lib.E_INVALID and b"16-byte aligned" in L.dsv41_last_error()


def test_capi_workspace_sizes_grow_with_tokens():
    L = _lib.load()
    sizes = []
    for T in (1, 8, 64, 256, 16384):
        n = C.c_size_t()
        assert L.dsv41_moe_workspace_size(T, 8, 384, 4096, 2048, None, C.byref(n)) == 0
        sizes.append(n.value)
    # (small batches carry split-K partials, so the sizes are not monotonic in T)
    assert all(s > 0 for s in sizes) and sizes[-1] == max(sizes)
    # activations dominate: 4 row buffers per route at H=4096/I=2048 fp16
    assert sizes[-1] >= 16384 * 8 * (3 * 4096 + 2048) * 2


def test_layer_validation_on_cpu_tensors():
    from dsv41_flash_offload_b200.exl3 import Exl3MoELayer
    E, H, I = 2, 256, 256
    w13 = torch.zeros(E, 2, H // 16, I // 16, 48, dtype=torch.int16)
    w2 = torch.zeros(E, I // 16, H // 16, 48, dtype=torch.int16)
    s = lambda *sh: torch.zeros(*sh, dtype=torch.float16)
    with pytest.raises(ValueError):
        Exl3MoELayer(w13[:, :1], w2, s(E, 2, H), s(E, 2, I), s(E, I), s(E, H))
    with pytest.raises(ValueError):
        Exl3MoELayer(w13, w2, s(E, 2, H), s(E, 2, I + 16), s(E, I), s(E, H))
    with pytest.raises(ValueError):
        Exl3MoELayer(w13, w2.float(), s(E, 2, H), s(E, 2, I), s(E, I), s(E, H))


def test_ep_peer_buffer_layout_host_checks():
    """dsv41_ep_peer_buffer_size is pure host arithmetic (no device call): same size for every rank,
    growing with world and tokens_cap, and argument errors for bad groups."""
    import ctypes as C
    from dsv41_flash_offload_b200 import _lib
    L = _lib.load()
    layer = _lib.MoeLayer(192, 4096, 2048, 0, *([16] * 7))   # dummy non-null pointers: never dereferenced

    def size(world, rank, cap, E=384, topk=8):
        g = _lib.EpPeerGroup()
        g.rank, g.world, g.num_global_experts, g.tokens_cap = rank, world, E, cap
        for d in range(_lib.MAX_PEERS):
            g.bases[d] = 16
        lay = _lib.MoeLayer(E // world if world and E % world == 0 else 1, 4096, 2048, 0, *([16] * 7))
        n = C.c_size_t()
        rc = L.dsv41_ep_peer_buffer_size(C.byref(g), C.byref(lay), topk, 32, C.byref(n))
        return rc, n.value

    sizes = [size(2, r, 64) for r in range(2)]
    assert all(rc == 0 for rc, _ in sizes) and sizes[0][1] == sizes[1][1] > 0
    assert size(4, 3, 64)[1] > size(2, 0, 64)[1]        # more peers -> more routes to hold
    assert size(2, 0, 128)[1] > size(2, 0, 64)[1]
    assert size(9, 0, 64)[0] == _lib.E_INVALID           # more than DSV41_MAX_PEERS ranks
    assert size(2, 2, 64)[0] == _lib.E_INVALID           # rank out of range
    assert size(5, 0, 64, E=384)[0] == _lib.E_INVALID    # 384 experts do not shard over 5
    assert size(2, 0, 0)[0] == _lib.E_INVALID            # no capacity
    g = _lib.EpPeerGroup()
    g.rank, g.world, g.num_global_experts, g.tokens_cap = 0, 2, 384, 64
    for d in range(_lib.MAX_PEERS):
        g.bases[d] = 16
    lay = _lib.MoeLayer(192, 4096, 2048, 0, *([16] * 7))
    n = C.c_size_t()
    for lim, want in ((0, 0), (50000, 0), (2000000, 0), (-1, _lib.E_INVALID), (2000001, _lib.E_INVALID)):
        g.wait_limit_us = lim                             # exchange wait bound: 0 = 2 s, else 1 us .. 2 s
        assert L.dsv41_ep_peer_buffer_size(C.byref(g), C.byref(lay), 8, 32, C.byref(n)) == want, lim
    del layer


def test_vllm_plugin_install_uninstall_on_module():
    """install() swaps the module's apply_exl3_fused_moe and wraps Exl3MoEMethod's
    process_weights_after_loading (original first, then the B200 view), idempotently; uninstall
    restores both (the reference's install(X) pattern, ct/ct_vllm.py:446-456)."""
    import types
    from dsv41_flash_offload_b200 import exl3, vllm_plugin

    calls = []

    class Exl3MoEMethod:
        def process_weights_after_loading(self, layer):
            calls.append("orig")

    def orig_fused(*a, **k):
        return "orig"

    X = types.ModuleType("fake_vllm_exl3")
    X.apply_exl3_fused_moe = orig_fused
    X.Exl3MoEMethod = Exl3MoEMethod
    vllm_plugin.install(X)
    vllm_plugin.install(X)   # second call is a no-op
    assert X.apply_exl3_fused_moe is not orig_fused
    assert X.apply_exl3_fused_moe.__doc__ == exl3.apply_exl3_fused_moe.__doc__
    layer = types.SimpleNamespace(_dsv41="view")   # as_layer returns the cached view
    Exl3MoEMethod().process_weights_after_loading(layer)
    assert calls == ["orig"]
    vllm_plugin.uninstall(X)
    assert X.apply_exl3_fused_moe is orig_fused
    assert X.Exl3MoEMethod.process_weights_after_loading.__name__ == "process_weights_after_loading"
    Exl3MoEMethod().process_weights_after_loading(layer)
    assert calls == ["orig", "orig"]
