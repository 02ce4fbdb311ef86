"""dsv41_moe_forward_noalloc: the layer forward for callers that cannot allocate device memory.

Callers that run the layer inside someone else's CUDA-graph capture, plugins handed a stream but no
allocator, and processes whose device memory is reserved up front cannot provide the workspace
dsv41_moe_forward asks for. The no-allocation entry point keeps its scratch in a fixed 32 MiB
device array of the library. This test calls it through the C ABI (ctypes), twice in a row with
different inputs, and checks each result against the workspace entry point within the parity
tolerance of the other layer tests; it also checks that a request beyond the array's size is
refused with a clear error, and that the status word kept in that array -- which such callers have no
workspace pointer to read -- is reported by dsv41_moe_noalloc_read_status. It lives in its own file so
that it runs last and also passes alone.
"""
import ctypes as C

import pytest
import torch

from conftest import assert_close_layer
from dsv41_flash_offload_b200 import _lib, exl3, synth

pytestmark = pytest.mark.gpu
DEV = "cuda:0"
LIMIT = 10.0


@pytest.fixture(scope="module")
def layer():
    return exl3.Exl3MoELayer.synthetic(384, 4096, 2048, seed=0, device=DEV)


def _call_noalloc(layer, x, ids, w, out, fat=32, max_routes=0):
    L = _lib.load()
    opt = _lib.MoeOptions(fat, LIMIT, None, 0, 0, max_routes)
    stream = torch.cuda.current_stream(x.device)
    with torch.cuda.device(x.device):
        return L.dsv41_moe_forward_noalloc(C.byref(layer._c), x.data_ptr(), _lib.DTYPE_BF16, x.shape[0], ids.data_ptr(),
                                           w.data_ptr(), ids.shape[1], C.byref(opt), out.data_ptr(),
                                           C.c_void_p(stream.cuda_stream))


def _noalloc_status():
    st = C.c_int32(-1)
    stream = torch.cuda.current_stream(torch.device(DEV))
    with torch.cuda.device(DEV):
        _lib.check(_lib.load().dsv41_moe_noalloc_read_status(C.c_void_p(stream.cuda_stream), C.byref(st)),
                   "dsv41_moe_noalloc_read_status")
    return st.value


def _inputs(seed, T):
    x = torch.from_numpy(synth.hidden_np(seed, T, 4096)).to(DEV, torch.bfloat16)
    ids, w = synth.routing_np(seed, T, 384, 8)
    return x, torch.from_numpy(ids).to(DEV), torch.from_numpy(w).to(DEV)


def test_noalloc_matches_workspace_entry_point_twice(layer):
    for seed, T in ((71, 64), (72, 8)):
        x, ids, w = _inputs(seed, T)
        out = torch.full((T, 4096), float("nan"), dtype=torch.float32, device=DEV)
        rc = _call_noalloc(layer, x, ids, w, out)
        _lib.check(rc, "dsv41_moe_forward_noalloc")
        ref = exl3.apply_exl3_fused_moe(x, ids, w, layer, None, None, LIMIT)
        torch.cuda.synchronize()
        assert_close_layer(out.cpu().numpy(), ref.cpu().numpy(), f"noalloc T={T}")
        assert _noalloc_status() == 0


def test_noalloc_refuses_requests_beyond_its_scratch(layer):
    T = 4096
    x = torch.zeros(T, 4096, dtype=torch.bfloat16, device=DEV)
    ids = torch.zeros(T, 8, dtype=torch.int64, device=DEV)
    w = torch.zeros(T, 8, dtype=torch.float32, device=DEV)
    out = torch.zeros(T, 4096, dtype=torch.float32, device=DEV)
    rc = _call_noalloc(layer, x, ids, w, out)
    assert rc == _lib.E_WORKSPACE
    assert b"static scratch" in _lib.load().dsv41_last_error()


def test_noalloc_status_word_is_readable(layer):
    """A failure the kernels report through the status word must reach a caller without a workspace:
    a max_routes bound below the call's valid routes drops the call (zero output) and sets status 3,
    which dsv41_moe_noalloc_read_status returns once and then clears."""
    x, ids, w = _inputs(73, 8)
    out = torch.full((8, 4096), float("nan"), dtype=torch.float32, device=DEV)
    _lib.check(_call_noalloc(layer, x, ids, w, out, max_routes=63), "dsv41_moe_forward_noalloc")
    assert _noalloc_status() == 3
    assert float(out.abs().max()) == 0.0
    assert _noalloc_status() == 0
    _lib.check(_call_noalloc(layer, x, ids, w, out, max_routes=64), "dsv41_moe_forward_noalloc")
    assert _noalloc_status() == 0
    ref = exl3.apply_exl3_fused_moe(x, ids, w, layer, None, None, LIMIT)
    assert_close_layer(out.cpu().numpy(), ref.cpu().numpy(), "noalloc after a dropped call")
