"""Trellis tiles at 2 and 4 bits per weight (the reference's 2-bit cold packs and 4-bit layers,
patch:519-528, pack/prepare_pack.py:47): dense decode bit-exact against the oracle's K-generic
state formula, and the full layer (decode-GEMV and tcgen05 GEMM paths) within the parity bar."""
import numpy as np
import pytest
import torch

from conftest import assert_close_layer
from dsv41_flash_offload_b200 import exl3, synth
from moe_ref import oracle_out

pytestmark = pytest.mark.gpu
DEV = "cuda:0"


@pytest.mark.parametrize("bits", [2, 3, 4])
def test_decode_dense_bits_vs_oracle(oracle, bits):
    k, n = 256, 512
    rng = np.random.default_rng(bits)
    tr = rng.integers(-32768, 32768, (k // 16) * (n // 16) * 16 * bits, dtype=np.int16)
    W = exl3.decode_dense(torch.from_numpy(tr).to(DEV), k, n).cpu().numpy()
    prev = oracle.bits
    oracle.set_bits(bits)
    try:
        ref = oracle.decode_matrix(tr, k, n)
    finally:
        oracle.set_bits(prev)
    assert np.array_equal(W.view(np.uint16), ref.view(np.uint16))


@pytest.mark.parametrize("bits", [2, 4])
def test_layer_bits_vs_oracle(oracle, bits):
    layer = exl3.Exl3MoELayer.synthetic(16, 512, 256, seed=5, device=DEV, bits=bits)
    assert layer.bits == bits
    for T, k, kind, fat in ((37, 6, "uniform", 32), (300, 4, "zipf", 32)):
        x = torch.from_numpy(synth.hidden_np(90 + T, T, 512)).to(DEV, torch.bfloat16)
        ids, w = synth.routing_np(91 + T, T, 16, k, kind=kind, zipf_s=1.5)
        ids, w = torch.from_numpy(ids).to(DEV), torch.from_numpy(w).to(DEV)
        out = exl3.apply_exl3_fused_moe(x, ids, w, layer, None, None, 10.0, fat_threshold=fat)
        assert exl3.read_status(device=DEV) == 0
        assert_close_layer(out.cpu().numpy(), oracle_out(oracle, layer, x, ids, w, 10.0), f"bits {bits} T {T}")
