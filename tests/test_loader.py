"""EXL3 checkpoint loader (loader.py): a small two-shard checkpoint in the reference's naming is
written with the module's own safetensors writer, then loaded back: stacked arrays equal the
sources, expert-parallel shards select the right experts, unsupported layers/codebooks raise.
The GPU case checks the loaded layer computes exactly what the synthetic layer does."""
import json
import os

import numpy as np
import pytest
import torch

from dsv41_flash_offload_b200 import loader, synth

E, H, I, LAYER = 3, 256, 256, 5


def _write_ckpt(d, prefix="model.", bits_override=None, mcg=False, bad_mul1=False, bits=3):
    s13, v13, s2, v2 = synth.scales_np(9, E, H, I, LAYER)
    shards = [{}, {}]
    wm = {}
    for e in range(E):
        g, u, dn = synth.expert_trellis_np(9, H, I, e, LAYER, bits=bits)
        for w, tr, suh, svh in (("w1", g, s13[e, 0], v13[e, 0]), ("w3", u, s13[e, 1], v13[e, 1]), ("w2", dn, s2[e], v2[e])):
            key = f"{prefix}layers.{LAYER}.ffn.experts.{e}.{w}"
            sh = shards[e % 2]
            sh[key + ".trellis"] = tr
            sh[key + ".suh"] = suh
            sh[key + ".svh"] = svh
            sh[key + ".mul1"] = np.array([0x12345678 if (bad_mul1 and e == 1) else loader.MUL1], np.uint32)
            if mcg and e == 2:
                sh[key + ".mcg"] = np.array([1], np.uint32)
    for i, sh in enumerate(shards):
        fn = f"model-{i:05d}-of-00002.safetensors"
        loader.write_safetensors(os.path.join(d, fn), sh)
        wm.update({k: fn for k in sh})
    json.dump({"metadata": {}, "weight_map": wm}, open(os.path.join(d, "model.safetensors.index.json"), "w"))
    q = {"quant_method": "exl3", "bits": bits, "codebook": "mul1", "layer_bits": {str(LAYER + 1): 4}}
    if bits_override:
        q["layer_bits"][str(LAYER)] = bits_override
    json.dump({"quantization_config": q}, open(os.path.join(d, "config.json"), "w"))
    return s13, v13, s2, v2


def test_loader_round_trip_cpu(tmp_path):
    s13, v13, s2, v2 = _write_ckpt(str(tmp_path))
    ck = loader.Checkpoint(str(tmp_path))
    assert ck.layer_bits(LAYER) == 3 and ck.layer_bits(LAYER + 1) == 4
    lay = loader.load_moe_layer(ck, LAYER, device="cpu")
    for e in range(E):
        g, u, dn = synth.expert_trellis_np(9, H, I, e, LAYER)
        assert np.array_equal(lay.w13_trellis[e, 0].numpy(), g) and np.array_equal(lay.w13_trellis[e, 1].numpy(), u)
        assert np.array_equal(lay.w2_trellis[e].numpy(), dn)
    assert np.array_equal(lay.w13_suh.numpy(), s13) and np.array_equal(lay.w13_svh.numpy(), v13)
    assert np.array_equal(lay.w2_suh.numpy(), s2) and np.array_equal(lay.w2_svh.numpy(), v2)
    shard = loader.load_moe_layer(ck, LAYER, device="cpu", expert_range=(1, 3))
    assert torch.equal(shard.w13_trellis, lay.w13_trellis[1:3]) and torch.equal(shard.w2_svh, lay.w2_svh[1:3])


def test_loader_rejects_unsupported(tmp_path):
    for i, kw in enumerate(({"bits_override": 5}, {"mcg": True}, {"bad_mul1": True}, {"bits_override": 2})):
        d = tmp_path / str(i)
        d.mkdir()
        _write_ckpt(str(d), **kw)
        with pytest.raises(ValueError if i == 3 else NotImplementedError):   # 2-bit config, 3-bit tiles
            loader.load_moe_layer(str(d), LAYER, device="cpu")
    ok = tmp_path / "ok"
    ok.mkdir()
    _write_ckpt(str(ok))
    with pytest.raises(KeyError):
        loader.load_moe_layer(str(ok), LAYER + 7, device="cpu")
    with pytest.raises(ValueError):
        loader.load_moe_layer(str(ok), LAYER, device="cpu", expert_range=(2, 9))


def test_safetensors_header_layout(tmp_path):
    p = str(tmp_path / "x.safetensors")
    a = np.arange(12, dtype=np.float16).reshape(3, 4)
    loader.write_safetensors(p, {"a": a, "b": np.array([7], np.int64)}, metadata={"format": "pt"})
    hdr, start = loader.read_header(p)
    assert start % 8 == 0 and hdr["a"]["dtype"] == "F16" and hdr["a"]["shape"] == [3, 4]
    ck = loader.Checkpoint(p)
    assert np.array_equal(ck.tensor("a"), a) and int(ck.tensor("b")[0]) == 7


@pytest.mark.gpu
def test_loaded_layer_matches_synthetic_on_gpu(tmp_path):
    from dsv41_flash_offload_b200 import exl3
    _write_ckpt(str(tmp_path), prefix="")
    lay = loader.load_moe_layer(str(tmp_path), LAYER, device="cuda:0")
    ref = exl3.Exl3MoELayer.synthetic(E, H, I, seed=9, layer=LAYER, device="cuda:0")
    x = torch.from_numpy(synth.hidden_np(3, 20, H)).to("cuda:0", torch.bfloat16)
    ids, w = synth.routing_np(4, 20, E, 2)
    ids, w = torch.from_numpy(ids).cuda(), torch.from_numpy(w).cuda()
    assert torch.equal(exl3.apply_exl3_fused_moe(x, ids, w, lay, None, None, 10.0),
                       exl3.apply_exl3_fused_moe(x, ids, w, ref, None, None, 10.0))


def test_loader_four_bit_layer(tmp_path):
    _write_ckpt(str(tmp_path), bits=4)
    lay = loader.load_moe_layer(str(tmp_path), LAYER, device="cpu")
    g, u, dn = synth.expert_trellis_np(9, H, I, 2, LAYER, bits=4)
    assert lay.bits == 4 and np.array_equal(lay.w13_trellis[2, 1].numpy(), u) and np.array_equal(lay.w2_trellis[2].numpy(), dn)
