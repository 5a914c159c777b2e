"""On-disk packed-weight files (15642_moe_b200/packed_io.py): round trip, integrity checks.
The GPU test packs real weights, saves, loads and runs moe_forward from the loaded tensors."""
import importlib
import os

import numpy as np
import pytest
import torch


@pytest.fixture(scope="module")
def io():
    return importlib.import_module("15642_moe_b200.packed_io")


def _fake(E=1, seed=0):
    g = torch.Generator().manual_seed(seed)
    return dict(w13_packed=torch.randint(0, 256, (E, 16, 56, 256, 128), dtype=torch.uint8, generator=g),
                w13_scale=torch.rand((E, 32, 56), generator=g),
                w2_packed=torch.randint(0, 256, (E, 28, 16, 256, 128), dtype=torch.uint8, generator=g),
                w2_scale=torch.rand((E, 56, 16), generator=g))


def test_round_trip(io, tmp_path):
    w = _fake()
    path = os.path.join(tmp_path, "e.moeb")
    io.save_packed(path, w["w13_packed"], w["w13_scale"], w["w2_packed"], w["w2_scale"], local_expert_offset=96)
    h = io.read_header(path)
    assert h["E_local"] == 1 and h["local_expert_offset"] == 96
    assert all(s["offset"] % 4096 == 0 for s in h["sections"])
    got = io.load_packed(path, device="cpu")
    assert got["local_expert_offset"] == 96
    for k in io.SECTIONS:
        assert torch.equal(got[k], w[k]), k


def test_integrity_checks(io, tmp_path):
    w = _fake(seed=1)
    path = os.path.join(tmp_path, "e.moeb")
    io.save_packed(path, w["w13_packed"], w["w13_scale"], w["w2_packed"], w["w2_scale"])
    sec = {s["name"]: s for s in io.read_header(path)["sections"]}
    with open(path, "r+b") as f:                      # flip one byte of the W2 tiles
        f.seek(sec["w2_packed"]["offset"] + 12345)
        b = f.read(1)
        f.seek(sec["w2_packed"]["offset"] + 12345)
        f.write(bytes([b[0] ^ 0x40]))
    with pytest.raises(RuntimeError, match="checksum"):
        io.load_packed(path, device="cpu")
    assert io.load_packed(path, device="cpu", verify=False)["w13_packed"].shape[0] == 1
    with open(path, "r+b") as f:
        f.truncate(sec["w2_scale"]["offset"] + 100)
    with pytest.raises(RuntimeError, match="truncated"):
        io.load_packed(path, device="cpu", verify=False)
    bad = os.path.join(tmp_path, "bad.moeb")
    with open(bad, "wb") as f:
        f.write(b"NOTMOE00" + bytes(100))
    with pytest.raises(RuntimeError, match="not a packed-weight file"):
        io.load_packed(bad, device="cpu")


def test_shape_checked_on_save(io, tmp_path):
    w = _fake()
    with pytest.raises(RuntimeError, match="w2_scale"):
        io.save_packed(os.path.join(tmp_path, "x"), w["w13_packed"], w["w13_scale"], w["w2_packed"],
                       w["w2_scale"][:, :10])


@pytest.mark.gpu
def test_loaded_weights_run(pkg, io, tmp_path):
    cfg = pkg.CONFIGS[1].with_(T=32, E_local=4, local_expert_offset=64, seed=5)
    inp = pkg.make_inputs(cfg, "cuda")
    ref = pkg.run(**inp)
    path = os.path.join(tmp_path, "w.moeb")
    io.save_packed(path, pkg.pack_w13(inp["gemm1_weights"]), inp["gemm1_weights_scale"],
                   pkg.pack_w2(inp["gemm2_weights"]), inp["gemm2_weights_scale"], cfg.local_expert_offset)
    w = io.load_packed(path, device="cuda")
    out = pkg.moe_forward(inp["hidden_states"], inp["hidden_states_scale"].float().contiguous(), w["w13_packed"],
                          w["w13_scale"], w["w2_packed"], w["w2_scale"], inp["routing_logits"].float().contiguous(),
                          inp["routing_bias"].float().reshape(-1).contiguous(), cfg.routed_scaling_factor,
                          w["local_expert_offset"])
    assert torch.equal(out.view(torch.int16), ref.view(torch.int16))
