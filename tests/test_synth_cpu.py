"""The CPU side of the seeded generator: format conversions against torch, determinism,
distributions. (The GPU twin is compared bit for bit in tests/test_gpu_synth.py.)"""
import numpy as np
import torch


def test_quantile_table_symmetric(pkg):
    t = pkg.quantile_table()
    assert t.shape == ((1 << 16) + 1,)
    np.testing.assert_array_equal(t, -t[::-1])
    assert np.all(np.diff(t) > 0)


def test_generator_deterministic_and_sliceable(pkg):
    cfg = pkg.MoEConfig(T=8, E_local=2, local_expert_offset=5, seed=11)
    a = pkg.make_inputs(cfg, "cpu")
    b = pkg.make_inputs(cfg, "cpu")
    for k in a:
        if isinstance(a[k], torch.Tensor):
            assert torch.equal(a[k].view(torch.uint8), b[k].view(torch.uint8)), k
    # expert 6 of a [5, 7) slice equals expert 1 of a [5, 7) slice and expert 0 of [6, 7)
    c = pkg.make_inputs(cfg.with_(E_local=1, local_expert_offset=6), "cpu")
    assert torch.equal(a["gemm1_weights"][1].view(torch.uint8), c["gemm1_weights"][0].view(torch.uint8))
    assert torch.equal(a["gemm2_weights_scale"][1], c["gemm2_weights_scale"][0])


def test_e4m3_and_scales_match_torch_cast(pkg, oracle):
    """Generated codes equal torch's float8_e4m3fn cast of x / scale (RNE, in range)."""
    cfg = pkg.MoEConfig(T=64, E_local=1, seed=3)
    inp = pkg.make_inputs(cfg, "cpu")
    codes = inp["hidden_states"].view(torch.uint8).numpy()
    scale = inp["hidden_states_scale"].numpy()              # [56, T]
    vals = oracle.decode_e4m3(codes).reshape(64, 56, 128)
    amax_q = np.abs(vals).max(axis=2)
    assert np.allclose(amax_q, 448.0)                      # amax maps to the top code
    # dequantised values reproduce bf16 numbers within e4m3 precision
    deq = vals * scale.T[:, :, None]
    assert np.isfinite(deq).all() and 0.9 < deq.std() < 1.1
    # torch's cast of the dequantised/scale agrees with the stored code
    x = torch.from_numpy((deq / scale.T[:, :, None]).astype(np.float32))
    tc = x.to(torch.float8_e4m3fn).view(torch.uint8).numpy().reshape(64, 56, 128)
    np.testing.assert_array_equal(tc, codes.reshape(64, 56, 128))


def test_weight_distribution(pkg, oracle):
    inp = pkg.make_inputs(pkg.MoEConfig(T=1, E_local=1, seed=0), "cpu")
    w = oracle.dequant_block(inp["gemm2_weights"][0].view(torch.uint8).numpy(),
                             inp["gemm2_weights_scale"][0].numpy())
    assert abs(w.mean()) < 1e-4 and 0.018 < w.std() < 0.022
    bias = inp["routing_bias"].float().numpy()
    assert 0.07 < bias.std() < 0.13


def test_skew_bias(pkg):
    cfg = pkg.CONFIGS[4].with_(T=2, E_local=1)
    b = pkg.make_inputs(cfg, "cpu")["routing_bias"].float()
    hot = list(cfg.hot_experts)
    assert len(hot) == 16 and (b[hot] == 1.5).all()


def test_oracle_generator_restatement_matches(pkg, oracle):
    """oracle/synth_oracle.py (numpy, used by the benchmark's CPU arms so they load no compiled
    code of the package) produces the package generator's bytes: a slice with hot experts, an
    offset and a seed other than 0, and the e4m3 encoder against torch's cast on edge values."""
    from oracle import synth_oracle as S
    cfg = pkg.MoEConfig(T=48, E_local=2, local_expert_offset=31, seed=9, hot_experts=(0, 1, 32))
    a = oracle.to_numpy_inputs(pkg.make_inputs(cfg, "cpu"))
    b = S.make_inputs(**cfg.__dict__)
    for k, v in a.items():
        if isinstance(v, np.ndarray):
            assert np.array_equal(v.view(np.uint8), np.ascontiguousarray(b[k]).view(np.uint8)), k
        else:
            assert v == b[k], k
    part = S.make_inputs(**cfg.__dict__, experts=[1])
    assert np.array_equal(part["gemm2_weights"][1], b["gemm2_weights"][1]) and not part["gemm1_weights"][0].any()
    x = np.concatenate([np.random.default_rng(0).standard_normal(1 << 16).astype(np.float32) * 50,
                        np.array([0, -0.0, 448, 463.9, 2 ** -9, 2 ** -10, 3 * 2 ** -11, -2 ** -7, 1e-30],
                                 np.float32)])
    ref = torch.from_numpy(x).to(torch.float8_e4m3fn).view(torch.uint8).numpy()
    np.testing.assert_array_equal(S.e4m3_codes(x), ref)
