"""DeepSeek-V3 shared-expert branch (every token through one expert, weight 1) against the CPU
restatement, alone and added to the routed output before one rounding."""
import numpy as np
import pytest
import torch

from gpu_helpers import out_bits

pytestmark = pytest.mark.gpu


def _shared(pkg, cfg_seed_offset, T):
    # The shared expert's weights: the generator's expert stream 255, independent of the routed slice.
    cfg = pkg.CONFIGS[1].with_(T=T, E_local=1, local_expert_offset=255, seed=cfg_seed_offset)
    return cfg, pkg.make_inputs(cfg, "cuda")


@pytest.mark.parametrize("T", [1, 16, 300])
def test_shared_expert_matches_oracle(pkg, oracle, T):
    cfg, inp = _shared(pkg, 4, T)
    w13p, w2p = pkg.pack_w13(inp["gemm1_weights"]), pkg.pack_w2(inp["gemm2_weights"])
    args = (inp["hidden_states"], inp["hidden_states_scale"].float().contiguous(), w13p,
            inp["gemm1_weights_scale"].float().contiguous(), w2p, inp["gemm2_weights_scale"].float().contiguous())
    out = pkg.shared_expert_forward(*args)
    f32 = pkg.shared_expert_forward(*args, fp32_out=True)
    torch.cuda.synchronize()
    npi = oracle.to_numpy_inputs(inp)
    ref = oracle.shared_expert_forward(npi["hidden_states"], npi["hidden_states_scale"], npi["gemm1_weights"],
                                       npi["gemm1_weights_scale"], npi["gemm2_weights"], npi["gemm2_weights_scale"])
    r = oracle.check_tolerance(ref, out_bits(out))
    assert r["bad"] == 0, r
    np.testing.assert_array_equal(out_bits(f32.to(torch.bfloat16)), out_bits(out))
    assert pkg.device_status(reset=True) == 0


def test_layer_with_shared_expert(pkg, oracle):
    """Full DeepSeek-V3 MoE output of a 32-expert slice: bf16(routed_fp32 + shared_fp32)."""
    T = 48
    rcfg = pkg.CONFIGS[1].with_(T=T, seed=9)
    rin = pkg.make_inputs(rcfg, "cuda")
    _, sin = _shared(pkg, 9, T)                     # same seed: same hidden states and scales
    assert torch.equal(sin["hidden_states"].view(torch.uint8), rin["hidden_states"].view(torch.uint8))
    hs = rin["hidden_states_scale"].float().contiguous()
    routed = pkg.moe_forward(rin["hidden_states"], hs, pkg.pack_w13(rin["gemm1_weights"]),
                             rin["gemm1_weights_scale"].float().contiguous(), pkg.pack_w2(rin["gemm2_weights"]),
                             rin["gemm2_weights_scale"].float().contiguous(),
                             rin["routing_logits"].float().contiguous(),
                             rin["routing_bias"].float().reshape(-1).contiguous(), rcfg.routed_scaling_factor, 0,
                             fp32_out=True)
    shared = pkg.shared_expert_forward(sin["hidden_states"], hs, pkg.pack_w13(sin["gemm1_weights"]),
                                       sin["gemm1_weights_scale"].float().contiguous(),
                                       pkg.pack_w2(sin["gemm2_weights"]),
                                       sin["gemm2_weights_scale"].float().contiguous(), fp32_out=True)
    out = (routed + shared).to(torch.bfloat16)
    rn, sn = oracle.to_numpy_inputs(rin), oracle.to_numpy_inputs(sin)
    ref = oracle.f32_to_bf16_bits(oracle.moe_forward(**rn, return_fp32=True) + oracle.shared_expert_forward(
        sn["hidden_states"], sn["hidden_states_scale"], sn["gemm1_weights"], sn["gemm1_weights_scale"],
        sn["gemm2_weights"], sn["gemm2_weights_scale"], return_fp32=True))
    r = oracle.check_tolerance(ref, out_bits(out))
    assert r["bad"] == 0, r


def test_shared_expert_t0(pkg):
    _, inp = _shared(pkg, 1, 1)
    w13p, w2p = pkg.pack_w13(inp["gemm1_weights"]), pkg.pack_w2(inp["gemm2_weights"])
    out = pkg.shared_expert_forward(inp["hidden_states"][:0], inp["hidden_states_scale"][:, :0].contiguous(), w13p,
                                    inp["gemm1_weights_scale"].float().contiguous(), w2p,
                                    inp["gemm2_weights_scale"].float().contiguous())
    assert out.shape == (0, 7168)
