"""HostPipeline: the serving loop from pinned host memory through the layer and back, with the
copies of neighbouring steps overlapping the forward on three streams, returns for every step
exactly moe_forward's output on that step's inputs (bit for bit), at several slot depths."""
import pytest
import torch

pytestmark = pytest.mark.gpu


def _step_inputs(base, n):
    """n distinct activation sets from one input set: rows rotated, logits perturbed."""
    g = torch.Generator(device="cuda").manual_seed(5)
    out = []
    for k in range(n):
        out.append({"hidden_states": torch.roll(base["hidden_states"].view(torch.uint8), k, 0).view(torch.float8_e4m3fn),
                    "hidden_states_scale": torch.roll(base["hidden_states_scale"].float(), k, 1).contiguous(),
                    "routing_logits": (base["routing_logits"].float()
                                       + 0.5 * torch.randn(base["routing_logits"].shape, device="cuda", generator=g))})
    return out


@pytest.mark.parametrize("depth", [1, 2, 3])
def test_pipeline_matches_moe_forward(pkg, depth):
    cfg = pkg.CONFIGS[1].with_(T=48)
    base = pkg.make_inputs(cfg, "cuda")
    w13p, w2p = pkg.pack_w13(base["gemm1_weights"]), pkg.pack_w2(base["gemm2_weights"])
    s13 = base["gemm1_weights_scale"].float().contiguous()
    s2 = base["gemm2_weights_scale"].float().contiguous()
    bias = base["routing_bias"].float().reshape(-1).contiguous()
    rsf, off = float(base["routed_scaling_factor"]), int(base["local_expert_offset"])
    pipe = pkg.HostPipeline.for_layer(w13p, s13, w2p, s2, base["routing_bias"], rsf, off, cfg.T, depth=depth)
    steps = _step_inputs(base, 5)
    host_in, host_out, expect = [], [], []
    for inp in steps:
        h = inp["hidden_states"].cpu().pin_memory()
        sc = inp["hidden_states_scale"].float().cpu().pin_memory()
        lg = inp["routing_logits"].float().cpu().pin_memory()
        host_in.append((h, sc, lg))
        host_out.append(torch.empty((cfg.T, 7168), dtype=torch.bfloat16).pin_memory())
        ref = pkg.moe_forward(inp["hidden_states"], inp["hidden_states_scale"].float().contiguous(), w13p, s13, w2p,
                              s2, inp["routing_logits"].float().contiguous(), bias, rsf, off)
        expect.append(ref.cpu())
    for (h, sc, lg), o in zip(host_in, host_out):
        pipe.submit(h, sc, lg, o)
    pipe.synchronize()
    assert pkg.device_status(reset=True) == 0
    for got, ref in zip(host_out, expect):
        assert torch.equal(got.view(torch.int16), ref.view(torch.int16))


def test_pipeline_argument_checks(pkg):
    pipe = pkg.HostPipeline(lambda h, s, lg, o: None, 4)
    h = torch.zeros((4, 7168), dtype=torch.float8_e4m3fn).pin_memory()
    sc = torch.zeros((56, 4)).pin_memory()
    lg = torch.zeros((4, 256)).pin_memory()
    o = torch.zeros((4, 7168), dtype=torch.bfloat16).pin_memory()
    with pytest.raises(RuntimeError, match="pinned"):
        pipe.submit(h, sc, lg, torch.zeros((4, 7168), dtype=torch.bfloat16))
    with pytest.raises(RuntimeError, match="shape"):
        pipe.submit(h, sc, torch.zeros((5, 256)).pin_memory(), o)
    pipe.submit(h, sc, lg, o)
    pipe.synchronize()


def test_pipeline_with_expert_parallel_forward(pkg):
    """The pipeline around an expert-parallel context (single rank: dispatch, flag barriers,
    owner-side and final combine on one GPU) on the pipeline's compute stream returns, for every
    step, moe_forward's output on that step's inputs."""
    cfg = pkg.CONFIGS[1].with_(T=40)
    base = pkg.make_inputs(cfg, "cuda")
    w13p, w2p = pkg.pack_w13(base["gemm1_weights"]), pkg.pack_w2(base["gemm2_weights"])
    s13 = base["gemm1_weights_scale"].float().contiguous()
    s2 = base["gemm2_weights_scale"].float().contiguous()
    bias = base["routing_bias"].float().reshape(-1).contiguous()
    rsf = float(base["routed_scaling_factor"])
    steps = _step_inputs(base, 4)
    with pkg.ExpertParallel(t_rank_max=cfg.T, e_rank=32) as ep:
        def layer(h, sc, lg, o):
            ep.forward(h, sc, w13p, s13, w2p, s2, lg, bias, rsf, out=o)

        pipe = pkg.HostPipeline(layer, cfg.T, depth=2)
        outs = []
        for inp in steps:
            o = torch.empty((cfg.T, 7168), dtype=torch.bfloat16).pin_memory()
            pipe.submit(inp["hidden_states"].cpu().pin_memory(), inp["hidden_states_scale"].cpu().pin_memory(),
                        inp["routing_logits"].cpu().pin_memory(), o)
            outs.append(o)
        pipe.synchronize()
    assert pkg.device_status(reset=True) == 0
    for inp, got in zip(steps, outs):
        ref = pkg.moe_forward(inp["hidden_states"], inp["hidden_states_scale"], w13p, s13, w2p, s2,
                              inp["routing_logits"], bias, rsf, 0)
        assert torch.equal(got.view(torch.int16), ref.cpu().view(torch.int16))
