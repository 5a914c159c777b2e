"""CUDA-graph capture of the forward (the launch-bound decode case). Every launch of
moe_forward and of the expert-parallel forward goes on the caller's stream with no host
synchronisation and no per-call host state (the expert-parallel epoch lives in device memory),
so a captured graph replays correctly with new inputs copied into the captured buffers."""
import numpy as np
import pytest
import torch

from gpu_helpers import out_bits

pytestmark = pytest.mark.gpu


def _packed(pkg, cfg):
    inp = pkg.make_inputs(cfg, "cuda")
    return inp, dict(w13p=pkg.pack_w13(inp["gemm1_weights"]), w2p=pkg.pack_w2(inp["gemm2_weights"]),
                     s13=inp["gemm1_weights_scale"].float().contiguous(),
                     s2=inp["gemm2_weights_scale"].float().contiguous(),
                     b=inp["routing_bias"].float().reshape(-1).contiguous(), rsf=float(inp["routed_scaling_factor"]))


def _activations(pkg, cfg, seed):
    inp = pkg.make_inputs(cfg.with_(seed=seed, E_local=1), "cuda")
    return (inp["hidden_states"], inp["hidden_states_scale"].float().contiguous(),
            inp["routing_logits"].float().contiguous())


def test_moe_forward_graph_replay(pkg):
    cfg = pkg.CONFIGS[1]                                   # T = 64 decode shape
    _, w = _packed(pkg, cfg)
    T = cfg.T
    h, hs, lg = (t.clone() for t in _activations(pkg, cfg, 100))
    out = torch.empty((T, 7168), dtype=torch.bfloat16, device="cuda")
    ws = torch.empty(pkg.workspace_bytes(T, 32), dtype=torch.uint8, device="cuda")
    call = lambda: pkg.moe_forward(h, hs, w["w13p"], w["s13"], w["w2p"], w["s2"], lg, w["b"], w["rsf"], 0,
                                   out=out, workspace=ws)
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        call()                                             # one-time set-up outside the capture
    torch.cuda.current_stream().wait_stream(s)
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        call()
    for seed in (101, 102, 103):
        nh, nhs, nlg = _activations(pkg, cfg, seed)
        h.copy_(nh); hs.copy_(nhs); lg.copy_(nlg)
        g.replay()
        torch.cuda.synchronize()
        ref = pkg.moe_forward(nh, nhs, w["w13p"], w["s13"], w["w2p"], w["s2"], nlg, w["b"], w["rsf"], 0)
        np.testing.assert_array_equal(out_bits(out), out_bits(ref))
    assert pkg.device_status(reset=True) == 0


def test_expert_parallel_graph_replay(pkg):
    """Single-rank expert-parallel layer: the barriers' epoch advances on the device, so each
    replay is a new epoch."""
    cfg = pkg.CONFIGS[1]
    _, w = _packed(pkg, cfg)
    T = cfg.T
    h, hs, lg = (t.clone() for t in _activations(pkg, cfg, 200))
    out = torch.empty((T, 7168), dtype=torch.bfloat16, device="cuda")
    with pkg.ExpertParallel(t_rank_max=T, e_rank=32) as ep:
        call = lambda: ep.forward(h, hs, w["w13p"], w["s13"], w["w2p"], w["s2"], lg, w["b"], w["rsf"], out=out)
        call()
        torch.cuda.synchronize()
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g):
            call()
        for seed in (201, 202, 203, 204):
            nh, nhs, nlg = _activations(pkg, cfg, seed)
            h.copy_(nh); hs.copy_(nhs); lg.copy_(nlg)
            g.replay()
            torch.cuda.synchronize()
            ref = pkg.moe_forward(nh, nhs, w["w13p"], w["s13"], w["w2p"], w["s2"], nlg, w["b"], w["rsf"], 0)
            np.testing.assert_array_equal(out_bits(out), out_bits(ref))
        call()                                             # eager after replays: epochs stay in step
        torch.cuda.synchronize()
        np.testing.assert_array_equal(out_bits(out), out_bits(ref))
        del g
    assert pkg.device_status(reset=True) == 0
