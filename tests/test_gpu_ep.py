"""Expert-parallel layer on the GPU.

On one GPU the expert-parallel path runs as a single rank (its own buffer is its only peer):
dispatch, the flag barriers, the owner-side combine and the final combine all run, and the
result must equal moe_forward bit for bit (one owner: the output is its partial, rounded once).
With two or more GPUs, tests/ep_gpu_worker.py runs under torchrun, one process per GPU, and
checks every rank against the slice-by-slice layer (bit for bit) and the CPU layer oracle
(tolerance).
"""
import os
import socket
import subprocess
import sys

import numpy as np
import pytest
import torch

from gpu_helpers import out_bits

pytestmark = pytest.mark.gpu
HERE = os.path.dirname(os.path.abspath(__file__))


def _args(pkg, inp):
    return dict(hidden=inp["hidden_states"], hs=inp["hidden_states_scale"].float().contiguous(),
                w13p=pkg.pack_w13(inp["gemm1_weights"]), s13=inp["gemm1_weights_scale"].float().contiguous(),
                w2p=pkg.pack_w2(inp["gemm2_weights"]), s2=inp["gemm2_weights_scale"].float().contiguous(),
                lg=inp["routing_logits"].float().contiguous(),
                b=inp["routing_bias"].float().reshape(-1).contiguous(), rsf=float(inp["routed_scaling_factor"]))


def _single(pkg, k):
    return pkg.moe_forward(k["hidden"], k["hs"], k["w13p"], k["s13"], k["w2p"], k["s2"], k["lg"], k["b"],
                           k["rsf"], 0)


def _ep(ctx, k):
    return ctx.forward(k["hidden"], k["hs"], k["w13p"], k["s13"], k["w2p"], k["s2"], k["lg"], k["b"], k["rsf"])


def test_fp32_out_rounds_to_moe_forward(pkg):
    """moe_forward(fp32_out=True) is the sum before the final rounding: its bf16 rounding is
    moe_forward's output bit for bit."""
    cfg = pkg.CONFIGS[1].with_(T=200, seed=6)
    k = _args(pkg, pkg.make_inputs(cfg, "cuda"))
    ref = _single(pkg, k)
    f32 = pkg.moe_forward(k["hidden"], k["hs"], k["w13p"], k["s13"], k["w2p"], k["s2"], k["lg"], k["b"],
                          k["rsf"], 0, fp32_out=True)
    assert f32.dtype == torch.float32
    np.testing.assert_array_equal(out_bits(f32.to(torch.bfloat16)), out_bits(ref))


@pytest.mark.parametrize("T,E", [(64, 32), (1000, 32), (48, 256)])
def test_single_rank_equals_moe_forward(pkg, T, E):
    cfg = pkg.CONFIGS[1].with_(T=T, E_local=E, seed=3)
    k = _args(pkg, pkg.make_inputs(cfg, "cuda"))
    ref = _single(pkg, k)
    with pkg.ExpertParallel(t_rank_max=T, e_rank=E) as ctx:
        for _ in range(3):                      # three epochs over the same buffers
            out = _ep(ctx, k)
            torch.cuda.synchronize()
            np.testing.assert_array_equal(out_bits(out), out_bits(ref))
    assert pkg.device_status(reset=True) == 0


def test_single_rank_varying_T(pkg):
    cfg = pkg.CONFIGS[1].with_(T=128, seed=8)
    full = pkg.make_inputs(cfg, "cuda")
    k_all = _args(pkg, full)
    with pkg.ExpertParallel(t_rank_max=128, e_rank=32) as ctx:
        for T in (0, 1, 128, 17, 0, 64):
            k = dict(k_all, hidden=k_all["hidden"][:T].contiguous(), hs=k_all["hs"][:, :T].contiguous(),
                     lg=k_all["lg"][:T].contiguous())
            out = _ep(ctx, k)
            ref = _single(pkg, k)
            torch.cuda.synchronize()
            np.testing.assert_array_equal(out_bits(out), out_bits(ref))
        with pytest.raises(RuntimeError, match="t_rank_max"):
            k = _args(pkg, pkg.make_inputs(cfg.with_(T=129), "cuda"))
            _ep(ctx, k)
    assert pkg.device_status(reset=True) == 0


def test_single_rank_permuted_placement(pkg):
    """Experts held in reversed local order: the owner still sums a token's routes in ascending
    global expert order, so the result equals moe_forward bit for bit."""
    cfg = pkg.CONFIGS[1].with_(T=96, seed=12)
    inp = pkg.make_inputs(cfg, "cuda")
    k = _args(pkg, inp)
    ref = _single(pkg, k)
    order = list(range(31, -1, -1))
    w = pkg.make_weights(cfg, order, "cuda")
    kp = dict(k, w13p=pkg.pack_w13(w["gemm1_weights"]), s13=w["gemm1_weights_scale"],
              w2p=pkg.pack_w2(w["gemm2_weights"]), s2=w["gemm2_weights_scale"])
    with pkg.ExpertParallel(t_rank_max=96, e_rank=32, placement=[order]) as ctx:
        assert ctx.experts == order
        out = _ep(ctx, kp)
        torch.cuda.synchronize()
    np.testing.assert_array_equal(out_bits(out), out_bits(ref))
    assert pkg.device_status(reset=True) == 0


def test_run_surface(pkg):
    """ExpertParallel.run takes reference.run's keywords for the rank's tokens and experts."""
    cfg = pkg.CONFIGS[1].with_(T=32, seed=4)
    inp = pkg.make_inputs(cfg, "cuda")
    ref = pkg.run(**inp)
    kw = {k: v for k, v in inp.items() if k != "local_expert_offset"}
    with pkg.ExpertParallel(t_rank_max=32, e_rank=32) as ctx:
        out = ctx.run(**kw)
    np.testing.assert_array_equal(out_bits(out), out_bits(ref))


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _run_worker(n, cases, timeout):
    cmd = [sys.executable, "-m", "torch.distributed.run", "--nnodes=1", f"--nproc-per-node={n}",
           "--master-addr", "127.0.0.1", "--master-port", str(_free_port()),
           os.path.join(HERE, "ep_gpu_worker.py"), "--cases", cases]
    env = dict(os.environ, NCCL_NVLS_ENABLE="0")
    p = subprocess.run(["timeout", "-k", "30", str(timeout)] + cmd, capture_output=True, text=True, env=env)
    # The cases that passed, then the first traceback of any rank, then the launcher's tail.
    lines = (p.stdout + p.stderr).splitlines()
    ok = [ln for ln in lines if "EP_CASE_OK" in ln]
    first = next((i for i, ln in enumerate(lines) if "Traceback" in ln), None)
    tb = lines[first:first + 40] if first is not None else []
    tail = "\n".join(ok + ["--- first traceback ---"] + tb + ["--- tail ---"]) + "\n" + (p.stdout + p.stderr)[-1500:]
    assert p.returncode == 0, tail
    for c in cases.split(","):
        for r in range(n):
            assert f"EP_CASE_OK {c} rank={r}" in p.stdout, tail


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs")
def test_two_ranks():
    _run_worker(2, "oracle,ragged,weak,layer,skew,graph,placement", 900)


@pytest.mark.skipif(torch.cuda.device_count() < 8, reason="needs 8 GPUs")
def test_eight_ranks():
    _run_worker(8, "oracle,ragged,weak,layer,skew,graph,placement", 1200)
