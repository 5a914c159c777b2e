"""The reference's own CUDA path timed on this GPU - the GPU BASELINE (test infrastructure).

Runs the reference's extension as its ``run_custom`` does (``moe_layer.py:99-120``): pack W13 /
W2 once with its ``pack_w13`` / ``pack_w2`` (``kernels/moe.cu:700-742``), then call its
``moe_forward`` (``kernels/moe.cu:744-900``: route_dispatch -> stage1 mma.sync GEMM1+SwiGLU ->
stage2 mma.sync GEMM2 + fp32 atomicAdd scatter -> bf16 convert) on the same device tensors the
benchmark feeds this package. The module is built by ``oracle/build_ref.py`` into ``oracle/_ref``.
Used by ``bench.py``'s ``ref_cuda`` baseline leg and by ``tests/``; never by the product.
"""
from __future__ import annotations

import torch

from . import build_ref


class RefCuda:
    """The reference extension bound to one workload (packed weights resident, inputs cast once
    the way run_custom casts them)."""

    def __init__(self, inp: dict, mod=None):
        self.mod = mod if mod is not None else build_ref.load()
        m = self.mod
        self.w13p = m.pack_w13(inp["gemm1_weights"].contiguous())
        self.w2p = m.pack_w2(inp["gemm2_weights"].contiguous())
        self.args = (inp["hidden_states"].contiguous(),
                     inp["hidden_states_scale"].to(torch.float32).contiguous(), self.w13p,
                     inp["gemm1_weights_scale"].to(torch.float32).contiguous(), self.w2p,
                     inp["gemm2_weights_scale"].to(torch.float32).contiguous(),
                     inp["routing_logits"].to(torch.float32).contiguous(),
                     inp["routing_bias"].to(torch.float32).reshape(-1).contiguous(),
                     float(inp["routed_scaling_factor"]), int(inp["local_expert_offset"]))

    def __call__(self) -> torch.Tensor:
        return self.mod.moe_forward(*self.args)

    def time_us(self, steps: int = 10, warmup: int = 3) -> float:
        """Mean device microseconds per call, CUDA events on the current stream."""
        for _ in range(warmup):
            self()
        torch.cuda.synchronize()
        s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s.record()
        for _ in range(steps):
            self()
        e.record()
        torch.cuda.synchronize()
        return s.elapsed_time(e) * 1e3 / steps
