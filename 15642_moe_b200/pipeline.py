"""Serving loop with activations in pinned host memory: the host→device copy of a step's inputs,
the layer's forward and the device→host copy of its output run on three CUDA streams, so the
copies of neighbouring steps overlap the forward of the current one (the reference moves no data:
its layer runs on tensors the caller already placed, reference/moe_ref.py:5-16).

Step i uses device slot i % depth for its inputs and output. Events order the streams:
  h2d:      wait until the forward of step i - depth has read slot s      -> copy inputs  -> in_ready[s]
  forward:  wait in_ready[s] and the D2H of step i - depth out of slot s  -> forward       -> in_free[s], out_ready[s]
  d2h:      wait out_ready[s]                                             -> copy output  -> out_free[s]
Every step still moves its own inputs in and its own output out; forwards run in submission order
on one stream (one workspace serves them all).
"""
from __future__ import annotations

from typing import Callable

import torch

from .layer import E_GLOBAL, H, H_BLOCKS, _check, moe_forward, workspace_bytes


class HostPipeline:
    """`forward(hidden, hidden_scale, logits, out)` enqueues one layer on the current stream for
    device tensors hidden e4m3 [T, 7168], hidden_scale fp32 [56, T], logits fp32 [T, 256] and
    writes bf16 [T, 7168] into `out`. `submit` takes pinned host tensors of those shapes and a
    pinned host bf16 [T, 7168] output; results are complete after `synchronize()` (or the
    caller's own wait on `d2h_stream`). The caller keeps each host buffer unchanged until then."""

    def __init__(self, forward: Callable, T: int, device: torch.device | str | None = None, depth: int = 2):
        _check(T >= 1, "T must be at least 1")
        _check(depth >= 1, "depth must be at least 1")
        self.forward, self.T, self.depth = forward, int(T), int(depth)
        self.device = torch.device(device) if device is not None else torch.device("cuda", torch.cuda.current_device())
        dev = self.device
        self.h2d_stream = torch.cuda.Stream(dev)
        self.compute_stream = torch.cuda.Stream(dev)
        self.d2h_stream = torch.cuda.Stream(dev)
        self._hidden = [torch.empty((T, H), dtype=torch.float8_e4m3fn, device=dev) for _ in range(depth)]
        self._scale = [torch.empty((H_BLOCKS, T), dtype=torch.float32, device=dev) for _ in range(depth)]
        self._logits = [torch.empty((T, E_GLOBAL), dtype=torch.float32, device=dev) for _ in range(depth)]
        self._out = [torch.empty((T, H), dtype=torch.bfloat16, device=dev) for _ in range(depth)]
        self._in_ready = [torch.cuda.Event() for _ in range(depth)]
        self._in_free = [torch.cuda.Event() for _ in range(depth)]
        self._out_ready = [torch.cuda.Event() for _ in range(depth)]
        self._out_free = [torch.cuda.Event() for _ in range(depth)]
        self._used = [False] * depth
        self.steps = 0

    @classmethod
    def for_layer(cls, W13_packed, W13_scale, W2_packed, W2_scale, bias, rsf: float, local_offset: int, T: int,
                  depth: int = 2) -> "HostPipeline":
        """One local-expert slice on one GPU (moe_forward with resident packed weights)."""
        dev = W13_packed.device
        ws = torch.empty(workspace_bytes(T, int(W13_packed.size(0))), dtype=torch.uint8, device=dev)
        bias = bias.to(torch.float32).reshape(-1).contiguous()

        def forward(h, s, lg, out):
            moe_forward(h, s, W13_packed, W13_scale, W2_packed, W2_scale, lg, bias, rsf, local_offset,
                        out=out, workspace=ws)

        return cls(forward, T, dev, depth)

    def submit(self, hidden: torch.Tensor, hidden_scale: torch.Tensor, logits: torch.Tensor,
               out: torch.Tensor) -> None:
        T = self.T
        for t, shape, name in ((hidden, (T, H), "hidden"), (hidden_scale, (H_BLOCKS, T), "hidden_scale"),
                               (logits, (T, E_GLOBAL), "logits"), (out, (T, H), "out")):
            _check(not t.is_cuda and tuple(t.shape) == shape and t.is_contiguous(),
                   f"{name} must be a contiguous host tensor of shape {shape}")
            _check(t.is_pinned(), f"{name} must be in pinned host memory")
        _check(hidden.element_size() == 1, "hidden must be an FP8 tensor")
        _check(hidden_scale.dtype == torch.float32 and logits.dtype == torch.float32,
               "hidden_scale and logits must be float32")
        _check(out.dtype == torch.bfloat16, "out must be bfloat16")
        s = self.steps % self.depth
        used = self._used[s]
        with torch.cuda.stream(self.h2d_stream):
            if used:
                self.h2d_stream.wait_event(self._in_free[s])
            self._hidden[s].view(torch.uint8).copy_(hidden.view(torch.uint8), non_blocking=True)
            self._scale[s].copy_(hidden_scale, non_blocking=True)
            self._logits[s].copy_(logits, non_blocking=True)
            self._in_ready[s].record(self.h2d_stream)
        with torch.cuda.stream(self.compute_stream):
            self.compute_stream.wait_event(self._in_ready[s])
            if used:
                self.compute_stream.wait_event(self._out_free[s])
            self.forward(self._hidden[s], self._scale[s], self._logits[s], self._out[s])
            self._in_free[s].record(self.compute_stream)
            self._out_ready[s].record(self.compute_stream)
        with torch.cuda.stream(self.d2h_stream):
            self.d2h_stream.wait_event(self._out_ready[s])
            out.copy_(self._out[s], non_blocking=True)
            self._out_free[s].record(self.d2h_stream)
        self._used[s] = True
        self.steps += 1

    def synchronize(self) -> None:
        self.d2h_stream.synchronize()
