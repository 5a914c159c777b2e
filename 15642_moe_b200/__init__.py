"""B200 (sm_100a) DeepSeek-V3/R1 FP8 block-scaled MoE forward.

The package directory name starts with a digit, so import it with
``importlib.import_module("15642_moe_b200")``.

Public surface (mirrors the reference's Python API):
  run(**inputs)                  drop-in for reference.run (reference/moe_ref.py:5)
  run_custom(ops, **inputs)      moe_layer.py:99
  pack_w13 / pack_w2 / moe_forward  the extension functions of kernels/moe.cu:902-909
  route(logits, bias, rsf)       the device router alone (expert indices + weights)
  quantize_hidden(x_bf16)        FP8 activation quantiser (e4m3 codes + [56, T] block scales)
  pack_gate / gate_quantize      router GEMM fused with the quantiser: logits + codes + scales
  shared_expert_forward(...)     DeepSeek-V3 shared expert (all tokens, weight 1) on the same kernels
  make_inputs(cfg, device)       seeded synthetic inputs of the benchmark configurations
  ExpertParallel                 expert-parallel layer over the GPUs of one node (ep.py)
  save_packed / load_packed      packed weights on disk (packed_io.py)
  HostPipeline                   serving loop from/to pinned host memory on three streams (pipeline.py)
"""
from .layer import (_cached_pack, _load_custom_ops, gate_quantize, moe_forward, ops, pack_gate, pack_w13,
                    pack_w2, quantize_hidden, route, run, run_custom, shared_expert_forward, workspace_bytes)
from .synth import CONFIGS, MoEConfig, make_inputs, make_weights, quantile_table
from ._native import MoEError, device_status, set_wait_limit_ns, wait_limit_ns, workspace_layout
from .ep import ExpertParallel, balanced_placement, expert_range, owner_of, token_range
from .packed_io import load_packed, save_packed
from .pipeline import HostPipeline

__all__ = [
    "run", "run_custom", "ops", "pack_w13", "pack_w2", "moe_forward", "route", "workspace_bytes",
    "quantize_hidden", "shared_expert_forward", "pack_gate", "gate_quantize",
    "make_inputs", "make_weights", "MoEConfig", "CONFIGS", "quantile_table", "MoEError", "device_status", "set_wait_limit_ns", "wait_limit_ns",
    "workspace_layout", "_cached_pack", "_load_custom_ops", "ExpertParallel", "expert_range",
    "owner_of", "token_range", "balanced_placement", "save_packed", "load_packed", "HostPipeline",
]
