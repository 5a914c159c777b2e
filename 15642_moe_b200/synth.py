"""Seeded synthetic inputs for the five benchmark configurations.

The reference publishes no dataset; its own generator (moe_layer.py:47-74) draws uniform
FP8 values. The configurations of this build instead use the DeepSeek-like distributions
named in the benchmark description: logits N(0,1), bias N(0,0.1) in bf16, hidden N(0,1) in
bf16 quantised to e4m3 per (token, 128 columns), weights N(0,0.02) in bf16 quantised to e4m3
per 128x128 block, all scales = amax / 448.

Bits are produced by a counter-based generator implemented twice (C for the host,
CUDA for the device) with identical results, see csrc/synth_core.h. Expert ``g`` of a weight
tensor always comes from the stream of global expert id ``g``, so any slice
``[local_expert_offset, local_expert_offset + E_local)`` of the 256-expert layer is
reproducible on its own (expert-parallel ranks generate only their own experts).
"""
from __future__ import annotations

import dataclasses
import functools
import statistics

import numpy as np
import torch

from . import _native

H, I_DIM, E_GLOBAL, BLOCK = 7168, 2048, 256, 128
TABLE_BITS = 16


@functools.lru_cache(maxsize=None)
def quantile_table() -> np.ndarray:
    """fp32 [2^16 + 1] standard-normal quantiles at (i + 0.5) / (2^16 + 1)."""
    n = 1 << TABLE_BITS
    nd = statistics.NormalDist()
    return np.array([nd.inv_cdf((i + 0.5) / (n + 1)) for i in range(n + 1)], dtype=np.float32)


@functools.lru_cache(maxsize=None)
def _table_on(device: str) -> torch.Tensor:
    return torch.from_numpy(quantile_table()).to(device)


@dataclasses.dataclass(frozen=True)
class MoEConfig:
    """One synthetic workload. ``T`` tokens, experts [offset, offset + E_local) of 256."""
    T: int
    E_local: int = 32
    local_expert_offset: int = 0
    seed: int = 0
    routed_scaling_factor: float = 2.5
    hidden_std: float = 1.0
    weight_std: float = 0.02
    bias_std: float = 0.1
    hot_experts: tuple = ()
    hot_bias: float = 1.5
    name: str = ""

    def with_(self, **kw) -> "MoEConfig":
        return dataclasses.replace(self, **kw)


# Configurations of the benchmark description (0..4). 3 and 4 are expert-parallel layers
# over 256 experts; their per-rank slices set E_local = 256 / world and the offset.
CONFIGS = {
    0: MoEConfig(T=16, name="cpu_oracle_t16"),
    1: MoEConfig(T=64, name="decode_t64"),
    2: MoEConfig(T=4096, name="prefill_t4096"),
    3: MoEConfig(T=8192, E_local=256, name="ep_layer_t8192"),
    4: MoEConfig(T=16384, E_local=256, hot_experts=tuple(e for g in range(8) for e in (32 * g, 32 * g + 1)),
                 name="ep_skew_t16384"),
}


def _ptr(t) -> int:
    return t.data_ptr() if isinstance(t, torch.Tensor) else t.ctypes.data


def make_inputs(cfg: MoEConfig, device: str | torch.device = "cuda") -> dict:
    """Inputs of ``reference.run`` / ``moe_forward`` for ``cfg`` (keyword names of
    reference/moe_ref.py:5-16), generated on ``device`` (CPU or CUDA, same bytes)."""
    device = torch.device(device)
    if device.type == "cuda":
        return _make_gpu(cfg, device)
    return _make_cpu(cfg)


def _kwargs(cfg, logits, bias, hidden, hscale, w13, s13, w2, s2) -> dict:
    return dict(
        routing_logits=logits,
        routing_bias=bias,
        hidden_states=hidden,
        hidden_states_scale=hscale,
        gemm1_weights=w13,
        gemm1_weights_scale=s13,
        gemm2_weights=w2,
        gemm2_weights_scale=s2,
        local_expert_offset=int(cfg.local_expert_offset),
        routed_scaling_factor=float(cfg.routed_scaling_factor),
    )


def _make_cpu(cfg: MoEConfig) -> dict:
    lib = _native.synth_cpu_lib()
    tab = quantile_table()
    T, E = cfg.T, cfg.E_local
    logits = np.empty((T, E_GLOBAL), np.float32)
    bias = np.empty((E_GLOBAL,), np.uint16)
    hidden = np.empty((T, H), np.uint8)
    hscale = np.empty((H // BLOCK, T), np.float32)
    w13 = np.empty((E, 2 * I_DIM, H), np.uint8)
    s13 = np.empty((E, 2 * I_DIM // BLOCK, H // BLOCK), np.float32)
    w2 = np.empty((E, H, I_DIM), np.uint8)
    s2 = np.empty((E, H // BLOCK, I_DIM // BLOCK), np.float32)
    hot = np.array(cfg.hot_experts or [0], np.int32)
    lib.moe_synth_cpu_logits(_ptr(tab), cfg.seed, T, E_GLOBAL, _ptr(logits))
    lib.moe_synth_cpu_bias(_ptr(tab), cfg.seed, E_GLOBAL, cfg.bias_std, _ptr(hot),
                           len(cfg.hot_experts), cfg.hot_bias, _ptr(bias))
    lib.moe_synth_cpu_hidden(_ptr(tab), cfg.seed, T, cfg.hidden_std, _ptr(hidden), _ptr(hscale))
    lib.moe_synth_cpu_w13(_ptr(tab), cfg.seed, cfg.local_expert_offset, E, cfg.weight_std,
                          _ptr(w13), _ptr(s13))
    lib.moe_synth_cpu_w2(_ptr(tab), cfg.seed, cfg.local_expert_offset, E, cfg.weight_std,
                         _ptr(w2), _ptr(s2))
    t = torch.from_numpy
    return _kwargs(cfg, t(logits), t(bias.view(np.int16)).view(torch.bfloat16),
                   t(hidden).view(torch.float8_e4m3fn), t(hscale),
                   t(w13).view(torch.float8_e4m3fn), t(s13), t(w2).view(torch.float8_e4m3fn), t(s2))


def _make_gpu(cfg: MoEConfig, device: torch.device) -> dict:
    lib = _native.cuda_lib()
    T, E = cfg.T, cfg.E_local
    with torch.cuda.device(device):
        tab = _table_on(str(device))
        st = torch.cuda.current_stream(device).cuda_stream
        logits = torch.empty((T, E_GLOBAL), dtype=torch.float32, device=device)
        bias = torch.empty((E_GLOBAL,), dtype=torch.bfloat16, device=device)
        hidden = torch.empty((T, H), dtype=torch.uint8, device=device)
        hscale = torch.empty((H // BLOCK, T), dtype=torch.float32, device=device)
        w13 = torch.empty((E, 2 * I_DIM, H), dtype=torch.uint8, device=device)
        s13 = torch.empty((E, 2 * I_DIM // BLOCK, H // BLOCK), dtype=torch.float32, device=device)
        w2 = torch.empty((E, H, I_DIM), dtype=torch.uint8, device=device)
        s2 = torch.empty((E, H // BLOCK, I_DIM // BLOCK), dtype=torch.float32, device=device)
        hot = torch.tensor(list(cfg.hot_experts) or [0], dtype=torch.int32, device=device)
        chk = _native.check
        chk(lib.moe_synth_logits(tab.data_ptr(), cfg.seed, T, E_GLOBAL, logits.data_ptr(), st))
        chk(lib.moe_synth_bias(tab.data_ptr(), cfg.seed, E_GLOBAL, cfg.bias_std, hot.data_ptr(),
                               len(cfg.hot_experts), cfg.hot_bias, bias.data_ptr(), st))
        chk(lib.moe_synth_hidden(tab.data_ptr(), cfg.seed, T, cfg.hidden_std, hidden.data_ptr(),
                                 hscale.data_ptr(), st))
        chk(lib.moe_synth_w13(tab.data_ptr(), cfg.seed, cfg.local_expert_offset, E, cfg.weight_std,
                              w13.data_ptr(), s13.data_ptr(), st))
        chk(lib.moe_synth_w2(tab.data_ptr(), cfg.seed, cfg.local_expert_offset, E, cfg.weight_std,
                             w2.data_ptr(), s2.data_ptr(), st))
    return _kwargs(cfg, logits, bias, hidden.view(torch.float8_e4m3fn), hscale,
                   w13.view(torch.float8_e4m3fn), s13, w2.view(torch.float8_e4m3fn), s2)


def make_weights(cfg: MoEConfig, experts, device: str | torch.device = "cuda") -> dict:
    """W13 / W2 (e4m3) and their scales of the listed global experts, stacked in that order (for
    a rank of an expert-parallel layer with an arbitrary placement); expert g is the same as in
    any slice make_inputs generates."""
    device = torch.device(device)
    experts = [int(g) for g in experts]
    E = len(experts)
    lib = _native.cuda_lib()
    with torch.cuda.device(device):
        tab = _table_on(str(device))
        st = torch.cuda.current_stream(device).cuda_stream
        w13 = torch.empty((E, 2 * I_DIM, H), dtype=torch.uint8, device=device)
        s13 = torch.empty((E, 2 * I_DIM // BLOCK, H // BLOCK), dtype=torch.float32, device=device)
        w2 = torch.empty((E, H, I_DIM), dtype=torch.uint8, device=device)
        s2 = torch.empty((E, H // BLOCK, I_DIM // BLOCK), dtype=torch.float32, device=device)
        for i, g in enumerate(experts):
            _native.check(lib.moe_synth_w13(tab.data_ptr(), cfg.seed, g, 1, cfg.weight_std, w13[i].data_ptr(),
                                            s13[i].data_ptr(), st))
            _native.check(lib.moe_synth_w2(tab.data_ptr(), cfg.seed, g, 1, cfg.weight_std, w2[i].data_ptr(),
                                           s2[i].data_ptr(), st))
    return dict(gemm1_weights=w13.view(torch.float8_e4m3fn), gemm1_weights_scale=s13,
                gemm2_weights=w2.view(torch.float8_e4m3fn), gemm2_weights_scale=s2)
