"""The reference test suite's own input generator, restated for the parity tests.

``build_moe_inputs(T, device, seed)`` of the reference (``moe_layer.py:47-74``) draws, from one
``torch.Generator`` seeded with ``seed`` and in this order: logits ``randn[T, 256]``; hidden
``rand[T, 7168] * 2 - 1`` cast to e4m3; hidden scales ``rand[56, T] * 0.1 + 0.01``; W13
``rand[32, 4096, 7168] * 2 - 1`` cast to e4m3 and its scales ``rand[32, 32, 56] * 0.1 + 0.01``;
W2 ``rand[32, 7168, 2048] * 2 - 1`` cast to e4m3 and its scales ``rand[32, 56, 16] * 0.1 + 0.01``;
the bias is zero, ``local_expert_offset`` 0 and ``routed_scaling_factor`` 1.0. The reference's
test calls it with ``seed = T`` (``tests/test_moe.py:44``).

Generated on the CPU, so the bytes do not depend on the GPU; ``tests/golden/ref_t*.npz`` store
the sha256 digests of the tensors the real reference generator produced, and the tests check
this restatement against them before using its inputs. Test infrastructure only.
"""
from __future__ import annotations

import hashlib

import torch

H, I_DIM, E_GLOBAL, E_LOCAL, BLOCK = 7168, 2048, 256, 32, 128


def build_moe_inputs(T: int, seed: int) -> dict:
    gen = torch.Generator(device="cpu")
    gen.manual_seed(seed)

    def rfp8(*shape):
        return (torch.rand(*shape, generator=gen) * 2 - 1).to(torch.float8_e4m3fn)

    def rscale(*shape):
        return torch.rand(*shape, generator=gen) * 0.1 + 0.01

    logits = torch.randn(T, E_GLOBAL, generator=gen)
    hidden = rfp8(T, H)
    hidden_scale = rscale(H // BLOCK, T)
    w13 = rfp8(E_LOCAL, 2 * I_DIM, H)
    w13_scale = rscale(E_LOCAL, 2 * I_DIM // BLOCK, H // BLOCK)
    w2 = rfp8(E_LOCAL, H, I_DIM)
    w2_scale = rscale(E_LOCAL, H // BLOCK, I_DIM // BLOCK)
    return dict(
        routing_logits=logits,
        routing_bias=torch.zeros(E_GLOBAL),
        hidden_states=hidden,
        hidden_states_scale=hidden_scale,
        gemm1_weights=w13,
        gemm1_weights_scale=w13_scale,
        gemm2_weights=w2,
        gemm2_weights_scale=w2_scale,
        local_expert_offset=0,
        routed_scaling_factor=1.0,
    )


def digests(inputs: dict) -> dict:
    """sha256 of every tensor's bytes (the form tests/golden/ stores)."""
    out = {}
    for k, v in inputs.items():
        if isinstance(v, torch.Tensor):
            out[k] = hashlib.sha256(v.contiguous().view(torch.uint8).numpy().tobytes()).hexdigest()
    return out
