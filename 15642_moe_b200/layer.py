"""Host API of the B200 MoE forward: the drop-in for the reference's Python surface.

Mirrors, with the same names, argument order and error text:
  * the extension functions ``pack_w13``, ``pack_w2``, ``moe_forward``
    (kernels/moe.cu:700-909) - TORCH_CHECK failures become ``RuntimeError`` here too;
  * ``run_custom(ops, **inputs)`` and the packed-weight cache of moe_layer.py:77-120;
  * ``run(**inputs)``, a replacement for ``reference.run`` (reference/moe_ref.py:5-16).

Every call goes to ``libmoe_b200.so`` on the tensors' CUDA device and the current stream.
There is no CPU path: CPU tensors are rejected.
"""
from __future__ import annotations

import weakref

import torch

from . import _native

H, I_DIM, E_GLOBAL, BLOCK = 7168, 2048, 256, 128
H_BLOCKS, I_BLOCKS, G1_BLOCKS = H // BLOCK, I_DIM // BLOCK, 2 * I_DIM // BLOCK
W13_PACKED_SHAPE = (16, 56, 256, 128)   # per expert: [j, kb, rows, bytes]
W2_PACKED_SHAPE = (28, 16, 256, 128)    # per expert: [nt, ib, rows, bytes]


def _check(cond: bool, msg: str) -> None:
    if not cond:
        raise RuntimeError(msg)


def _cuda(t: torch.Tensor, name: str) -> None:
    _check(t.is_cuda, f"{name} must be a CUDA tensor")


def _stream(device: torch.device) -> int:
    return torch.cuda.current_stream(device).cuda_stream


def pack_w13(W13: torch.Tensor) -> torch.Tensor:
    """FP8 W13 [E, 4096, 7168] -> packed uint8 [E, 16, 56, 256, 128] (kernels/moe.cu:700-720)."""
    _check(W13.dim() == 3, "W13 must be [E_local, 4096, 7168]")
    _check(W13.element_size() == 1, "W13 must be an FP8 tensor")
    _check(W13.is_contiguous(), "W13 must be contiguous")
    _check(W13.size(1) == 2 * I_DIM and W13.size(2) == H, "W13 must be [E_local, 4096, 7168]")
    _cuda(W13, "W13")
    E = int(W13.size(0))
    lib = _native.cuda_lib()
    out = torch.empty((E, *W13_PACKED_SHAPE), dtype=torch.uint8, device=W13.device)
    with torch.cuda.device(W13.device):
        _native.check(lib.moe_pack_w13(W13.data_ptr(), E, out.data_ptr(), _stream(W13.device)))
    return out


def pack_w2(W2: torch.Tensor) -> torch.Tensor:
    """FP8 W2 [E, 7168, 2048] -> packed uint8 [E, 28, 16, 256, 128] (kernels/moe.cu:722-742)."""
    _check(W2.dim() == 3, "W2 must be [E_local, 7168, 2048]")
    _check(W2.element_size() == 1, "W2 must be an FP8 tensor")
    _check(W2.is_contiguous(), "W2 must be contiguous")
    _check(W2.size(1) == H and W2.size(2) == I_DIM, "W2 must be [E_local, 7168, 2048]")
    _cuda(W2, "W2")
    E = int(W2.size(0))
    lib = _native.cuda_lib()
    out = torch.empty((E, *W2_PACKED_SHAPE), dtype=torch.uint8, device=W2.device)
    with torch.cuda.device(W2.device):
        _native.check(lib.moe_pack_w2(W2.data_ptr(), E, out.data_ptr(), _stream(W2.device)))
    return out


def workspace_bytes(T: int, E_local: int) -> int:
    return int(_native.cuda_lib().moe_forward_workspace_bytes(T, E_local))


def moe_forward(hidden, hidden_scale, W13_packed, W13_scale, W2_packed, W2_scale, logits, bias,
                rsf: float, local_offset: int, out: torch.Tensor | None = None,
                workspace: torch.Tensor | None = None, *, fp32_out: bool = False) -> torch.Tensor:
    """bf16 [T, 7168] MoE output; argument order of kernels/moe.cu:744-754.

    ``out`` and ``workspace`` may be passed to reuse buffers (e.g. inside a CUDA graph);
    otherwise they come from the PyTorch caching allocator like the reference's scratch.
    ``fp32_out=True`` returns the fp32 sum before the final bf16 rounding (moe_forward_f32).
    """
    # Shape / dtype / contiguity checks with the reference's messages (kernels/moe.cu:759-817).
    _check(hidden.dim() == 2, "hidden must be [T, 7168]")
    _check(hidden_scale.dim() == 2, "hidden_scale must be [56, T]")
    _check(W13_packed.dim() == 5, "W13_packed must be [E_local, 16, 56, 256, 128]")
    _check(W13_scale.dim() == 3, "W13_scale must be [E_local, 32, 56]")
    _check(W2_packed.dim() == 5, "W2_packed must be [E_local, 28, 16, 256, 128]")
    _check(W2_scale.dim() == 3, "W2_scale must be [E_local, 56, 16]")
    _check(logits.dim() == 2, "logits must be [T, 256]")
    _check(hidden.element_size() == 1, "hidden must be an FP8 tensor")
    _check(hidden_scale.dtype == torch.float32, "hidden_scale must be float32")
    _check(W13_packed.dtype == torch.uint8, "W13_packed must be packed FP8 bytes from pack_w13")
    _check(W13_scale.dtype == torch.float32, "W13_scale must be float32")
    _check(W2_packed.dtype == torch.uint8, "W2_packed must be packed FP8 bytes from pack_w2")
    _check(W2_scale.dtype == torch.float32, "W2_scale must be float32")
    _check(logits.dtype == torch.float32, "logits must be float32")
    _check(bias.dtype == torch.float32, "bias must be float32")
    T, E_local = int(hidden.size(0)), int(W13_packed.size(0))
    _check(int(hidden.size(1)) == H, "hidden must have hidden dim 7168")
    _check(tuple(hidden_scale.shape) == (H_BLOCKS, T), "hidden_scale must be [56, T]")
    _check(tuple(logits.shape) == (T, E_GLOBAL), "logits must be [T, 256]")
    _check(bias.numel() == E_GLOBAL, "bias must have 256 elements")
    _check(tuple(W13_packed.shape[1:]) == W13_PACKED_SHAPE, "W13_packed must be [E_local, 16, 56, 256, 128]")
    _check(tuple(W13_scale.shape) == (E_local, G1_BLOCKS, H_BLOCKS), "W13_scale must be [E_local, 32, 56]")
    _check(int(W2_packed.size(0)) == E_local and tuple(W2_packed.shape[1:]) == W2_PACKED_SHAPE,
           "W2_packed must be [E_local, 28, 16, 256, 128]")
    _check(tuple(W2_scale.shape) == (E_local, H_BLOCKS, I_BLOCKS), "W2_scale must be [E_local, 56, 16]")
    for t, n in ((hidden, "hidden"), (hidden_scale, "hidden_scale"), (W13_packed, "W13_packed"),
                 (W13_scale, "W13_scale"), (W2_packed, "W2_packed"), (W2_scale, "W2_scale"),
                 (logits, "logits"), (bias, "bias")):
        _check(t.is_contiguous(), f"{n} must be contiguous")
        _cuda(t, n)
    dev = hidden.device
    _check(all(t.device == dev for t in (hidden_scale, W13_packed, W13_scale, W2_packed, W2_scale,
                                          logits, bias)), "all tensors must be on one device")
    lib = _native.cuda_lib()
    out_dtype = torch.float32 if fp32_out else torch.bfloat16
    if out is None:
        out = torch.empty((T, H), dtype=out_dtype, device=dev)
    _check(out.dtype == out_dtype and tuple(out.shape) == (T, H) and out.is_contiguous(),
           f"out must be a contiguous {'fp32' if fp32_out else 'bf16'} [T, 7168] tensor")
    nbytes = int(lib.moe_forward_workspace_bytes(T, E_local)) if T > 0 else 0
    if workspace is None:
        workspace = torch.empty((max(nbytes, 1),), dtype=torch.uint8, device=dev)
    _check(workspace.numel() >= nbytes, f"workspace must hold {nbytes} bytes")
    if T == 0:
        return out
    fn = lib.moe_forward_f32 if fp32_out else lib.moe_forward
    with torch.cuda.device(dev):
        _native.check(fn(
            hidden.data_ptr(), hidden_scale.data_ptr(), W13_packed.data_ptr(), W13_scale.data_ptr(),
            W2_packed.data_ptr(), W2_scale.data_ptr(), logits.data_ptr(), bias.data_ptr(),
            float(rsf), int(local_offset), T, E_local, out.data_ptr(), workspace.data_ptr(),
            workspace.numel(), _stream(dev)))
    return out


def shared_expert_forward(hidden, hidden_scale, W13_packed, W13_scale, W2_packed, W2_scale,
                          fp32_out: bool = False, out: torch.Tensor | None = None,
                          workspace: torch.Tensor | None = None) -> torch.Tensor:
    """DeepSeek-V3 shared expert: every token through one FP8 block-scaled expert (packed with
    pack_w13 / pack_w2, E = 1) with weight 1. bf16 [T, 7168], or fp32 with ``fp32_out`` (add it
    to ``moe_forward(..., fp32_out=True)`` and round once for the full layer output)."""
    _check(hidden.dim() == 2 and int(hidden.size(1)) == H and hidden.element_size() == 1,
           "hidden must be FP8 [T, 7168]")
    T, dev = int(hidden.size(0)), hidden.device
    _check(tuple(hidden_scale.shape) == (H_BLOCKS, T) and hidden_scale.dtype == torch.float32,
           "hidden_scale must be float32 [56, T]")
    _check(tuple(W13_packed.shape) == (1, *W13_PACKED_SHAPE) and W13_packed.dtype == torch.uint8,
           "W13_packed must be [1, 16, 56, 256, 128] from pack_w13")
    _check(tuple(W2_packed.shape) == (1, *W2_PACKED_SHAPE) and W2_packed.dtype == torch.uint8,
           "W2_packed must be [1, 28, 16, 256, 128] from pack_w2")
    _check(tuple(W13_scale.shape) == (1, G1_BLOCKS, H_BLOCKS) and W13_scale.dtype == torch.float32,
           "W13_scale must be float32 [1, 32, 56]")
    _check(tuple(W2_scale.shape) == (1, H_BLOCKS, I_BLOCKS) and W2_scale.dtype == torch.float32,
           "W2_scale must be float32 [1, 56, 16]")
    for t, n in ((hidden, "hidden"), (hidden_scale, "hidden_scale"), (W13_packed, "W13_packed"),
                 (W13_scale, "W13_scale"), (W2_packed, "W2_packed"), (W2_scale, "W2_scale")):
        _check(t.is_contiguous(), f"{n} must be contiguous")
        _cuda(t, n)
    lib = _native.cuda_lib()
    out_dtype = torch.float32 if fp32_out else torch.bfloat16
    if out is None:
        out = torch.empty((T, H), dtype=out_dtype, device=dev)
    _check(out.dtype == out_dtype and tuple(out.shape) == (T, H) and out.is_contiguous(), "bad out tensor")
    nbytes = int(lib.moe_forward_workspace_bytes(T, 1)) if T > 0 else 0
    if workspace is None:
        workspace = torch.empty((max(nbytes, 1),), dtype=torch.uint8, device=dev)
    _check(workspace.numel() >= nbytes, f"workspace must hold {nbytes} bytes")
    if T == 0:
        return out
    with torch.cuda.device(dev):
        _native.check(lib.moe_shared_expert_forward(
            hidden.data_ptr(), hidden_scale.data_ptr(), W13_packed.data_ptr(), W13_scale.data_ptr(),
            W2_packed.data_ptr(), W2_scale.data_ptr(), T, out.data_ptr(), 1 if fp32_out else 0,
            workspace.data_ptr(), workspace.numel(), _stream(dev)))
    return out


def quantize_hidden(hidden: torch.Tensor, out: torch.Tensor | None = None,
                    scale: torch.Tensor | None = None):
    """bf16 hidden [T, 7168] -> (e4m3 codes [T, 7168], fp32 scales [56, T]): per (token,
    128-column block) scale = amax / 448, code = e4m3(x / scale) (the configurations'
    quantisation), ready for moe_forward / run."""
    _check(hidden.dim() == 2 and int(hidden.size(1)) == H, "hidden must be [T, 7168]")
    _check(hidden.dtype == torch.bfloat16, "hidden must be bfloat16")
    _check(hidden.is_contiguous(), "hidden must be contiguous")
    _cuda(hidden, "hidden")
    T, dev = int(hidden.size(0)), hidden.device
    if out is None:
        out = torch.empty((T, H), dtype=torch.float8_e4m3fn, device=dev)
    if scale is None:
        scale = torch.empty((H_BLOCKS, T), dtype=torch.float32, device=dev)
    _check(out.element_size() == 1 and tuple(out.shape) == (T, H) and out.is_contiguous(),
           "out must be a contiguous FP8 [T, 7168] tensor")
    _check(scale.dtype == torch.float32 and tuple(scale.shape) == (H_BLOCKS, T) and scale.is_contiguous(),
           "scale must be a contiguous float32 [56, T] tensor")
    with torch.cuda.device(dev):
        _native.check(_native.cuda_lib().moe_quantize_hidden(hidden.data_ptr(), T, out.data_ptr(),
                                                             scale.data_ptr(), _stream(dev)))
    return out, scale


GATE_PACKED_SHAPE = (H_BLOCKS, 2, E_GLOBAL, 128)   # per 128-column block: two swizzled halves


def pack_gate(w_gate: torch.Tensor) -> torch.Tensor:
    """W_gate bf16 [256, 7168] (the DeepSeek-V3 router weight) -> packed uint8 images for
    gate_quantize, once per weight set."""
    _check(w_gate.dim() == 2 and tuple(w_gate.shape) == (E_GLOBAL, H), "W_gate must be [256, 7168]")
    _check(w_gate.dtype == torch.bfloat16, "W_gate must be bfloat16")
    _check(w_gate.is_contiguous(), "W_gate must be contiguous")
    _cuda(w_gate, "W_gate")
    lib = _native.cuda_lib()
    out = torch.empty(int(lib.moe_gate_packed_bytes()), dtype=torch.uint8, device=w_gate.device)
    with torch.cuda.device(w_gate.device):
        _native.check(lib.moe_pack_gate(w_gate.data_ptr(), out.data_ptr(), _stream(w_gate.device)))
    return out.view(GATE_PACKED_SHAPE)


def gate_quantize(hidden: torch.Tensor, gate_packed: torch.Tensor, logits: torch.Tensor | None = None,
                  out: torch.Tensor | None = None, scale: torch.Tensor | None = None):
    """MoE prologue in one pass over bf16 hidden [T, 7168]: (routing logits fp32 [T, 256] =
    hidden . W_gate^T, e4m3 codes [T, 7168], fp32 scales [56, T]). The codes and scales equal
    quantize_hidden's; the three outputs are moe_forward's routing_logits, hidden_states and
    hidden_states_scale."""
    _check(hidden.dim() == 2 and int(hidden.size(1)) == H, "hidden must be [T, 7168]")
    _check(hidden.dtype == torch.bfloat16, "hidden must be bfloat16")
    _check(hidden.is_contiguous(), "hidden must be contiguous")
    _cuda(hidden, "hidden")
    _check(gate_packed.dtype == torch.uint8 and tuple(gate_packed.shape) == GATE_PACKED_SHAPE
           and gate_packed.is_contiguous(), "gate_packed must come from pack_gate")
    _check(gate_packed.device == hidden.device, "gate_packed must be on the device of hidden")
    T, dev = int(hidden.size(0)), hidden.device
    if logits is None:
        logits = torch.empty((T, E_GLOBAL), dtype=torch.float32, device=dev)
    if out is None:
        out = torch.empty((T, H), dtype=torch.float8_e4m3fn, device=dev)
    if scale is None:
        scale = torch.empty((H_BLOCKS, T), dtype=torch.float32, device=dev)
    _check(logits.dtype == torch.float32 and tuple(logits.shape) == (T, E_GLOBAL) and logits.is_contiguous(),
           "logits must be a contiguous float32 [T, 256] tensor")
    _check(out.element_size() == 1 and tuple(out.shape) == (T, H) and out.is_contiguous(),
           "out must be a contiguous FP8 [T, 7168] tensor")
    _check(scale.dtype == torch.float32 and tuple(scale.shape) == (H_BLOCKS, T) and scale.is_contiguous(),
           "scale must be a contiguous float32 [56, T] tensor")
    with torch.cuda.device(dev):
        _native.check(_native.cuda_lib().moe_gate_quantize(hidden.data_ptr(), gate_packed.data_ptr(), T,
                                                           logits.data_ptr(), out.data_ptr(), scale.data_ptr(),
                                                           _stream(dev)))
    return logits, out, scale


def route(logits: torch.Tensor, bias: torch.Tensor, rsf: float):
    """(topk_idx int32 [T, 8], topk_w fp32 [T, 8]) from the device router."""
    _check(logits.dim() == 2 and logits.size(1) == E_GLOBAL and logits.dtype == torch.float32,
           "logits must be float32 [T, 256]")
    _cuda(logits, "logits")
    logits = logits.contiguous()
    bias = bias.to(torch.float32).reshape(-1).contiguous()
    T = int(logits.size(0))
    idx = torch.empty((T, 8), dtype=torch.int32, device=logits.device)
    w = torch.empty((T, 8), dtype=torch.float32, device=logits.device)
    with torch.cuda.device(logits.device):
        _native.check(_native.cuda_lib().moe_route(logits.data_ptr(), bias.data_ptr(), float(rsf), T,
                                                   idx.data_ptr(), w.data_ptr(), _stream(logits.device)))
    return idx, w


class _Ops:
    """Stand-in for the reference's loaded extension module (``ops`` in moe_layer.py)."""
    pack_w13 = staticmethod(pack_w13)
    pack_w2 = staticmethod(pack_w2)
    moe_forward = staticmethod(moe_forward)


ops = _Ops()
_packed_weight_cache: dict = {}


def _load_custom_ops():
    """Counterpart of moe_layer.py:31-43; the library is prebuilt, not JIT-compiled."""
    _native.cuda_lib()
    return ops


def _cached_pack(cache_name, tensor, pack_fn):
    """Packed-weight cache keyed like moe_layer.py:77-95, with a weakref owner check."""
    tensor = tensor.contiguous()
    key = (cache_name, int(tensor.data_ptr()), tuple(tensor.shape), str(tensor.dtype),
           str(tensor.device), int(tensor._version))
    entry = _packed_weight_cache.get(key)
    if entry is not None:
        owner_ref, packed = entry
        if owner_ref() is tensor:
            return packed
    packed = pack_fn(tensor)
    _packed_weight_cache[key] = (weakref.ref(tensor), packed)
    return packed


@torch.no_grad()
def run_custom(ops, routing_logits, routing_bias, hidden_states, hidden_states_scale,
               gemm1_weights, gemm1_weights_scale, gemm2_weights, gemm2_weights_scale,
               local_expert_offset, routed_scaling_factor):
    """moe_layer.py:99-120: pack (cached), cast scales/logits/bias to fp32, call moe_forward."""
    w13p = _cached_pack("w13", gemm1_weights, ops.pack_w13)
    w2p = _cached_pack("w2", gemm2_weights, ops.pack_w2)
    return ops.moe_forward(
        hidden_states.contiguous(),
        hidden_states_scale.to(torch.float32).contiguous(),
        w13p,
        gemm1_weights_scale.to(torch.float32).contiguous(),
        w2p,
        gemm2_weights_scale.to(torch.float32).contiguous(),
        routing_logits.to(torch.float32).contiguous(),
        routing_bias.to(torch.float32).reshape(-1).contiguous(),
        float(routed_scaling_factor),
        int(local_expert_offset),
    )


@torch.no_grad()
def run(routing_logits, routing_bias, hidden_states, hidden_states_scale, gemm1_weights,
        gemm1_weights_scale, gemm2_weights, gemm2_weights_scale, local_expert_offset: int,
        routed_scaling_factor: float) -> torch.Tensor:
    """Drop-in for ``reference.run`` (reference/moe_ref.py:5-16) on CUDA tensors."""
    # Same geometry assertions as the oracle (moe_ref.py:35-52).
    T = routing_logits.shape[0]
    E_local = gemm1_weights.shape[0]
    assert routing_logits.shape[1] == E_GLOBAL
    assert hidden_states.shape == (T, H)
    assert hidden_states_scale.shape == (H_BLOCKS, T)
    assert gemm1_weights.shape == (E_local, 2 * I_DIM, H)
    assert gemm1_weights_scale.shape == (E_local, G1_BLOCKS, H_BLOCKS)
    assert gemm2_weights.shape == (E_local, H, I_DIM)
    assert gemm2_weights_scale.shape == (E_local, H_BLOCKS, I_BLOCKS)
    assert routing_bias.shape[-1] == E_GLOBAL
    return run_custom(ops, routing_logits, routing_bias, hidden_states, hidden_states_scale,
                      gemm1_weights, gemm1_weights_scale, gemm2_weights, gemm2_weights_scale,
                      local_expert_offset, routed_scaling_factor)
