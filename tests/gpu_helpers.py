"""Shared helpers of the GPU parity tests (run the CUDA path, read its workspace)."""
import numpy as np
import torch

from oracle import moe_oracle as O


def forward_with_workspace(pkg, inp):
    """Run moe_forward through the public API with a caller-owned workspace."""
    w13p = pkg.pack_w13(inp["gemm1_weights"])
    w2p = pkg.pack_w2(inp["gemm2_weights"])
    T, E = inp["hidden_states"].shape[0], inp["gemm1_weights"].shape[0]
    ws = torch.zeros(pkg.workspace_bytes(T, E), dtype=torch.uint8, device="cuda")
    out = pkg.moe_forward(
        inp["hidden_states"], inp["hidden_states_scale"].float().contiguous(), w13p,
        inp["gemm1_weights_scale"].float().contiguous(), w2p,
        inp["gemm2_weights_scale"].float().contiguous(), inp["routing_logits"].float().contiguous(),
        inp["routing_bias"].float().reshape(-1).contiguous(), inp["routed_scaling_factor"],
        inp["local_expert_offset"], workspace=ws)
    torch.cuda.synchronize()
    return out, ws


def region(ws, layout, name, dtype, count=None):
    off = layout[name]
    names = list(layout)
    end = layout[names[names.index(name) + 1]]
    raw = ws[off:end]
    t = raw.view(dtype)
    return (t[:count] if count is not None else t).cpu().numpy()


def unswizzle(tiles: np.ndarray) -> np.ndarray:
    """[..., 128 rows, 128 bytes] K-major 128B-swizzled tiles -> logical byte order."""
    shp = tiles.shape
    ch = tiles.reshape(-1, 128, 8, 16)
    phys = np.arange(8)[None, :] ^ (np.arange(128)[:, None] & 7)          # [128, 8]
    out = np.take_along_axis(ch, phys[None, :, :, None], axis=2)
    return out.reshape(shp)


def out_bits(t: torch.Tensor) -> np.ndarray:
    return t.contiguous().view(torch.int16).cpu().numpy().view(np.uint16)


def oracle_inputs(inp):
    return O.to_numpy_inputs(inp)
