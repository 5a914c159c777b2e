"""CPU oracle for the DeepSeek-V3/R1 FP8 MoE forward - TEST INFRASTRUCTURE ONLY.

A numpy restatement of the reference PyTorch oracle ``reference/moe_ref.py:run`` used as the
checker for the CUDA path. Only ``tests/``, ``__graft_entry__.smoke()`` and the CPU-baseline
leg of ``bench.py`` may import it; the product path never calls it.

Pinning: ``tests/golden/`` holds outputs and routing indices produced by running the real
``reference/moe_ref.py`` in the build container (script: ``tests/golden/make_golden.py``);
``tests/test_oracle_golden.py`` checks this restatement against them.

Two deliberate, documented definitions where the reference leaves bits unspecified:
  * sigmoid is rounded once: fp32(1 / (1 + exp(-x)) evaluated in float64). torch's fp32
    sigmoid rounds several times and differs by 1 ulp on ~30% of inputs, so expert indices
    can differ from the reference's only where two candidates lie within an ulp;
  * exact ties in the group and expert top-k go to the lower index, the convention of the
    reference CUDA kernel (kernels/moe.cu:146-158, 261-305); torch.topk's tie order is
    unspecified (on CPU it currently prefers higher indices).
The routing weight sum runs in ascending expert order (moe_ref.py:105 sums a dense row).
"""
from __future__ import annotations

import os
from concurrent.futures import ThreadPoolExecutor

import numpy as np

H = 7168
I = 2048
E_GLOBAL = 256
N_GROUP = 8
GROUP_SIZE = 32
TOP_K = 8
TOPK_GROUP = 4
BLOCK = 128


def _threads() -> int:
    return max(1, min(16, os.cpu_count() or 1))


# ---------------------------------------------------------------------------- number formats
def _e4m3_table() -> np.ndarray:
    """Values of the 256 e4m3fn codes (OCP FP8: bias 7, no inf, 0x7F/0xFF = NaN)."""
    vals = np.empty(256, np.float32)
    for code in range(256):
        s = -1.0 if code & 0x80 else 1.0
        e = (code >> 3) & 0xF
        m = code & 0x7
        if e == 0xF and m == 0x7:
            vals[code] = np.nan
        elif e == 0:
            vals[code] = s * m * 2.0 ** -9
        else:
            vals[code] = s * (1.0 + m / 8.0) * 2.0 ** (e - 7)
    return vals


E4M3 = _e4m3_table()


def decode_e4m3(u8: np.ndarray) -> np.ndarray:
    return E4M3[np.asarray(u8, dtype=np.uint8)]


def bf16_bits_to_f32(bits: np.ndarray) -> np.ndarray:
    return (np.asarray(bits, np.uint16).astype(np.uint32) << 16).view(np.float32)


def f32_to_bf16_bits(x: np.ndarray) -> np.ndarray:
    """Round-to-nearest-even fp32 -> bf16 (finite inputs), as torch's .to(torch.bfloat16)."""
    b = np.ascontiguousarray(x, np.float32).view(np.uint32).astype(np.uint64)
    b = (b + 0x7FFF + ((b >> 16) & 1)) >> 16
    return b.astype(np.uint16)


def sigmoid_rn(x: np.ndarray) -> np.ndarray:
    x64 = np.asarray(x, np.float32).astype(np.float64)
    return (1.0 / (1.0 + np.exp(-x64))).astype(np.float32)


# ---------------------------------------------------------------------------- routing
def route(logits: np.ndarray, bias: np.ndarray, rsf: float):
    """No-aux-loss grouped routing, reference/moe_ref.py:82-107.

    Returns (topk_idx int32 [T, 8] in selection order - descending biased score, ties to the
    lower index - and topk_w float32 [T, 8] aligned with it).
    """
    logits = np.asarray(logits, np.float32)
    bias = np.asarray(bias, np.float32).reshape(-1)
    T = logits.shape[0]
    s = sigmoid_rn(logits)                                   # moe_ref.py:85
    sb = (s + bias[None, :]).astype(np.float32)              # moe_ref.py:86
    grouped = sb.reshape(T, N_GROUP, GROUP_SIZE)             # moe_ref.py:89
    top2 = np.sort(grouped, axis=2)[:, :, -2:]               # moe_ref.py:91
    gscore = (top2[:, :, 1] + top2[:, :, 0]).astype(np.float32)  # moe_ref.py:92
    gorder = np.argsort(-gscore, axis=1, kind="stable")      # moe_ref.py:94 (ties -> lower)
    keep = np.zeros((T, N_GROUP), bool)
    np.put_along_axis(keep, gorder[:, :TOPK_GROUP], True, axis=1)
    mask = np.repeat(keep, GROUP_SIZE, axis=1)               # moe_ref.py:95-97
    pruned = np.where(mask, sb, -np.inf).astype(np.float32)  # moe_ref.py:99-100
    topk_idx = np.argsort(-pruned, axis=1, kind="stable")[:, :TOP_K].astype(np.int32)  # :101
    s_sel = np.take_along_axis(s, topk_idx, axis=1)
    asc = np.argsort(topk_idx, axis=1)
    wsum = np.zeros(T, np.float32)
    for k in range(TOP_K):                                   # moe_ref.py:105, ascending experts
        wsum = (wsum + np.take_along_axis(s_sel, asc[:, k:k + 1], axis=1)[:, 0]).astype(np.float32)
    wsum = (wsum + np.float32(1e-20)).astype(np.float32)
    w = ((s_sel / wsum[:, None]).astype(np.float32) * np.float32(rsf)).astype(np.float32)  # :106
    return topk_idx, w


# ---------------------------------------------------------------------------- quantiser
def encode_e4m3(y: np.ndarray) -> np.ndarray:
    """fp32 -> e4m3fn codes, round to nearest even, saturating to +-448 (NaN not produced)."""
    y = np.asarray(y, np.float32)
    pos = _e4m3_table()[:127].astype(np.float64)           # codes 0x00..0x7E, increasing
    a = np.minimum(np.abs(y).astype(np.float64), 448.0)
    i = np.clip(np.searchsorted(pos, a, side="right") - 1, 0, 126)
    j = np.minimum(i + 1, 126)
    lo, hi = pos[i], pos[j]
    up = (a - lo > hi - a) | ((a - lo == hi - a) & (i % 2 == 1))
    code = np.where(up & (j != i), j, i).astype(np.uint8)
    return np.where(np.signbit(y), code | np.uint8(0x80), code).astype(np.uint8)


def quantize_hidden(x: np.ndarray):
    """bf16-valued fp32 [T, 7168] -> (e4m3 codes [T, 7168], fp32 scales [56, T]) with the
    benchmark configurations' convention: per (token, 128-column block) scale = amax / 448
    (1 for an all-zero block), code = e4m3(x / scale). Restates the quantisation the configs
    apply to hidden states before reference/moe_ref.py:run (test infrastructure)."""
    x = np.asarray(x, np.float32)
    T = x.shape[0]
    blk = x.reshape(T, H // BLOCK, BLOCK)
    amax = np.abs(blk).max(axis=2)
    scale = np.where(amax > 0, amax / np.float32(448.0), np.float32(1.0)).astype(np.float32)
    codes = encode_e4m3(blk / scale[:, :, None])
    return codes.reshape(T, H), np.ascontiguousarray(scale.T)


# ---------------------------------------------------------------------------- gate (router) GEMM
def gate_logits(x: np.ndarray, w_gate: np.ndarray):
    """Routing logits of the DeepSeek-V3 gate, logits = x . W_gate^T over the fp32-upcast bf16
    operands (transformers' DeepseekV3TopkRouter.forward, models/deepseek_v3/
    modeling_deepseek_v3.py:150, F.linear in float32). Returns (fp64 logits, fp64 sum_k |x w|):
    the exact dot products (every bf16 product is exact and fp64 holds the sums of 7168 of them
    to about 2^-40 relative), and the scale against which an fp32 accumulation's error is bounded.
    Test infrastructure: the reference receives the logits as an input."""
    x64 = np.asarray(x, np.float64)
    w64 = np.asarray(w_gate, np.float64)
    return x64 @ w64.T, np.abs(x64) @ np.abs(w64).T


def bf16_bits_to_f32(u: np.ndarray) -> np.ndarray:
    """bf16 bit patterns (uint16) -> the fp32 values they represent."""
    return (np.asarray(u, np.uint16).astype(np.uint32) << 16).view(np.float32)


# ---------------------------------------------------------------------------- expert compute
def dequant_hidden(hidden_u8: np.ndarray, hidden_scale: np.ndarray) -> np.ndarray:
    """A = fp8(hidden) * scale[h/128, t] (moe_ref.py:59-67)."""
    T = hidden_u8.shape[0]
    a = decode_e4m3(hidden_u8).reshape(T, H // BLOCK, BLOCK)
    return (a * np.asarray(hidden_scale, np.float32).T[:, :, None]).reshape(T, H).astype(np.float32)


def dequant_block(w_u8: np.ndarray, scale: np.ndarray, out: np.ndarray | None = None) -> np.ndarray:
    """W = fp8(w) * S[r/128, c/128] for one expert matrix (moe_ref.py:69-79), written in place
    into ``out`` when given (no temporaries: the CPU cost of this step is memory traffic)."""
    R, C = w_u8.shape
    if out is None:
        out = np.empty((R, C), np.float32)
    np.take(E4M3, np.asarray(w_u8, np.uint8), out=out)
    o4 = out.reshape(R // BLOCK, BLOCK, C // BLOCK, BLOCK)
    np.multiply(o4, np.asarray(scale, np.float32)[:, None, :, None], out=o4)
    return out


def expert_rows(topk_idx: np.ndarray, ge: int) -> np.ndarray:
    """Tokens that selected global expert ge, ascending (moe_ref.py:118-122)."""
    return np.nonzero((topk_idx == ge).any(axis=1))[0]


def moe_forward(routing_logits, routing_bias, hidden_states, hidden_states_scale, gemm1_weights,
                gemm1_weights_scale, gemm2_weights, gemm2_weights_scale, local_expert_offset,
                routed_scaling_factor, experts=None, return_fp32=False, return_routing=False,
                accumulate=None):
    """bf16 bits [T, 7168] of reference/moe_ref.py:run on numpy inputs.

    ``hidden_states``/``gemm*_weights`` are e4m3 codes (uint8); ``routing_bias`` float32.
    ``experts`` optionally restricts the computation to a subset of local expert indices
    (the output then holds only their contributions - used for bounded CPU timing samples).
    ``accumulate`` (fp32 [T, 7168]) replaces the zero tensor of moe_ref.py:110, so calls over
    consecutive expert slices chain into one layer of more experts with a single final rounding
    (the semantics moe_ref.py would have with all those experts local).
    """
    logits = np.asarray(routing_logits, np.float32)
    T = logits.shape[0]
    E_local = gemm1_weights.shape[0]
    assert logits.shape[1] == E_GLOBAL
    assert hidden_states.shape == (T, H)
    assert hidden_states_scale.shape == (H // BLOCK, T)
    assert gemm1_weights.shape == (E_local, 2 * I, H)
    assert gemm2_weights.shape == (E_local, H, I)
    topk_idx, topk_w = route(logits, routing_bias, routed_scaling_factor)
    A = dequant_hidden(hidden_states, hidden_states_scale)
    out = np.zeros((T, H), np.float32) if accumulate is None else np.array(accumulate, np.float32)  # :110
    work = []
    for le in (range(E_local) if experts is None else experts):
        ge = int(local_expert_offset) + le
        if ge < 0 or ge >= E_GLOBAL:                         # moe_ref.py:115-116
            continue
        tok = expert_rows(topk_idx, ge)
        if tok.size:
            work.append((le, ge, tok))

    # The fp32 dequantisation of moe_ref.py:69-79 is elementwise; numpy runs it on one core,
    # so experts are dequantised on a thread pool (numpy releases the GIL) a batch at a time,
    # into per-worker buffers reused across batches.
    batch = max(1, min(len(work), _threads()))
    bufs = [(np.empty((2 * I, H), np.float32), np.empty((H, I), np.float32)) for _ in range(batch)]

    def deq(slot_le):
        slot, le = slot_le
        return (dequant_block(gemm1_weights[le], gemm1_weights_scale[le], bufs[slot][0]),
                dequant_block(gemm2_weights[le], gemm2_weights_scale[le], bufs[slot][1]))

    with ThreadPoolExecutor(max_workers=batch) as ex:
        for b0 in range(0, len(work), batch):
            chunk = work[b0:b0 + batch]
            weights = list(ex.map(deq, [(i, le) for i, (le, _, _) in enumerate(chunk)]))
            for (le, ge, tok), (W13, W2) in zip(chunk, weights):
                G1 = A[tok] @ W13.T                          # moe_ref.py:128
                X1, X2 = G1[:, :I], G1[:, I:]                # moe_ref.py:129
                C = ((X2 / (np.float32(1.0) + np.exp(-X2))) * X1).astype(np.float32)  # :130
                O = C @ W2.T                                 # moe_ref.py:131
                w_tok = topk_w[tok][topk_idx[tok] == ge]     # moe_ref.py:133
                out[tok] += (O * w_tok[:, None]).astype(np.float32)  # moe_ref.py:134
            del weights
    res = out if return_fp32 else f32_to_bf16_bits(out)      # moe_ref.py:136
    if return_routing:
        return res, topk_idx, topk_w
    return res


def shared_expert_forward(hidden_states, hidden_states_scale, gemm1_weights, gemm1_weights_scale,
                          gemm2_weights, gemm2_weights_scale, return_fp32=False):
    """DeepSeek-V3 shared expert: the expert computation of moe_ref.py:126-134 applied to every
    token with weight 1 (one expert, E = 1 arrays). Test infrastructure."""
    A = dequant_hidden(hidden_states, hidden_states_scale)
    W13 = dequant_block(gemm1_weights[0], gemm1_weights_scale[0])
    W2 = dequant_block(gemm2_weights[0], gemm2_weights_scale[0])
    G1 = A @ W13.T
    X1, X2 = G1[:, :I], G1[:, I:]
    C = ((X2 / (np.float32(1.0) + np.exp(-X2))) * X1).astype(np.float32)
    O = (C @ W2.T).astype(np.float32)
    return O if return_fp32 else f32_to_bf16_bits(O)


def to_numpy_inputs(inputs: dict) -> dict:
    """Convert the torch keyword inputs of reference.run to the numpy form used here."""
    import torch

    def u8(t):
        return t.detach().cpu().contiguous().view(torch.uint8).numpy()

    def f32(t):
        return t.detach().cpu().to(torch.float32).contiguous().numpy()

    return dict(
        routing_logits=f32(inputs["routing_logits"]),
        routing_bias=f32(inputs["routing_bias"]),
        hidden_states=u8(inputs["hidden_states"]),
        hidden_states_scale=f32(inputs["hidden_states_scale"]),
        gemm1_weights=u8(inputs["gemm1_weights"]),
        gemm1_weights_scale=f32(inputs["gemm1_weights_scale"]),
        gemm2_weights=u8(inputs["gemm2_weights"]),
        gemm2_weights_scale=f32(inputs["gemm2_weights_scale"]),
        local_expert_offset=int(inputs["local_expert_offset"]),
        routed_scaling_factor=float(inputs["routed_scaling_factor"]),
    )


def check_tolerance(ref_bits: np.ndarray, got_bits: np.ndarray, atol=1e-2, rtol=2e-2) -> dict:
    """The reference test's elementwise check |got - ref| <= atol + rtol * |ref|
    (tests/test_moe.py:21-38), reported at rtol 2e-2 and 5e-2."""
    ref = bf16_bits_to_f32(ref_bits).astype(np.float64)
    got = bf16_bits_to_f32(got_bits).astype(np.float64)
    err = np.abs(ref - got)
    tol = atol + rtol * np.abs(ref)
    return dict(
        max_abs_err=float(err.max()) if err.size else 0.0,
        max_tol_ratio=float((err / tol).max()) if err.size else 0.0,
        bad=int((err > tol).sum()),
        bad_rtol5=int((err > atol + 5e-2 * np.abs(ref)).sum()),
        n=int(err.size),
    )
