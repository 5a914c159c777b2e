"""Seeded synthetic inputs of the benchmark configurations, restated in numpy - TEST INFRASTRUCTURE.

An independent implementation of the generator the package builds into its native libraries
(counter-based splitmix64 bits, a 2^16-interval inverse-normal table, bf16 and e4m3 rounding,
amax/448 block scales), so the CPU baseline and the reference arm of the benchmark can build
their inputs without loading any of the package's compiled code. The recipe, step by step:

  * bits of element ``idx`` of stream (seed, kind, sub):
    ``mix64(base + (idx + 1) * 0x9E3779B97F4A7C15) >> 32`` with
    ``base = mix64(mix64(seed * 0x9E3779B97F4A7C15 + kind) ^ (sub * 0xD1B54A32D192ED03 + 0x632BE59BD9B4E019))``
    and ``mix64`` the splitmix64 finaliser (shifts 30/27/31, multipliers 0xBF58476D1CE4E5B9,
    0x94D049BB133111EB); kinds 1..5 = logits, bias, hidden, W13, W2; ``sub`` = global expert id;
  * normal: ``lo + frac * (hi - lo)`` between table entries ``i = bits >> 16`` and ``i + 1``,
    ``frac = (bits & 0xFFFF) * 2^-16``, each operation rounded to fp32; the table holds the
    fp32 standard-normal quantiles at ``(i + 0.5) / (2^16 + 1)``;
  * value = bf16(std * normal) (round to nearest even), then e4m3 (round to nearest even,
    saturating) of value / scale with scale = amax / 448 per block (1 for an all-zero block):
    per (token, 128 columns) for hidden states, per 128 x 128 block for weights;
  * bias = bf16(0.1 * normal), replaced by +1.5 on the configured hot experts.

Checked against the package's generator byte for byte (``tests/test_synth_cpu.py``).
"""
from __future__ import annotations

import functools
import os
import statistics
from concurrent.futures import ThreadPoolExecutor

import numpy as np

H, I_DIM, E_GLOBAL, BLOCK = 7168, 2048, 256, 128
TABLE_BITS = 16
GOLDEN = 0x9E3779B97F4A7C15
KIND = dict(logits=1, bias=2, hidden=3, w13=4, w2=5)
_M64 = (1 << 64) - 1


def _mix64_int(z: int) -> int:
    z &= _M64
    z = ((z ^ (z >> 30)) * 0xBF58476D1CE4E5B9) & _M64
    z = ((z ^ (z >> 27)) * 0x94D049BB133111EB) & _M64
    return z ^ (z >> 31)


def stream_base(seed: int, kind: int, sub: int) -> int:
    a = _mix64_int((seed * GOLDEN + kind) & _M64)
    b = (sub * 0xD1B54A32D192ED03 + 0x632BE59BD9B4E019) & _M64
    return _mix64_int(a ^ b)


def _mix64(z: np.ndarray) -> np.ndarray:
    z = np.bitwise_xor(z, z >> np.uint64(30))
    z *= np.uint64(0xBF58476D1CE4E5B9)
    z ^= z >> np.uint64(27)
    z *= np.uint64(0x94D049BB133111EB)
    z ^= z >> np.uint64(31)
    return z


@functools.lru_cache(maxsize=None)
def quantile_table() -> np.ndarray:
    n = 1 << TABLE_BITS
    nd = statistics.NormalDist()
    return np.array([nd.inv_cdf((i + 0.5) / (n + 1)) for i in range(n + 1)], dtype=np.float32)


def normals(base: int, start: int, count: int) -> np.ndarray:
    """fp32 standard normals of elements start .. start+count-1 of the stream at ``base``."""
    idx = np.arange(start + 1, start + count + 1, dtype=np.uint64)
    idx *= np.uint64(GOLDEN)
    idx += np.uint64(base)
    u = (_mix64(idx) >> np.uint64(32)).astype(np.uint32)
    tab = quantile_table()
    i = u >> np.uint32(32 - TABLE_BITS)
    frac = (u & np.uint32((1 << (32 - TABLE_BITS)) - 1)).astype(np.float32) * np.float32(2.0 ** -(32 - TABLE_BITS))
    lo = tab[i]
    d = tab[i + 1] - lo
    return lo + frac * d


def bf16_round(x: np.ndarray) -> np.ndarray:
    b = np.ascontiguousarray(x, np.float32).view(np.uint32).copy()
    b += np.uint32(0x7FFF) + ((b >> np.uint32(16)) & np.uint32(1))
    b &= np.uint32(0xFFFF0000)
    return b.view(np.float32)


def e4m3_codes(y: np.ndarray) -> np.ndarray:
    """fp32 -> e4m3fn bytes, round to nearest even, saturating to +-448 (bit arithmetic)."""
    b = np.ascontiguousarray(y, np.float32).view(np.uint32)
    sign = ((b >> np.uint32(24)) & np.uint32(0x80)).astype(np.uint8)
    a = b & np.uint32(0x7FFFFFFF)
    e = (a >> np.uint32(23)).astype(np.int32) - 127
    # normal range: 3 mantissa bits, RNE on the 20 dropped bits
    r = (a & np.uint32(0x7FFFFF)) >> np.uint32(20)
    rem = a & np.uint32(0xFFFFF)
    up = (rem > 0x80000) | ((rem == 0x80000) & ((r & np.uint32(1)) == 1))
    r = r + up.astype(np.uint32)
    e_n = e + (r == 8).astype(np.int32)
    r = np.where(r == 8, np.uint32(0), r)
    code = np.clip(((e_n + 7).astype(np.int64) << 3) | r.astype(np.int64), 0, 0x7E)
    # subnormal range (e < -6): value = m * 2^-9, m in 0..8
    mant = (a & np.uint32(0x7FFFFF)) | np.uint32(0x800000)
    shift = np.clip(14 - e, 1, 31).astype(np.uint32)
    m = mant >> shift
    remd = mant & ((np.uint32(1) << shift) - np.uint32(1))
    half = np.uint32(1) << (shift - np.uint32(1))
    m = m + ((remd > half) | ((remd == half) & ((m & np.uint32(1)) == 1))).astype(np.uint32)
    m = np.where((a == 0) | (14 - e > 31), np.uint32(0), m)
    code = np.where(e < -6, m.astype(np.int64), code)
    code = np.where(a >= 0x43E80000, 0x7E, code)
    return (sign | code.astype(np.uint8)).astype(np.uint8)


def _threads() -> int:
    return max(1, min(16, os.cpu_count() or 1))


def logits(seed: int, T: int) -> np.ndarray:
    base = stream_base(seed, KIND["logits"], 0)
    return normals(base, 0, T * E_GLOBAL).reshape(T, E_GLOBAL)


def bias_bits(seed: int, std: float, hot: tuple, hot_value: float) -> np.ndarray:
    base = stream_base(seed, KIND["bias"], 0)
    v = np.float32(std) * normals(base, 0, E_GLOBAL)
    for h in hot:
        v[h] = np.float32(hot_value)
    b = v.view(np.uint32).astype(np.uint64)
    return ((b + 0x7FFF + ((b >> 16) & 1)) >> 16).astype(np.uint16)


def _quant_rows(v: np.ndarray):
    """v [R, 128] -> codes [R, 128], scales [R] (amax/448 per row; 1 for an all-zero row)."""
    amax = np.abs(v).max(axis=1)
    scale = np.where(amax > 0, amax / np.float32(448.0), np.float32(1.0)).astype(np.float32)
    return e4m3_codes(v / scale[:, None]), scale


def hidden(seed: int, T: int, std: float = 1.0):
    """(e4m3 codes [T, 7168], scales [56, T])."""
    base = stream_base(seed, KIND["hidden"], 0)
    codes = np.empty((T, H), np.uint8)
    scale = np.empty((H // BLOCK, T), np.float32)
    rows = max(1, 65536 // H * 8)

    def job(t0):
        t1 = min(T, t0 + rows)
        v = bf16_round(np.float32(std) * normals(base, t0 * H, (t1 - t0) * H))
        q, s = _quant_rows(v.reshape(-1, BLOCK))
        codes[t0:t1] = q.reshape(t1 - t0, H)
        scale[:, t0:t1] = s.reshape(t1 - t0, H // BLOCK).T
    with ThreadPoolExecutor(_threads()) as ex:
        list(ex.map(job, range(0, T, rows)))
    return codes, scale


def _weight_matrix(base: int, R: int, C: int, std: float, ex):
    codes = np.empty((R, C), np.uint8)
    scale = np.empty((R // BLOCK, C // BLOCK), np.float32)

    def job(br):
        v = bf16_round(np.float32(std) * normals(base, br * BLOCK * C, BLOCK * C)).reshape(BLOCK, C // BLOCK, BLOCK)
        amax = np.abs(v).max(axis=(0, 2))
        s = np.where(amax > 0, amax / np.float32(448.0), np.float32(1.0)).astype(np.float32)
        codes[br * BLOCK:(br + 1) * BLOCK] = e4m3_codes(v / s[None, :, None]).reshape(BLOCK, C)
        scale[br] = s
    list(ex.map(job, range(R // BLOCK)))
    return codes, scale


def weights(seed: int, experts, std: float = 0.02):
    """W13 / W2 codes and scales of the listed global experts, stacked in that order."""
    experts = list(experts)
    E = len(experts)
    w13 = np.empty((E, 2 * I_DIM, H), np.uint8)
    s13 = np.empty((E, 2 * I_DIM // BLOCK, H // BLOCK), np.float32)
    w2 = np.empty((E, H, I_DIM), np.uint8)
    s2 = np.empty((E, H // BLOCK, I_DIM // BLOCK), np.float32)
    with ThreadPoolExecutor(_threads()) as ex:
        for i, g in enumerate(experts):
            w13[i], s13[i] = _weight_matrix(stream_base(seed, KIND["w13"], g), 2 * I_DIM, H, std, ex)
            w2[i], s2[i] = _weight_matrix(stream_base(seed, KIND["w2"], g), H, I_DIM, std, ex)
    return w13, s13, w2, s2


def make_inputs(T: int, E_local: int = 32, local_expert_offset: int = 0, seed: int = 0,
                routed_scaling_factor: float = 2.5, hidden_std: float = 1.0, weight_std: float = 0.02,
                bias_std: float = 0.1, hot_experts: tuple = (), hot_bias: float = 1.5,
                experts=None, **_ignored) -> dict:
    """numpy inputs of the oracle (``moe_oracle.moe_forward`` keyword form) for a configuration.
    ``experts`` restricts the generated weights to those local indices (the others stay zero),
    which is all a forward over that expert subset reads."""
    lg = logits(seed, T)
    bias = bias_bits(seed, bias_std, tuple(hot_experts), hot_bias)
    hs, hsc = hidden(seed, T, hidden_std)
    sel = list(range(E_local)) if experts is None else list(experts)
    w13 = np.zeros((E_local, 2 * I_DIM, H), np.uint8)
    s13 = np.zeros((E_local, 2 * I_DIM // BLOCK, H // BLOCK), np.float32)
    w2 = np.zeros((E_local, H, I_DIM), np.uint8)
    s2 = np.zeros((E_local, H // BLOCK, I_DIM // BLOCK), np.float32)
    if sel:
        a, b, c, d = weights(seed, [local_expert_offset + e for e in sel], weight_std)
        w13[sel], s13[sel], w2[sel], s2[sel] = a, b, c, d
    return dict(routing_logits=lg,
                routing_bias=(bias.astype(np.uint32) << 16).view(np.float32),
                hidden_states=hs, hidden_states_scale=hsc,
                gemm1_weights=w13, gemm1_weights_scale=s13, gemm2_weights=w2, gemm2_weights_scale=s2,
                local_expert_offset=int(local_expert_offset),
                routed_scaling_factor=float(routed_scaling_factor))
