"""CPU checks of the quantisers (csrc/quant.cuh quotient2, used by quantize_hidden_kernel and
gate_quantize_kernel) and of the fused gate kernel (csrc/gate.cuh) that need no GPU: the
division (Markstein's method with two corrections) restated over exact rationals and compared
with the correctly rounded quotient, the scale tables against direct division, the router-GEMM
restatement against torch's fp32 linear, and the C ABI's argument checks."""
import importlib
from fractions import Fraction

import numpy as np
import torch


def rn32(v: Fraction) -> float:
    """Round an exact rational to the nearest fp32 value, ties to even (subnormals included)."""
    if v == 0:
        return 0.0
    a = abs(v)
    e = a.numerator.bit_length() - a.denominator.bit_length()
    if Fraction(2) ** e > a:
        e -= 1
    quantum = Fraction(2) ** (max(e, -126) - 23)
    n = a / quantum
    f = n.numerator // n.denominator
    rem = n - f
    if rem > Fraction(1, 2) or (rem == Fraction(1, 2) and f % 2 == 1):
        f += 1
    r = float(f * quantum)
    return -r if v < 0 else r


def fma32(a: float, b: float, c: float) -> float:
    return rn32(Fraction(a) * Fraction(b) + Fraction(c))


def markstein_quotient(x: float, s: float) -> float:
    """The kernel's x / s: y = RN(1/s), q = RN(x y), then twice q = RN(q + RN(x - s q) y)."""
    y = rn32(1 / Fraction(s))
    q = rn32(Fraction(x) * Fraction(y))
    for _ in range(2):
        q = fma32(fma32(q, -s, x), y, q)
    return q


def test_rn32_matches_numpy_division():
    rng = np.random.default_rng(0)
    a = rng.standard_normal(200).astype(np.float32)
    b = rng.standard_normal(200).astype(np.float32)
    for p, q in zip(a, b):
        assert rn32(Fraction(float(p)) / Fraction(float(q))) == float(np.float32(p) / np.float32(q))


def test_markstein_two_corrections_give_the_correctly_rounded_quotient():
    rng = np.random.default_rng(1)
    bits = rng.integers(0x1780, 0x7F7F, 3000).astype(np.uint32)          # block maxima >= 2^-80
    amax = (bits << 16).view(np.float32)
    scale = amax / np.float32(448.0)
    # block values within 28 binades below the maximum (every value with a nonzero code)
    xb = np.maximum(bits.astype(np.int64) - rng.integers(0, 28 * 128, bits.size), 0x0080).astype(np.uint32)
    x = (xb << 16).view(np.float32)
    for xv, sv in zip(x, scale):
        exact = rn32(Fraction(float(xv)) / Fraction(float(sv)))
        assert markstein_quotient(float(xv), float(sv)) == exact, (float(xv), float(sv))


def test_gate_oracle_against_torch_linear(oracle):
    g = torch.Generator().manual_seed(0)
    x = torch.randn((16, 7168), generator=g).to(torch.bfloat16)
    w = (0.02 * torch.randn((256, 7168), generator=g)).to(torch.bfloat16)
    ref, bound = oracle.gate_logits(x.float().numpy(), w.float().numpy())
    cpu = torch.nn.functional.linear(x.float(), w.float()).numpy()
    assert ref.shape == (16, 256) and (bound > 0).all()
    assert (np.abs(cpu - ref) <= 2.0 ** -14 * bound).all()
    u = np.array([0x3F80, 0xBF80, 0x0000, 0x8000, 0x4049], np.uint16)
    np.testing.assert_array_equal(oracle.bf16_bits_to_f32(u), np.float32([1.0, -1.0, 0.0, -0.0, 3.140625]))


def test_gate_capi_argument_errors(pkg):
    native = importlib.import_module("15642_moe_b200._native")
    lib = native.cuda_lib()
    assert lib.moe_gate_packed_bytes() == 256 * 7168 * 2
    assert lib.moe_gate_quantize(None, None, -1, None, None, None, None) == 1
    assert b"[T, 7168]" in lib.moe_last_error()
    assert lib.moe_gate_quantize(None, None, 0, None, None, None, None) == 0      # T = 0: nothing to do
    assert lib.moe_gate_quantize(None, None, 65537, None, None, None, None) == 1
    assert b"65536" in lib.moe_last_error()
    assert lib.moe_gate_quantize(None, None, 4, None, None, None, None) == 1
    assert b"null" in lib.moe_last_error()
    assert lib.moe_pack_gate(None, None, None) == 1
    assert b"null" in lib.moe_last_error()
    # Misaligned (non-null) pointers are refused on the host, before any device work.
    odd, ok = 0x1008, 0x2000
    assert lib.moe_gate_quantize(odd, ok, 4, ok, ok, ok, None) == 1
    assert b"16-byte aligned" in lib.moe_last_error()
    assert lib.moe_gate_quantize(ok, ok, 4, ok, ok, odd, None) == 1
    assert lib.moe_pack_gate(ok, odd, None) == 1
    assert b"16-byte aligned" in lib.moe_last_error()


def test_scale_tables_equal_direct_division_for_every_fast_exponent():
    """csrc/gate.cuh block_scale: for amax = (1 + f/128) 2^(E-127) with E in [47, 254], the block
    scale RN(amax / 448) and its reciprocal RN(1 / scale) equal the f-th table entries scaled by
    2^(E-127) (exponent-field addition), for all 128 mantissas."""
    f = np.arange(128, dtype=np.uint32)
    tab_s = (np.float32(1.0) + f.astype(np.float32) * np.float32(1 / 128)) / np.float32(448.0)
    tab_y = np.float32(1.0) / tab_s
    for E in range(47, 255):
        amax = ((np.uint32(E) << 23) | (f << 16)).view(np.float32)
        s = amax / np.float32(448.0)
        y = np.float32(1.0) / s
        adj = np.int64(E - 127) << 23
        s_tab = (tab_s.view(np.uint32).astype(np.int64) + adj).astype(np.uint32).view(np.float32)
        y_tab = (tab_y.view(np.uint32).astype(np.int64) - adj).astype(np.uint32).view(np.float32)
        np.testing.assert_array_equal(s_tab.view(np.uint32), s.view(np.uint32))
        np.testing.assert_array_equal(y_tab.view(np.uint32), y.view(np.uint32))
