"""moe_forward on the reference test suite's own inputs.

The reference's test (tests/test_moe.py:18,44) runs T in {1, 4, 32, 64, 256, 2048, 4096, 8192,
16384} with inputs from its build_moe_inputs(T, seed=T) (moe_layer.py:47-74: uniform e4m3
values, U(0.01, 0.11) scales, zero bias, routed_scaling_factor 1). tests/ref_inputs.py restates
that generator on the CPU; tests/golden/ref_t*.npz hold, for T <= 256, the digests of the real
generator's tensors and the real reference.run output (tests/golden/make_golden.py).

* T <= 256: the restated inputs must match the stored digests byte for byte, the selected
  experts must equal the reference's, and the output must meet the reference tolerance
  (|got - ref| <= 1e-2 + 2e-2 |ref|). On these inputs the outputs are small (|out| < ~0.02),
  so the test also bounds the error by 1% of the largest output magnitude.
* T >= 2048: sampled rows against the CPU oracle (the oracle is pinned to the reference by the
  goldens), same two bounds.
"""
import json
import os

import numpy as np
import pytest
import torch

from gpu_helpers import out_bits
from ref_inputs import build_moe_inputs, digests
from test_gpu_parity_large import rows_of

pytestmark = pytest.mark.gpu
GOLDEN = os.path.join(os.path.dirname(__file__), "golden")
ATOL, RTOL = 1e-2, 2e-2
SCALED = 1e-2        # max |err| <= SCALED * max |ref|


@pytest.fixture(autouse=True)
def _status_clean(pkg):
    pkg.device_status(reset=True)
    yield
    assert pkg.device_status(reset=True) == 0, "a kernel reported a timeout or bad metadata"


def _cuda(inp):
    return {k: (v.cuda() if isinstance(v, torch.Tensor) else v) for k, v in inp.items()}


def _check(oracle, ref_bits, got_bits):
    r = oracle.check_tolerance(ref_bits, got_bits, ATOL, RTOL)
    ref = oracle.bf16_bits_to_f32(ref_bits).astype(np.float64)
    got = oracle.bf16_bits_to_f32(got_bits).astype(np.float64)
    r["max_abs_ref"] = float(np.abs(ref).max()) if ref.size else 0.0
    r["scaled_err"] = r["max_abs_err"] / r["max_abs_ref"] if r["max_abs_ref"] > 0 else 0.0
    return r


@pytest.mark.parametrize("T", [1, 4, 32, 64, 256])
def test_reference_golden(pkg, oracle, T):
    g = np.load(os.path.join(GOLDEN, f"ref_t{T}.npz"))
    inp = build_moe_inputs(T, T)
    assert digests(inp) == json.loads(str(g["inputs_sha256"])), "generator restatement drifted"
    dinp = _cuda(inp)
    idx, _ = pkg.route(dinp["routing_logits"], dinp["routing_bias"], 1.0)
    np.testing.assert_array_equal(np.sort(idx.cpu().numpy(), axis=1), g["topk_sorted"].astype(np.int64))
    got = out_bits(pkg.run(**dinp))
    r = _check(oracle, g["out_bf16"], got)
    print(f"T={T}", r)
    assert r["bad"] == 0, r
    assert r["max_abs_err"] <= SCALED * r["max_abs_ref"], r


@pytest.mark.parametrize("T", [2048, 4096, 8192, 16384])
def test_reference_generator_sampled_rows(pkg, oracle, T):
    inp = build_moe_inputs(T, T)
    got = out_bits(pkg.run(**_cuda(inp)))
    npi = oracle.to_numpy_inputs(inp)
    rng = np.random.default_rng(T)
    rows = np.unique(np.concatenate([[0, T - 1], rng.choice(T, 254, replace=False)]))
    ref = oracle.moe_forward(**rows_of(npi, rows))
    r = _check(oracle, ref, got[rows])
    print(f"T={T} rows={rows.size}", r)
    assert r["bad"] == 0, r
    assert r["max_abs_err"] <= SCALED * r["max_abs_ref"], r
