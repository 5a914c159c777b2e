"""The CPU oracle against golden vectors produced by the real reference (tests/golden/).

These pin oracle/moe_oracle.py before it is trusted as the checker of the CUDA path:
same expert indices as reference/moe_ref.py on every token, and bf16 outputs within the
reference test's tolerance (tests/test_moe.py:21-38; in practice within 1 bf16 ulp).
"""
import hashlib
import json
import os

import numpy as np
import pytest
import torch

GOLDEN = os.path.join(os.path.dirname(__file__), "golden")
FULL = ["cfg0_t16", "cfg1_t64", "t1_seed1", "t1_seed3", "t4_off224"]
ROUTING = ["route_cfg2_t4096", "route_cfg4_t16384_skew"]


def load(name):
    g = np.load(os.path.join(GOLDEN, name + ".npz"))
    return g, json.loads(str(g["config"]))


def digests(inputs):
    return {k: hashlib.sha256(v.contiguous().view(torch.uint8).numpy().tobytes()).hexdigest()
            for k, v in inputs.items() if isinstance(v, torch.Tensor)}


@pytest.fixture(scope="module")
def cpu_inputs(pkg):
    cache = {}

    def get(name):
        if name not in cache:
            g, cfg = load(name)
            cache[name] = pkg.make_inputs(pkg.MoEConfig(**cfg), "cpu")
        return cache[name]
    return get


@pytest.mark.parametrize("name", FULL)
def test_generator_reproduces_golden_inputs(name, cpu_inputs):
    g, _ = load(name)
    assert digests(cpu_inputs(name)) == json.loads(str(g["inputs_sha256"]))


@pytest.mark.parametrize("name", FULL)
def test_oracle_matches_reference_golden(name, cpu_inputs, oracle):
    g, _ = load(name)
    out, idx, _ = oracle.moe_forward(**oracle.to_numpy_inputs(cpu_inputs(name)), return_routing=True)
    np.testing.assert_array_equal(np.sort(idx, axis=1), g["topk_sorted"])
    r = oracle.check_tolerance(g["out_bf16"], out)
    assert r["bad"] == 0, r
    # The restatement differs from torch only by fp32 summation order: within 1 bf16 ulp,
    # or 2^-14 absolute where cancellation leaves a value near zero.
    diff = np.abs(oracle.bf16_bits_to_f32(out) - oracle.bf16_bits_to_f32(g["out_bf16"]))
    ulp = np.abs(oracle.bf16_bits_to_f32(g["out_bf16"])) * 2.0 ** -7 + 2.0 ** -14
    assert (diff <= ulp).all()
    assert (out == g["out_bf16"]).mean() > 0.99


@pytest.mark.parametrize("name", ROUTING)
def test_oracle_routing_matches_reference(name, pkg, oracle):
    g, cfg = load(name)
    inp = pkg.make_inputs(pkg.MoEConfig(**cfg).with_(E_local=1), "cpu")
    idx, w = oracle.route(inp["routing_logits"].numpy(), inp["routing_bias"].float().numpy(),
                          cfg["routed_scaling_factor"])
    np.testing.assert_array_equal(np.sort(idx, axis=1), g["topk_sorted"])
    # weights renormalise to the scaling factor
    np.testing.assert_allclose(w.sum(axis=1), cfg["routed_scaling_factor"], rtol=1e-5)


def test_planted_mistake_is_caught(cpu_inputs, oracle, monkeypatch):
    """A wrong oracle (SiLU on the wrong half) must fail the golden comparison."""
    g, _ = load("cfg0_t16")
    real = oracle.moe_forward

    def swapped(**kw):
        kw = dict(kw)
        w13 = kw["gemm1_weights"]
        kw["gemm1_weights"] = np.concatenate([w13[:, 2048:], w13[:, :2048]], axis=1)
        s13 = kw["gemm1_weights_scale"]
        kw["gemm1_weights_scale"] = np.concatenate([s13[:, 16:], s13[:, :16]], axis=1)
        return real(**kw)

    out = swapped(**oracle.to_numpy_inputs(cpu_inputs("cfg0_t16")))
    assert oracle.check_tolerance(g["out_bf16"], out)["bad"] > 1000


# Goldens on the reference test suite's own inputs (moe_layer.build_moe_inputs, seed = T;
# restated in tests/ref_inputs.py). T = 256 takes a few seconds more than the others.
REF_FULL = ["ref_t1", "ref_t4", "ref_t32", "ref_t64", "ref_t256"]


@pytest.mark.parametrize("name", REF_FULL)
def test_oracle_matches_reference_on_its_own_generator(name, oracle):
    from ref_inputs import build_moe_inputs, digests as ref_digests
    g, cfg = load(name)
    inp = build_moe_inputs(cfg["T"], cfg["seed"])
    assert ref_digests(inp) == json.loads(str(g["inputs_sha256"])), "generator restatement drifted"
    out, idx, _ = oracle.moe_forward(**oracle.to_numpy_inputs(inp), return_routing=True)
    np.testing.assert_array_equal(np.sort(idx, axis=1), g["topk_sorted"])
    r = oracle.check_tolerance(g["out_bf16"], out)
    assert r["bad"] == 0, r
    diff = np.abs(oracle.bf16_bits_to_f32(out) - oracle.bf16_bits_to_f32(g["out_bf16"]))
    ulp = np.abs(oracle.bf16_bits_to_f32(g["out_bf16"])) * 2.0 ** -7 + 2.0 ** -20
    assert (diff <= ulp).all(), float(diff.max())
    assert (out == g["out_bf16"]).mean() > 0.99


@pytest.mark.parametrize("name", FULL + REF_FULL)
def test_reference_rows_without_local_routes_are_plus_zero(name):
    """The reference's output starts as a zero tensor and only local routes add to it
    (reference/moe_ref.py:110-136), so a token without a local route gets the bf16 bits of +0
    and every other token a row that is not all zeros. The CUDA path writes such rows directly
    (without summing anything) from 1024 tokens on; this pins that they must be exactly +0."""
    g, cfg = load(name)
    off = cfg.get("local_expert_offset", 0)
    e_local = cfg.get("E_local", 32)                  # the reference generator's 32 local experts
    idx = g["topk_sorted"].astype(np.int64)
    nlocal = ((idx >= off) & (idx < off + e_local)).sum(axis=1)
    rows_zero = (g["out_bf16"] == 0).all(axis=1)
    np.testing.assert_array_equal(rows_zero, nlocal == 0)
