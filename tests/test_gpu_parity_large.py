"""moe_forward against the CPU oracle at the benchmark's own sizes.

* Configuration 2 exactly as the benchmark runs it (T = 4096, experts 0-31 of 256, seed 0), and
  T = 2048: every element of the output.
* T = 8192 and T = 16384 (configuration 4's skewed routing on one 32-expert slice): a few
  hundred sampled rows. Routing and every expert row are per token, so the oracle run on just
  those tokens' rows gives exactly those rows of the full layer.

Tolerance (the reference test's, tests/test_moe.py:21-38): |got - ref| <= 1e-2 + 2e-2 |ref|
elementwise, every element checked.
"""
import numpy as np
import pytest
import torch

from gpu_helpers import out_bits

pytestmark = pytest.mark.gpu
ATOL, RTOL = 1e-2, 2e-2


@pytest.fixture(autouse=True)
def _status_clean(pkg):
    pkg.device_status(reset=True)
    yield
    assert pkg.device_status(reset=True) == 0, "a kernel reported a timeout or bad metadata"


def rows_of(npi: dict, rows: np.ndarray) -> dict:
    """The oracle's inputs restricted to a set of tokens."""
    out = dict(npi)
    out["routing_logits"] = npi["routing_logits"][rows]
    out["hidden_states"] = npi["hidden_states"][rows]
    out["hidden_states_scale"] = np.ascontiguousarray(npi["hidden_states_scale"][:, rows])
    return out


@pytest.mark.parametrize("name,kw", [("config2_t4096", dict(ci=2)),
                                     ("t2048_seed2048", dict(ci=2, T=2048, seed=2048))])
def test_full_output(pkg, oracle, name, kw):
    ci = kw.pop("ci")
    cfg = pkg.CONFIGS[ci].with_(**kw)
    inp = pkg.make_inputs(cfg, "cuda")
    got = out_bits(pkg.run(**inp))
    npi = oracle.to_numpy_inputs(inp)
    ref = oracle.moe_forward(**npi)
    r = oracle.check_tolerance(ref, got, ATOL, RTOL)
    r["identical_frac"] = float((ref == got).mean())
    print(name, r)
    assert r["bad"] == 0, r


@pytest.mark.parametrize("name,ci,kw", [("t8192_seed0", 2, dict(T=8192)),
                                        ("skew_t16384", 4, dict(T=16384, E_local=32))])
def test_sampled_rows(pkg, oracle, name, ci, kw):
    cfg = pkg.CONFIGS[ci].with_(**kw)
    inp = pkg.make_inputs(cfg, "cuda")
    got = out_bits(pkg.run(**inp))
    npi = oracle.to_numpy_inputs(inp)
    rng = np.random.default_rng(cfg.T)
    rows = np.unique(np.concatenate([np.arange(8), np.arange(cfg.T - 8, cfg.T),
                                     rng.choice(cfg.T, 368, replace=False)]))
    ref = oracle.moe_forward(**rows_of(npi, rows))
    r = oracle.check_tolerance(ref, got[rows], ATOL, RTOL)
    idx, _ = oracle.route(npi["routing_logits"][rows], npi["routing_bias"], cfg.routed_scaling_factor)
    r["rows"], r["rows_with_local_route"] = int(rows.size), int(((idx >= 0) & (idx < 32)).any(axis=1).sum())
    print(name, r)
    assert r["rows_with_local_route"] > rows.size // 8
    assert r["bad"] == 0, r
