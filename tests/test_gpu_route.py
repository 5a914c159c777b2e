"""Device router vs the CPU oracle: identical expert indices (selection order included) and
identical weights, bit for bit (reference/moe_ref.py:82-107 restated in oracle/)."""
import json
import os

import numpy as np
import pytest
import torch

from test_routing_kat import kat_cases

pytestmark = pytest.mark.gpu
GOLDEN = os.path.join(os.path.dirname(__file__), "golden")


def _route_both(pkg, oracle, logits_np, bias_np, rsf):
    idx, w = pkg.route(torch.from_numpy(logits_np).cuda(), torch.from_numpy(bias_np).cuda(), rsf)
    ridx, rw = oracle.route(logits_np, bias_np, rsf)
    return idx.cpu().numpy(), w.cpu().numpy(), ridx, rw


@pytest.mark.parametrize("T,cfg_i,seed", [(1, 0, 1), (64, 1, 0), (4096, 2, 0), (16384, 4, 0), (3000, 0, 9)])
def test_router_bit_exact(pkg, oracle, T, cfg_i, seed):
    cfg = pkg.CONFIGS[cfg_i].with_(T=T, E_local=1, seed=seed)
    inp = pkg.make_inputs(cfg, "cuda")
    lg = inp["routing_logits"].cpu().numpy()
    b = inp["routing_bias"].float().cpu().numpy()
    idx, w, ridx, rw = _route_both(pkg, oracle, lg, b, cfg.routed_scaling_factor)
    np.testing.assert_array_equal(idx, ridx)
    np.testing.assert_array_equal(w.view(np.uint32), rw.view(np.uint32))


@pytest.mark.parametrize("name", ["route_cfg2_t4096", "route_cfg4_t16384_skew"])
def test_router_matches_reference_golden(pkg, name):
    g = np.load(os.path.join(GOLDEN, name + ".npz"))
    cfg = pkg.MoEConfig(**json.loads(str(g["config"]))).with_(E_local=1)
    inp = pkg.make_inputs(cfg, "cuda")
    idx, _ = pkg.route(inp["routing_logits"], inp["routing_bias"], cfg.routed_scaling_factor)
    np.testing.assert_array_equal(np.sort(idx.cpu().numpy(), axis=1), g["topk_sorted"])


@pytest.mark.parametrize("case", kat_cases(), ids=lambda c: c[0])
def test_router_kat(pkg, oracle, case):
    name, lg, b, expect = case
    idx, w, ridx, rw = _route_both(pkg, oracle, lg, b, 2.5)
    np.testing.assert_array_equal(idx, ridx)
    np.testing.assert_array_equal(w, rw)
    if expect is not None:
        assert np.sort(idx, axis=1).tolist() == expect
