"""The reference's own CUDA extension (built by oracle/build_ref.py) on this GPU: the baseline
the benchmark times next to this package. Checks that the baseline computes the layer (its
output on the reference test's own inputs meets the reference tolerance against the reference
oracle's golden), and prints how it fares on the benchmark configuration's inputs, where its
single-e4m3 intermediate (kernels/moe.cu:516-541) exceeds that tolerance. Skipped when the
module was not built (it needs the reference checkout at build time)."""
import os

import numpy as np
import pytest
import torch

from gpu_helpers import out_bits
from ref_inputs import build_moe_inputs

pytestmark = pytest.mark.gpu
GOLDEN = os.path.join(os.path.dirname(__file__), "golden")


@pytest.fixture(scope="module")
def ref_mod():
    from oracle import build_ref
    if not os.path.exists(build_ref.so_path()):
        pytest.skip("oracle/_ref/moe_fused_ref.so not built")
    return build_ref.load()


def test_reference_cuda_on_its_own_inputs(ref_mod, oracle):
    from oracle.ref_cuda import RefCuda
    g = np.load(os.path.join(GOLDEN, "ref_t64.npz"))
    inp = {k: (v.cuda() if isinstance(v, torch.Tensor) else v) for k, v in build_moe_inputs(64, 64).items()}
    got = out_bits(RefCuda(inp, ref_mod)())
    r = oracle.check_tolerance(g["out_bf16"], got)
    print("reference CUDA, its own inputs, T=64:", r)
    assert r["bad"] == 0, r


def test_reference_cuda_on_benchmark_inputs(ref_mod, pkg, oracle):
    from oracle.ref_cuda import RefCuda
    g = np.load(os.path.join(GOLDEN, "cfg1_t64.npz"))
    inp = pkg.make_inputs(pkg.CONFIGS[1], "cuda")
    ref_cuda = oracle.check_tolerance(g["out_bf16"], out_bits(RefCuda(inp, ref_mod)()))
    ours = oracle.check_tolerance(g["out_bf16"], out_bits(pkg.run(**inp)))
    print("configuration 1: reference CUDA", ref_cuda, "this package", ours)
    assert ours["bad"] == 0
    assert ours["max_abs_err"] <= ref_cuda["max_abs_err"]
