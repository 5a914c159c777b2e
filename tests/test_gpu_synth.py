"""The GPU input generator produces exactly the CPU generator's bytes."""
import pytest
import torch

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("cfg_kw", [dict(T=16, E_local=2, seed=0),
                                    dict(T=33, E_local=1, seed=5, local_expert_offset=200),
                                    dict(T=8, E_local=1, seed=2, hot_experts=(0, 1, 32), hot_bias=1.5)])
def test_gpu_generator_matches_cpu(pkg, cfg_kw):
    cfg = pkg.MoEConfig(**cfg_kw)
    g = pkg.make_inputs(cfg, "cuda")
    c = pkg.make_inputs(cfg, "cpu")
    for k, v in c.items():
        if isinstance(v, torch.Tensor):
            assert torch.equal(g[k].cpu().view(torch.uint8), v.view(torch.uint8)), k
        else:
            assert g[k] == v
