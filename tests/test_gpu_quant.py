"""Device FP8 activation quantiser vs the CPU restatement, bit for bit (codes and scales)."""
import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu


def _inputs(T, seed):
    g = torch.Generator().manual_seed(seed)
    x = torch.randn((T, 7168), generator=g)
    mag = torch.tensor([1e-6, 1e-2, 1.0, 300.0])[torch.randint(0, 4, (T, 56), generator=g)]
    x = (x.view(T, 56, 128) * mag[:, :, None]).view(T, 7168)
    if T > 2:
        x[1] = 0.0
        x[2, 256:384] = -0.0
    return x.to(torch.bfloat16)


@pytest.mark.parametrize("T", [1, 3, 97, 4096])
def test_quantize_matches_oracle(pkg, oracle, T):
    x = _inputs(T, T)
    q, s = pkg.quantize_hidden(x.cuda())
    torch.cuda.synchronize()
    codes, scale = oracle.quantize_hidden(x.float().numpy())
    np.testing.assert_array_equal(q.view(torch.uint8).cpu().numpy(), codes)
    np.testing.assert_array_equal(s.cpu().numpy().view(np.uint32), scale.view(np.uint32))


def test_quantize_feeds_moe_forward(pkg, oracle):
    """bf16 hidden -> device quantiser -> moe_forward equals the forward on the oracle's bytes."""
    cfg = pkg.CONFIGS[1].with_(T=16, seed=2)
    inp = pkg.make_inputs(cfg, "cuda")
    x = _inputs(16, 7).cuda()
    q, s = pkg.quantize_hidden(x)
    out = pkg.run(**dict(inp, hidden_states=q, hidden_states_scale=s))
    codes, scale = oracle.quantize_hidden(x.float().cpu().numpy())
    ref = pkg.run(**dict(inp, hidden_states=torch.from_numpy(codes).view(torch.float8_e4m3fn).cuda(),
                         hidden_states_scale=torch.from_numpy(scale).cuda()))
    assert torch.equal(out.view(torch.int16), ref.view(torch.int16))


def test_quantize_t0_and_errors(pkg):
    q, s = pkg.quantize_hidden(torch.empty((0, 7168), dtype=torch.bfloat16, device="cuda"))
    assert q.shape == (0, 7168) and s.shape == (56, 0)
    with pytest.raises(RuntimeError, match="bfloat16"):
        pkg.quantize_hidden(torch.zeros((2, 7168), device="cuda"))
