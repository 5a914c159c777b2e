"""Fused gate GEMM + FP8 quantiser (gate_quantize) on the GPU against the CPU restatements:
codes and scales bit for bit (oracle quantize_hidden, and the standalone device quantiser),
logits within the fp32-accumulation bound of the exact dot products, batch invariance of the
logits, and the division's correct rounding over every relevant bf16 magnitude."""
import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu

# An fp32 accumulation of 7168 exact bf16 products in K slices of 1792, 16 products per tensor
# core step, errs by at most a few hundred fp32 roundings of partial sums bounded by sum|x w|;
# 2^-14 * sum|x w| leaves a wide margin over the ~2^-16 worst case of that argument.
LOGIT_TOL = 2.0 ** -14


def _hidden(T, seed):
    g = torch.Generator().manual_seed(seed)
    x = torch.randn((T, 7168), generator=g)
    mag = torch.tensor([1e-6, 1e-2, 1.0, 300.0])[torch.randint(0, 4, (T, 56), generator=g)]
    x = (x.view(T, 56, 128) * mag[:, :, None]).view(T, 7168)
    if T > 2:
        x[1] = 0.0
        x[2, 256:384] = -0.0
    return x.to(torch.bfloat16)


def _gate(seed):
    g = torch.Generator().manual_seed(1000 + seed)
    return (0.02 * torch.randn((256, 7168), generator=g)).to(torch.bfloat16)


def _check_logits(oracle, x, w, logits):
    ref, bound = oracle.gate_logits(x.float().numpy(), w.float().numpy())
    err = np.abs(logits.cpu().numpy().astype(np.float64) - ref)
    assert (err <= LOGIT_TOL * bound + 1e-30).all(), float((err / np.maximum(bound, 1e-30)).max())
    return float((err / np.maximum(bound, 1e-30)).max())


def test_pack_gate_layout(pkg):
    w = _gate(0)
    packed = pkg.pack_gate(w.cuda()).cpu().numpy()
    src = w.view(torch.int16).numpy().view(np.uint8).reshape(256, 56, 2, 8, 16)   # row, kb, half, chunk
    r = np.arange(256)[:, None]
    c = np.arange(8)[None, :]
    for kb in (0, 13, 55):
        for half in (0, 1):
            img = packed[kb, half].reshape(256, 8, 16)                          # row, stored chunk
            np.testing.assert_array_equal(img[r, c ^ (r & 7)], src[:, kb, half])


@pytest.mark.parametrize("T", [1, 3, 127, 128, 129, 1000, 4096])
def test_gate_quantize_matches_oracle(pkg, oracle, T):
    x, w = _hidden(T, T), _gate(T)
    gp = pkg.pack_gate(w.cuda())
    logits, q, s = pkg.gate_quantize(x.cuda(), gp)
    q_alone, s_alone = pkg.quantize_hidden(x.cuda())
    torch.cuda.synchronize()
    codes, scale = oracle.quantize_hidden(x.float().numpy())
    np.testing.assert_array_equal(q.view(torch.uint8).cpu().numpy(), codes)
    np.testing.assert_array_equal(s.cpu().numpy().view(np.uint32), scale.view(np.uint32))
    assert torch.equal(q.view(torch.uint8), q_alone.view(torch.uint8))
    assert torch.equal(s.view(torch.int32), s_alone.view(torch.int32))
    _check_logits(oracle, x, w, logits)


def test_gate_logits_agree_with_fp32_linear(pkg, oracle):
    """Against torch's fp32 linear on the CPU (the published router's arithmetic): both lie
    within the same bound of the exact products."""
    T = 512
    g = torch.Generator().manual_seed(5)
    x = torch.randn((T, 7168), generator=g).to(torch.bfloat16)
    w = _gate(5)
    logits, _, _ = pkg.gate_quantize(x.cuda(), pkg.pack_gate(w.cuda()))
    cpu = torch.nn.functional.linear(x.float(), w.float()).numpy().astype(np.float64)
    ref, bound = oracle.gate_logits(x.float().numpy(), w.float().numpy())
    assert (np.abs(cpu - ref) <= LOGIT_TOL * bound).all()
    rel = _check_logits(oracle, x, w, logits)
    assert rel < 2.0 ** -17, rel


def test_gate_logits_batch_invariant(pkg):
    """A token's logits do not depend on T or on its position in the batch."""
    x, w = _hidden(4096, 11).cuda(), _gate(11).cuda()
    gp = pkg.pack_gate(w)
    full, _, _ = pkg.gate_quantize(x, gp)
    part, _, _ = pkg.gate_quantize(x[1000:1300].contiguous(), gp)
    one, _, _ = pkg.gate_quantize(x[4095:4096].contiguous(), gp)
    again, _, _ = pkg.gate_quantize(x, gp)
    assert torch.equal(full[1000:1300].view(torch.int32), part.view(torch.int32))
    assert torch.equal(full[4095:4096].view(torch.int32), one.view(torch.int32))
    assert torch.equal(full.view(torch.int32), again.view(torch.int32))


def _division_blocks(seed):
    """Blocks that put every bf16 magnitude within 2^28 of the block maximum (all the values
    whose code can be nonzero) under many block maxima, with random signs and positions."""
    rng = np.random.default_rng(seed)
    maxima = list(rng.integers(0x0080, 0x7F80, 600))                 # normal bf16 amax patterns
    maxima += [0x3F7F, 0x3F80, 0x437F, 0x4380, 0x7F7F, 0x0080, 0x00FF, 0x0001, 0x0040,
               0x1A00, 0x1AFF, 0x1B80, 0x177F, 0x1780, 0x1781]       # edge mantissas, tiny, subnormal,
    #                                                                  either side of the 2^-80 switch
    blocks = []
    for a in maxima:
        vals = np.arange(max(0, a - 28 * 128), a + 1, dtype=np.int64)
        for i in range(0, len(vals), 127):
            chunk = vals[i:i + 127]
            blk = np.concatenate([[a], chunk, rng.choice(vals, 127 - len(chunk))]).astype(np.uint16)
            blk = rng.permutation(blk)
            blk |= (rng.integers(0, 2, 128) << 15).astype(np.uint16)
            blocks.append(blk)
    blocks = np.stack(blocks)
    pad = (-len(blocks)) % 56
    blocks = np.concatenate([blocks, blocks[:pad]])
    return blocks.reshape(-1, 7168)


def test_gate_division_exhaustive_magnitudes(pkg, oracle):
    bits = _division_blocks(3)
    x = torch.from_numpy(bits.view(np.int16)).view(torch.bfloat16)
    T = x.shape[0]
    logits, q, s = pkg.gate_quantize(x.cuda(), pkg.pack_gate(_gate(3).cuda()))
    q_alone, _ = pkg.quantize_hidden(x.cuda())
    torch.cuda.synchronize()
    codes, scale = oracle.quantize_hidden(oracle.bf16_bits_to_f32(bits))
    np.testing.assert_array_equal(s.cpu().numpy().view(np.uint32), scale.view(np.uint32))
    got = q.view(torch.uint8).cpu().numpy()
    bad = np.nonzero(got != codes)
    assert bad[0].size == 0, (T, bad[0][:5], bad[1][:5])
    assert torch.equal(q.view(torch.uint8), q_alone.view(torch.uint8))


def test_gate_zero_rows_and_t0(pkg):
    gp = pkg.pack_gate(_gate(1).cuda())
    x = torch.zeros((130, 7168), dtype=torch.bfloat16, device="cuda")
    x[129, 5] = 2.0
    logits, q, s = pkg.gate_quantize(x, gp)
    torch.cuda.synchronize()
    assert (logits[:129] == 0).all() and (q[:129].view(torch.uint8) == 0).all()
    assert (s[:, :129] == 1.0).all() and float(s[0, 129]) == float(np.float32(2.0) / np.float32(448.0))
    e = pkg.gate_quantize(torch.empty((0, 7168), dtype=torch.bfloat16, device="cuda"), gp)
    assert e[0].shape == (0, 256) and e[1].shape == (0, 7168) and e[2].shape == (56, 0)
    with pytest.raises(RuntimeError, match="bfloat16"):
        pkg.gate_quantize(torch.zeros((2, 7168), device="cuda"), gp)
    with pytest.raises(RuntimeError, match="pack_gate"):
        pkg.gate_quantize(x, gp.view(-1))


def test_gate_quantize_feeds_moe_forward(pkg, oracle):
    """hidden -> gate_quantize -> moe_forward equals moe_forward on the same logits and the
    oracle's quantised bytes."""
    cfg = pkg.CONFIGS[1].with_(T=64, seed=4)
    inp = pkg.make_inputs(cfg, "cuda")
    x = _hidden(64, 9)
    logits, q, s = pkg.gate_quantize(x.cuda(), pkg.pack_gate(_gate(9).cuda()))
    out = pkg.run(**dict(inp, routing_logits=logits, hidden_states=q, hidden_states_scale=s))
    codes, scale = oracle.quantize_hidden(x.float().numpy())
    ref = pkg.run(**dict(inp, routing_logits=logits,
                         hidden_states=torch.from_numpy(codes).view(torch.float8_e4m3fn).cuda(),
                         hidden_states_scale=torch.from_numpy(scale).cuda()))
    assert torch.equal(out.view(torch.int16), ref.view(torch.int16))
