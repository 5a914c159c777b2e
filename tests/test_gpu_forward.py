"""moe_forward on the B200 against the reference goldens and the CPU oracle.

Tolerance (the reference test's, tests/test_moe.py:21-38): |got - ref| <= 1e-2 + 2e-2 |ref|
elementwise, every element. The stage tests check the intermediate buffers of the same run
(gathered rows bit-exact, SwiGLU output and weighted expert rows within the precision of the
two-term e4m3 intermediate) so a failure points at one kernel.
"""
import json
import os

import numpy as np
import pytest
import torch

from gpu_helpers import forward_with_workspace, out_bits, region, unswizzle

pytestmark = pytest.mark.gpu
GOLDEN = os.path.join(os.path.dirname(__file__), "golden")
ATOL, RTOL = 1e-2, 2e-2


def _golden(name):
    g = np.load(os.path.join(GOLDEN, name + ".npz"))
    return g, json.loads(str(g["config"]))


@pytest.fixture(autouse=True)
def _status_clean(pkg):
    pkg.device_status(reset=True)
    yield
    assert pkg.device_status(reset=True) == 0, "a kernel reported a timeout or bad metadata"


@pytest.mark.parametrize("name", ["t1_seed1", "t1_seed3", "t4_off224", "cfg0_t16", "cfg1_t64"])
def test_forward_matches_reference_golden(pkg, oracle, name):
    g, cfg = _golden(name)
    inp = pkg.make_inputs(pkg.MoEConfig(**cfg), "cuda")
    out = pkg.run(**inp)
    torch.cuda.synchronize()
    r = oracle.check_tolerance(g["out_bf16"], out_bits(out), ATOL, RTOL)
    print(name, r)
    assert r["bad"] == 0, r


@pytest.mark.parametrize("kw", [dict(T=256, seed=1), dict(T=1024, seed=2),
                                dict(T=200, seed=3, E_local=8, local_expert_offset=96),
                                dict(T=160, seed=4, local_expert_offset=240)])
def test_forward_matches_oracle(pkg, oracle, kw):
    cfg = pkg.MoEConfig(**kw)
    inp = pkg.make_inputs(cfg, "cuda")
    out = out_bits(pkg.run(**inp))
    ref = oracle.moe_forward(**oracle.to_numpy_inputs(inp))
    r = oracle.check_tolerance(ref, out, ATOL, RTOL)
    print(kw, r)
    assert r["bad"] == 0, r


def test_forward_skewed_routing(pkg, oracle):
    """Config-4 bias (+1.5 on two experts per group): all traffic on the hot experts."""
    cfg = pkg.CONFIGS[4].with_(T=1536, E_local=32)
    inp = pkg.make_inputs(cfg, "cuda")
    out = out_bits(pkg.run(**inp))
    ref = oracle.moe_forward(**oracle.to_numpy_inputs(inp))
    r = oracle.check_tolerance(ref, out, ATOL, RTOL)
    print(r)
    assert r["bad"] == 0, r


def test_forward_deterministic(pkg):
    inp = pkg.make_inputs(pkg.MoEConfig(T=512, seed=5), "cuda")
    a = pkg.run(**inp).clone()
    b = pkg.run(**inp)
    assert torch.equal(a.view(torch.int16), b.view(torch.int16))


def test_forward_t0(pkg):
    inp = pkg.make_inputs(pkg.MoEConfig(T=0, E_local=1), "cuda")
    out = pkg.run(**inp)
    assert out.shape == (0, 7168)


def test_max_tokens_rows_are_independent(pkg):
    """At the largest T the API takes (65536), every token's output equals the output of a small
    forward over just that token's row: routing and every GEMM row are per token, so the batch
    around a token (tile membership, slot order, how many tiles each expert has) changes nothing.
    Checked bit for bit on the first and last 300 tokens; one more token is refused."""
    cfg = pkg.CONFIGS[2].with_(T=65536, seed=13)
    inp = pkg.make_inputs(cfg, "cuda")
    big = pkg.run(**inp)
    torch.cuda.synchronize()
    assert pkg.device_status(reset=True) == 0
    for lo, hi in ((0, 300), (65536 - 300, 65536)):
        part = dict(inp, hidden_states=inp["hidden_states"][lo:hi].contiguous(),
                    hidden_states_scale=inp["hidden_states_scale"][:, lo:hi].contiguous(),
                    routing_logits=inp["routing_logits"][lo:hi].contiguous())
        small = pkg.run(**part)
        np.testing.assert_array_equal(out_bits(big[lo:hi]), out_bits(small))
    del big
    x = torch.empty((65537, 7168), dtype=torch.uint8, device="cuda").view(torch.float8_e4m3fn)
    with pytest.raises(RuntimeError, match="65536"):
        pkg.moe_forward(x, torch.ones((56, 65537), device="cuda"), pkg.pack_w13(inp["gemm1_weights"][:1]),
                        inp["gemm1_weights_scale"][:1].float().contiguous(), pkg.pack_w2(inp["gemm2_weights"][:1]),
                        inp["gemm2_weights_scale"][:1].float().contiguous(), torch.zeros((65537, 256), device="cuda"),
                        torch.zeros(256, device="cuda"), 2.5, 0)


def test_stages(pkg, oracle):
    """Intermediate buffers of one run against numpy restatements."""
    cfg = pkg.MoEConfig(T=96, seed=6)
    inp = pkg.make_inputs(cfg, "cuda")
    out, ws = forward_with_workspace(pkg, inp)
    T, E = cfg.T, cfg.E_local
    lay = pkg.workspace_layout(T, E)
    npi = oracle.to_numpy_inputs(inp)
    idx, w = oracle.route(npi["routing_logits"], npi["routing_bias"], cfg.routed_scaling_factor)

    # routing metadata: per-expert slot lists (any order) and each token's ascending list
    counts = region(ws, lay, "counts", torch.int32, E)
    exp_counts = np.array([(idx == e).any(axis=1).sum() for e in range(E)])
    np.testing.assert_array_equal(counts, exp_counts)
    route_token = region(ws, lay, "route_token", torch.int32, E * T).reshape(E, T)
    route_w = region(ws, lay, "route_w", torch.float32, E * T).reshape(E, T)
    token_nr = region(ws, lay, "token_nr", torch.int32, T)
    token_route = region(ws, lay, "token_route", torch.int32, T * 8).reshape(T, 8)
    dense_base = region(ws, lay, "dense_base", torch.int32, E + 1)
    np.testing.assert_array_equal(dense_base, np.concatenate([[0], np.cumsum(exp_counts)]))
    for e in range(E):
        toks = np.nonzero((idx == e).any(axis=1))[0]
        got = route_token[e, :exp_counts[e]]
        np.testing.assert_array_equal(np.sort(got), toks)
        wexp = np.array([w[t][idx[t] == e][0] for t in got], np.float32)
        np.testing.assert_array_equal(route_w[e, :exp_counts[e]], wexp)
    for t in range(T):
        local = sorted(int(g) for g in idx[t] if g < E)
        assert token_nr[t] == len(local)
        for k, g in enumerate(local):
            le, slot = token_route[t, k] >> 16, token_route[t, k] & 0xFFFF
            assert le == g and route_token[le, slot] == t

    # gather: bit-exact FP8 rows and scales in the experts' swizzled tile images
    n_tiles = int(sum((c + 127) // 128 for c in exp_counts))
    a = region(ws, lay, "a_tiled", torch.uint8, n_tiles * 56 * 128 * 128).reshape(n_tiles, 56, 128, 128)
    a = unswizzle(a).transpose(0, 2, 1, 3).reshape(n_tiles * 128, 7168)
    asc = region(ws, lay, "a_scale", torch.float32, n_tiles * 56 * 128).reshape(n_tiles, 56, 128)
    asc = asc.transpose(0, 2, 1).reshape(n_tiles * 128, 56)
    t0 = 0
    for e in range(E):
        toks = route_token[e, :exp_counts[e]]
        rows = t0 * 128 + np.arange(exp_counts[e])
        np.testing.assert_array_equal(a[rows], npi["hidden_states"][toks])
        np.testing.assert_array_equal(asc[rows], npi["hidden_states_scale"].T[toks])
        t0 += (exp_counts[e] + 127) // 128

    # GEMM1 + SwiGLU: C = scale * (hi + lo) vs the fp32 oracle
    A = oracle.dequant_hidden(npi["hidden_states"], npi["hidden_states_scale"])
    hi = unswizzle(region(ws, lay, "c_hi", torch.uint8, n_tiles * 16 * 128 * 128).reshape(n_tiles, 16, 128, 128))
    lo = unswizzle(region(ws, lay, "c_lo", torch.uint8, n_tiles * 16 * 128 * 128).reshape(n_tiles, 16, 128, 128))
    cs = region(ws, lay, "c_scale", torch.float32, n_tiles * 16 * 128).reshape(n_tiles, 16, 128)
    cval = (oracle.decode_e4m3(hi) + oracle.decode_e4m3(lo)) * cs[..., None]
    cval = cval.transpose(0, 2, 1, 3).reshape(n_tiles * 128, 2048)
    routes = int(exp_counts.sum())
    # weighted route rows: dense rows in blocks of 128, each block as [224 column groups][128 rows][32]
    nblk = (routes + 127) // 128
    partial = (region(ws, lay, "partial", torch.float32, nblk * 128 * 7168).reshape(nblk, 224, 128, 32)
               .transpose(0, 2, 1, 3).reshape(nblk * 128, 7168))
    out_f = out.float().cpu().numpy()
    assert (token_nr == 1).any() and (token_nr > 1).any()
    t0 = 0
    worst_c, worst_o = 0.0, 0.0
    for e in range(E):
        nt = (exp_counts[e] + 127) // 128
        if nt == 0:
            continue
        rows = np.arange(t0 * 128, t0 * 128 + exp_counts[e])      # tile rows = slots
        drows = dense_base[e] + np.arange(exp_counts[e])
        toks = route_token[e, :exp_counts[e]]
        W13 = oracle.dequant_block(npi["gemm1_weights"][e], npi["gemm1_weights_scale"][e])
        G1 = A[toks] @ W13.T
        C = (G1[:, 2048:] / (1.0 + np.exp(-G1[:, 2048:]))) * G1[:, :2048]
        blk_max = np.abs(C).reshape(len(toks), 16, 128).max(axis=2, keepdims=True)
        err = np.abs(cval[rows] - C).reshape(len(toks), 16, 128) / (blk_max + 1e-30)
        worst_c = max(worst_c, float(err.max()))
        W2 = oracle.dequant_block(npi["gemm2_weights"][e], npi["gemm2_weights_scale"][e])
        Oe = (C @ W2.T) * route_w[e, :exp_counts[e]][:, None]
        # a token's only local route goes straight to its output row (bf16); the others to `partial`
        multi = token_nr[toks] > 1
        got = np.where(multi[:, None], partial[drows], out_f[toks])
        rel = np.abs(got - Oe).max(axis=1) / (np.abs(Oe).max(axis=1) + 1e-30)
        worst_o = max(worst_o, float(rel.max()))
        t0 += nt
    print("worst C block-relative err", worst_c, "worst route-row relative err", worst_o)
    assert worst_c < 2.0 ** -7
    assert worst_o < 1e-2


def test_forward_two_tile_experts(pkg, oracle):
    """Skewed routing with T=1536: hot experts span several 128-row tiles (gather across tiles)."""
    cfg = pkg.CONFIGS[4].with_(T=1536, E_local=32, seed=3)
    inp = pkg.make_inputs(cfg, "cuda")
    out, ws = forward_with_workspace(pkg, inp)
    counts = region(ws, pkg.workspace_layout(cfg.T, 32), "counts", torch.int32, 32)
    assert counts.max() > 256
    ref = oracle.moe_forward(**oracle.to_numpy_inputs(inp))
    r = oracle.check_tolerance(ref, out_bits(out), ATOL, RTOL)
    assert r["bad"] == 0, r


def test_forward_tile_size_boundaries(pkg, oracle):
    """Local expert counts chosen at the kernels' tile-shape boundaries: 64 routes (one tile run with
    M = 64 MMAs), 65 (one M = 128 tile), 128 (one full tile), 129 (a full tile plus a one-route M = 64
    tile) and 1. The logits make each token's eight picks explicit: +10 on the chosen experts (group 0
    holds the local ones, groups 1-3 the rest of the eight), -10 elsewhere, zero bias."""
    T = 129
    cfg = pkg.MoEConfig(T=T, seed=11)
    inp = pkg.make_inputs(cfg, "cuda")
    logits = torch.full((T, 256), -10.0)
    want = {0: 64, 1: 65, 2: 128, 3: 129, 4: 1}
    for t in range(T):
        local = [e for e, n in want.items() if t < n]
        others = [32 * (1 + g) + t % 4 * 3 + i for g in range(3) for i in range(3)][:8 - len(local)]
        for e in local + others:
            logits[t, e] = 10.0
    inp["routing_logits"] = logits.to(inp["routing_logits"].dtype).to("cuda")
    inp["routing_bias"] = torch.zeros_like(inp["routing_bias"])
    out, ws = forward_with_workspace(pkg, inp)
    counts = region(ws, pkg.workspace_layout(T, 32), "counts", torch.int32, 32)
    assert [int(counts[e]) for e in range(5)] == [64, 65, 128, 129, 1]
    assert int(counts[5:].sum()) == 0
    ref = oracle.moe_forward(**oracle.to_numpy_inputs(inp))
    r = oracle.check_tolerance(ref, out_bits(out), ATOL, RTOL)
    print(r)
    assert r["bad"] == 0, r


@pytest.mark.parametrize("fp32_out", [False, True])
def test_output_16_byte_aligned_only(pkg, fp32_out):
    """The output need only be 16-byte aligned. At T >= 1024 the GEMM2 kernel writes the rows of
    one-route tokens itself and the router the zero rows of tokens without a local route; an
    output 16 bytes past a 32-byte boundary must give the same bits, with no row left unwritten."""
    T = 1024
    inp = pkg.make_inputs(pkg.MoEConfig(T=T, seed=2), "cuda")
    f32 = {k: inp[k].to(torch.float32).contiguous() for k in
           ("hidden_states_scale", "gemm1_weights_scale", "gemm2_weights_scale", "routing_logits")}
    args = (inp["hidden_states"].contiguous(), f32["hidden_states_scale"], pkg.pack_w13(inp["gemm1_weights"]),
            f32["gemm1_weights_scale"], pkg.pack_w2(inp["gemm2_weights"]), f32["gemm2_weights_scale"],
            f32["routing_logits"], inp["routing_bias"].to(torch.float32).reshape(-1).contiguous(),
            float(inp["routed_scaling_factor"]), int(inp["local_expert_offset"]))
    dtype = torch.float32 if fp32_out else torch.bfloat16
    step = 16 // (4 if fp32_out else 2)
    ref = pkg.moe_forward(*args, fp32_out=fp32_out)
    big = torch.full((T * 7168 + step,), float("nan"), dtype=dtype, device="cuda")
    out = big[step:].view(T, 7168)
    assert out.data_ptr() % 32 == 16
    pkg.moe_forward(*args, out=out, fp32_out=fp32_out)
    torch.cuda.synchronize()
    iview = torch.int32 if fp32_out else torch.int16
    assert torch.equal(out.view(iview), ref.view(iview))
    assert not torch.isnan(out.float()).any()               # every row written over the NaN fill
    zero_rows = (out.view(iview) == 0).all(dim=1).sum().item()
    assert zero_rows > 0                                     # tokens without a local route: +0 rows
