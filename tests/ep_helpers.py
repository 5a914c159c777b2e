"""Expected results of the expert-parallel layer, built from the CPU oracle.

The expert-parallel forward (15642_moe_b200/ep.py) returns, per token, the fp32 sum over owner
ranks (ascending) of each owner's fp32 partial (the sum of its experts' weighted outputs in
ascending expert order), rounded once to bf16. The layer oracle sums over all experts in
ascending order and rounds once (reference/moe_ref.py:110-136 with every owned expert local);
the two differ only in the association of the fp32 additions. Both are computed here from
per-expert oracle outputs.
"""
from __future__ import annotations

import numpy as np

H = 7168


def per_expert_outputs(pkg, oracle, cfg, experts) -> dict:
    """fp32 [T, 7168] weighted output of each global expert in `experts` over all cfg.T tokens
    (zero rows for tokens that did not pick it), each expert generated on its own."""
    res = {}
    for ge in sorted(set(int(g) for g in experts)):
        inp = pkg.make_inputs(cfg.with_(E_local=1, local_expert_offset=ge), "cpu")
        res[ge] = oracle.moe_forward(**oracle.to_numpy_inputs(inp), return_fp32=True)
    return res


def owner_map(world: int, e_rank: int, placement=None) -> dict:
    """Global expert -> owner rank (contiguous ranges unless a placement is given)."""
    if placement is None:
        placement = [range(d * e_rank, (d + 1) * e_rank) for d in range(world)]
    return {int(g): d for d, experts in enumerate(placement) for g in experts}


def owned_picks(topk_row, world: int, e_rank: int, placement=None) -> list[int]:
    own = owner_map(world, e_rank, placement)
    return sorted(int(g) for g in topk_row if int(g) in own)


def owner_partial(contrib: dict, topk_idx, t: int, d: int, world: int, e_rank: int, placement=None):
    """fp32 [7168] partial of owner d for token t (None if t picked none of d's experts)."""
    own = owner_map(world, e_rank, placement)
    picks = [g for g in owned_picks(topk_idx[t], world, e_rank, placement) if own[g] == d]
    if not picks:
        return None
    part = np.zeros(H, np.float32)
    for g in picks:
        part = part + contrib[g][t]
    return part


def ep_combine_bits(oracle, partials: list) -> np.ndarray:
    """Final combine of one token: fp32 sum of the present owners' partials in ascending owner
    order from +0, one bf16 rounding."""
    acc = np.zeros(H, np.float32)
    for p in partials:
        if p is not None:
            acc = acc + p
    return oracle.f32_to_bf16_bits(acc)


def ep_expected_bits(oracle, contrib: dict, topk_idx, tokens, world: int, e_rank: int,
                     placement=None) -> np.ndarray:
    """bf16 bits [len(tokens), 7168] of the expert-parallel result."""
    rows = [ep_combine_bits(oracle, [owner_partial(contrib, topk_idx, t, d, world, e_rank, placement)
                                     for d in range(world)]) for t in tokens]
    return np.stack(rows) if rows else np.zeros((0, H), np.uint16)


def layer_oracle_bits(oracle, contrib: dict, topk_idx, tokens, world: int, e_rank: int,
                      placement=None) -> np.ndarray:
    """bf16 bits of the single-rounding layer oracle over all owned experts."""
    out = np.zeros((len(tokens), H), np.float32)
    for i, t in enumerate(tokens):
        for g in owned_picks(topk_idx[t], world, e_rank, placement):
            out[i] = out[i] + contrib[g][t]
    return oracle.f32_to_bf16_bits(out)


def gloo_worker(rank: int, world: int, port: int, T_global: int, e_rank: int, seed: int,
                interleaved: bool = False) -> None:
    """One gloo rank of the CPU emulation of the expert-parallel data flow: handle exchange,
    token / expert partition (contiguous expert ranges, or rank d owning the experts g with
    g mod world == d), owner-side partials, exchange, source-side combine."""
    import importlib
    import os
    import sys

    import torch.distributed as dist

    sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
    pkg = importlib.import_module("15642_moe_b200")
    ep = importlib.import_module("15642_moe_b200.ep")
    from oracle import moe_oracle as oracle

    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world)
    try:
        blob = bytes([rank + 1]) * 64
        handles = ep.exchange_handles(blob)
        assert handles == [bytes([r + 1]) * 64 for r in range(world)], "handles out of rank order"
        # Buffer geometry agreed across ranks: every rank sees every rank's (t_rank_max, e_rank).
        assert ep.agree_shapes(rank + 3, e_rank) == [(r + 3, e_rank) for r in range(world)]

        cfg = pkg.MoEConfig(T=T_global, E_local=1, seed=seed)
        inp = pkg.make_inputs(cfg, "cpu")
        idx, _ = oracle.route(inp["routing_logits"].numpy(), inp["routing_bias"].float().numpy(),
                              cfg.routed_scaling_factor)
        placement = ([[g for g in range(world * e_rank) if g % world == d] for d in range(world)]
                     if interleaved else None)
        own = owner_map(world, e_rank, placement)
        mine = sorted({int(g) for g in idx.ravel() if own.get(int(g)) == rank})
        if not interleaved:
            lo_e, hi_e = ep.expert_range(rank, e_rank)
            assert all(lo_e <= g < hi_e and ep.owner_of(g, world, e_rank) == rank for g in mine)
        contrib = per_expert_outputs(pkg, oracle, cfg, mine)
        # Owner side: one fp32 partial per (token, this owner), for every global token.
        partials = {t: owner_partial(contrib, idx, t, rank, world, e_rank, placement) for t in range(T_global)}
        gathered = [None] * world
        dist.all_gather_object(gathered, partials)
        # Source side: combine the own tokens' partials in ascending owner order.
        lo, hi = ep.token_range(T_global, world, rank)
        out = [ep_combine_bits(oracle, [gathered[d][t] for d in range(world)]) for t in range(lo, hi)]
        outs = [None] * world
        dist.all_gather_object(outs, out)
        if rank == 0:
            got = np.stack([r for o in outs for r in o])
            allx = sorted({int(g) for g in idx.ravel() if int(g) in own})
            full = per_expert_outputs(pkg, oracle, cfg, allx)
            tokens = list(range(T_global))
            np.testing.assert_array_equal(got, ep_expected_bits(oracle, full, idx, tokens, world, e_rank, placement))
            ref = layer_oracle_bits(oracle, full, idx, tokens, world, e_rank, placement)
            r = oracle.check_tolerance(ref, got)
            assert r["bad"] == 0, r
    finally:
        dist.destroy_process_group()
