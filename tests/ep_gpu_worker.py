"""One rank of the multi-GPU expert-parallel parity run (launched by tests/test_gpu_ep.py under
torchrun, one process per GPU). Every case compares this rank's expert-parallel output with

  * the same layer computed on this GPU alone, slice by slice: for each owner d (ascending),
    moe_forward_f32 over all ranks' tokens with d's experts (local_expert_offset =
    d * e_rank), summed in fp32, rounded once, rows of this rank - bit for bit. Owner d's GEMMs
    see exactly the routes that expert-parallel owner d receives, so both run the same tiles
    and the same schedule;
  * for the small case, the single-rounding CPU layer oracle, within the reference tolerance.

Prints EP_CASE_OK <name> per case; any mismatch raises (non-zero exit).
"""
from __future__ import annotations

import argparse
import datetime
import importlib
import os
import sys

import numpy as np
import torch
import torch.distributed as dist

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.dirname(HERE))
sys.path.insert(0, HERE)

import ep_helpers  # noqa: E402

pkg = importlib.import_module("15642_moe_b200")
ep_mod = importlib.import_module("15642_moe_b200.ep")


def bits(t: torch.Tensor) -> np.ndarray:
    return t.contiguous().view(torch.int16).cpu().numpy().view(np.uint16)


class Layer:
    """Every slice of the layer (packed) on this GPU, plus this rank's own slice."""

    def __init__(self, cfg, world, e_rank, device):
        self.slices = []
        for d in range(world):
            inp = pkg.make_inputs(cfg.with_(E_local=e_rank, local_expert_offset=d * e_rank), device)
            self.slices.append(dict(
                w13p=pkg.pack_w13(inp["gemm1_weights"]), w2p=pkg.pack_w2(inp["gemm2_weights"]),
                s13=inp["gemm1_weights_scale"].float().contiguous(),
                s2=inp["gemm2_weights_scale"].float().contiguous(), offset=d * e_rank))
            if d == 0:
                self.inp = inp
            del inp
        torch.cuda.synchronize()

    def tokens(self, ranges):
        """Rows of the global batch given as [(lo, hi), ...], concatenated in that order."""
        inp = self.inp
        cat = lambda t, dim: torch.cat([t.narrow(dim, lo, hi - lo) for lo, hi in ranges], dim).contiguous()
        return dict(hidden=cat(inp["hidden_states"], 0), hs=cat(inp["hidden_states_scale"], 1).float(),
                    lg=cat(inp["routing_logits"], 0).float(),
                    b=inp["routing_bias"].float().reshape(-1).contiguous(),
                    rsf=float(inp["routed_scaling_factor"]))

    def reference(self, tok, lo, hi):
        """Rows [lo, hi) of the layer over all of `tok`'s tokens, slice by slice."""
        T = tok["hidden"].shape[0]
        acc = torch.zeros((T, 7168), dtype=torch.float32, device=tok["hidden"].device)
        if T > 0:
            for s in self.slices:
                acc += pkg.moe_forward(tok["hidden"], tok["hs"], s["w13p"], s["s13"], s["w2p"], s["s2"],
                                       tok["lg"], tok["b"], tok["rsf"], s["offset"], fp32_out=True)
        return acc[lo:hi].to(torch.bfloat16)

    def ep_forward(self, ctx, tok, rank):
        s = self.slices[rank]
        return ctx.forward(tok["hidden"], tok["hs"], s["w13p"], s["s13"], s["w2p"], s["s2"], tok["lg"],
                           tok["b"], tok["rsf"])


def check_equal(name, got, ref):
    g, r = bits(got), bits(ref)
    if not np.array_equal(g, r):
        bad = int((g != r).sum())
        raise AssertionError(f"{name}: {bad} of {g.size} bf16 values differ from the slice-by-slice layer")


def check_status(name):
    st = pkg.device_status(reset=True)
    if st != 0:
        raise AssertionError(f"{name}: device status {st}")


def case_layer(rank, world, device, T_global, e_rank, seed, skew=False, epochs=2):
    base = pkg.CONFIGS[4] if skew else pkg.CONFIGS[3]
    cfg = base.with_(T=T_global, seed=seed)
    layer = Layer(cfg, world, e_rank, device)
    lo, hi = ep_mod.token_range(T_global, world, rank)
    ref = layer.reference(layer.tokens([(0, T_global)]), lo, hi)
    tok = layer.tokens([(lo, hi)])
    with ep_mod.ExpertParallel(t_rank_max=hi - lo, e_rank=e_rank, device=device) as ctx:
        for _ in range(epochs):               # repeated epochs reuse every buffer
            out = layer.ep_forward(ctx, tok, rank)
            torch.cuda.synchronize()
            check_equal(f"layer T={T_global} e_rank={e_rank}", out, ref)
    check_status("layer")
    return layer, lo, hi, out


def case_oracle(rank, world, device):
    from oracle import moe_oracle as oracle
    T_global, e_rank = 4, 256 // world
    layer, lo, hi, out = case_layer(rank, world, device, T_global, e_rank, seed=0, epochs=1)
    cfg = pkg.CONFIGS[3].with_(T=T_global)
    cinp = pkg.make_inputs(cfg.with_(E_local=1), "cpu")
    idx, _ = oracle.route(cinp["routing_logits"].numpy(), cinp["routing_bias"].float().numpy(),
                          cfg.routed_scaling_factor)
    mine = sorted({int(g) for t in range(lo, hi) for g in idx[t]})
    contrib = ep_helpers.per_expert_outputs(pkg, oracle, cfg, mine)
    tokens = list(range(lo, hi))
    ref = ep_helpers.layer_oracle_bits(oracle, contrib, idx, tokens, world, e_rank)
    r = oracle.check_tolerance(ref, bits(out))
    if r["bad"] != 0:
        raise AssertionError(f"oracle: {r}")
    emu = ep_helpers.ep_expected_bits(oracle, contrib, idx, tokens, world, e_rank)
    rr = oracle.check_tolerance(emu, bits(out))
    if rr["bad"] != 0:
        raise AssertionError(f"oracle (expert-parallel rounding): {rr}")


def case_ragged(rank, world, device):
    """Token counts that differ per rank and per epoch, zeros included, over one context."""
    e_rank = 32
    plan = [[5, 0], [0, 7], [33, 17], [64, 64], [1, 1]]
    t_max = 64
    cfg = pkg.CONFIGS[3].with_(T=t_max * world, seed=5)
    layer = Layer(cfg, world, e_rank, device)
    with ep_mod.ExpertParallel(t_rank_max=t_max, e_rank=e_rank, device=device) as ctx:
        for ep_i, counts in enumerate(plan):
            counts = [counts[r % len(counts)] for r in range(world)]
            ranges = [(r * t_max, r * t_max + counts[r]) for r in range(world)]
            mine = sum(counts[:rank])
            ref = layer.reference(layer.tokens(ranges), mine, mine + counts[rank])
            tok = layer.tokens([ranges[rank]])
            out = layer.ep_forward(ctx, tok, rank)
            torch.cuda.synchronize()
            check_equal(f"ragged epoch {ep_i}", out, ref)
    check_status("ragged")


def case_graph(rank, world, device):
    """Each rank captures its expert-parallel forward in a CUDA graph and replays it with new
    tokens; every replay is a new epoch of the device-side barriers."""
    e_rank, t_max = 32, 64
    cfg = pkg.CONFIGS[3].with_(T=t_max * world, seed=11)
    layer = Layer(cfg, world, e_rank, device)
    s = layer.slices[rank]
    lo = rank * t_max
    tok = layer.tokens([(lo, lo + t_max)])
    st = {k: tok[k].clone() for k in ("hidden", "hs", "lg")}
    out = torch.empty((t_max, 7168), dtype=torch.bfloat16, device=device)
    with ep_mod.ExpertParallel(t_rank_max=t_max, e_rank=e_rank, device=device) as ctx:
        call = lambda: ctx.forward(st["hidden"], st["hs"], s["w13p"], s["s13"], s["w2p"], s["s2"], st["lg"],
                                   tok["b"], tok["rsf"], out=out)
        call()
        torch.cuda.synchronize()
        dist.barrier()
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g):
            call()
        for seed in (12, 13, 14):
            other = Layer.__new__(Layer)
            other.inp = pkg.make_inputs(cfg.with_(seed=seed, E_local=1), device)
            other.slices = layer.slices
            new = other.tokens([(lo, lo + t_max)])
            for k in ("hidden", "hs", "lg"):
                st[k].copy_(new[k])
            dist.barrier()
            g.replay()
            torch.cuda.synchronize()
            everyone = other.tokens([(0, t_max * world)])
            everyone["b"] = tok["b"]                    # the captured call keeps the first bias
            ref = other.reference(everyone, lo, lo + t_max)
            check_equal(f"graph replay seed {seed}", out, ref)
        del g
    check_status("graph")


def case_placement(rank, world, device):
    """Full layer with an interleaved placement (rank d owns the experts g with g % world == d).
    Reference: each expert's fp32 contribution over all tokens (moe_forward_f32 with that expert
    alone); owner d's partial is their sum in ascending expert order, the output the sum of the
    partials in ascending owner order, rounded once."""
    T_global, e_rank = 256, 256 // world
    cfg = pkg.CONFIGS[3].with_(T=T_global, seed=21)
    placement = [[g for g in range(256) if g % world == d] for d in range(world)]
    inp = pkg.make_inputs(cfg.with_(E_local=1), device)
    allt = dict(hidden=inp["hidden_states"], hs=inp["hidden_states_scale"].float().contiguous(),
                lg=inp["routing_logits"].float().contiguous(), b=inp["routing_bias"].float().reshape(-1).contiguous(),
                rsf=float(inp["routed_scaling_factor"]))
    partial = []
    for d in range(world):
        acc = torch.zeros((T_global, 7168), dtype=torch.float32, device=device)
        for g in placement[d]:
            w = pkg.make_weights(cfg, [g], device)
            acc += pkg.moe_forward(allt["hidden"], allt["hs"], pkg.pack_w13(w["gemm1_weights"]),
                                   w["gemm1_weights_scale"], pkg.pack_w2(w["gemm2_weights"]),
                                   w["gemm2_weights_scale"], allt["lg"], allt["b"], allt["rsf"], g, fp32_out=True)
        partial.append(acc)
    total = torch.zeros_like(partial[0])
    for p_ in partial:
        total += p_
    lo, hi = ep_mod.token_range(T_global, world, rank)
    ref = total[lo:hi].to(torch.bfloat16)
    mine = pkg.make_weights(cfg, placement[rank], device)
    with ep_mod.ExpertParallel(t_rank_max=hi - lo, e_rank=e_rank, device=device, placement=placement) as ctx:
        out = ctx.forward(allt["hidden"][lo:hi].contiguous(), allt["hs"][:, lo:hi].contiguous(),
                          pkg.pack_w13(mine["gemm1_weights"]), mine["gemm1_weights_scale"],
                          pkg.pack_w2(mine["gemm2_weights"]), mine["gemm2_weights_scale"],
                          allt["lg"][lo:hi].contiguous(), allt["b"], allt["rsf"])
        torch.cuda.synchronize()
    check_equal("interleaved placement", out, ref)
    check_status("placement")


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--cases", default="oracle,ragged,weak,layer")
    args = ap.parse_args()
    rank, world = int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"])
    local = int(os.environ.get("LOCAL_RANK", rank))
    torch.cuda.set_device(local)
    device = torch.device("cuda", local)
    dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300), device_id=device)
    try:
        for name in args.cases.split(","):
            if name == "oracle":
                case_oracle(rank, world, device)
            elif name == "ragged":
                case_ragged(rank, world, device)
            elif name == "weak":             # the benchmark's layer: 32 experts per rank
                case_layer(rank, world, device, 4096, 32, seed=0)
            elif name == "layer":            # configuration 3: T = 8192, 256 / world experts each
                case_layer(rank, world, device, 8192, 256 // world, seed=0)
            elif name == "placement":
                case_placement(rank, world, device)
            elif name == "graph":
                case_graph(rank, world, device)
            elif name == "skew":             # configuration 4's skewed routing, 256 / world each
                case_layer(rank, world, device, 16384 if world == 8 else 4096, 256 // world, seed=0,
                           skew=True)
            else:
                raise ValueError(name)
            torch.cuda.empty_cache()
            dist.barrier()
            print(f"EP_CASE_OK {name} rank={rank}", flush=True)
    finally:
        dist.barrier()
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
