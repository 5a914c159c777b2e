"""Generate the golden fixtures of tests/golden/ by running the REAL reference oracle.

Run in the build container (where the reference checkout is mounted), from the repo root:
    python tests/golden/make_golden.py --reference PATH_OF_THE_REFERENCE_CHECKOUT
Nothing at test or benchmark time runs this script or reads the reference.

For each case the inputs come from the package's seeded CPU generator (bit-identical to the
GPU generator); the script stores
  * ``out_bf16``    uint16 [T, 7168]  reference.run(**inputs) as bf16 bits (full cases only),
  * ``topk_sorted`` uint8  [T, 8]     the reference's top-8 expert ids per token, ascending,
                                       captured from its torch.topk(k=8) call (moe_ref.py:101),
  * ``inputs_sha256``                  digests of every generated input tensor, so a test can
                                       detect any drift of the generator,
  * the configuration fields.
Routing-only cases stop the reference right after its top-8 selection.

``ref_t*`` cases use the reference's OWN test generator instead (``moe_layer.build_moe_inputs``
on the CPU, ``seed = T`` as ``tests/test_moe.py:44`` calls it: uniform e4m3 values, U(0.01,
0.11) scales, zero bias, routed_scaling_factor 1) at the reference test's token counts up to
256 (``tests/test_moe.py:18``). They store the same fields; ``tests/ref_inputs.py`` restates
that generator and must reproduce the stored digests.
"""
from __future__ import annotations

import argparse
import hashlib
import importlib
import json
import os
import sys

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))
REPO = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, REPO)
pkg = importlib.import_module("15642_moe_b200")

# (name, config index, overrides, routing_only)
CASES = [
    ("cfg0_t16", 0, {}, False),
    ("cfg1_t64", 1, {}, False),
    ("t1_seed3", 0, {"T": 1, "seed": 3}, False),          # no local expert: all-zero output
    ("t1_seed1", 0, {"T": 1, "seed": 1}, False),          # two local experts (2 and 17)
    ("t4_off224", 0, {"T": 4, "seed": 7, "local_expert_offset": 224}, False),
    ("route_cfg2_t4096", 2, {}, True),
    ("route_cfg4_t16384_skew", 4, {"E_local": 32}, True),
]


# The reference test's token counts that fit a committed fixture (T = 2048 and up: the
# oracle-parity tests on the GPU cover those sizes).
REF_CASES = [1, 4, 32, 64, 256]


class _Stop(Exception):
    pass


def digests(inputs: dict) -> dict:
    out = {}
    for k, v in inputs.items():
        if isinstance(v, torch.Tensor):
            out[k] = hashlib.sha256(v.contiguous().view(torch.uint8).numpy().tobytes()).hexdigest()
    return out


def run_reference(reference, inputs: dict, routing_only: bool):
    captured = []
    orig = torch.topk

    def spy(input, k, dim=None, largest=True, sorted=True, **kw):
        r = orig(input, k, dim=dim, largest=largest, sorted=sorted, **kw)
        if k == 8:
            captured.append(r.indices.clone())
            if routing_only:
                raise _Stop()
        return r

    torch.topk = spy
    try:
        out = reference.run(**inputs)
    except _Stop:
        out = None
    finally:
        torch.topk = orig
    idx = np.sort(captured[-1].numpy().astype(np.int64), axis=1).astype(np.uint8)
    return out, idx


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", required=True, help="root of the reference checkout (contains reference/)")
    ap.add_argument("--only", default=None)
    args = ap.parse_args()
    sys.path.insert(0, args.reference)
    reference = importlib.import_module("reference")
    torch.set_num_threads(os.cpu_count())
    for name, ci, over, routing_only in CASES:
        if args.only and name != args.only:
            continue
        cfg = pkg.CONFIGS[ci].with_(**over)
        inputs = pkg.make_inputs(cfg, "cpu")
        dig = digests(inputs)
        out, idx = run_reference(reference, inputs, routing_only)
        rec = dict(topk_sorted=idx, config=json.dumps(cfg.__dict__), inputs_sha256=json.dumps(dig))
        if out is not None:
            rec["out_bf16"] = out.contiguous().view(torch.int16).numpy().view(np.uint16)
        np.savez_compressed(os.path.join(HERE, f"{name}.npz"), **rec)
        print(name, "T=%d" % cfg.T, "routing_only" if routing_only else "full", flush=True)
    moe_layer = importlib.import_module("moe_layer")
    sys.path.insert(0, os.path.dirname(HERE))
    ref_inputs = importlib.import_module("ref_inputs")
    for T in REF_CASES:
        name = f"ref_t{T}"
        if args.only and name != args.only:
            continue
        inputs = moe_layer.build_moe_inputs(T, device="cpu", seed=T)
        dig = digests(inputs)
        mine = ref_inputs.digests(ref_inputs.build_moe_inputs(T, T))
        assert mine == dig, f"tests/ref_inputs.py does not reproduce the reference generator at T={T}"
        out, idx = run_reference(reference, inputs, False)
        cfg = dict(generator="reference moe_layer.build_moe_inputs (cpu)", T=T, seed=T,
                   local_expert_offset=0, routed_scaling_factor=1.0)
        np.savez_compressed(os.path.join(HERE, f"{name}.npz"), topk_sorted=idx, config=json.dumps(cfg),
                            inputs_sha256=json.dumps(dig),
                            out_bf16=out.contiguous().view(torch.int16).numpy().view(np.uint16))
        print(name, "T=%d" % T, "full (reference generator)", flush=True)


if __name__ == "__main__":
    main()
