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


if __name__ == "__main__":
    main()
