"""Build recipe for the reference's own CUDA extension, the GPU baseline - TEST INFRASTRUCTURE.

Compiles the reference's ``kernels/moe.cu`` unchanged, from where it lies in the reference
checkout, the way its own loader does (``moe_layer.py:31-43``: ``torch.utils.cpp_extension.load``
with ``-O3 --use_fast_math -arch=sm_{major}{minor}``; a B200 reports compute capability 10.0,
so ``-arch=sm_100``). The module (pybind name ``moe_fused_ref``; exports ``pack_w13``,
``pack_w2``, ``moe_forward`` as ``kernels/moe.cu:902-909``) lands in ``oracle/_ref/``, which
is git-ignored and travels to the GPU box with the other built libraries. Nothing of the
reference's source is copied into this repository.

Only ``bench.py``'s baseline leg (``ref_cuda``) and ``tests/`` load it, as the comparison arm;
the product never does.

    python -m oracle.build_ref [--reference PATH]      # default PATH: the reference checkout
"""
from __future__ import annotations

import argparse
import importlib.util
import os
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
OUT_DIR = os.path.join(HERE, "_ref")
NAME = "moe_fused_ref"
DEFAULT_REFERENCE = os.environ.get("MOE_REFERENCE_DIR", "/root/reference")


def so_path() -> str:
    return os.path.join(OUT_DIR, NAME + ".so")


def build(reference: str = DEFAULT_REFERENCE, verbose: bool = False) -> str:
    """Compile ``<reference>/kernels/moe.cu`` into ``oracle/_ref/moe_fused_ref.so``."""
    src = os.path.join(reference, "kernels", "moe.cu")
    if not os.path.exists(src):
        raise FileNotFoundError(f"reference CUDA source not found: {src}")
    from torch.utils import cpp_extension
    os.makedirs(OUT_DIR, exist_ok=True)
    # The reference's flags; an explicit -arch flag makes cpp_extension add no -gencode of its own.
    cpp_extension.load(name=NAME, sources=[src], build_directory=OUT_DIR, verbose=verbose,
                       extra_cuda_cflags=["-O3", "--use_fast_math", "-arch=sm_100"])
    return so_path()


def load():
    """Import the prebuilt module from ``oracle/_ref`` (no compilation; torch must be importable)."""
    import torch  # noqa: F401  (the extension links against torch's libraries)
    path = so_path()
    if not os.path.exists(path):
        raise FileNotFoundError(f"{path} is missing: run python -m oracle.build_ref where the reference is present")
    spec = importlib.util.spec_from_file_location(NAME, path)
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


if __name__ == "__main__":
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", default=DEFAULT_REFERENCE)
    ap.add_argument("-v", action="store_true")
    a = ap.parse_args()
    print(build(a.reference, verbose=a.v))
    sys.exit(0)
