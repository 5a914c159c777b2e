"""On-disk format of packed expert weights, so a server loads them ready for moe_forward
instead of repacking at start-up (the counterpart of the reference's in-process packed-weight
cache, moe_layer.py:77-95, made persistent).

File layout (little-endian):
  magic      8 bytes   b"MOEB200P"
  header     4 bytes   length H of the JSON header that follows
  JSON       H bytes   {"version", "layout", "E_local", "local_expert_offset", "sections":
                        [{"name", "dtype", "shape", "offset", "nbytes", "crc32"}, ...]}
  sections   each at its 4096-byte aligned offset: w13_packed (uint8 [E, 16, 56, 256, 128]),
             w13_scale (fp32 [E, 32, 56]), w2_packed (uint8 [E, 28, 16, 256, 128]),
             w2_scale (fp32 [E, 56, 16])
The packed sections are this library's shared-memory tile images (pack_w13 / pack_w2); `layout`
names that layout and a reader refuses any other.
"""
from __future__ import annotations

import json
import os
import zlib

import numpy as np
import torch

from .layer import G1_BLOCKS, H_BLOCKS, I_BLOCKS, W13_PACKED_SHAPE, W2_PACKED_SHAPE, _check

MAGIC = b"MOEB200P"
VERSION = 1
LAYOUT = "sm100-sw128-kmajor-v1"
ALIGN = 4096
SECTIONS = ("w13_packed", "w13_scale", "w2_packed", "w2_scale")


def _expected_shapes(E: int) -> dict:
    return {"w13_packed": (E, *W13_PACKED_SHAPE), "w13_scale": (E, G1_BLOCKS, H_BLOCKS),
            "w2_packed": (E, *W2_PACKED_SHAPE), "w2_scale": (E, H_BLOCKS, I_BLOCKS)}


def _as_numpy(t: torch.Tensor, dtype) -> np.ndarray:
    t = t.detach().contiguous()
    if t.is_cuda:
        t = t.cpu()
    return t.view(torch.uint8).numpy().view(dtype) if dtype == np.uint8 else t.to(torch.float32).numpy()


def save_packed(path: str, w13_packed: torch.Tensor, w13_scale: torch.Tensor, w2_packed: torch.Tensor,
                w2_scale: torch.Tensor, local_expert_offset: int = 0) -> None:
    """Write packed weights (from pack_w13 / pack_w2) and their fp32 scales to `path`."""
    E = int(w13_packed.shape[0])
    arrays = {"w13_packed": _as_numpy(w13_packed, np.uint8), "w13_scale": _as_numpy(w13_scale, np.float32),
              "w2_packed": _as_numpy(w2_packed, np.uint8), "w2_scale": _as_numpy(w2_scale, np.float32)}
    for name, shape in _expected_shapes(E).items():
        _check(tuple(arrays[name].shape) == shape, f"{name} must have shape {shape}")
    sections, off = [], 0
    for name in SECTIONS:
        a = np.ascontiguousarray(arrays[name])
        sections.append({"name": name, "dtype": str(a.dtype), "shape": list(a.shape), "nbytes": int(a.nbytes),
                         "crc32": zlib.crc32(memoryview(a).cast("B")) & 0xFFFFFFFF})
    header = {"version": VERSION, "layout": LAYOUT, "E_local": E,
              "local_expert_offset": int(local_expert_offset), "sections": sections}
    # Offsets depend on the header length; fix the header size with generous digit widths.
    for sec in sections:
        sec["offset"] = 0
    blob = json.dumps(header).encode()
    base = ((len(MAGIC) + 4 + len(blob) + 64 * len(sections) + ALIGN - 1) // ALIGN) * ALIGN
    off = base
    for sec in sections:
        sec["offset"] = off
        off = ((off + sec["nbytes"] + ALIGN - 1) // ALIGN) * ALIGN
    blob = json.dumps(header).encode()
    _check(len(MAGIC) + 4 + len(blob) <= base, "header too large")
    tmp = path + ".tmp"
    with open(tmp, "wb") as f:
        f.write(MAGIC)
        f.write(len(blob).to_bytes(4, "little"))
        f.write(blob)
        for sec in sections:
            f.seek(sec["offset"])
            f.write(memoryview(np.ascontiguousarray(arrays[sec["name"]])).cast("B"))
        f.truncate(off)
    os.replace(tmp, path)


def read_header(path: str) -> dict:
    with open(path, "rb") as f:
        magic = f.read(len(MAGIC))
        _check(magic == MAGIC, f"{path}: not a packed-weight file")
        n = int.from_bytes(f.read(4), "little")
        header = json.loads(f.read(n))
    _check(header.get("version") == VERSION, f"{path}: unsupported version {header.get('version')}")
    _check(header.get("layout") == LAYOUT, f"{path}: packed layout {header.get('layout')!r} is not {LAYOUT!r}")
    return header


def load_packed(path: str, device: str | torch.device = "cuda", verify: bool = True) -> dict:
    """Read a file written by save_packed: {"w13_packed", "w13_scale", "w2_packed", "w2_scale",
    "E_local", "local_expert_offset"} with the tensors on `device`, ready for moe_forward.
    `verify` checks every section's CRC32."""
    header = read_header(path)
    E = int(header["E_local"])
    shapes = _expected_shapes(E)
    size = os.path.getsize(path)
    out = {"E_local": E, "local_expert_offset": int(header["local_expert_offset"])}
    for sec in header["sections"]:
        name = sec["name"]
        _check(name in shapes and tuple(sec["shape"]) == shapes[name], f"{path}: bad section {name}")
        _check(sec["offset"] + sec["nbytes"] <= size, f"{path}: section {name} is truncated")
        dtype = np.dtype(sec["dtype"])
        a = np.memmap(path, dtype=dtype, mode="r", offset=sec["offset"], shape=tuple(sec["shape"]))
        if verify:
            _check(zlib.crc32(memoryview(np.ascontiguousarray(a)).cast("B")) & 0xFFFFFFFF == sec["crc32"],
                   f"{path}: section {name} fails its checksum")
        t = torch.from_numpy(np.array(a))
        out[name] = t.to(device) if torch.device(device).type != "cpu" else t
    _check(all(n in out for n in SECTIONS), f"{path}: missing sections")
    return out
