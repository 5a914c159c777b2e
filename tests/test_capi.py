"""The C ABI library loads without a GPU, exports every symbol include/moe_b200.h declares,
and rejects bad arguments on the host (no device work is issued by these calls)."""
import ctypes
import os
import re

import pytest

HEADER = os.path.join(os.path.dirname(os.path.dirname(__file__)), "include", "moe_b200.h")


def declared_functions():
    text = open(HEADER).read()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(moe_[a-z0-9_]+)\s*\(", text)))


def test_header_declares_the_reference_entry_points():
    names = declared_functions()
    for n in ("moe_pack_w13", "moe_pack_w2", "moe_forward"):
        assert n in names


def test_library_exports_every_declared_symbol(pkg):
    from importlib import import_module
    native = import_module("15642_moe_b200._native")
    lib = native.cuda_lib()
    for name in declared_functions():
        assert hasattr(lib, name), name
        assert name in native.CUDA_SIGNATURES, name


def test_sizes(pkg):
    native = __import__("importlib").import_module("15642_moe_b200._native")
    lib = native.cuda_lib()
    assert lib.moe_pack_w13_bytes(32) == 32 * 4096 * 7168
    assert lib.moe_pack_w2_bytes(32) == 32 * 7168 * 2048
    assert lib.moe_pack_w13_bytes(0) == 0
    ws = lib.moe_forward_workspace_bytes(64, 32)
    assert ws > 0 and lib.moe_forward_workspace_bytes(4096, 32) > ws
    lay = native.workspace_layout(64, 32)
    assert lay["total"] == ws
    offs = [v for k, v in lay.items()]
    assert offs == sorted(offs) and all(v % 1024 == 0 for v in offs)
    # expert outputs are stored densely, one fp32 row per local route (at most 8 per token)
    assert lay["partial"] + 64 * 8 * 7168 * 4 <= lay["total"]
    # SwiGLU tiles are padded per expert: every token routed to 8 local experts, each tile partial
    tiles = (64 * 8 + 32 * 127 + 127) // 128
    assert lay["c_lo"] - lay["c_hi"] >= tiles * 16 * 128 * 128
    # per-expert slot lists hold up to T routes each
    assert lay["route_w"] - lay["route_token"] >= 32 * 64 * 4


def test_host_side_argument_errors(pkg):
    native = __import__("importlib").import_module("15642_moe_b200._native")
    lib = native.cuda_lib()
    null = None
    rc = lib.moe_forward(null, null, null, null, null, null, null, null, 1.0, 0, 16, 0, null, null, 0, null)
    assert rc == 1 and b"E_local" in lib.moe_last_error()
    rc = lib.moe_forward(null, null, null, null, null, null, null, null, 1.0, 0, -1, 32, null, null, 0, null)
    assert rc == 1 and b"hidden must be [T, 7168]" in lib.moe_last_error()
    # T == 0 is a no-op
    assert lib.moe_forward(null, null, null, null, null, null, null, null, 1.0, 0, 0, 32, null, null, 0, null) == 0
    rc = lib.moe_forward(null, null, null, null, null, null, null, null, 1.0, 0, 4, 32, null, null, 0, null)
    assert rc == 1 and b"null" in lib.moe_last_error()
    buf = (ctypes.c_uint8 * 64)()
    p = ctypes.addressof(buf)
    p16 = (p + 15) & ~15
    rc = lib.moe_forward(p16, p16, p16, p16, p16, p16, p16, p16, 1.0, 0, 4, 32, p16, p16, 16, null)
    assert rc == 3 and b"workspace too small" in lib.moe_last_error()
    rc = lib.moe_forward(p16 + 1, p16, p16, p16, p16, p16, p16, p16, 1.0, 0, 4, 32, p16, p16, 16, null)
    assert rc == 1 and b"aligned" in lib.moe_last_error()
    assert lib.moe_pack_w13(null, 0, null, null) == 1
    assert b"W13 must be [E_local, 4096, 7168]" in lib.moe_last_error()
    assert lib.moe_pack_w2(null, 300, null, null) == 1


def test_python_api_rejects_cpu_tensors(pkg):
    import torch
    w = torch.zeros((1, 4096, 7168), dtype=torch.float8_e4m3fn)
    with pytest.raises(RuntimeError, match="CUDA tensor"):
        pkg.pack_w13(w)
    with pytest.raises(RuntimeError, match="W13 must be"):
        pkg.pack_w13(torch.zeros((1, 4096, 7000), dtype=torch.float8_e4m3fn))
    with pytest.raises(RuntimeError, match="FP8"):
        pkg.pack_w2(torch.zeros((1, 7168, 2048), dtype=torch.float32))


def test_workspace_alignment_is_checked(pkg):
    """The workspace must be 256-byte aligned (kernels store 32-byte vectors into it); a pointer
    that is only 16-byte aligned is refused on the host before anything is launched."""
    native = __import__("importlib").import_module("15642_moe_b200._native")
    lib = native.cuda_lib()
    p = 0x10000010   # host-side fake address: 16-byte aligned, not 256; nothing is dereferenced
    rc = lib.moe_forward(p, p, p, p, p, p, p, p, 2.5, 0, 16, 32, p, p, 1 << 40, None)
    assert rc == 1 and b"256-byte" in lib.moe_last_error()


@pytest.mark.parametrize("T,E", [(0, 32), (1, 1), (1, 32), (7, 3), (64, 32), (1000, 8), (1024, 32),
                                 (4096, 32), (16384, 256), (65536, 32), (65536, 256)])
def test_workspace_layout_covers_every_region(pkg, T, E):
    """Each scratch region holds the largest index its kernels address, for any routing: the
    per-expert 128-row tiles (each active expert pads its rows up to a multiple of 128), the dense
    route rows of `partial` in blocks of 128 rows x 224 groups of 32 floats, and the slot lists.
    Regions start on 1024-byte boundaries, so 256-bit stores at 32-byte offsets inside them stay
    aligned on a 256-byte aligned workspace."""
    import random
    native = __import__("importlib").import_module("15642_moe_b200._native")
    lay = native.workspace_layout(T, E)
    order = ["counts", "dense_base", "topk_idx", "topk_w", "token_nr", "token_route", "route_token",
             "route_w", "a_tiled", "a_scale", "c_hi", "c_lo", "c_scale", "partial", "tile_ready", "total"]
    offs = [lay[k] for k in order]
    assert offs == sorted(offs) and all(v % 1024 == 0 for v in offs)
    size = {k: lay[order[i + 1]] - lay[k] for i, k in enumerate(order[:-1])}
    kmax = min(E, 8)
    routes = T * kmax
    active = min(routes, E)
    tiles = (routes + active * 127 + 127) // 128
    need = {
        "counts": 4 * E, "dense_base": 4 * (E + 1), "topk_idx": 4 * 8 * T, "topk_w": 4 * 8 * T,
        "token_nr": 4 * T, "token_route": 4 * 8 * T, "route_token": 4 * E * T, "route_w": 4 * E * T,
        "a_tiled": tiles * 56 * 128 * 128, "a_scale": 4 * tiles * 56 * 128,
        "c_hi": tiles * 16 * 128 * 128, "c_lo": tiles * 16 * 128 * 128, "c_scale": 4 * tiles * 16 * 128,
        "partial": 4 * ((routes + 127) // 128) * 128 * 7168, "tile_ready": 4 * (tiles + 1),
    }
    for k, n in need.items():
        assert size[k] >= n, (k, size[k], n)
    if routes:
        # The last float a route row can address (partial_offset of dense row routes - 1, column 7167).
        d, col = routes - 1, 7167
        last = ((d // 128 * 224 + (col >> 5)) * 128 + d % 128) * 32 + (col & 31)
        assert 4 * (last + 1) <= size["partial"]
    # Any split of the routes over the experts fits in the tiles the layout provides.
    rng = random.Random(T * 1000 + E)
    for _ in range(20):
        counts = [0] * E
        for _ in range(min(routes, 4096)):
            counts[rng.randrange(E)] += 1
        scale = routes / max(1, sum(counts))
        counts = [min(T, int(c * scale)) for c in counts]
        assert sum((c + 127) // 128 for c in counts) <= tiles


def test_output_overlapping_an_input_is_refused(pkg):
    """Output rows are written while inputs are still being read, so an output that overlaps an
    input or the workspace is refused on the host, before anything is launched (fake addresses:
    nothing is dereferenced)."""
    native = __import__("importlib").import_module("15642_moe_b200._native")
    lib = native.cuda_lib()
    T, E = 16, 32
    ws = lib.moe_forward_workspace_bytes(T, E)
    base = 1 << 36
    names = ["hidden", "hidden_scale", "w13", "w13_scale", "w2", "w2_scale", "logits", "bias", "ws"]
    sizes = [T * 7168, 4 * 56 * T, E * 4096 * 7168, 4 * E * 32 * 56, E * 7168 * 2048, 4 * E * 56 * 16,
             4 * T * 256, 4 * 256, ws]
    addr, a = {}, base
    for n, s in zip(names, sizes):
        addr[n] = a
        a += (s + 4095) // 4096 * 4096 + 4096
    out_free = a

    def call(out):
        v = addr
        return lib.moe_forward(v["hidden"], v["hidden_scale"], v["w13"], v["w13_scale"], v["w2"],
                               v["w2_scale"], v["logits"], v["bias"], 2.5, 0, T, E, out, v["ws"], ws, None)

    # Every case here is refused on the host: a call whose fake addresses passed every host check
    # would launch kernels on them where a GPU is present, so no such call is made.
    for n, s in zip(names, sizes):
        for out in (addr[n], addr[n] + s - 16, addr[n] - T * 7168 * 2 + 16):
            rc = call(out)
            assert rc == 1 and b"overlaps" in lib.moe_last_error(), (n, out - addr[n])
    assert out_free > addr["ws"] + ws                 # the layout above keeps the ranges apart
