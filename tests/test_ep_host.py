"""Host side of the expert-parallel layer, on the CPU: the token / expert partition, the C ABI's
argument checks (no device work), and a two-rank gloo run of the whole data flow (handle
exchange, owner-side partials, exchange, source-side combine) checked against the
single-rounding layer oracle."""
import importlib
import socket

import numpy as np
import pytest
import torch.multiprocessing as mp

import ep_helpers


@pytest.fixture(scope="module")
def ep():
    return importlib.import_module("15642_moe_b200.ep")


@pytest.mark.parametrize("T,world", [(0, 2), (1, 2), (7, 3), (4096, 8), (8192, 2), (5, 8)])
def test_token_partition_covers_every_row_once(ep, T, world):
    ranges = [ep.token_range(T, world, r) for r in range(world)]
    assert ranges[0][0] == 0 and ranges[-1][1] == T
    for (lo0, hi0), (lo1, _) in zip(ranges, ranges[1:]):
        assert hi0 == lo1 and lo0 <= hi0
    sizes = [hi - lo for lo, hi in ranges]
    assert max(sizes) - min(sizes) <= 1


@pytest.mark.parametrize("world,e_rank", [(1, 256), (2, 128), (4, 64), (8, 32), (2, 32)])
def test_expert_owner(ep, world, e_rank):
    for g in range(256):
        d = ep.owner_of(g, world, e_rank)
        if g < world * e_rank:
            lo, hi = ep.expert_range(d, e_rank)
            assert lo <= g < hi
        else:
            assert d == -1


def test_capi_rejects_bad_ep_shapes(pkg):
    import ctypes
    native = importlib.import_module("15642_moe_b200._native")
    lib = native.cuda_lib()
    assert lib.moe_ep_symmetric_bytes(9, 16, 32) == 0
    assert lib.moe_ep_symmetric_bytes(8, 16, 33) == 0          # 8 * 33 > 256 experts
    assert lib.moe_ep_symmetric_bytes(8, 8193, 32) == 0        # more than 65536 received rows
    assert lib.moe_ep_workspace_bytes(2, 0, 128) == 0
    small = lib.moe_ep_symmetric_bytes(2, 16, 128)
    assert 0 < small < lib.moe_ep_symmetric_bytes(2, 4096, 128)
    # The workspace is the single-GPU layout over world * t_rank_max received rows, plus the
    # source side (route counts, slot bases, route lists over all 256 experts).
    extra = lib.moe_ep_workspace_bytes(8, 512, 32) - lib.moe_forward_workspace_bytes(4096, 32)
    assert 256 * 512 * 8 <= extra <= 256 * 512 * 8 + 512 * 40 + 16 * 1024
    ctx = ctypes.c_void_p()
    handle = ctypes.create_string_buffer(64)
    assert lib.moe_ep_create(2, 2, 16, 128, None, ctypes.byref(ctx), handle) == 1
    assert b"rank" in lib.moe_last_error()
    assert lib.moe_ep_create(0, 9, 16, 16, None, ctypes.byref(ctx), handle) == 1
    assert b"world" in lib.moe_last_error()
    assert lib.moe_ep_create(0, 2, 16, 129, None, ctypes.byref(ctx), handle) == 1
    assert b"e_rank" in lib.moe_last_error()
    dup = (ctypes.c_int * 4)(3, 7, 3, 9)               # expert 3 listed twice
    assert lib.moe_ep_create(0, 2, 16, 2, dup, ctypes.byref(ctx), handle) == 1
    assert b"placement" in lib.moe_last_error()
    out_of_range = (ctypes.c_int * 2)(5, 256)
    assert lib.moe_ep_create(0, 1, 16, 2, out_of_range, ctypes.byref(ctx), handle) == 1
    assert ctx.value is None
    assert lib.moe_ep_forward(None, None, None, None, None, None, None, None, None, 1.0, 0, None,
                              None, 0, None) == 1
    assert b"not connected" in lib.moe_last_error()
    assert lib.moe_ep_destroy(None) == 0


def test_balanced_placement(ep):
    rng = np.random.default_rng(0)
    loads = rng.gamma(0.6, 100.0, 256)
    loads[[0, 1, 2, 3]] = 5000.0                     # four hot experts, contiguous at rank 0
    world, e_rank = 8, 32
    place = ep.balanced_placement(loads, world, e_rank)
    assert sorted(g for p in place for g in p) == list(range(256))
    assert all(len(p) == e_rank and p == sorted(p) for p in place)
    per = [loads[p].sum() for p in place]
    contiguous = [loads[r * e_rank:(r + 1) * e_rank].sum() for r in range(world)]
    assert max(per) < 0.5 * max(contiguous)
    # Largest-first greedy stays within 4/3 of the lower bound max(mean, largest single load).
    assert max(per) <= 4 / 3 * max(np.mean(per), loads.max())
    # A subset of the experts (fewer ranks than the full layer).
    sub = ep.balanced_placement(loads, 2, 32, experts=range(64))
    assert sorted(g for p in sub for g in p) == list(range(64))


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


@pytest.mark.parametrize("interleaved", [False, True], ids=["contiguous", "interleaved"])
def test_two_rank_gloo_dataflow_matches_layer_oracle(interleaved):
    """Full 256-expert layer over 2 ranks (128 experts each), 4 tokens split 2 + 2, with contiguous
    expert ranges or an interleaved placement."""
    world = 2
    mp.start_processes(ep_helpers.gloo_worker, args=(world, _free_port(), 4, 128, 0, interleaved), nprocs=world,
                       join=True, start_method="spawn")
