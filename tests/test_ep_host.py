"""Host side of the expert-parallel layer, on the CPU: the token / expert partition, the C ABI's
argument checks (no device work), and a two-rank gloo run of the whole data flow (handle
exchange, owner-side partials, exchange, source-side combine) checked against the
single-rounding layer oracle."""
import importlib
import socket

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
    # source side's local route counts and reserved slot bases (256 ints each).
    assert lib.moe_ep_workspace_bytes(8, 512, 32) == lib.moe_forward_workspace_bytes(4096, 32) + 2048
    ctx = ctypes.c_void_p()
    handle = ctypes.create_string_buffer(64)
    assert lib.moe_ep_create(2, 2, 16, 128, ctypes.byref(ctx), handle) == 1
    assert b"rank" in lib.moe_last_error()
    assert lib.moe_ep_create(0, 9, 16, 16, ctypes.byref(ctx), handle) == 1
    assert b"world" in lib.moe_last_error()
    assert lib.moe_ep_create(0, 2, 16, 129, ctypes.byref(ctx), handle) == 1
    assert b"e_rank" in lib.moe_last_error()
    assert ctx.value is None
    assert lib.moe_ep_forward(None, None, None, None, None, None, None, None, None, 1.0, 0, None,
                              None, 0, None) == 1
    assert b"not connected" in lib.moe_last_error()
    assert lib.moe_ep_destroy(None) == 0


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def test_two_rank_gloo_dataflow_matches_layer_oracle():
    """Full 256-expert layer over 2 ranks (128 experts each), 4 tokens split 2 + 2."""
    world = 2
    mp.start_processes(ep_helpers.gloo_worker, args=(world, _free_port(), 4, 128, 0), nprocs=world,
                       join=True, start_method="spawn")
