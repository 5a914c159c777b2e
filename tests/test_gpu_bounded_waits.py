"""Bounded waits run out on purpose, on one GPU, without a fault: the wait limit is shortened
through the C ABI, a kernel waits on something nothing will ever signal, gives up after the
limit, reports its status bit and returns; the context stays usable (a forward right after
is bit-identical to one before). The limit and the status word are restored afterwards."""
import time

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu
SHORT_NS = 50_000_000          # 50 ms


@pytest.fixture
def short_limit(pkg):
    pkg.device_status(reset=True)
    old = pkg.wait_limit_ns()
    assert old == 2_000_000_000
    pkg.set_wait_limit_ns(SHORT_NS)
    assert pkg.wait_limit_ns() == SHORT_NS
    yield
    pkg.set_wait_limit_ns(old)
    assert pkg.wait_limit_ns() == old
    assert pkg.device_status(reset=True) == 0


def _forward_bits(pkg):
    inp = pkg.make_inputs(pkg.MoEConfig(T=16, seed=21), "cuda")
    return pkg.run(**inp).view(torch.int16).cpu().numpy()


def test_ep_barrier_gives_up_on_a_missing_rank(pkg, short_limit):
    native = pkg._native
    before = _forward_bits(pkg)
    buf = torch.zeros(256, dtype=torch.uint8, device="cuda")
    t0 = time.perf_counter()
    native.check(native.cuda_lib().moe_probe_ep_barrier_timeout(buf.data_ptr(), torch.cuda.current_stream().cuda_stream))
    status = pkg.device_status(reset=True)
    dt = time.perf_counter() - t0
    assert status == native.ST_EP_TIMEOUT, status
    assert dt < 1.0, dt                          # gave up after ~50 ms, not the 2 s default
    flags = buf.view(torch.int32).cpu().numpy()
    assert flags[0] == 1 and flags[16] == 1 and flags[17] == 0   # epoch 1, own flag set, rank 1 never
    np.testing.assert_array_equal(_forward_bits(pkg), before)


@pytest.mark.parametrize("who", [1, 2, 4])
def test_mbarrier_wait_gives_up(pkg, short_limit, who):
    native = pkg._native
    aborted = torch.full((1,), -1, dtype=torch.int32, device="cuda")
    t0 = time.perf_counter()
    native.check(native.cuda_lib().moe_probe_mbar_timeout(who, aborted.data_ptr(), torch.cuda.current_stream().cuda_stream))
    status = pkg.device_status(reset=True)
    dt = time.perf_counter() - t0
    assert status == who and int(aborted.item()) == 1, (status, aborted)
    assert dt < 1.0, dt


def test_wait_limit_range_checked(pkg):
    with pytest.raises(pkg.MoEError, match="limit"):
        pkg.set_wait_limit_ns(10)
    assert pkg.wait_limit_ns() == 2_000_000_000
