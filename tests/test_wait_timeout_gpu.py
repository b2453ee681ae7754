"""Failure detection without a GPU fault: a kernel whose mbarrier wait can
never complete (nothing arrives) gives up after its poll limit, records the
expired-wait code in the device error word and returns; the host reads it
(DHDeviceError) and the context stays usable.  The same give-up path bounds
every pipeline wait of the GEMM and head kernels; the attention kernel's
suspending waits give up after a wall-time limit, checked the same way."""

import pytest

pytestmark = pytest.mark.gpu


def test_expired_wait_is_reported_and_the_context_survives(cuda):
    torch = cuda
    from diffusionhard_b200 import _lib

    _lib.check_device_error()  # start clean
    done = torch.full((1,), 7, dtype=torch.int32, device="cuda")
    # a wait that completes: its single arrival is made
    _lib.call("dh_wait_selftest", 4096, 1, done.data_ptr(), None)
    assert int(done.item()) == 1
    _lib.check_device_error()
    # a wait on a barrier nothing arrives on: gives up, reports code 1
    _lib.call("dh_wait_selftest", 4096, 0, done.data_ptr(), None)
    assert int(done.item()) == 0
    with pytest.raises(_lib.DHDeviceError) as err:
        _lib.check_device_error()
    assert err.value.code == 1
    _lib.check_device_error()  # the word was cleared by the read above
    # the context is still usable: the same kernel and a library op run normally
    _lib.call("dh_wait_selftest", 4096, 1, done.data_ptr(), None)
    assert int(done.item()) == 1
    assert float((torch.ones(1024, device="cuda") * 2).sum().item()) == 2048.0
    _lib.check_device_error()


def test_expired_suspending_wait_is_reported(cuda):
    """The attention kernel's waits sleep on the mbarrier and are bounded by
    wall time: a wait nothing completes gives up after its limit (here 20 ms)
    with the same code, and a completed one returns at once."""
    torch = cuda
    import time

    from diffusionhard_b200 import _lib

    _lib.check_device_error()
    done = torch.full((1,), 7, dtype=torch.int32, device="cuda")
    _lib.call("dh_wait_suspend_selftest", 20_000_000, 1, done.data_ptr(), None)
    assert int(done.item()) == 1
    _lib.check_device_error()
    t0 = time.perf_counter()
    _lib.call("dh_wait_suspend_selftest", 20_000_000, 0, done.data_ptr(), None)
    assert int(done.item()) == 0
    assert time.perf_counter() - t0 >= 0.02
    with pytest.raises(_lib.DHDeviceError) as err:
        _lib.check_device_error()
    assert err.value.code == 1
    _lib.call("dh_wait_suspend_selftest", 20_000_000, 1, done.data_ptr(), None)
    assert int(done.item()) == 1
    _lib.check_device_error()


def test_selftest_argument_checks(cuda):
    from diffusionhard_b200 import _lib

    assert _lib.raw("dh_wait_selftest", 4096, 1, None, None) == 100
    assert _lib.raw("dh_wait_selftest", 0, 1, 16, None) == 105
    assert _lib.raw("dh_wait_selftest", (1 << 16) + 1, 1, 16, None) == 105
    assert _lib.raw("dh_wait_suspend_selftest", 1000, 1, None, None) == 100
    assert _lib.raw("dh_wait_suspend_selftest", 0, 1, 16, None) == 105
    assert _lib.raw("dh_wait_suspend_selftest", 2_000_000_001, 1, 16, None) == 105
