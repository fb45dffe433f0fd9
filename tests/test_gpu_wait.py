"""The bounded device waits of the tensor-core kernels (tc_common.cuh), run to expiry for real:
a probe kernel waits on an mbarrier that nothing completes, with a limit of about a millisecond.
The wait must give up, the host must read FLETCHER_ERR_DEVICE_WAIT, and the context must stay
usable.  No fault and no hang is involved."""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu

ERR_DEVICE_WAIT = 5


@pytest.fixture(scope="module")
def be():
    import build
    build.build()
    import fletcher
    yield fletcher.Backend(0)


@pytest.mark.parametrize("sleeping", [0, 1])
def test_expired_wait_is_reported_and_context_survives(be, sleeping):
    import fletcher as fl
    with pytest.raises(fl.FletcherError) as e:
        be.check(fl.lib().Cuda_Debug_WaitTimeoutProbe(be.ctx, 2_000_000, sleeping))
    assert e.value.code == ERR_DEVICE_WAIT
    assert "bounded wait expired (device code 1)" in str(e.value)
    # The flag was cleared by the report, and the context still runs work.
    be.synchronize()
    x = np.arange(4 * 128, dtype=np.float32).reshape(4, 128) / 100
    t = be.new_tensor(4, 128, x)
    np.testing.assert_array_equal(t.to_host(), x)
    be.synchronize()


def test_probe_rejects_bad_limits(be):
    import fletcher as fl
    assert fl.lib().Cuda_Debug_WaitTimeoutProbe(be.ctx, 0, 0) != 0
    assert fl.lib().Cuda_Debug_WaitTimeoutProbe(be.ctx, 10**12, 0) != 0
    be.synchronize()
