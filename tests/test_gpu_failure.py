"""Failure detection on the GPU without faulting it.

Every device-side wait in the library is bounded: after a limit it records
RV_ERR_TIMEOUT in the device error word and the kernel returns.  These tests
make such a wait run out on purpose -- an mbarrier phase no thread arrives
on, a flag no peer sets -- and check that the timeout is reported by
rv_device_status and that the device keeps working afterwards (the
reference's analogue: injected EBUSY driving the typed-error path,
crates/core/src/io/stream.rs:2794-2830, and its retryable error kinds,
stream.rs:58-70).  Nothing here traps, faults or hangs: each wait gives up
after about 10 ms of SM cycles.
"""
import time

import numpy as np
import pytest

torch = pytest.importorskip("torch")

pytestmark = pytest.mark.gpu

CYCLES = 20_000_000  # ~10 ms at 1.9 GHz


@pytest.fixture(scope="module")
def rv():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    import ramvamp_b200

    ramvamp_b200.device_status(0)  # start from a clean error word
    return ramvamp_b200


@pytest.mark.parametrize("what", ["mbarrier", "flag"])
def test_bounded_wait_reports_timeout_and_device_recovers(rv, orc, what):
    code = rv.WAIT_MBARRIER if what == "mbarrier" else rv.WAIT_FLAG
    t0 = time.perf_counter()
    rv.wait_probe(code, CYCLES)
    with pytest.raises(rv.KernelError) as e:
        rv.device_status(0)
    assert e.value.kind == "Timeout"
    assert time.perf_counter() - t0 < 30.0
    # The error word was read and cleared; the next calls run normally.
    rv.device_status(0)
    x = np.random.default_rng(5).standard_normal(1024).astype(np.float32)
    out = torch.empty(4 * 292, dtype=torch.uint8, device="cuda")
    rv.quantize_row_q8_k(torch.from_numpy(x).cuda(), out)
    torch.cuda.synchronize()
    want = orc.quantize_row_q8_k(x)
    assert out.cpu().numpy().tobytes() == want.tobytes()
    rv.device_status(0)


def test_wait_probe_rejects_bad_arguments(rv):
    for what, cycles in ((2, CYCLES), (0, 0), (1, 1 << 40)):
        with pytest.raises(rv.KernelError) as e:
            rv.wait_probe(what, cycles)
        assert e.value.kind == "InvalidArgument"
    rv.device_status(0)
