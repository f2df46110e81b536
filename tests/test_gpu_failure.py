"""Failure detection on the GPU without a fault: a bounded device wait that runs out
reports PTQ8_ERR_TIMEOUT instead of hanging, the context stays usable, and the error
word is per engine (another engine on the same device is unaffected).

The failure is made by the engine's test switch (ptq8_engine_set_wait_test): the first
operand load of the first tensor-core conv's CTA 0 is announced to its barrier but never
issued, so the MMA warp, the epilogue and the producer's drain wait on a barrier that
nothing completes.  Each wait gives up after the short limit set here (about 20 ms).
Nothing traps, faults or hangs; every memory access stays where it always is."""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu

PTQ8_ERR_TIMEOUT = 4


def test_wait_timeout_is_reported_and_engine_recovers(make_model):
    from ptq_int8_lab_b200 import engine as E
    p = make_model("resnet18", seed=0, bn="data")
    a = E.open_engine(p["model"], p["calib"], p["plan"], max_batch=8)
    b = E.open_engine(p["model"], p["calib"], p["plan"], max_batch=8)
    x = np.random.default_rng(41).standard_normal((4, 3, 32, 32)).astype(np.float32)
    want = a.forward(x)
    assert np.array_equal(b.forward(x), want)

    a.set_wait_test(wait_limit_cycles=40_000_000, stall_first_load=True)
    with pytest.raises(E.Ptq8Error) as ei:
        a.forward(x)
    assert ei.value.status == PTQ8_ERR_TIMEOUT, str(ei.value)
    assert "timed out" in str(ei.value)

    # the other engine on the same device has its own error word
    assert np.array_equal(b.forward(x), want)
    b.check_device_error()

    # the report cleared the word; with the switch off the same engine is exact again
    a.set_wait_test(0, False)
    assert np.array_equal(a.forward(x), want)
    a.check_device_error()
