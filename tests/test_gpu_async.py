"""ptq8_engine_forward_async: the pipelined host-buffer forward (two input slots, the
next call's H2D overlapping the current forward) gives exactly the logits of the
synchronous ptq8_engine_forward for every call, across slot reuse, batch changes and a
synchronous call in between (fp32 logits: the tolerance is zero)."""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def test_async_matches_sync(make_model):
    import torch
    from ptq_int8_lab_b200 import engine as E
    p = make_model(0)
    eng = E.open_engine(p["model"], p["calib"], p["plan"], max_batch=16)
    rng = np.random.default_rng(31)
    sizes = [16, 16, 9, 16, 5]
    xs = [rng.standard_normal((n, 3, 32, 32)).astype(np.float32) for n in sizes]
    want = [eng.forward(x) for x in xs]

    xh = [torch.from_numpy(x).pin_memory() for x in xs]
    lh = [torch.empty(n, 10, dtype=torch.float32).pin_memory() for n in sizes]
    for i in range(3):   # calls 0-2 in flight together (slots 0, 1, 0)
        eng.forward_async(xh[i].data_ptr(), sizes[i], lh[i].data_ptr())
    eng.sync()
    mid = eng.forward(xs[0])   # a synchronous call between pipelined ones
    for i in range(3, 5):
        eng.forward_async(xh[i].data_ptr(), sizes[i], lh[i].data_ptr())
    eng.sync()
    assert np.array_equal(mid, want[0])
    for i in range(5):
        assert np.array_equal(lh[i].numpy(), want[i]), i


def test_async_right_after_device_forward(make_model):
    """ptq8_engine_forward_device (enqueued, not waited for) reads input slot 0; the first
    pipelined call right after it copies its input into slot 0 on the copy stream, which
    must wait until that forward has read the slot."""
    import torch
    from ptq_int8_lab_b200 import engine as E
    p = make_model(0)
    n = 256
    eng = E.open_engine(p["model"], p["calib"], p["plan"], max_batch=n)
    rng = np.random.default_rng(37)
    x0 = rng.standard_normal((n, 3, 32, 32)).astype(np.float32)
    x1 = rng.standard_normal((n, 3, 32, 32)).astype(np.float32)
    want0, want1 = eng.forward(x0), eng.forward(x1)
    for _ in range(3):
        eng2 = E.open_engine(p["model"], p["calib"], p["plan"], max_batch=n)   # no pipelined call yet
        xd = torch.from_numpy(x0).cuda()
        ld = torch.empty(n, 10, device="cuda")
        x1h = torch.from_numpy(x1).pin_memory()
        l1h = torch.empty(n, 10, dtype=torch.float32).pin_memory()
        torch.cuda.synchronize()
        eng2.forward_device(xd.data_ptr(), n, ld.data_ptr())
        eng2.forward_async(x1h.data_ptr(), n, l1h.data_ptr())
        eng2.forward_device(xd.data_ptr(), n, ld.data_ptr())
        eng2.forward_async(x1h.data_ptr(), n, l1h.data_ptr())   # slot 1
        eng2.forward_async(x1h.data_ptr(), n, l1h.data_ptr())   # slot 0 again
        eng2.sync()
        assert np.array_equal(ld.cpu().numpy(), want0)
        assert np.array_equal(l1h.numpy(), want1)
