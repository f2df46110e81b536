"""8-bit pixel input (CIFAR-10 records): the stem kernel decodes, normalises and quantizes
on the device.  Every conv's input codes and the final fp32 map must be bit-exact with the
oracle run on the reference's fp32 normalisation of the same pixels (ref_e2e.py:261-276,
main.cpp:245-261), and the pipelined / device-pointer forms must give the synchronous
form's logits exactly."""
import numpy as np
import pytest

from oracle import ptq8_oracle as O
from tests.parity import compare

pytestmark = pytest.mark.gpu


def _pixels(n, seed):
    px = np.random.default_rng(seed).integers(0, 256, size=(n, 3, 32, 32), dtype=np.uint8)
    px[0] = (np.arange(3 * 1024) % 256).reshape(3, 32, 32)   # every value in every channel
    return px


@pytest.mark.parametrize("mode", [0, 1])
def test_u8_matches_oracle(make_model, mode):
    from ptq_int8_lab_b200 import engine as E
    p = make_model(0)
    n = 7
    eng = E.open_engine(p["model"], p["calib"], p["plan"], max_batch=16)
    eng.set_input_norm(mode)
    px = _pixels(n, 41 + mode)
    logits = eng.forward_u8(px)
    om = O.read_model(p["model"])
    tr = O.Oracle(om, O.read_ptqc(p["calib"])).forward(O.normalize_u8(px, mode))
    compare(eng, tr, om, n, logits)


def test_u8_records_and_forms(make_model):
    """Raw CIFAR-10 records (label byte + 3072 pixels): record_bytes 3073 from the file's
    second byte; pipelined and device-pointer forms; fp32 input in between."""
    import torch
    from ptq_int8_lab_b200 import engine as E
    p = make_model(0)
    n = 12
    eng = E.open_engine(p["model"], p["calib"], p["plan"], max_batch=16)
    px = _pixels(n, 43)
    want = eng.forward_u8(px)
    x = O.normalize_u8(px, 0)
    assert np.array_equal(eng.forward(x), want)   # the fp32 path on the same normalised input
    rec = np.concatenate([np.arange(n, dtype=np.uint8)[:, None], px.reshape(n, -1)], axis=1).reshape(-1)
    assert np.array_equal(eng.forward_u8(rec[1:], n=n, record_bytes=3073), want)

    rh = torch.from_numpy(rec).pin_memory()
    lh = [torch.empty(n, 10, dtype=torch.float32).pin_memory() for _ in range(3)]
    for k in range(3):   # slots 0, 1, 0
        eng.forward_u8_async(rh.data_ptr() + 1, n, 3073, lh[k].data_ptr())
    eng.sync()
    for k in range(3):
        assert np.array_equal(lh[k].numpy(), want), k

    xd = torch.from_numpy(px).cuda()
    ld = torch.empty(n, 10, device="cuda")
    torch.cuda.synchronize()
    eng.forward_device_u8(xd.data_ptr(), n, 0, ld.data_ptr())
    eng.sync()
    assert np.array_equal(ld.cpu().numpy(), want)
