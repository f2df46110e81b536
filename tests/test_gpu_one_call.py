"""The one-call C ABI (ptq8_load / ptq8_capture_graph / ptq8_forward / ptq8_forward_debug /
ptq8_destroy) gives the same logits and int8 codes as the stepwise engine API."""
import ctypes

import numpy as np
import pytest

from oracle import ptq8_oracle as O
from tests.parity import stem_rows

pytestmark = pytest.mark.gpu


def test_one_call_matches_stepwise(make_model):
    import torch
    from ptq_int8_lab_b200 import engine as E
    p = make_model(0)
    n = 6
    x = np.random.default_rng(21).standard_normal((n, 3, 32, 32)).astype(np.float32)

    ref = E.open_engine(p["model"], p["calib"], p["plan"], max_batch=8)
    want_logits = ref.forward(x)
    m = E.Model.load(p["model"])
    want_codes = {i: ref.dump_codes(i, n) for i in range(m.n_conv)}

    L = E.lib()
    eng = ctypes.c_void_p()
    err = ctypes.create_string_buffer(1024)
    opts = E.Opts(0, 8, 8, E.ACT_ABSMAX, 0, 8)
    assert L.ptq8_load(p["model"].encode(), p["calib"].encode(), p["plan"].encode(), ctypes.byref(opts),
                       ctypes.byref(eng), err, len(err)) == 0, err.value
    try:
        assert L.ptq8_capture_graph(eng, n) == 0, L.ptq8_last_error(eng)
        xd = torch.from_numpy(x).cuda()
        ld = torch.empty(n, 10, device="cuda")
        stream = torch.cuda.current_stream().cuda_stream
        assert L.ptq8_forward(eng, xd.data_ptr(), n, ld.data_ptr(), stream) == 0, L.ptq8_last_error(eng)
        torch.cuda.synchronize()
        assert np.array_equal(ld.cpu().numpy(), want_logits)

        got = {}

        def on_dump(user, conv, codes, nn, h, w, ld_):
            got[conv] = np.ctypeslib.as_array(codes, shape=(nn, h, w, ld_)).copy()

        cb = E.DUMP_FN(on_dump)
        ld.zero_()
        assert L.ptq8_forward_debug(eng, xd.data_ptr(), n, ld.data_ptr(), stream, cb, None) == 0
        assert np.array_equal(ld.cpu().numpy(), want_logits)
        assert sorted(got) == list(range(m.n_conv))
        for i in range(m.n_conv):
            assert np.array_equal(got[i], want_codes[i]), i
        # the stem's rows against the oracle's codes of the input
        om = O.read_model(p["model"])
        tr = O.Oracle(om, O.read_ptqc(p["calib"])).forward(x)
        assert np.array_equal(got[0], stem_rows(tr.codes[0], om.convs[0], got[0].shape[-1]))
    finally:
        L.ptq8_destroy(eng)
