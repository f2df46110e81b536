"""Engine-vs-oracle comparison helpers shared by the GPU parity tests."""
import numpy as np

from oracle import ptq8_oracle as O


def stem_rows(codes_nchw: np.ndarray, conv: O.Conv, kpad: int) -> np.ndarray:
    """Expected stem im2col rows [N, OH, OW, kpad], k = (i*KW + j)*C + c, from oracle codes."""
    N, C, H, W = codes_nchw.shape
    OH = (H + 2 * conv.ph - conv.kh) // conv.sh + 1
    OW = (W + 2 * conv.pw - conv.kw) // conv.sw + 1
    xp = np.zeros((N, C, H + 2 * conv.ph, W + 2 * conv.pw), dtype=np.int8)
    xp[:, :, conv.ph:conv.ph + H, conv.pw:conv.pw + W] = codes_nchw
    out = np.zeros((N, OH, OW, kpad), dtype=np.int8)
    for i in range(conv.kh):
        for j in range(conv.kw):
            tap = xp[:, :, i:i + conv.sh * (OH - 1) + 1:conv.sh, j:j + conv.sw * (OW - 1) + 1:conv.sw]
            k0 = (i * conv.kw + j) * C
            out[..., k0:k0 + C] = tap.transpose(0, 2, 3, 1)
    return out


def _dump_images(dump, images):
    """dump(n, n0) for each engine image in `images` (any order), stacked."""
    return np.concatenate([dump(1, int(k)) for k in images], axis=0)


def compare(engine, trace: O.Trace, model: O.Model, n: int, logits: np.ndarray, rtol: float = 1e-5,
            images=None):
    """Assert bit-exact int8 conv-input codes and final fp32 map; logits within rtol.

    `images` (optional): the engine batch positions of the trace's n images (trace row k is
    engine image images[k]), for checks of a few images of a large batch; `logits` are then
    the engine logits of those images."""
    bad = []
    for i, conv in enumerate(model.convs):
        if images is None:
            got = engine.dump_codes(i, n)
        else:
            got = _dump_images(lambda c, k: engine.dump_codes(i, c, k), images)
        want = trace.codes[i]
        if i == model.stem:
            exp = stem_rows(want, conv, got.shape[-1])
            ok = np.array_equal(got, exp)
        else:
            C = want.shape[1]
            if got.shape[1:3] != want.shape[2:4]:
                # a 1x1 stride-2 conv fused into its block's last conv keeps only the input
                # codes it reads: the even positions
                assert (conv.kh, conv.kw, conv.sh, conv.sw, conv.ph, conv.pw) == (1, 1, 2, 2, 0, 0), i
                want = want[:, :, ::2, ::2]
                assert got.shape[1:3] == want.shape[2:4], (i, got.shape, want.shape)
            ok = np.array_equal(got[..., :C], want.transpose(0, 2, 3, 1))
            if not ok:
                d = got[..., :C].astype(np.int32) - want.transpose(0, 2, 3, 1)
                bad.append((i, int((d != 0).sum()), int(np.abs(d).max()), d.size))
                continue
        if not ok:
            bad.append((i, -1, -1, got.size))
    assert not bad, f"int8 code mismatches (conv, n_diff, max|diff|, size): {bad}"
    fin = engine.dump_final(n) if images is None else _dump_images(engine.dump_final, images)
    want = trace.block_out[-1].transpose(0, 2, 3, 1) if trace.block_out else trace.stem_out.transpose(0, 2, 3, 1)
    assert np.array_equal(fin, want), f"final fp32 map differs: max|diff|={np.abs(fin - want).max()}"
    # logits within rtol = 1e-5 relative (per image, against the image's largest |logit|) of the
    # oracle's float64 head and of its float32 head (ref_e2e.py:255-256 arithmetic)
    ok, err = O.logits_close(logits, trace.logits, rtol)
    assert ok, f"logits rel err {err:.3e} > {rtol} (float64 head)"
    ok32, err32 = O.logits_close(logits, trace.logits_f32, rtol)
    assert ok32, f"logits rel err {err32:.3e} > {rtol} (float32 head)"
    return max(err, err32)
