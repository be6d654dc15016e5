"""The C restatement (oracle/qx_oracle.c) against the reference on inputs
that exercise its selection and conversion edge cases: exact router ties that
cut the top-8 inside a tied group, exact argmax ties in the head, and fp16
block scales with exponent 31.  The GPU tests use the same images
(tests/test_gpu_exact.py), so these pin the checker they are compared with.
"""
import numpy as np
import pytest

import qxlib
import qximg

TIE_CFG = dict(experts=128)
TOKEN = 42


@pytest.fixture(scope="module")
def tie_img():
    return qximg.tie_image(qxlib.mini_config(7, **TIE_CFG))


@pytest.fixture(scope="module")
def inf_img():
    return qximg.fp16_inf_image(qxlib.mini_config(7), TOKEN)


def _decode(model, steps, ctx=32):
    kv = model.new_kv(ctx)
    tok, out = TOKEN, []
    for s in range(steps):
        r = model.decode_step(tok, s, kv)
        out.append((r["token"], r["experts"].copy(), r["residual"].copy()))
        tok = r["token"]
    return out, kv


def test_tie_image_cuts_top8_inside_a_tied_triple(ref, port, tie_img):
    R = ref.open_image(tie_img)
    P = port.open_image(tie_img)
    cut = 0
    for seed in (1, 2, 3, 4):
        x = qxlib.normal_vector(seed, R.hidden)
        for layer in range(R.layers):
            _, rmoe, rsel, rw = R.moe_layer(layer, x)
            _, pmoe, psel, pw = P.moe_layer(layer, x)
            assert list(psel) == list(rsel)
            np.testing.assert_array_equal(pw, rw)
            np.testing.assert_array_equal(pmoe.view(np.uint32), rmoe.view(np.uint32))
            sel = set(int(e) for e in rsel)
            for e in range(0, 126, 3):
                members = [e in sel, e + 1 in sel, e + 2 in sel]
                if sum(members) in (1, 2):
                    assert members[0] and (members[1] or not members[2]), "a tie went to a higher index"
                    cut += 1
    assert cut >= 4


def test_tie_image_decode_matches_reference(ref, port, tie_img):
    want, _ = _decode(ref.open_image(tie_img), 6)
    got, _ = _decode(port.open_image(tie_img), 6)
    V = ref.open_image(tie_img).vocab
    for (rt, re_, rr), (pt, pe, pr) in zip(want, got):
        assert pt == rt and rt < V // 2
        np.testing.assert_array_equal(pe, re_)
        np.testing.assert_array_equal(pr.view(np.uint32), rr.view(np.uint32))


def test_fp16_exponent31_scales_match_reference(ref, port, inf_img):
    R = ref.open_image(inf_img)
    P = port.open_image(inf_img)
    np.testing.assert_array_equal(P.embed(TOKEN), R.embed(TOKEN))
    assert np.max(np.abs(R.embed(TOKEN))) > 1e6          # the +-65504 scales are in use
    want, rkv = _decode(R, 3)
    got, pkv = _decode(P, 3)
    for (rt, re_, rr), (pt, pe, pr) in zip(want, got):
        assert pt == rt
        np.testing.assert_array_equal(pe, re_)
        np.testing.assert_array_equal(pr.view(np.uint32), rr.view(np.uint32))
    for k in ("k", "v", "ks", "vs"):
        np.testing.assert_array_equal(pkv[k], rkv[k])
