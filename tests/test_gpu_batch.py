"""The batched MoE layer (qx_cuda_moe_batch): many tokens through one MoE
FFN layer with the expert projections as grouped GEMMs on the tcgen05 tensor
cores (BASELINE config 5's grouped-expert contraction).

The reference has no batched path: it runs qx_apply_real_moe_layer
(src/qx_format.c:5198-5317) once per token.  Every token of a batch must
therefore equal that per-token result: the top-8 experts exactly, the outputs
within 1e-4 of the reference (tests/qxtol.py).  Against the engine's own
per-token entry point (qx_cuda_moe_layer), which forms the same exact integer
block sums, the outputs must be identical bit for bit.
"""
import numpy as np
import pytest

import qxlib
import qximg
from qxtol import assert_close

pytestmark = pytest.mark.gpu


def inputs(n, hidden, seed0=100):
    return np.stack([qxlib.normal_vector(seed0 + t, hidden) for t in range(n)])


def check_against_per_token(eng, layer, x, sample):
    out, moe, sel, w = eng.moe_batch(layer, x)
    for t in sample:
        lo, m1, s1, w1 = eng.moe_layer(layer, x[t])
        assert list(sel[t]) == list(s1), "token %d" % t
        np.testing.assert_array_equal(w[t], w1, err_msg="routing weights token %d" % t)
        np.testing.assert_array_equal(moe[t].view(np.uint32), m1.view(np.uint32), err_msg="moe output token %d" % t)
        np.testing.assert_array_equal(out[t].view(np.uint32), lo.view(np.uint32), err_msg="layer output token %d" % t)
    return out, moe, sel, w


@pytest.mark.parametrize("n", [1, 13, 40, 300])
def test_moe_batch_mini_equals_per_token(mini_image, n):
    eng = qxlib.Engine(mini_image, ctx=16)
    try:
        for layer in range(eng.layers):
            check_against_per_token(eng, layer, inputs(n, eng.hidden, 100 * layer), range(n))
    finally:
        eng.close()


def test_moe_batch_full_geometry(full_image, ref):
    """Full Qwen3-30B-A3B geometry (128 experts of 768, hidden 2048), layer 3:
    512 tokens in one call; 48 of them against the per-token path bit for bit,
    4 against the reference itself."""
    eng = qxlib.Engine(full_image, ctx=16)
    try:
        x = inputs(512, eng.hidden)
        out, moe, sel, w = check_against_per_token(eng, 3, x, range(0, 512, 11))
        R = ref.open_image(full_image)
        for t in (0, 77, 300, 511):
            rlo, rmoe, rsel, rw = R.moe_layer(3, x[t])
            assert list(sel[t]) == list(rsel)
            assert_close(moe[t], rmoe, what="moe output token %d" % t)
            assert_close(out[t], rlo, what="layer output token %d" % t)
    finally:
        eng.close()


def test_moe_batch_router_ties(ref):
    """Router rows in tied triples (tests/qximg.py): the batched top-8 cuts
    inside a tied group exactly like the reference's strict-> scan."""
    img = qximg.tie_image(qxlib.mini_config(7, experts=128))
    eng = qxlib.Engine(img, ctx=16)
    try:
        R = ref.open_image(img)
        x = inputs(24, eng.hidden, 7)
        out, moe, sel, w = check_against_per_token(eng, 1, x, range(24))
        for t in range(0, 24, 5):
            _, rmoe, rsel, _ = R.moe_layer(1, x[t])
            assert list(sel[t]) == list(rsel)
    finally:
        eng.close()


def test_moe_batch_arguments(mini_image):
    eng = qxlib.Engine(mini_image, ctx=16)
    try:
        with pytest.raises(RuntimeError, match="invalid batched expert argument"):
            eng.moe_batch(eng.layers, inputs(2, eng.hidden))
        with pytest.raises(RuntimeError, match="invalid batched expert argument"):
            eng.moe_batch(0, np.zeros((0, eng.hidden), np.float32))
        x = inputs(3, eng.hidden)
        x[1, 5] = np.nan                        # the reference fails such a token's router softmax (:5268)
        with pytest.raises(RuntimeError, match="invalid selected router weights"):
            eng.moe_batch(0, x)
        x[1, 5] = 0.0                           # and the engine is usable afterwards
        check_against_per_token(eng, 0, x, range(3))
    finally:
        eng.close()
