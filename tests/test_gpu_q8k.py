"""The reference's q8_k_compat activation mode (src/qx_format.c:3869-4205)
through QX_CUDA_Q8K_COMPAT: greedy tokens and top-8 experts equal to the
reference's own C path run with --activation q8_k_compat, final residuals and
the MoE stage within 1e-4, for the benchmark mix and two real-GGUF mixes."""
import numpy as np
import pytest

import qxlib
import workloads as W
from qxtol import assert_close

pytestmark = pytest.mark.gpu
Q8K_COMPAT = 0x8

MIXES = {
    "benchmark": {},
    "q5k-iq2s-iq3s": dict(attn_type=13, gate_type=22, up_type=22, down_type=21),
    "q6k-iq2s-iq4xs": dict(attn_type=14, gate_type=22, up_type=22, down_type=23),
}


@pytest.fixture
def ref_q8(ref):
    ref.lib.qxref_set_activation(1)
    yield ref
    ref.lib.qxref_set_activation(0)      # the checker is shared: back to f32


@pytest.mark.parametrize("mix", sorted(MIXES))
def test_q8_k_compat_decode_matches_reference(mix, ref_q8):
    img = qxlib.build_image(qxlib.mini_config(7, **MIXES[mix]))
    eng = qxlib.Engine(img, ctx=64, flags=Q8K_COMPAT)
    try:
        m = ref_q8.open_image(img)
        kv = m.new_kv(64)
        tok = W.START_TOKEN
        for s in range(10):
            r = m.decode_step(tok, s, kv)
            e = eng.decode_step(tok, s, want_residual=True, want_experts=True)
            assert e["token"] == r["token"], "%s step %d" % (mix, s)
            np.testing.assert_array_equal(e["experts"], r["experts"], err_msg="%s step %d" % (mix, s))
            assert_close(e["residual"], r["residual"], what="%s final residual step %d" % (mix, s))
            tok = r["token"]
        for layer in range(eng.layers):
            x = qxlib.normal_vector(60 + layer, eng.hidden)
            lo, moe, sel, w = eng.moe_layer(layer, x)
            rlo, rmoe, rsel, rw = m.moe_layer(layer, x)
            assert list(sel) == list(rsel)
            assert_close(moe, rmoe, what="%s q8 moe layer %d" % (mix, layer))
        normed, logits, tt, tl = eng.final_head(W.head_input(eng.hidden), 8)
        rn, rlogits, rtt, rtl = m.final_head(W.head_input(eng.hidden), top_n=8)
        assert list(tt) == list(rtt)
        assert_close(logits, rlogits, what="%s q8 logits" % mix)
    finally:
        eng.close()


def test_q8_k_compat_rejects_non_finite_activations(mini_image):
    eng = qxlib.Engine(mini_image, ctx=16, flags=Q8K_COMPAT)
    try:
        x = qxlib.normal_vector(1, eng.hidden)
        x[7] = np.inf
        with pytest.raises(RuntimeError, match="Q8_K activation contains NaN or Inf"):
            eng.final_head(x, 1)
    finally:
        eng.close()


def test_q8_k_compat_full_model_first_steps(full_image, ref_q8):
    """Full geometry (48 layers, 128 experts, 151936 vocab): two greedy steps."""
    eng = qxlib.Engine(full_image, ctx=8, flags=Q8K_COMPAT)
    try:
        m = ref_q8.open_image(full_image)
        kv = m.new_kv(8)
        tok = W.START_TOKEN
        for s in range(2):
            r = m.decode_step(tok, s, kv)
            e = eng.decode_step(tok, s, want_residual=True, want_experts=True)
            assert e["token"] == r["token"], "step %d" % s
            np.testing.assert_array_equal(e["experts"], r["experts"], err_msg="step %d" % s)
            assert_close(e["residual"], r["residual"], what="final residual step %d" % s)
            tok = r["token"]
    finally:
        eng.close()
