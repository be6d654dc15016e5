"""Quant mixes of the real Qwen3-30B-A3B GGUF files (IQ2_S gate/up,
IQ3_S or IQ4_XS down, Q5_K or Q6_K attention) through the per-stage path,
checked against the reference's own C decode (src/qx_format.c, through
oracle/_ref/libqxref.so): greedy tokens and top-8 experts exact, final
residual within 1e-4; the MoE and attention stage entry points too."""
import numpy as np
import pytest

import qxlib
import workloads as W
from qxtol import assert_close

pytestmark = pytest.mark.gpu

# ggml types: Q5_K 13, Q6_K 14, IQ2_XS 17, IQ3_XXS 18, IQ3_S 21, IQ2_S 22, IQ4_XS 23
MIXES = {
    "q5k-iq2s-iq3s": dict(attn_type=13, gate_type=22, up_type=22, down_type=21),
    "q6k-iq2s-iq4xs": dict(attn_type=14, gate_type=22, up_type=22, down_type=23),
    "iq4xs-iq2xs-iq3s": dict(attn_type=23, gate_type=17, up_type=17, down_type=21),
}


@pytest.mark.parametrize("mix", sorted(MIXES))
def test_mixed_quant_decode_matches_reference(mix, ref):
    img = qxlib.build_image(qxlib.mini_config(7, **MIXES[mix]))
    eng = qxlib.Engine(img, ctx=64)
    try:
        m = ref.open_image(img)
        kv = m.new_kv(64)
        tok = W.START_TOKEN
        p0 = eng.profile()["kernel_launches"]
        for s in range(10):
            r = m.decode_step(tok, s, kv)
            e = eng.decode_step(tok, s, want_residual=True, want_experts=True)
            assert e["token"] == r["token"], "%s step %d" % (mix, s)
            np.testing.assert_array_equal(e["experts"], r["experts"], err_msg="%s step %d" % (mix, s))
            assert_close(e["residual"], r["residual"], what="%s final residual step %d" % (mix, s))
            tok = r["token"]
        assert eng.profile()["kernel_launches"] - p0 > 10     # the per-stage path ran, not the one-launch kernel
        for layer in range(eng.layers):
            x = qxlib.normal_vector(40 + layer, eng.hidden)
            lo, moe, sel, w = eng.moe_layer(layer, x)
            rlo, rmoe, rsel, rw = m.moe_layer(layer, x)
            assert list(sel) == list(rsel)
            assert_close(moe, rmoe, what="%s moe layer %d" % (mix, layer))
            assert_close(lo, rlo, what="%s layer output %d" % (mix, layer))
    finally:
        eng.close()


def test_gate_and_up_of_different_types_are_rejected():
    # the engine needs one type for a layer's gate and up experts
    img = qxlib.build_image(qxlib.mini_config(7, gate_type=17, up_type=22))
    with pytest.raises(RuntimeError, match="gate and up experts must share one type"):
        qxlib.Engine(img, ctx=16)
