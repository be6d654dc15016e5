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


def stepwise(eng, prompt, position=0):
    r = None
    for p, t in enumerate(prompt):
        r = eng.decode_step(int(t), position + p, want_residual=True)
    return r


@pytest.mark.parametrize("geometry,n", [("mini", 1), ("mini", 77), ("full4", 300)])
def test_prefill_equals_the_per_token_prompt_loop(geometry, n):
    """qx_cuda_prefill against the prompt run one token at a time through the
    decode step (the reference's prompt loop, src/qx_format.c:6250-6547):
    the next token, the last token's final residual and every INT8 K/V row
    and scale of every layer must be identical."""
    cfg = qxlib.mini_config(7) if geometry == "mini" else qxlib.synth_config(7, layers=4)
    eng = qxlib.Engine(qxlib.build_image(cfg), ctx=n + 24)
    try:
        prompt = np.random.default_rng(n).integers(0, eng.vocab, n).astype(np.uint32)
        eng.reset()
        nxt, res = eng.prefill(prompt, 0, want_residual=True)
        kv_pre = [eng.kv_read(layer, 0, n) for layer in range(eng.layers)]
        cont = eng.generate(nxt, n, 8)            # decoding continues from the prefilled cache
        eng.reset()
        r = stepwise(eng, prompt)
        assert nxt == r["token"]
        np.testing.assert_array_equal(res.view(np.uint32), r["residual"].view(np.uint32))
        for layer in range(eng.layers):
            k, v, ks, vs = eng.kv_read(layer, 0, n)
            np.testing.assert_array_equal(kv_pre[layer][0], k)
            np.testing.assert_array_equal(kv_pre[layer][1], v)
            np.testing.assert_array_equal(kv_pre[layer][2].view(np.uint32), ks.view(np.uint32))
            np.testing.assert_array_equal(kv_pre[layer][3].view(np.uint32), vs.view(np.uint32))
        assert list(eng.generate(nxt, n, 8)) == list(cont)
    finally:
        eng.close()


def test_prefill_mini_matches_the_reference(ref, mini_image):
    """The reference's own C path (the shim's decode step, pinned to its
    unmodified state loop) decodes 5 tokens and then a 24-token prompt one
    token at a time; the engine decodes the same 5 tokens and prefills the
    prompt at position 5.  The next token and the whole INT8 K/V cache must
    agree."""
    eng = qxlib.Engine(mini_image, ctx=64)
    try:
        R = ref.open_image(mini_image)
        kv = R.new_kv(64)
        prompt = np.random.default_rng(3).integers(0, eng.vocab, 24).astype(np.uint32)
        lead = [42]
        for p in range(5):
            lead.append(R.decode_step(lead[-1], p, kv)["token"])
        rt = None
        for p, t in enumerate(prompt):
            rt = R.decode_step(int(t), 5 + p, kv)
        eng.reset()
        for p in range(5):
            eng.decode_step(lead[p], p)
        assert eng.prefill(prompt, 5) == rt["token"]
        for layer in range(eng.layers):
            k, v, ks, vs = eng.kv_read(layer, 0, 29)
            np.testing.assert_array_equal(k, kv["k"][layer, :29])
            np.testing.assert_array_equal(v, kv["v"][layer, :29])
            np.testing.assert_array_equal(ks, kv["ks"][layer, :29])
    finally:
        eng.close()


def test_prefill_arguments(mini_image):
    eng = qxlib.Engine(mini_image, ctx=32)
    try:
        with pytest.raises(RuntimeError, match="steps exceed ctx"):
            eng.prefill(np.zeros(40, np.uint32), 0)
        with pytest.raises(RuntimeError, match="prompt token out of range"):
            eng.prefill(np.array([1, eng.vocab], np.uint32), 0)
    finally:
        eng.close()


@pytest.mark.parametrize("geometry", ["mini", "full4"])
def test_decode_batch_equals_single_sequence(geometry):
    """qx_cuda_decode_batch: several sequences, each in its own KV slot,
    joining at different steps, must produce the same greedy tokens as the
    single-sequence step decoding each of them alone."""
    cfg = qxlib.mini_config(7) if geometry == "mini" else qxlib.synth_config(7, layers=4)
    eng = qxlib.Engine(qxlib.build_image(cfg), ctx=64)
    try:
        starts = [42, 7, 1000, 5, 42, 3000]
        joins = [0, 0, 0, 3, 5, 5]                # step at which each sequence starts (position 0)
        steps = 14
        slots = [9, 0, 63, 4, 17, 2]
        cur = list(starts)
        got = [[] for _ in starts]
        for step in range(steps):
            live = [i for i in range(len(starts)) if joins[i] <= step]
            nxt = eng.decode_batch([slots[i] for i in live], [cur[i] for i in live],
                                   [step - joins[i] for i in live])
            for i, t in zip(live, nxt):
                got[i].append(int(t))
                cur[i] = int(t)
        for i, s0 in enumerate(starts):
            eng.reset()
            want = eng.generate(s0, 0, steps - joins[i])
            assert got[i] == list(want), "sequence %d" % i
    finally:
        eng.close()


def test_decode_batch_arguments(mini_image):
    eng = qxlib.Engine(mini_image, ctx=16)
    try:
        with pytest.raises(RuntimeError, match="appears twice"):
            eng.decode_batch([1, 1], [42, 43], [0, 0])
        with pytest.raises(RuntimeError, match="steps exceed ctx"):
            eng.decode_batch([1], [42], [16])
        with pytest.raises(RuntimeError, match="invalid batched decode argument"):
            eng.decode_batch([64], [42], [0])
    finally:
        eng.close()


def test_decode_batch_long_context_equals_single_sequence():
    """Past ~3470 positions the 8 query heads' softmax weights no longer fit
    the grouped attention kernel's shared memory, and the batched step takes
    the per-head kernel.  Four sequences at positions 3600..3700, in fresh
    slots (zero history), two batched steps: each sequence's tokens must equal
    the single-sequence step's from the same zero history."""
    eng = qxlib.Engine(qxlib.build_image(qxlib.synth_config(7, layers=4)), ctx=3712)
    try:
        starts, pos0, slots = [42, 7, 1000, 3000], [3600, 3601, 3700, 3650], [5, 0, 63, 11]
        cur, got = list(starts), [[] for _ in starts]
        for step in range(2):
            nxt = eng.decode_batch(slots, cur, [p + step for p in pos0])
            for i, t in enumerate(nxt):
                got[i].append(int(t))
                cur[i] = int(t)
        for i in range(len(starts)):
            eng.reset()
            t0 = eng.decode_step(starts[i], pos0[i])["token"]
            t1 = eng.decode_step(t0, pos0[i] + 1)["token"]
            assert got[i] == [t0, t1], "sequence %d" % i
    finally:
        eng.close()
