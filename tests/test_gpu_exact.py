"""Bit-exact parity of the CUDA engine's integer and selection work.

Through the C ABI on a B200, against the reference (oracle/_ref/libqxref.so,
src/qx_format.c compiled unchanged) or the C restatement that
tests/test_oracle_pin.py and tests/test_ties_and_specials.py pin to it:
  - the INT8 K/V cache and its scales after a multi-step decode, byte for
    byte (one lrintf(x / scale) per value, one scale per layer and token,
    src/qx_format.c:4449-4463, :6343-6399);
  - exact router ties that cut the top-8 inside a tied group, and exact
    argmax ties in the head (lower index wins, :5272-5285, :3723-3730);
  - fp16 block scales with exponent 31 (+-65504, :1868-1869);
  - the reference's own unmodified state loop (:6721) for 4 greedy steps;
  - decode near the end of a 4096-token context through the one-launch step;
  - the loader entry point the reference binding calls
    (qx_cuda_engine_create_from_qxf with QX_CUDA_VERIFY_CHECKSUMS).
"""
import json
import os

import numpy as np
import pytest

import qxlib
import qximg
import workloads as W
from qxtol import assert_close

pytestmark = pytest.mark.gpu
GOLD = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")


def fnv1a64(b):
    h = 1469598103934665603
    for x in bytes(b):
        h = ((h ^ x) * 1099511628211) & 0xFFFFFFFFFFFFFFFF
    return h


def engine_decode(eng, steps, token=W.START_TOKEN, first=0):
    out, tok = [], token
    for s in range(first, first + steps):
        r = eng.decode_step(tok, s, want_residual=True, want_experts=True)
        out.append(r)
        tok = r["token"]
    return out


def checker_decode(model, steps, kv, token=W.START_TOKEN, first=0):
    out, tok = [], token
    for s in range(first, first + steps):
        r = model.decode_step(tok, s, kv)
        out.append(r)
        tok = r["token"]
    return out


def assert_kv_equal(eng, kv, positions, layers, first=0):
    for layer in range(layers):
        k, v, ks, vs = eng.kv_read(layer, first, positions)
        np.testing.assert_array_equal(k, kv["k"][layer, first:first + positions], err_msg="K layer %d" % layer)
        np.testing.assert_array_equal(v, kv["v"][layer, first:first + positions], err_msg="V layer %d" % layer)
        np.testing.assert_array_equal(ks.view(np.uint32), kv["ks"][layer, first:first + positions].view(np.uint32))
        np.testing.assert_array_equal(vs.view(np.uint32), kv["vs"][layer, first:first + positions].view(np.uint32))


@pytest.mark.parametrize("geometry,steps", [("mini", 64), ("full4", 24)])
def test_kv_cache_is_bit_exact_after_decode(port, geometry, steps):
    cfg = qxlib.mini_config(7) if geometry == "mini" else qxlib.synth_config(7, layers=4)
    img = qxlib.build_image(cfg)
    eng = qxlib.Engine(img, ctx=steps + 8)
    try:
        got = engine_decode(eng, steps)
        P = port.open_image(img)
        kv = P.new_kv(steps + 8)
        want = checker_decode(P, steps, kv)
        for s, (g, w) in enumerate(zip(got, want)):
            assert g["token"] == w["token"], "step %d" % s
            np.testing.assert_array_equal(g["experts"], w["experts"], err_msg="step %d" % s)
        res_bits = sum(int(np.count_nonzero(g["residual"].view(np.uint32) != w["residual"].view(np.uint32)))
                       for g, w in zip(got, want))
        print("%s: final-residual floats differing in any bit: %d of %d" % (geometry, res_bits, steps * eng.hidden))
        assert_close(got[-1]["residual"], want[-1]["residual"], what="final residual")
        assert_kv_equal(eng, kv, steps, cfg.layers)
    finally:
        eng.close()


def test_router_and_head_ties_follow_the_reference(ref):
    img = qximg.tie_image(qxlib.mini_config(7, experts=128))
    eng = qxlib.Engine(img, ctx=48)
    try:
        R = ref.open_image(img)
        # stage entry point: the top-8 cut inside a tied triple
        cut = 0
        for seed in range(1, 9):
            x = qxlib.normal_vector(seed, eng.hidden)
            for layer in range(eng.layers):
                lo, moe, sel, w = eng.moe_layer(layer, x)
                rlo, rmoe, rsel, rw = R.moe_layer(layer, x)
                assert list(sel) == list(rsel), "seed %d layer %d" % (seed, layer)
                assert_close(moe, rmoe, what="moe output")
                s = set(int(e) for e in sel)
                cut += sum(1 for e in range(0, 126, 3) if sum((e in s, e + 1 in s, e + 2 in s)) in (1, 2))
        assert cut >= 8
        # greedy decode through the one-launch step: experts and tied argmaxes
        got = engine_decode(eng, 40)
        kv = R.new_kv(48)
        want = checker_decode(R, 40, kv)
        for s, (g, w) in enumerate(zip(got, want)):
            assert g["token"] == w["token"] < eng.vocab // 2, "step %d" % s
            np.testing.assert_array_equal(g["experts"], w["experts"], err_msg="step %d" % s)
        assert_kv_equal(eng, kv, 40, eng.layers)
    finally:
        eng.close()


def test_fp16_exponent31_scales_on_the_device(ref):
    img = qximg.fp16_inf_image(qxlib.mini_config(7), W.START_TOKEN)
    eng = qxlib.Engine(img, ctx=16)
    try:
        R = ref.open_image(img)
        np.testing.assert_array_equal(eng.embed(W.START_TOKEN), R.embed(W.START_TOKEN))
        got = engine_decode(eng, 4)
        kv = R.new_kv(16)
        want = checker_decode(R, 4, kv)
        for s, (g, w) in enumerate(zip(got, want)):
            assert g["token"] == w["token"], "step %d" % s
            np.testing.assert_array_equal(g["experts"], w["experts"])
            assert_close(g["residual"], w["residual"], what="residual step %d" % s)
        assert_kv_equal(eng, kv, 4, eng.layers)
        # the head rows with +-65504 scales, alone
        normed, logits, tt, tl = eng.final_head(W.head_input(eng.hidden), 8)
        rn, rl, rtt, rtl = R.final_head(W.head_input(eng.hidden), 8)
        assert list(tt) == list(rtt)
        assert_close(logits, rl, what="logits")
    finally:
        eng.close()


@pytest.fixture(scope="module")
def full(full_image):
    e = qxlib.Engine(full_image, ctx=4096)
    yield e
    e.close()


def test_state_loop_of_the_reference(full):
    """The reference's own CLI state loop (state-loop-probe --full-moe
    --final-head --dump-residuals), recorded by tests/golden/make_golden.py."""
    with open(os.path.join(GOLD, "golden_full.json")) as f:
        sl = json.load(f)["state_loop"]
    full.reset()
    tok = W.START_TOKEN
    for s, st in enumerate(sl["steps"]):
        assert st["input"] == tok
        r = full.decode_step(tok, s, want_logits=True, want_residual=True, want_experts=True)
        assert r["token"] == st["token"] == st["argmax"], "step %d" % s
        np.testing.assert_array_equal(r["experts"], np.asarray(st["experts"], np.uint32))
        assert_close(r["residual"], st["residual"], what="final residual step %d" % s)
        assert_close(r["logits"][sl["logits_sample_idx"]], st["logits_sample"], what="logits step %d" % s)
        for layer in range(full.layers):
            k, v, ks, vs = full.kv_read(layer, s, 1)
            assert fnv1a64(k[0].tobytes()) == st["k_checksum"][layer], "K row layer %d step %d" % (layer, s)
            assert fnv1a64(v[0].tobytes()) == st["v_checksum"][layer], "V row layer %d step %d" % (layer, s)
            assert ks[0] == np.float32(st["k_scale"][layer]) and vs[0] == np.float32(st["v_scale"][layer])
        tok = r["token"]
    assert tok == sl["final_token"]


def test_long_context_decode_through_the_one_launch_step(full, full_image, port):
    """Positions 4088..4091 of a 4096-token context: the history 0..4087 of
    every layer is seeded INT8 data (written through qx_cuda_kv_write), the
    step runs in one launch (the ctx cap is src/qx_format.c:6125-6129)."""
    first, steps, ctx = 4088, 4, 4096
    rng = np.random.default_rng(5)
    P = port.open_image(full_image)
    kv = P.new_kv(ctx)
    full.reset()
    kvv = full.kv_heads * full.head_dim
    for layer in range(full.layers):
        k = rng.integers(-127, 128, (first, kvv), dtype=np.int8)
        v = rng.integers(-127, 128, (first, kvv), dtype=np.int8)
        ks = (rng.random(first, dtype=np.float32) * 0.02 + 0.005).astype(np.float32)
        vs = (rng.random(first, dtype=np.float32) * 0.02 + 0.005).astype(np.float32)
        kv["k"][layer, :first], kv["v"][layer, :first], kv["ks"][layer, :first], kv["vs"][layer, :first] = k, v, ks, vs
        full.kv_write(layer, 0, k, v, ks, vs)
    p0 = full.profile()["kernel_launches"]
    got = engine_decode(full, steps, first=first)
    assert full.profile()["kernel_launches"] - p0 == steps       # one launch per token
    want = checker_decode(P, steps, kv, first=first)
    for s, (g, w) in enumerate(zip(got, want)):
        assert g["token"] == w["token"], "position %d" % (first + s)
        np.testing.assert_array_equal(g["experts"], w["experts"], err_msg="position %d" % (first + s))
        assert_close(g["residual"], w["residual"], what="residual position %d" % (first + s))
    assert_kv_equal(full, kv, steps, full.layers, first=first)


def test_create_from_qxf_with_checksums(mini_image, tmp_path):
    """The entry point the reference-side binding calls: a QXF1 file on disk,
    mapped, verified (FNV-1a of every tensor) and uploaded."""
    path = str(tmp_path / "mini.qxf")
    mini_image.tofile(path)
    with open(os.path.join(GOLD, "golden_mini.json")) as f:
        g = json.load(f)["decode"]
    eng = qxlib.Engine(path=path, ctx=32, flags=qxlib.VERIFY_CHECKSUMS)
    try:
        tok = g[0]["input"]
        for s, st in enumerate(g):
            r = eng.decode_step(tok, s, want_experts=True)
            assert r["token"] == st["token"]
            np.testing.assert_array_equal(r["experts"], np.asarray(st["experts"], np.uint32))
            tok = r["token"]
    finally:
        eng.close()
    bad = mini_image.copy()
    _, off, size, _, _ = qximg.tensors(bad)["blk.1.ffn_down_exps.weight"]
    bad[off + size // 2] ^= 0x40
    bad_path = str(tmp_path / "bad.qxf")
    bad.tofile(bad_path)
    with pytest.raises(RuntimeError, match="tensor checksum mismatch"):
        qxlib.Engine(path=bad_path, ctx=32, flags=qxlib.VERIFY_CHECKSUMS)
    # without the flag the file opens (the reference also verifies only on request)
    qxlib.Engine(path=bad_path, ctx=32).close()


def test_smaller_engine_created_later_does_not_break_the_first(full, mini_image):
    """The step kernel's shared-memory limit is per device and per function:
    creating a smaller model's engine after the full one must not lower it
    below what the full engine's launches need."""
    with open(os.path.join(GOLD, "golden_full.json")) as f:
        g = json.load(f)["decode"]
    small = qxlib.Engine(mini_image, ctx=16)
    try:
        small.decode_step(W.START_TOKEN, 0)
        full.reset()
        assert full.decode_step(g[0]["input"], 0)["token"] == g[0]["token"]
    finally:
        small.close()


def test_device_exp_against_host_libm():
    """The softmaxes and SiLU call CUDA's double exp; the reference calls the
    C library's (src/qx_format.c:2511-2513, :5131-5167, :5257-5285).  Both are
    within an ulp of e^x but need not round alike.  Count how often they
    differ on the ranges the engine feeds them: softmax arguments (score -
    max, logit - max) in [-40, 0] and SiLU arguments in [-20, 20]."""
    import math
    import torch
    rng = np.random.default_rng(9)
    for lo, hi in ((-40.0, 0.0), (-20.0, 20.0)):
        x = rng.uniform(lo, hi, 200000)
        dev = torch.exp(torch.from_numpy(x).cuda()).cpu().numpy()
        host = np.array([math.exp(v) for v in x])
        diff = int(np.count_nonzero(dev != host))
        ulps = np.abs(dev.view(np.int64) - host.view(np.int64))
        print("exp on [%g, %g]: %d of %d differ (max %d ulp)" % (lo, hi, diff, x.size, int(ulps.max())))
        assert ulps.max() <= 1        # both faithful; how often they differ is reported, not bounded
