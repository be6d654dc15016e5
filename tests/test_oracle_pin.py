"""Pin the C restatement (oracle/qx_oracle.c) before trusting it as the GPU
checker: bit-identical to the reference's own compiled C on the same inputs,
and to the golden fixtures the reference produced (tests/golden/)."""
import json
import math
import os

import numpy as np
import pytest

import qxlib
import workloads as W

GOLD = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")


def load(name):
    path = os.path.join(GOLD, name)
    if not os.path.exists(path):
        pytest.skip("%s not generated" % name)
    with open(path) as f:
        return json.load(f)


def f32(a):
    return np.asarray(a, np.float32)


def test_port_matches_reference_mini(ref, port, mini_image):
    R, P = ref.open_image(mini_image), port.open_image(mini_image)
    x = W.head_input(R.hidden)
    for a, b in zip(R.final_head(x, 16), P.final_head(x, 16)):
        np.testing.assert_array_equal(a, b)
    for layer in range(R.layers):
        for a, b in zip(R.moe_layer(layer, x), P.moe_layer(layer, x)):
            np.testing.assert_array_equal(a, b)
    kr, kp = R.new_kv(160), P.new_kv(160)
    for step in range(0, 140):
        xi = qxlib.normal_vector(100 + step, R.hidden)
        for a, b in zip(R.attention_layer(1, step, kr, xi), P.attention_layer(1, step, kp, xi)):
            np.testing.assert_array_equal(a, b)
    for key in ("k", "v", "ks", "vs"):
        np.testing.assert_array_equal(kr[key], kp[key])


def test_port_matches_golden_mini(port, mini_image):
    g = load("golden_mini.json")
    m = port.open_image(mini_image)
    np.testing.assert_array_equal(m.embed(g["embed_token"]), f32(g["embed"]))
    normed, logits, tt, tl = m.final_head(W.head_input(m.hidden), 32)
    np.testing.assert_array_equal(logits, f32(g["head"]["logits"]))
    np.testing.assert_array_equal(normed, f32(g["head"]["normalized"]))
    assert list(tt) == g["head"]["top_tokens"]
    lo, moe, sel, w = m.moe_layer(g["moe"]["layer"], W.moe_input(m.hidden))
    assert list(sel) == g["moe"]["selected"]
    np.testing.assert_array_equal(moe, f32(g["moe"]["moe_output"]))
    np.testing.assert_array_equal(w, np.asarray(g["moe"]["weights"]))
    kv = m.new_kv(16)
    tok = g["decode"][0]["input"]
    for s, st in enumerate(g["decode"]):
        r = m.decode_step(tok, s, kv)
        assert r["token"] == st["token"]
        np.testing.assert_array_equal(r["experts"], np.asarray(st["experts"], np.uint32))
        tok = r["token"]


def test_port_attention_history_matches_golden_mini(port, mini_image):
    g = load("golden_mini.json")
    m = port.open_image(mini_image)
    layer = g["attention"]["layer"]
    KVV = m.kv_heads * m.head_dim

    def q(vec):
        vec = np.ascontiguousarray(vec, np.float32)
        out = np.zeros(vec.size, np.int8)
        s = port.f["quantize_int8"](vec.ctypes.data, out.ctypes.data, vec.size)
        return out, np.float32(s)

    for case in g["attention"]["cases"]:
        P = case["position"]
        kv = m.new_kv(P + 1)
        k, v, ks, vs = W.attn_history(P, KVV, q)
        kv["k"][layer, :P], kv["v"][layer, :P], kv["ks"][layer, :P], kv["vs"][layer, :P] = k, v, ks, vs
        res, ao, ctxv, _, _ = m.attention_layer(layer, P, kv, W.attn_input(m.hidden))
        np.testing.assert_array_equal(res, f32(case["residual"]))
        np.testing.assert_array_equal(ctxv, f32(case["context"]))
        assert list(kv["k"][layer, P]) == case["k_row"]


def test_port_decoders_match_golden(port):
    for name in ("golden_mini.json", "golden_full.json"):
        path = os.path.join(GOLD, name)
        if not os.path.exists(path):
            continue
        for d in json.load(open(path))["decoders"]:
            raw = np.frombuffer(bytes.fromhex(d["bytes"]), np.uint8).copy()
            out = np.zeros(256, np.float32)
            assert port.f["decode_block"](d["ggml_type"], raw.ctypes.data, out.ctypes.data)
            np.testing.assert_array_equal(out, f32(d["values"]), err_msg=d["tensor"])


def _rope_probe(port, tokens, q_heads_run):
    """The reference's rope/GQA known-answer probe (src/qx_format.c:4643-4731)
    rebuilt from the restatement's RoPE and INT8 primitives."""
    D, KVH, group = 128, 4, 8
    q = np.array([((i % 17) - 8) / 8.0 for i in range(q_heads_run * D)], np.float32)
    port.f["rope"](q.ctypes.data, q_heads_run, D, tokens - 1)
    kq = np.zeros((tokens, KVH * D), np.int8)
    vq = np.zeros((tokens, KVH * D), np.int8)
    ks = np.zeros(tokens, np.float32)
    vs = np.zeros(tokens, np.float32)
    for t in range(tokens):
        k = np.array([((((t + 1) * (i + 3)) % 23) - 11) / 11.0 for i in range(KVH * D)], np.float32)
        v = np.array([((((t + 2) * (i + 5)) % 19) - 9) / 9.0 for i in range(KVH * D)], np.float32)
        port.f["rope"](k.ctypes.data, KVH, D, t)
        ks[t] = port.f["quantize_int8"](k.ctypes.data, kq[t].ctypes.data, KVH * D)
        vs[t] = port.f["quantize_int8"](v.ctypes.data, vq[t].ctypes.data, KVH * D)
    scores = np.zeros((q_heads_run, tokens))
    weights = np.zeros((q_heads_run, tokens))
    ctx = np.zeros(q_heads_run * D)
    for h in range(q_heads_run):
        g = h // group
        for t in range(tokens):
            s = 0.0
            for d in range(D):
                s += float(q[h * D + d]) * float(kq[t, g * D + d]) * float(ks[t])
            scores[h, t] = s / math.sqrt(D)
        e = np.exp(scores[h] - scores[h].max())
        weights[h] = e / e.sum()
        for t in range(tokens):
            ctx[h * D:(h + 1) * D] += weights[h, t] * vq[t, g * D:(g + 1) * D].astype(np.float64) * float(vs[t])
    return scores, weights, ctx


def test_rope_gqa_known_answers():
    import oracle_bind
    port = oracle_bind.Checker("port")
    for case in load("golden_mini.json")["rope_gqa_golden"]:
        T, QR = case["args"]["tokens"], case["args"]["q_heads_run"]
        if T > 20:
            continue
        scores, weights, ctx = _rope_probe(port, T, QR)
        last, st = QR - 1, (1 if T > 1 else 0)
        want_s = [scores[0, 0], scores[0, st], scores[last, 0], scores[last, st]]
        want_w = [weights[0, 0], weights[0, st], weights[last, 0], weights[last, st]]
        want_c = [ctx[0], ctx[64], ctx[last * 128], ctx[last * 128 + 64]]
        np.testing.assert_allclose(case["score_samples"], want_s, rtol=1e-12, atol=1e-12)
        np.testing.assert_allclose(case["weight_samples"], want_w, rtol=1e-12, atol=1e-12)
        np.testing.assert_allclose(case["context_samples"], want_c, rtol=1e-12, atol=1e-12)


def test_port_matches_golden_full_head_and_moe(port, full_image):
    g = load("golden_full.json")
    m = port.open_image(full_image)
    normed, logits, tt, tl = m.final_head(W.head_input(m.hidden), 32)
    assert list(tt) == g["head"]["top_tokens"]
    np.testing.assert_array_equal(tl, np.asarray(g["head"]["top_logits"]))
    np.testing.assert_array_equal(logits[g["head"]["logits_sample_idx"]], f32(g["head"]["logits_sample"]))
    lo, moe, sel, w = m.moe_layer(g["moe"]["layer"], W.moe_input(m.hidden))
    assert list(sel) == g["moe"]["selected"]
    np.testing.assert_array_equal(moe, f32(g["moe"]["moe_output"]))
    np.testing.assert_array_equal(m.embed(g["embed_token"]), f32(g["embed"]))


def test_state_loop_fixture_agrees_with_the_decode_fixture():
    """golden_full.json holds two records of config 4's first greedy steps:
    "decode" from the shim's composed step (oracle/ref_shim.c) and
    "state_loop" from the reference's own unmodified CLI state loop
    (src/qx_format.c:6721, checked step by step against the shim when the
    fixture was written).  They must agree."""
    g = load("golden_full.json")
    sl = g["state_loop"]["steps"]
    for d, s in zip(g["decode"], sl):
        assert d["input"] == s["input"] and d["token"] == s["token"]
        assert d["experts"] == s["experts"]
        if d["residual"] is not None:
            np.testing.assert_array_equal(f32(d["residual"]), f32(s["residual"]))


def test_port_matches_the_reference_state_loop(port, full_image):
    """The C restatement against the reference's unmodified state loop: two
    greedy steps of config 4, K/V rows by FNV-1a checksum and scale."""
    sl = load("golden_full.json")["state_loop"]["steps"]
    m = port.open_image(full_image)
    kv = m.new_kv(4)
    tok = W.START_TOKEN
    for s, st in enumerate(sl[:2]):
        r = m.decode_step(tok, s, kv)
        assert r["token"] == st["token"]
        assert r["experts"].tolist() == st["experts"]
        np.testing.assert_array_equal(r["residual"], f32(st["residual"]))
        for layer in range(m.layers):
            assert port.f["fnv1a64"](kv["k"][layer, s].ctypes.data, kv["k"].shape[2]) == st["k_checksum"][layer]
            assert port.f["fnv1a64"](kv["v"][layer, s].ctypes.data, kv["v"].shape[2]) == st["v_checksum"][layer]
            assert kv["ks"][layer, s] == np.float32(st["k_scale"][layer])
        tok = r["token"]
