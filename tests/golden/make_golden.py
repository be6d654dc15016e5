"""Regenerate the golden fixtures in tests/golden/ from the reference itself.

Run in a tree that has the reference sources and a built oracle
(`make -C oracle`): every value written here comes from the reference's own C
code (oracle/_ref/libqxref.so, i.e. src/qx_format.c compiled unchanged) on the
seeded synthetic inputs of qx-mini-c_b200/workloads.py.  The GPU tests compare
the engine against these files; the CPU tests also use them to pin the C
restatement in oracle/ without the reference tree.

    python tests/golden/make_golden.py            # mini + full-size fixtures
    python tests/golden/make_golden.py --mini     # mini only (seconds)
    python tests/golden/make_golden.py --state-loop   # add the state-loop pin to golden_full.json
"""
import argparse
import json
import os
import sys
import tempfile

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, os.path.join(ROOT, "qx-mini-c_b200"))
sys.path.insert(0, os.path.join(ROOT, "oracle"))

import oracle_bind  # noqa: E402
import qxlib  # noqa: E402
import workloads as W  # noqa: E402


def fl(a):
    return [float(v) for v in np.asarray(a).ravel()]


def quantizer(ref):
    def q(vec):
        vec = np.ascontiguousarray(vec, np.float32)
        out = np.zeros(vec.size, np.int8)
        s = ref.f["quantize_int8"](vec.ctypes.data, out.ctypes.data, vec.size)
        return out, np.float32(s)
    return q


def model_fixture(ref, img, full, decode_steps, attn_positions):
    m = ref.open_image(img)
    H, V = m.hidden, m.vocab
    out = {"model_seed": W.MODEL_SEED, "full": full}
    # embedding known answer
    out["embed_token"] = W.START_TOKEN
    out["embed"] = fl(m.embed(W.START_TOKEN))
    # config 1: head
    x = W.head_input(H)
    normed, logits, tt, tl = m.final_head(x, top_n=32)
    out["head"] = {"top_tokens": [int(t) for t in tt], "top_logits": fl(tl), "normalized": fl(normed),
                   "logits_sample_idx": list(range(0, V, max(1, V // 512))),
                   "logits_sum": float(np.sum(logits, dtype=np.float64)),
                   "logits_sumsq": float(np.sum(np.asarray(logits, np.float64) ** 2))}
    out["head"]["logits_sample"] = fl(logits[out["head"]["logits_sample_idx"]])
    if not full:
        out["head"]["logits"] = fl(logits)
    # config 2: one MoE layer
    layer = min(W.MOE_LAYER, m.layers - 1)
    lo, moe, sel, w = m.moe_layer(layer, W.moe_input(H))
    out["moe"] = {"layer": layer, "selected": [int(s) for s in sel], "weights": fl(w), "moe_output": fl(moe),
                  "layer_output": fl(lo)}
    # config 3: attention with INT8 N(0,1) history at several context lengths
    layer = min(W.ATTN_LAYER, m.layers - 1)
    KVV = m.kv_heads * m.head_dim
    out["attention"] = {"layer": layer, "cases": []}
    for P in attn_positions:
        kv = m.new_kv(P + 1)
        k, v, ks, vs = W.attn_history(P, KVV, quantizer(ref))
        kv["k"][layer, :P] = k
        kv["v"][layer, :P] = v
        kv["ks"][layer, :P] = ks
        kv["vs"][layer, :P] = vs
        res, ao, ctxv, kcur, vcur = m.attention_layer(layer, P, kv, W.attn_input(H))
        out["attention"]["cases"].append({"position": P, "residual": fl(res), "attn_out": fl(ao), "context": fl(ctxv),
                                          "k_scale": float(kv["ks"][layer, P]), "v_scale": float(kv["vs"][layer, P]),
                                          "k_row": [int(a) for a in kv["k"][layer, P]],
                                          "v_row": [int(a) for a in kv["v"][layer, P]]})
    # config 4: greedy decode from START_TOKEN
    kv = m.new_kv(max(decode_steps, 1) + 1)
    tok = W.START_TOKEN
    steps = []
    for s in range(decode_steps):
        r = m.decode_step(tok, s, kv, want_logits=False)
        steps.append({"position": s, "input": tok, "token": r["token"], "experts": r["experts"].tolist(),
                      "routing": fl(r["routing"]), "top2": fl(r["top2"]),
                      "residual": fl(r["residual"]) if s in (0, decode_steps - 1) else None})
        tok = r["token"]
    out["decode"] = steps
    m.close()
    return out


def decoder_fixture(ref, img):
    """One block of each GGUF type in the model, decoded by the reference."""
    import struct
    hdr = img[:272].tobytes()
    count = struct.unpack_from("<I", hdr, 16)[0]
    diro = struct.unpack_from("<Q", hdr, 24)[0]
    seen, out = set(), []
    bsz = {12: 144, 14: 210, 17: 74, 18: 98, 23: 136}
    for i in range(count):
        e = img[diro + 208 * i: diro + 208 * (i + 1)].tobytes()
        name = e[:96].split(b"\0")[0].decode()
        flags = struct.unpack_from("<I", e, 164)[0]
        offset = struct.unpack_from("<Q", e, 144)[0]
        if flags not in bsz or flags in seen:
            continue
        seen.add(flags)
        for blk_i in (0, 1, 7):
            raw = np.ascontiguousarray(img[offset + blk_i * bsz[flags]: offset + (blk_i + 1) * bsz[flags]])
            vals = np.zeros(256, np.float32)
            ref.f["decode_block"](flags, raw.ctypes.data, vals.ctypes.data)
            out.append({"tensor": name, "ggml_type": flags, "block": blk_i, "bytes": raw.tobytes().hex(),
                        "values": fl(vals)})
    return out


def rope_golden(ref):
    outs = []
    for tokens, heads in ((2, 9), (17, 32), (64, 32)):
        with tempfile.NamedTemporaryFile(suffix=".json", delete=False) as f:
            path = f.name
        err = __import__("ctypes").create_string_buffer(256)
        assert ref.lib.qxref_rope_gqa_golden_json(tokens, heads, path.encode(), err, 256)
        with open(path) as fh:
            js = json.load(fh)
        os.unlink(path)
        js["args"] = {"tokens": tokens, "q_heads_run": heads}
        outs.append(js)
    return outs


def state_loop_fixture(ref, img, steps):
    """The reference's own, unmodified state loop (src/qx_format.c:6721, the
    CLI's `state-loop-probe --full-moe --final-head --dump-residuals`) on the
    image written to disk.  Records per step the greedy token, per layer the
    selected experts, routing weights, K/V row checksums and scales, and the
    final residual and logits sample from the dump files.  The shim's composed
    decode step (oracle/ref_shim.c) must reproduce every one of them."""
    import ctypes
    import glob
    import shutil
    tmp = tempfile.mkdtemp(prefix="qxsl")
    try:
        path = os.path.join(tmp, "model.qxf")
        img.tofile(path)
        dump = os.path.join(tmp, "dump")
        os.mkdir(dump)
        js_path = os.path.join(tmp, "out.json")
        err = ctypes.create_string_buffer(512)
        ok = ref.lib.qxref_state_loop_json(path.encode(), W.START_TOKEN, steps, steps + 1, js_path.encode(),
                                           dump.encode(), err, 512)
        assert ok, err.value
        with open(js_path) as fh:
            js = json.load(fh)
        if os.environ.get("QX_STATE_LOOP_KEEP"):
            shutil.copy(js_path, os.environ["QX_STATE_LOOP_KEEP"])
        m = ref.open_image(img)
        V = m.vocab
        sample = list(range(0, V, max(1, V // 512)))
        out = {"steps": [], "k_cache_checksum": js["k_cache_checksum"], "v_cache_checksum": js["v_cache_checksum"],
               "final_token": js["final_token"], "logits_sample_idx": sample}
        kv = m.new_kv(steps + 1)
        tok = W.START_TOKEN
        for s, st in enumerate(js["tokens"]):
            layers = st["layers"]
            res = np.fromfile(os.path.join(dump, "step-%d-layer-%d-output.f32" % (s, m.layers - 1)), np.float32)
            logits = np.fromfile(os.path.join(dump, "step-%d-logits.f32" % s), np.float32)
            assert st["input_token"] == tok and st["position"] == s
            rec = {"position": s, "input": tok, "token": st["selected_token"],
                   "experts": [l["selected_experts"] for l in layers],
                   "routing": [l["routing_weights"] for l in layers],
                   "k_checksum": [l["k_checksum"] for l in layers], "v_checksum": [l["v_checksum"] for l in layers],
                   "k_scale": [l["k_scale"] for l in layers], "v_scale": [l["v_scale"] for l in layers],
                   "residual": fl(res), "logits_sample": fl(logits[sample]), "argmax": int(np.argmax(logits))}
            # the shim's decode step must agree with the unmodified loop
            r = m.decode_step(tok, s, kv, want_logits=True)
            assert r["token"] == rec["token"], (s, r["token"], rec["token"])
            assert r["experts"].tolist() == rec["experts"], s
            assert np.array_equal(r["residual"].view(np.uint32), res.view(np.uint32)), s
            assert np.array_equal(r["logits"].view(np.uint32), logits.view(np.uint32)), s
            for layer in range(m.layers):
                assert ref.f["fnv1a64"](kv["k"][layer, s].ctypes.data, kv["k"].shape[2]) == rec["k_checksum"][layer]
                assert ref.f["fnv1a64"](kv["v"][layer, s].ctypes.data, kv["v"].shape[2]) == rec["v_checksum"][layer]
                assert np.float32(kv["ks"][layer, s]) == np.float32(rec["k_scale"][layer])
            out["steps"].append(rec)
            tok = rec["token"]
        m.close()
        assert len(glob.glob(os.path.join(dump, "*.f32"))) > 0
        return out
    finally:
        shutil.rmtree(tmp, ignore_errors=True)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--mini", action="store_true")
    ap.add_argument("--state-loop", action="store_true")
    a = ap.parse_args()
    ref = oracle_bind.Checker("ref")
    if a.state_loop:
        path = os.path.join(HERE, "golden_full.json")
        with open(path) as f:
            fx = json.load(f)
        fx["state_loop"] = state_loop_fixture(ref, qxlib.build_image(W.model_config(full=True)), steps=4)
        with open(path, "w") as f:
            json.dump(fx, f)
        print("added state_loop to golden_full.json")
        return
    mini = qxlib.build_image(W.model_config(full=False))
    fx = model_fixture(ref, mini, False, decode_steps=8, attn_positions=[0, 1, 63, 64, 130])
    fx["decoders"] = decoder_fixture(ref, mini)
    fx["rope_gqa_golden"] = rope_golden(ref)
    with open(os.path.join(HERE, "golden_mini.json"), "w") as f:
        json.dump(fx, f)
    print("wrote golden_mini.json")
    if a.mini:
        return
    full = qxlib.build_image(W.model_config(full=True))
    fx = model_fixture(ref, full, True, decode_steps=3, attn_positions=[511, 4095])
    fx["decoders"] = decoder_fixture(ref, full)
    fx["state_loop"] = state_loop_fixture(ref, full, steps=4)
    with open(os.path.join(HERE, "golden_full.json"), "w") as f:
        json.dump(fx, f)
    print("wrote golden_full.json")


if __name__ == "__main__":
    main()
