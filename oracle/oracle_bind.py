"""TEST INFRASTRUCTURE ONLY: ctypes bindings for the two CPU checkers.

  _ref/libqxref.so    - the reference's own C (src/qx_format.c) behind ref_shim.c
  _ref/libqxoracle.so - this repo's C restatement (qx_oracle.c)

Both export the same entry points under the prefixes ``qxref_`` and ``qxo_``,
so `Checker("ref")` and `Checker("port")` are interchangeable.  Only tests/,
__graft_entry__.smoke() and bench.py's CPU legs import this module.
"""
import ctypes as C
import os

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
P = C.c_void_p
U32, U64, F32 = C.c_uint32, C.c_uint64, C.c_float


def _path(kind):
    return os.path.join(HERE, "_ref", "libqxref.so" if kind == "ref" else "libqxoracle.so")


def available(kind):
    return os.path.exists(_path(kind))


def _ptr(a):
    return None if a is None else a.ctypes.data


class Checker:
    def __init__(self, kind="port"):
        path = _path(kind)
        if not os.path.exists(path):
            raise RuntimeError("checker %s not built: %s (make -C oracle)" % (kind, path))
        self.kind = kind
        self.lib = C.CDLL(path)
        pre = "qxref_" if kind == "ref" else "qxo_"
        sig = {
            "open_path": ([C.c_char_p, C.c_int, C.POINTER(P), C.c_char_p, U64], C.c_int),
            "open_image": ([P, U64, C.POINTER(P), C.c_char_p, U64], C.c_int),
            "close": ([P], None),
            "embed": ([P, U32, P, C.c_char_p, U64], C.c_int),
            "final_head": ([P, P, P, P, U32, P, P, C.c_char_p, U64], C.c_int),
            "moe_layer": ([P, U32, P, P, P, P, P, C.c_char_p, U64], C.c_int),
            "attention_layer": ([P, U32, U32, U32, P, P, P, P, P, P, P, P, P, C.c_char_p, U64], C.c_int),
            "decode_step": ([P, U32, U32, U32, P, P, P, P, P, P, P, P, P, P, C.c_char_p, U64], C.c_int),
            "quantize_int8": ([P, P, U32], F32),
            "rope": ([P, U32, U32, U32], None),
            "decode_block": ([U32, P, P], C.c_int),
            "fp16_to_f32": ([C.c_uint16], F32),
            "fnv1a64": ([P, U64], U64),
        }
        self.f = {}
        for name, (args, res) in sig.items():
            fn = getattr(self.lib, pre + name, None)
            if fn is None:
                continue
            fn.argtypes = args
            fn.restype = res
            self.f[name] = fn
        if kind == "ref":
            self.lib.qxref_table.argtypes = [U32]
            self.lib.qxref_table.restype = P
            self.lib.qxref_state_loop_json.argtypes = [C.c_char_p, U32, U32, U32, C.c_char_p, C.c_char_p,
                                                       C.c_char_p, U64]
            self.lib.qxref_rope_gqa_golden_json.argtypes = [U32, U32, C.c_char_p, C.c_char_p, U64]
        if kind == "port":
            self.lib.qxo_set_threads.argtypes = [U32]

    def _err(self):
        return C.create_string_buffer(512)

    def _check(self, ok, err, what):
        if not ok:
            raise RuntimeError("%s %s: %s" % (self.kind, what, err.value.decode(errors="replace")))

    def open_image(self, img):
        m = P()
        err = self._err()
        self._check(self.f["open_image"](img.ctypes.data, img.nbytes, C.byref(m), err, len(err)), err, "open_image")
        return Model(self, m, img)

    def open_path(self, path):
        m = P()
        err = self._err()
        self._check(self.f["open_path"](path.encode(), 1, C.byref(m), err, len(err)), err, "open_path")
        return Model(self, m, None, path)


class Model:
    """One opened model on a checker; keeps the image alive."""

    def __init__(self, checker, handle, image, path=None):
        self.c, self.h, self.image = checker, handle, image
        if image is not None:
            raw = image[:272].tobytes()
        else:
            with open(path, "rb") as fh:
                raw = fh.read(272)
        hdr = np.frombuffer(raw, dtype=np.uint32)
        m = hdr[14:27]
        (self.layers, self.hidden, self.q_heads, self.kv_heads, self.head_dim, self.vocab, self.experts,
         self.moe_intermediate) = (int(m[2]), int(m[3]), int(m[5]), int(m[6]), int(m[7]), int(m[8]), int(m[10]),
                                   int(m[12]))

    def close(self):
        if self.h:
            self.c.f["close"](self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def _call(self, name, *args):
        err = self.c._err()
        self.c._check(self.c.f[name](self.h, *args, err, len(err)), err, name)

    def embed(self, token):
        out = np.zeros(self.hidden, np.float32)
        self._call("embed", token, _ptr(out))
        return out

    def final_head(self, residual, top_n=8):
        residual = np.ascontiguousarray(residual, np.float32)
        normed = np.zeros(self.hidden, np.float32)
        logits = np.zeros(self.vocab, np.float32)
        tt = np.zeros(top_n, np.uint32)
        tl = np.zeros(top_n, np.float64)
        self._call("final_head", _ptr(residual), _ptr(normed), _ptr(logits), top_n, _ptr(tt), _ptr(tl))
        return normed, logits, tt, tl

    def moe_layer(self, layer, x):
        x = np.ascontiguousarray(x, np.float32)
        out = np.zeros(self.hidden, np.float32)
        moe = np.zeros(self.hidden, np.float32)
        sel = np.zeros(8, np.uint32)
        w = np.zeros(8, np.float64)
        self._call("moe_layer", layer, _ptr(x), _ptr(out), _ptr(moe), _ptr(sel), _ptr(w))
        return out, moe, sel, w

    def new_kv(self, ctx):
        kvv = self.kv_heads * self.head_dim
        return dict(ctx=ctx, k=np.zeros((self.layers, ctx, kvv), np.int8), v=np.zeros((self.layers, ctx, kvv), np.int8),
                    ks=np.zeros((self.layers, ctx), np.float32), vs=np.zeros((self.layers, ctx), np.float32))

    def attention_layer(self, layer, step, kv, residual):
        """Returns (residual after attention, attention output, context, k, v)."""
        res = np.array(residual, np.float32, copy=True)
        ao = np.zeros(self.hidden, np.float32)
        ctxv = np.zeros(self.q_heads * self.head_dim, np.float32)
        kvv = self.kv_heads * self.head_dim
        k = np.zeros(kvv, np.float32)
        v = np.zeros(kvv, np.float32)
        self._call("attention_layer", layer, step, kv["ctx"], _ptr(kv["k"]), _ptr(kv["v"]), _ptr(kv["ks"]),
                   _ptr(kv["vs"]), _ptr(res), _ptr(ao), _ptr(ctxv), _ptr(k), _ptr(v))
        return res, ao, ctxv, k, v

    def decode_step(self, token, step, kv, want_logits=False):
        experts = np.zeros((self.layers, 8), np.uint32)
        routing = np.zeros((self.layers, 8), np.float64)
        res = np.zeros(self.hidden, np.float32)
        logits = np.zeros(self.vocab, np.float32) if want_logits else None
        nxt = np.zeros(1, np.uint32)
        top2 = np.zeros(2, np.float64)
        self._call("decode_step", token, step, kv["ctx"], _ptr(kv["k"]), _ptr(kv["v"]), _ptr(kv["ks"]), _ptr(kv["vs"]),
                   _ptr(experts), _ptr(routing), _ptr(res), _ptr(logits), _ptr(nxt), _ptr(top2))
        return dict(token=int(nxt[0]), experts=experts, routing=routing, residual=res, logits=logits, top2=top2)
