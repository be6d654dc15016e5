"""ctypes bindings over the engine's two in-tree libraries.

libqxhost.so holds the host plumbing (QXF1 containers, the seeded synthetic
model); libqxcuda.so is the C-ABI decode engine declared in include/qx_cuda.h.
Nothing here computes: every call goes straight to native code, and the engine
entry points raise if libqxcuda.so is missing instead of falling back.
"""
import ctypes as C
import os

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))

F32 = 0
Q4_K, Q6_K, IQ2_XS, IQ3_XXS, IQ4_XS = 12, 14, 17, 18, 23


class SynthConfig(C.Structure):
    _fields_ = [(n, C.c_uint32) for n in (
        "layers", "hidden", "q_heads", "kv_heads", "head_dim", "vocab", "experts", "experts_per_token",
        "moe_intermediate", "attn_type", "gate_type", "up_type", "down_type", "embd_type", "head_type")] + [
        ("seed", C.c_uint64), ("threads", C.c_uint32)]


class CudaModel(C.Structure):
    _fields_ = [(n, C.c_uint32) for n in (
        "layers", "hidden", "q_heads", "kv_heads", "head_dim", "vocab", "experts", "experts_per_token",
        "moe_intermediate")]


class CudaOptions(C.Structure):
    _fields_ = [("device", C.c_int32), ("ctx_tokens", C.c_uint32), ("flags", C.c_uint32),
                ("ep_rank", C.c_uint32), ("ep_world", C.c_uint32), ("reserved", C.c_uint32),
                ("stream", C.c_void_p), ("nccl_comm", C.c_void_p)]


class CudaProfile(C.Structure):
    _fields_ = [("backend", C.c_char * 32), ("device_bytes", C.c_uint64), ("host_to_device_bytes", C.c_uint64),
                ("device_to_host_bytes", C.c_uint64), ("kernel_launches", C.c_uint64),
                ("graph_replays", C.c_uint64), ("decode_steps", C.c_uint64)]


def _load(name):
    path = os.path.join(HERE, name)
    if not os.path.exists(path):
        raise RuntimeError("%s is not built (run make in %s)" % (name, HERE))
    return C.CDLL(path)


_host = None
_cuda = None


def host():
    global _host
    if _host is None:
        lib = _load("libqxhost.so")
        lib.qxh_synth_image_size.argtypes = [C.POINTER(SynthConfig), C.POINTER(C.c_uint64), C.c_char_p, C.c_uint64]
        lib.qxh_synth_build.argtypes = [C.POINTER(SynthConfig), C.c_void_p, C.c_uint64, C.c_char_p, C.c_uint64]
        lib.qxh_synth_default.argtypes = [C.POINTER(SynthConfig), C.c_uint64]
        lib.qxh_normal_vector.argtypes = [C.c_uint64, C.c_void_p, C.c_uint64]
        lib.qxh_fp16_to_f32.argtypes = [C.c_uint16]
        lib.qxh_fp16_to_f32.restype = C.c_float
        lib.qxh_f32_to_fp16.argtypes = [C.c_float]
        lib.qxh_f32_to_fp16.restype = C.c_uint16
        lib.qxh_tables.restype = C.c_void_p
        lib.qxh_sha256_init.argtypes = [C.c_void_p]
        lib.qxh_sha256_update.argtypes = [C.c_void_p, C.c_void_p, C.c_uint64]
        lib.qxh_sha256_final.argtypes = [C.c_void_p, C.c_void_p]
        VP, U32 = C.c_void_p, C.c_uint32
        lib.qxh_kv_snapshot_write.argtypes = [C.c_char_p, U32, U32, U32, U32, U32, U32, U32, VP, VP, VP, VP,
                                              C.c_char_p, C.c_uint64]
        lib.qxh_kv_snapshot_read.argtypes = [C.c_char_p, U32, U32, U32, U32, U32, VP, VP, VP, VP, VP, VP,
                                             C.c_char_p, C.c_uint64]
        _host = lib
    return _host


def err_buf():
    return C.create_string_buffer(512)


def check(ok, err, what):
    if not ok:
        raise RuntimeError("%s failed: %s" % (what, err.value.decode(errors="replace")))


def synth_config(seed=7, **over):
    cfg = SynthConfig()
    host().qxh_synth_default(C.byref(cfg), seed)
    for k, v in over.items():
        setattr(cfg, k, v)
    return cfg


def mini_config(seed=7, **over):
    """A small model of the same structure (fast CPU oracles): 2 layers,
    hidden 512, 8 query / 2 KV heads of 128, 4096 vocab, 16 experts of 256."""
    base = dict(layers=2, hidden=512, q_heads=8, kv_heads=2, head_dim=128, vocab=4096, experts=16,
                experts_per_token=8, moe_intermediate=256)
    base.update(over)
    return synth_config(seed, **base)


def build_image(cfg):
    """Return a numpy uint8 array holding a complete QXF1 container."""
    size = C.c_uint64()
    err = err_buf()
    check(host().qxh_synth_image_size(C.byref(cfg), C.byref(size), err, len(err)), err, "qxh_synth_image_size")
    img = np.empty(size.value, dtype=np.uint8)
    check(host().qxh_synth_build(C.byref(cfg), img.ctypes.data, size.value, err, len(err)), err, "qxh_synth_build")
    return img


def normal_vector(seed, n):
    out = np.empty(n, dtype=np.float32)
    host().qxh_normal_vector(seed, out.ctypes.data, n)
    return out


# ---- engine (libqxcuda.so) ---------------------------------------------------
ENGINE_SYMBOLS = [
    "qx_cuda_engine_create", "qx_cuda_engine_create_from_qxf", "qx_cuda_engine_create_from_image",
    "qx_cuda_engine_destroy", "qx_cuda_reset", "qx_cuda_decode_step", "qx_cuda_generate", "qx_cuda_final_head",
    "qx_cuda_moe_layer", "qx_cuda_attention_layer", "qx_cuda_embed", "qx_cuda_kv_write", "qx_cuda_kv_read",
    "qx_cuda_profile_get", "qx_cuda_time_kernels", "qx_cuda_phase_trace", "qx_cuda_stream",
    "qx_cuda_ep_handle", "qx_cuda_ep_connect", "qx_cuda_ep_partition", "qx_cuda_kv_export", "qx_cuda_kv_import",
    "qx_cuda_moe_batch", "qx_cuda_prefill", "qx_cuda_decode_batch",
]

VERIFY_CHECKSUMS = 0x1
NO_GRAPH = 0x2
PER_STAGE = 0x4


def cuda():
    """Load libqxcuda.so and declare its C signatures (include/qx_cuda.h)."""
    global _cuda
    if _cuda is None:
        lib = _load("libqxcuda.so")
        P, U32, U64, I32 = C.c_void_p, C.c_uint32, C.c_uint64, C.c_int32
        E = C.c_char_p
        sig = {
            "qx_cuda_engine_create_from_qxf": [C.c_char_p, C.POINTER(CudaOptions), C.POINTER(P), E, U64],
            "qx_cuda_engine_create_from_image": [P, U64, C.POINTER(CudaOptions), C.POINTER(P), E, U64],
            "qx_cuda_reset": [P, E, U64],
            "qx_cuda_decode_step": [P, U32, U32, P, P, P, P, P, E, U64],
            "qx_cuda_generate": [P, U32, U32, U32, P, E, U64],
            "qx_cuda_final_head": [P, P, P, P, U32, P, P, E, U64],
            "qx_cuda_moe_layer": [P, U32, P, P, P, P, P, E, U64],
            "qx_cuda_moe_batch": [P, U32, U32, P, P, P, P, P, E, U64],
            "qx_cuda_prefill": [P, P, U32, U32, P, P, E, U64],
            "qx_cuda_decode_batch": [P, U32, P, P, P, P, E, U64],
            "qx_cuda_attention_layer": [P, U32, U32, P, P, P, E, U64],
            "qx_cuda_embed": [P, U32, P, E, U64],
            "qx_cuda_kv_write": [P, U32, U32, U32, P, P, P, P, E, U64],
            "qx_cuda_kv_read": [P, U32, U32, U32, P, P, P, P, E, U64],
            "qx_cuda_profile_get": [P, C.POINTER(CudaProfile)],
            "qx_cuda_time_kernels": [P, U32, U32, U32, C.c_char_p, U64, P, P, U32, P, E, U64],
            "qx_cuda_phase_trace": [P, U32, U32, P, U32, P, E, U64],
            "qx_cuda_ep_handle": [P, P, U64, E, U64],
            "qx_cuda_ep_connect": [P, P, U64, U32, E, U64],
            "qx_cuda_ep_partition": [U32, U32, U32, U32, P],
            "qx_cuda_kv_export": [P, C.c_char_p, U32, U32, U32, E, U64],
            "qx_cuda_kv_import": [P, C.c_char_p, U32, P, P, E, U64],
        }
        for name, args in sig.items():
            fn = getattr(lib, name)
            fn.argtypes = args
            fn.restype = C.c_int
        lib.qx_cuda_engine_destroy.argtypes = [P]
        lib.qx_cuda_engine_destroy.restype = None
        lib.qx_cuda_stream.argtypes = [P]
        lib.qx_cuda_stream.restype = P
        _cuda = lib
    return _cuda


def _p(a):
    return None if a is None else a.ctypes.data


def sha256(data):
    """SHA-256 digest (bytes) by the host library's implementation."""
    state = C.create_string_buffer(128)
    buf = bytes(data)
    out = C.create_string_buffer(32)
    host().qxh_sha256_init(state)
    host().qxh_sha256_update(state, buf, len(buf))
    host().qxh_sha256_final(state, out)
    return out.raw


def kv_snapshot_write(path, k, v, ks, vs, positions, next_token, seed, kv_heads, head_dim):
    """Host writer of a QXKVSNP1 file from arrays k, v [layers][ctx][kv_heads*head_dim]
    (int8) and ks, vs [layers][ctx] (float32)."""
    layers, ctx = ks.shape
    err = err_buf()
    ok = host().qxh_kv_snapshot_write(str(path).encode(), layers, positions, ctx, kv_heads, head_dim, next_token, seed,
                                      _p(k), _p(v), _p(ks), _p(vs), err, len(err))
    check(ok, err, "qxh_kv_snapshot_write")


def kv_snapshot_read(path, layers, ctx, kv_heads, head_dim, seed):
    """Host reader; returns (k, v, ks, vs, positions, next_token)."""
    kvv = kv_heads * head_dim
    k = np.zeros((layers, ctx, kvv), np.int8)
    v = np.zeros((layers, ctx, kvv), np.int8)
    ks = np.zeros((layers, ctx), np.float32)
    vs = np.zeros((layers, ctx), np.float32)
    pos, nt = np.zeros(1, np.uint32), np.zeros(1, np.uint32)
    err = err_buf()
    ok = host().qxh_kv_snapshot_read(str(path).encode(), layers, ctx, kv_heads, head_dim, seed, _p(k), _p(v), _p(ks),
                                     _p(vs), _p(pos), _p(nt), err, len(err))
    check(ok, err, "qxh_kv_snapshot_read")
    return k, v, ks, vs, int(pos[0]), int(nt[0])


def ep_partition(experts, vocab, world, rank):
    """(expert_begin, expert_end, head_row_begin, head_row_end) of `rank`
    (qx_cuda_ep_partition; host-only, no GPU needed)."""
    out = np.zeros(4, np.uint32)
    if not cuda().qx_cuda_ep_partition(experts, vocab, world, rank, out.ctypes.data):
        raise ValueError("invalid expert-parallel partition arguments")
    return tuple(int(v) for v in out)


def connect_ep(engine, all_gather):
    """Map every rank's exchange buffer into `engine`.  all_gather(obj) must
    return the list of every rank's obj in rank order (e.g. a wrapper of
    torch.distributed.all_gather_object)."""
    handles = all_gather(engine.ep_handle())
    engine.ep_connect(handles)
    return handles


class Engine:
    """Thin owner of a qx_cuda_engine*; every method is one C-ABI call."""

    def __init__(self, image=None, path=None, ctx=4096, device=-1, flags=0, stream=None, ep_rank=0, ep_world=1):
        lib = cuda()
        opt = CudaOptions()
        opt.device = device
        opt.ctx_tokens = ctx
        opt.flags = flags
        opt.stream = stream
        opt.ep_rank = ep_rank
        opt.ep_world = ep_world
        h = C.c_void_p()
        err = err_buf()
        if path is not None:
            ok = lib.qx_cuda_engine_create_from_qxf(path.encode(), C.byref(opt), C.byref(h), err, len(err))
        else:
            ok = lib.qx_cuda_engine_create_from_image(image.ctypes.data, image.nbytes, C.byref(opt), C.byref(h), err,
                                                      len(err))
        check(ok, err, "qx_cuda_engine_create")
        self.h = h
        self.lib = lib
        self.ctx = ctx
        hdr = np.frombuffer((image[:272].tobytes() if image is not None else open(path, "rb").read(272)), np.uint32)
        m = hdr[14:27]
        self.layers, self.hidden, self.q_heads, self.kv_heads, self.head_dim = (int(m[2]), int(m[3]), int(m[5]),
                                                                                  int(m[6]), int(m[7]))
        self.vocab, self.experts, self.moe_intermediate = int(m[8]), int(m[10]), int(m[12])

    EP_HANDLE_BYTES = 64

    def kv_export(self, path, positions, next_token, seed):
        self._call("qx_cuda_kv_export", str(path).encode(), positions, next_token, seed)

    def kv_import(self, path, seed):
        """Returns (positions, next_token)."""
        pos, nt = np.zeros(1, np.uint32), np.zeros(1, np.uint32)
        self._call("qx_cuda_kv_import", str(path).encode(), seed, _p(pos), _p(nt))
        return int(pos[0]), int(nt[0])

    def ep_handle(self):
        """This rank's exchange-buffer handle (bytes) for qx_cuda_ep_connect."""
        buf = C.create_string_buffer(self.EP_HANDLE_BYTES)
        self._call("qx_cuda_ep_handle", buf, self.EP_HANDLE_BYTES)
        return buf.raw

    def ep_connect(self, handles):
        """Map every rank's exchange buffer; handles: list of bytes in rank order."""
        blob = b"".join(h.ljust(self.EP_HANDLE_BYTES, b"\0")[:self.EP_HANDLE_BYTES] for h in handles)
        buf = C.create_string_buffer(blob, len(blob))
        self._call("qx_cuda_ep_connect", buf, self.EP_HANDLE_BYTES, len(handles))

    def close(self):
        if getattr(self, "h", None):
            self.lib.qx_cuda_engine_destroy(self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def _call(self, name, *args):
        err = err_buf()
        check(getattr(self.lib, name)(self.h, *args, err, len(err)), err, name)

    def reset(self):
        self._call("qx_cuda_reset")

    def decode_step(self, token, position, want_logits=False, want_residual=False, want_experts=False):
        nxt = np.zeros(1, np.uint32)
        logits = np.zeros(self.vocab, np.float32) if want_logits else None
        res = np.zeros(self.hidden, np.float32) if want_residual else None
        ex = np.zeros((self.layers, 8), np.uint32) if want_experts else None
        rw = np.zeros((self.layers, 8), np.float32) if want_experts else None
        self._call("qx_cuda_decode_step", token, position, _p(nxt), _p(logits), _p(res), _p(ex), _p(rw))
        return dict(token=int(nxt[0]), logits=logits, residual=res, experts=ex, routing=rw)

    def generate(self, token, position, steps):
        out = np.zeros(steps, np.uint32)
        self._call("qx_cuda_generate", token, position, steps, _p(out))
        return out

    def final_head(self, residual, top_n=8):
        residual = np.ascontiguousarray(residual, np.float32)
        normed = np.zeros(self.hidden, np.float32)
        logits = np.zeros(self.vocab, np.float32)
        tt = np.zeros(top_n, np.uint32)
        tl = np.zeros(top_n, np.float32)
        self._call("qx_cuda_final_head", _p(residual), _p(normed), _p(logits), top_n, _p(tt), _p(tl))
        return normed, logits, tt, tl

    def moe_layer(self, layer, x):
        x = np.ascontiguousarray(x, np.float32)
        out = np.zeros(self.hidden, np.float32)
        moe = np.zeros(self.hidden, np.float32)
        sel = np.zeros(8, np.uint32)
        w = np.zeros(8, np.float32)
        self._call("qx_cuda_moe_layer", layer, _p(x), _p(out), _p(moe), _p(sel), _p(w))
        return out, moe, sel, w

    def moe_batch(self, layer, x):
        """x: [tokens][hidden] residuals; returns (layer_output, moe_output,
        selected [tokens][8], weights [tokens][8]) of qx_cuda_moe_batch."""
        x = np.ascontiguousarray(x, np.float32)
        t = x.shape[0]
        out = np.zeros_like(x)
        moe = np.zeros_like(x)
        sel = np.zeros((t, 8), np.uint32)
        w = np.zeros((t, 8), np.float32)
        self._call("qx_cuda_moe_batch", layer, t, _p(x), _p(out), _p(moe), _p(sel), _p(w))
        return out, moe, sel, w

    def prefill(self, tokens, position=0, want_residual=False):
        """Prompt prefill (qx_cuda_prefill): returns the greedy next token (and
        the last prompt token's final residual)."""
        tokens = np.ascontiguousarray(tokens, np.uint32)
        nxt = np.zeros(1, np.uint32)
        res = np.zeros(self.hidden, np.float32) if want_residual else None
        self._call("qx_cuda_prefill", _p(tokens), tokens.size, position, _p(nxt), _p(res))
        return (int(nxt[0]), res) if want_residual else int(nxt[0])

    def decode_batch(self, slots, tokens, positions):
        """One greedy step of several sequences (qx_cuda_decode_batch)."""
        slots = np.ascontiguousarray(slots, np.uint32)
        tokens = np.ascontiguousarray(tokens, np.uint32)
        positions = np.ascontiguousarray(positions, np.uint32)
        nxt = np.zeros(slots.size, np.uint32)
        self._call("qx_cuda_decode_batch", slots.size, _p(slots), _p(tokens), _p(positions), _p(nxt))
        return nxt

    def attention_layer(self, layer, position, residual):
        res = np.array(residual, np.float32, copy=True)
        ao = np.zeros(self.hidden, np.float32)
        ctxv = np.zeros(self.q_heads * self.head_dim, np.float32)
        self._call("qx_cuda_attention_layer", layer, position, _p(res), _p(ao), _p(ctxv))
        return res, ao, ctxv

    def embed(self, token):
        out = np.zeros(self.hidden, np.float32)
        self._call("qx_cuda_embed", token, _p(out))
        return out

    def kv_write(self, layer, first, k, v, ks, vs):
        k, v = np.ascontiguousarray(k, np.int8), np.ascontiguousarray(v, np.int8)
        ks, vs = np.ascontiguousarray(ks, np.float32), np.ascontiguousarray(vs, np.float32)
        self._call("qx_cuda_kv_write", layer, first, len(ks), _p(k), _p(v), _p(ks), _p(vs))

    def kv_read(self, layer, first, count):
        kvv = self.kv_heads * self.head_dim
        k = np.zeros((count, kvv), np.int8)
        v = np.zeros((count, kvv), np.int8)
        ks = np.zeros(count, np.float32)
        vs = np.zeros(count, np.float32)
        self._call("qx_cuda_kv_read", layer, first, count, _p(k), _p(v), _p(ks), _p(vs))
        return k, v, ks, vs

    def profile(self):
        p = CudaProfile()
        self.lib.qx_cuda_profile_get(self.h, C.byref(p))
        return {f: (getattr(p, f).decode() if f == "backend" else int(getattr(p, f))) for f, _ in p._fields_}

    def time_kernels(self, token, position, steps):
        names = C.create_string_buffer(4096)
        ms = np.zeros(64, np.float32)
        ln = np.zeros(64, np.uint32)
        cnt = np.zeros(1, np.uint32)
        self._call("qx_cuda_time_kernels", token, position, steps, names, len(names), _p(ms), _p(ln), 64, _p(cnt))
        keys = names.value.decode().split(";")
        return {k: (float(ms[i]), int(ln[i])) for i, k in enumerate(keys[:int(cnt[0])])}

    PHASES = ("qkv", "scores", "context", "oproj", "router", "gateup", "down")

    def phase_trace(self, token, position, detail=False):
        """Run one persistent decode step with %globaltimer stamps at every grid
        barrier; returns {"qkv": [us per layer], ..., "head": us, "total": us}.
        The "qkv" phase of layer 0 includes the embedding lookup.  With
        detail=True also "markers" (epochs x 8 in-phase stamps of CTA 0, us from
        the previous barrier exit, NaN where unset) and "arrivals" (epochs x
        CTAs, us from the previous barrier exit)."""
        P = len(self.PHASES)
        n = 3 + P * self.layers
        cap = n * (9 + 1024)
        st = np.zeros(cap, np.uint64)
        cnt = np.zeros(1, np.uint32)
        self._call("qx_cuda_phase_trace", token, position, _p(st), cap, _p(cnt))
        st = st[:int(cnt[0])].astype(np.int64)
        ex = st[:n - 1]
        d = np.diff(ex) / 1000.0
        out = {name: d[i:P * self.layers:P].tolist() for i, name in enumerate(self.PHASES)}
        out["head"] = float(d[P * self.layers:].sum())
        out["total"] = float(d.sum())
        if detail:
            grid = (len(st) - 9 * n) // n
            prev = np.concatenate([[ex[0]], ex[:-1]])[:, None]          # exit of epoch e-1
            mk = st[n:9 * n].reshape(n, 8)[:n - 1].astype(np.float64)
            mk = np.where(mk > 0, (mk - prev) / 1000.0, np.nan)
            ar = st[9 * n:].reshape(n, grid)[:n - 1].astype(np.float64)
            ar = np.where(ar > 0, (ar - prev) / 1000.0, np.nan)
            out["markers"], out["arrivals"] = mk, ar
        return out

    def stream(self):
        return self.lib.qx_cuda_stream(self.h)
