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
