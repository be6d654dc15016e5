"""The allocation-free head entry point (qx_cuda_final_head_noalloc).

Some callers cannot allocate device memory themselves: a plugin living inside
a host that owns every allocation, or code that must not allocate between
stream-ordered steps.  For them the library offers one head entry point whose
scratch lives in a fixed array inside the library; the caller passes only its
own input and output buffers.  This test allocates those buffers itself (with
torch) and checks, over two calls in a row, that the entry point matches the
regular qx_cuda_final_head on the same residual within the suite's tolerance
(tests/qxtol.py) and picks the same argmax token.  It sits in its own file,
collected last, and runs alone or after the other tests.
"""
import ctypes as C
import struct

import numpy as np
import pytest

import qxlib
import workloads as W
from qxtol import assert_close

pytestmark = pytest.mark.gpu


def tensor_bytes(img, name):
    hdr = img[:272].tobytes()
    count = struct.unpack_from("<I", hdr, 16)[0]
    diro = struct.unpack_from("<Q", hdr, 24)[0]
    for i in range(count):
        e = img[diro + 208 * i: diro + 208 * (i + 1)].tobytes()
        if e[:96].split(b"\0")[0].decode() == name:
            off, size = struct.unpack_from("<QQ", e, 144)
            return img[off: off + size]
    raise KeyError(name)


def test_final_head_noalloc_matches_final_head(mini_image):
    import torch
    lib = qxlib.cuda()
    fn = lib.qx_cuda_final_head_noalloc
    fn.argtypes = [C.c_void_p, C.c_void_p, C.c_void_p, C.c_uint32, C.c_uint32, C.c_void_p, C.c_void_p, C.c_void_p,
                   C.c_char_p, C.c_uint64]
    fn.restype = C.c_int
    eng = qxlib.Engine(mini_image, ctx=16, device=0)
    H, V = eng.hidden, eng.vocab
    dev = torch.device("cuda", 0)
    norm = torch.from_numpy(np.frombuffer(tensor_bytes(mini_image, "output_norm.weight").tobytes(),
                                          np.float32).copy()).to(dev)
    head = torch.from_numpy(tensor_bytes(mini_image, "output.weight").copy()).to(dev)
    logits = torch.empty(V, dtype=torch.float32, device=dev)
    argmax = torch.empty(1, dtype=torch.int32, device=dev)
    stream = torch.cuda.current_stream(dev)
    for seed in (1, 2):                      # two calls in a row share the library's scratch
        x = qxlib.normal_vector(seed, H)
        _, want_logits, want_top, _ = eng.final_head(x, 1)
        xd = torch.from_numpy(x).to(dev)
        err = qxlib.err_buf()
        ok = fn(xd.data_ptr(), norm.data_ptr(), head.data_ptr(), H, V, logits.data_ptr(), argmax.data_ptr(),
                C.c_void_p(stream.cuda_stream), err, len(err))
        assert ok, err.value
        torch.cuda.synchronize(dev)
        assert_close(logits.cpu().numpy(), want_logits, what="no-alloc logits")
        assert int(argmax.cpu().item()) == int(want_top[0])
    eng.close()


def _fn():
    fn = qxlib.cuda().qx_cuda_final_head_noalloc
    fn.argtypes = [C.c_void_p, C.c_void_p, C.c_void_p, C.c_uint32, C.c_uint32, C.c_void_p, C.c_void_p, C.c_void_p,
                   C.c_char_p, C.c_uint64]
    fn.restype = C.c_int
    return fn


def test_final_head_noalloc_full_geometry_matches_the_reference(full_image):
    """H = 2048, V = 151936 (config 1): argmax and logits sample against the
    reference's own head (tests/golden/golden_full.json), twice in a row, the
    second call without a logits buffer."""
    import json
    import os
    import torch
    with open(os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden", "golden_full.json")) as f:
        g = json.load(f)["head"]
    fn = _fn()
    dev = torch.device("cuda", 0)
    H, V = 2048, 151936
    norm = torch.from_numpy(np.frombuffer(tensor_bytes(full_image, "output_norm.weight").tobytes(),
                                          np.float32).copy()).to(dev)
    head = torch.from_numpy(tensor_bytes(full_image, "output.weight").copy()).to(dev)
    xd = torch.from_numpy(W.head_input(H)).to(dev)
    logits = torch.empty(V, dtype=torch.float32, device=dev)
    argmax = torch.empty(1, dtype=torch.int32, device=dev)
    stream = C.c_void_p(torch.cuda.current_stream(dev).cuda_stream)
    for with_logits in (True, False):
        argmax.fill_(-7)
        err = qxlib.err_buf()
        ok = fn(xd.data_ptr(), norm.data_ptr(), head.data_ptr(), H, V, logits.data_ptr() if with_logits else None,
                argmax.data_ptr(), stream, err, len(err))
        assert ok, err.value
        torch.cuda.synchronize(dev)
        assert int(argmax.cpu().item()) == g["top_tokens"][0]
        if with_logits:
            got = logits.cpu().numpy()
            assert_close(got[g["logits_sample_idx"]], g["logits_sample"], what="no-alloc logits")


def test_final_head_noalloc_non_finite_and_misaligned(mini_image):
    import torch
    fn = _fn()
    dev = torch.device("cuda", 0)
    H, V = 512, 4096
    norm = torch.from_numpy(np.frombuffer(tensor_bytes(mini_image, "output_norm.weight").tobytes(),
                                          np.float32).copy()).to(dev)
    raw = tensor_bytes(mini_image, "output.weight")
    head = torch.zeros(raw.size + 64, dtype=torch.uint8, device=dev)
    head[:raw.size] = torch.from_numpy(raw.copy()).to(dev)
    x = qxlib.normal_vector(3, H)
    x[17] = np.inf
    xd = torch.from_numpy(x).to(dev)
    argmax = torch.zeros(1, dtype=torch.int32, device=dev)
    stream = C.c_void_p(torch.cuda.current_stream(dev).cuda_stream)
    err = qxlib.err_buf()
    ok = fn(xd.data_ptr(), norm.data_ptr(), head.data_ptr(), H, V, None, argmax.data_ptr(), stream, err, len(err))
    assert ok, err.value
    torch.cuda.synchronize(dev)
    assert int(argmax.cpu().item()) & 0xFFFFFFFF == 0xFFFFFFFF
    # a head pointer off a 16-byte boundary is refused on the host
    err = qxlib.err_buf()
    ok = fn(xd.data_ptr(), norm.data_ptr(), head.data_ptr() + 8, H, V, None, argmax.data_ptr(), stream, err, len(err))
    assert ok == 0 and b"16-byte aligned" in err.value


def test_final_head_noalloc_rejects_oversize():
    lib = qxlib.cuda()
    fn = lib.qx_cuda_final_head_noalloc
    err = qxlib.err_buf()
    one = C.c_void_p(16)
    ok = fn(one, one, one, 4096, 4096, None, one, None, err, len(err))
    assert ok == 0 and b"at most 2048" in err.value
