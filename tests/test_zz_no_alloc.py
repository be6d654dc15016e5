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


def test_final_head_noalloc_rejects_oversize():
    lib = qxlib.cuda()
    fn = lib.qx_cuda_final_head_noalloc
    err = qxlib.err_buf()
    one = C.c_void_p(16)
    ok = fn(one, one, one, 4096, 4096, None, one, None, err, len(err))
    assert ok == 0 and b"at most 2048" in err.value
