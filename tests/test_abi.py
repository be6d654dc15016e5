"""The C ABI: header is valid C, the library loads without a GPU and exports
every entry point the header declares, and argument validation happens before
any device work."""
import ctypes as C
import os
import re
import subprocess

import qxlib

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HEADER = os.path.join(ROOT, "include", "qx_cuda.h")


def declared_functions():
    text = open(HEADER).read()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(qx_cuda_\w+)\s*\(", text)))


def test_header_declares_the_engine_surface():
    names = declared_functions()
    assert set(qxlib.ENGINE_SYMBOLS) <= set(names)
    assert len(names) >= 16


def test_library_exports_every_declared_symbol():
    lib = C.CDLL(os.path.join(ROOT, "qx-mini-c_b200", "libqxcuda.so"))
    missing = [n for n in declared_functions() if not hasattr(lib, n)]
    assert not missing, missing


def test_header_compiles_as_c17(tmp_path):
    src = tmp_path / "t.c"
    src.write_text('#include "qx_cuda.h"\nint main(void){qx_cuda_options o={0}; (void)o; return 0;}\n')
    subprocess.check_call(["gcc", "-std=c17", "-Wall", "-Werror", "-I", os.path.dirname(HEADER), "-c", str(src),
                           "-o", str(tmp_path / "t.o")])


def test_create_rejects_bad_geometry_before_touching_a_device():
    lib = qxlib.cuda()
    lib.qx_cuda_engine_create.argtypes = [C.c_void_p, C.c_void_p, C.c_uint32, C.c_void_p, C.c_void_p, C.c_char_p,
                                          C.c_uint64]
    model = qxlib.CudaModel(layers=1, hidden=100, q_heads=32, kv_heads=4, head_dim=128, vocab=151936, experts=128,
                            experts_per_token=8, moe_intermediate=768)
    tensor = (C.c_uint8 * 64)()
    h = C.c_void_p()
    err = qxlib.err_buf()
    ok = lib.qx_cuda_engine_create(C.addressof(model), C.addressof(tensor), 1, None, C.addressof(h), err, len(err))
    assert ok == 0 and b"geometry" in err.value
    ok = lib.qx_cuda_engine_create(None, None, 0, None, None, err, len(err))
    assert ok == 0 and err.value == b"invalid argument"


def test_create_from_image_rejects_corrupt_container(mini_image):
    bad = mini_image.copy()
    bad[0] = ord("X")
    opt = qxlib.CudaOptions(device=-1, ctx_tokens=64)
    h = C.c_void_p()
    err = qxlib.err_buf()
    ok = qxlib.cuda().qx_cuda_engine_create_from_image(bad.ctypes.data, bad.nbytes, C.byref(opt), C.byref(h), err,
                                                       len(err))
    assert ok == 0 and err.value == b"bad QXF magic"
