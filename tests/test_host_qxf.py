"""Host plumbing on CPU: QXF1 container rules, FNV, fp16, IQ tables, generator.

Pins against the reference's own compiled C where the reference tree is
available (fixture `ref`), otherwise against literal known answers.
"""
import ctypes as C
import os
import struct

import numpy as np
import pytest

import qxlib


def _host_open_image(img):
    buf = C.create_string_buffer(1024)          # qxh_file (header + pointers)
    err = qxlib.err_buf()
    lib = qxlib.host()
    lib.qxh_open_image.argtypes = [C.c_void_p, C.c_uint64, C.c_void_p, C.c_char_p, C.c_uint64]
    ok = lib.qxh_open_image(img.ctypes.data, img.nbytes, buf, err, len(err))
    return ok, err.value.decode()


def test_fnv_uses_reference_offset_basis():
    lib = qxlib.host()
    lib.qxh_fnv1a64.argtypes = [C.c_void_p, C.c_uint64]
    lib.qxh_fnv1a64.restype = C.c_uint64
    assert lib.qxh_fnv1a64(None, 0) == 1469598103934665603
    data = np.frombuffer(b"qx-mini-c", np.uint8)
    h = 1469598103934665603
    for b in data:
        h = ((h ^ int(b)) * 1099511628211) % (1 << 64)
    assert lib.qxh_fnv1a64(data.ctypes.data, data.size) == h


def test_fnv_matches_reference(ref):
    lib = qxlib.host()
    lib.qxh_fnv1a64.argtypes = [C.c_void_p, C.c_uint64]
    lib.qxh_fnv1a64.restype = C.c_uint64
    data = np.random.default_rng(1).integers(0, 256, 4097, dtype=np.uint8)
    assert lib.qxh_fnv1a64(data.ctypes.data, data.size) == ref.f["fnv1a64"](data.ctypes.data, data.size)


def test_fp16_all_codes_match_reference_rule():
    lib = qxlib.host()
    codes = np.arange(65536, dtype=np.uint16)
    got = np.array([lib.qxh_fp16_to_f32(int(c)) for c in codes], np.float32)
    want = codes.view(np.float16).astype(np.float32)
    special = ((codes >> 10) & 31) == 31
    np.testing.assert_array_equal(got[~special], want[~special])
    assert np.all(np.abs(got[special]) == 65504.0)
    assert np.all(np.signbit(got[special]) == ((codes[special] & 0x8000) != 0))


def test_fp16_matches_reference(ref):
    lib = qxlib.host()
    for c in list(range(0, 65536, 97)) + [0x7c00, 0xfc00, 0x7e00, 0x0001, 0x8001, 0x03ff]:
        assert lib.qxh_fp16_to_f32(c) == ref.f["fp16_to_f32"](c) or (
            np.isnan(lib.qxh_fp16_to_f32(c)) and np.isnan(ref.f["fp16_to_f32"](c)))


def test_f32_to_fp16_round_trip():
    lib = qxlib.host()
    for v in (0.0, 1.0, -2.5, 65504.0, 6.1e-5, 3e-8, 1e-3, 0.333333):
        assert lib.qxh_f32_to_fp16(v) == int(np.float16(v).view(np.uint16))


def _ref_table(ref, which, count, width):
    p = ref.lib.qxref_table(which)
    return np.frombuffer((C.c_uint8 * (count * width)).from_address(p), np.uint8).reshape(count, width)


def test_iq_tables_match_reference(ref):
    class T(C.Structure):
        _fields_ = [("iq2xs", C.c_uint8 * 4096), ("iq2s", C.c_uint8 * 8192), ("iq3xxs", C.c_uint8 * 1024),
                    ("iq3s", C.c_uint8 * 2048), ("ksigns", C.c_uint8 * 128)]
    lib = qxlib.host()
    t = T.from_address(lib.qxh_tables())
    np.testing.assert_array_equal(np.frombuffer(t.iq2xs, np.uint8).reshape(512, 8), _ref_table(ref, 0, 512, 8))
    np.testing.assert_array_equal(np.frombuffer(t.iq3xxs, np.uint8).reshape(256, 4), _ref_table(ref, 1, 256, 4))
    np.testing.assert_array_equal(np.frombuffer(t.iq2s, np.uint8).reshape(1024, 8), _ref_table(ref, 2, 1024, 8))
    np.testing.assert_array_equal(np.frombuffer(t.iq3s, np.uint8).reshape(512, 4), _ref_table(ref, 3, 512, 4))
    np.testing.assert_array_equal(np.frombuffer(t.ksigns, np.uint8), _ref_table(ref, 4, 128, 1).ravel())


def test_synthetic_model_is_deterministic(mini_image):
    again = qxlib.build_image(qxlib.mini_config(7))
    assert np.array_equal(again, mini_image)
    other = qxlib.build_image(qxlib.mini_config(8))
    assert not np.array_equal(other, mini_image)
    ok, msg = _host_open_image(mini_image)
    assert ok, msg


def test_synthetic_model_thread_count_does_not_matter():
    a = qxlib.build_image(qxlib.mini_config(7, threads=1))
    b = qxlib.build_image(qxlib.mini_config(7, threads=5))
    assert np.array_equal(a, b)


def test_reference_loader_accepts_synthetic_file(ref, mini_image, tmp_path):
    path = tmp_path / "mini.qxf"
    mini_image.tofile(path)
    m = ref.open_path(str(path))
    assert m.hidden == 512 and m.layers == 2 and m.vocab == 4096
    m.close()


def _corrupt(img, mutate):
    bad = img.copy()
    mutate(bad)
    return bad


def _entry_off(img, i):
    diro = struct.unpack_from("<Q", img[:272].tobytes(), 24)[0]
    return diro + 208 * i


# The structure-size check: qx_open_file has its own "unsupported QXF structure
# size" (src/qx_format.c:720-721), but qx_read_header (:443-445) runs first and
# rejects the same fields as "QXF struct size mismatch", so that is the message
# the reference's loader gives (test_loader_messages_match_reference below).
CORRUPTIONS = {
    "bad QXF magic": lambda b: b.__setitem__(0, ord("X")),
    "QXF struct size mismatch": lambda b: b.__setitem__(8, b[8] ^ 1),
    "empty tensor directory": lambda b: b.__setitem__(slice(16, 20), np.zeros(4, np.uint8)),
    "unsupported QXF version": lambda b: b.__setitem__(4, 2),
    "manifest checksum mismatch": lambda b: b.__setitem__(60, b[60] ^ 1),
    "invalid tensor dimensions": lambda b: b.__setitem__(slice(_entry_off(b, 3) + 112, _entry_off(b, 3) + 120),
                                                         np.zeros(8, np.uint8)),
    "tensor byte size inconsistent with dimensions": lambda b: b.__setitem__(_entry_off(b, 2) + 152,
                                                                             b[_entry_off(b, 2) + 152] ^ 16),
    "duplicate tensor name": lambda b: b.__setitem__(slice(_entry_off(b, 2), _entry_off(b, 2) + 96),
                                                     b[_entry_off(b, 1): _entry_off(b, 1) + 96]),
    "invalid tensor metadata": lambda b: b.__setitem__(_entry_off(b, 1) + 164, 99),
    "invalid tensor placement": lambda b: b.__setitem__(_entry_off(b, 1) + 145, b[_entry_off(b, 1) + 145] ^ 1),
}


@pytest.mark.parametrize("message", sorted(CORRUPTIONS))
def test_loader_rejects_corrupt_containers(mini_image, message):
    ok, msg = _host_open_image(_corrupt(mini_image, CORRUPTIONS[message]))
    assert not ok
    assert msg == message


@pytest.mark.parametrize("message", sorted(CORRUPTIONS))
def test_loader_messages_match_reference(ref, mini_image, message, tmp_path):
    path = tmp_path / "bad.qxf"
    _corrupt(mini_image, CORRUPTIONS[message]).tofile(path)
    with pytest.raises(RuntimeError) as e:
        ref.open_path(str(path))
    assert str(e.value).endswith(message)


def test_loader_rejects_truncated_file(mini_image):
    ok, msg = _host_open_image(mini_image[:-4096].copy())
    assert not ok and msg == "declared QXF file size does not match file"
