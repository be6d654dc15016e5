"""QXKVSNP1 snapshots between the engine and the reference's C path: the
engine exports its device KV after a greedy run, the reference reads the file
with its own reader and continues decoding, and both pick the same tokens and
experts; and the reverse, a snapshot written by the reference's writer
imported into the engine."""
import ctypes as C

import numpy as np
import pytest

import qxlib
import workloads as W

pytestmark = pytest.mark.gpu
SEED = 7
CTX = 64


def ref_read(ref, path, m):
    f = ref.lib.qxref_kv_snapshot_read
    P, U32 = C.c_void_p, C.c_uint32
    f.argtypes = [C.c_char_p, U32, U32, U32, U32, U32, P, P, P, P, P, P, C.c_char_p, C.c_uint64]
    kv = m.new_kv(CTX)
    pos, nt = np.zeros(1, np.uint32), np.zeros(1, np.uint32)
    err = qxlib.err_buf()
    ok = f(str(path).encode(), m.layers, CTX, m.kv_heads, m.head_dim, SEED, kv["k"].ctypes.data, kv["v"].ctypes.data,
           kv["ks"].ctypes.data, kv["vs"].ctypes.data, pos.ctypes.data, nt.ctypes.data, err, len(err))
    assert ok, err.value
    return kv, int(pos[0]), int(nt[0])


def ref_write(ref, path, m, kv, positions, next_token):
    f = ref.lib.qxref_kv_snapshot_write
    P, U32 = C.c_void_p, C.c_uint32
    f.argtypes = [C.c_char_p, U32, U32, U32, U32, U32, U32, U32, P, P, P, P, C.c_char_p, C.c_uint64]
    err = qxlib.err_buf()
    ok = f(str(path).encode(), m.layers, positions, CTX, m.kv_heads, m.head_dim, next_token, SEED,
           kv["k"].ctypes.data, kv["v"].ctypes.data, kv["ks"].ctypes.data, kv["vs"].ctypes.data, err, len(err))
    assert ok, err.value


@pytest.fixture(scope="module")
def eng(mini_image):
    e = qxlib.Engine(mini_image, ctx=CTX)
    yield e
    e.close()


def test_engine_snapshot_continues_in_the_reference(eng, ref, mini_image, tmp_path):
    eng.reset()
    first = eng.generate(W.START_TOKEN, 0, 20)
    path = tmp_path / "engine.kv"
    eng.kv_export(path, 20, int(first[-1]), SEED)
    m = ref.open_image(mini_image)
    kv, pos, nt = ref_read(ref, path, m)
    assert (pos, nt) == (20, int(first[-1]))
    want = eng.generate(nt, pos, 8)          # the engine continues from its own KV
    tok = nt
    for s in range(8):
        r = m.decode_step(tok, pos + s, kv)
        assert r["token"] == want[s], "step %d" % (pos + s)
        tok = r["token"]


def test_reference_snapshot_continues_in_the_engine(eng, ref, mini_image, tmp_path):
    m = ref.open_image(mini_image)
    kv = m.new_kv(CTX)
    tok = W.START_TOKEN
    for s in range(16):
        tok = m.decode_step(tok, s, kv)["token"]
    path = tmp_path / "ref.kv"
    ref_write(ref, path, m, kv, 16, tok)
    eng.reset()
    assert eng.kv_import(path, SEED) == (16, tok)
    k, v, ks, vs = eng.kv_read(0, 0, 16)
    np.testing.assert_array_equal(k, kv["k"][0, :16])
    np.testing.assert_array_equal(vs, kv["vs"][0, :16])
    for s in range(16, 24):
        r = m.decode_step(tok, s, kv)
        e = eng.decode_step(tok, s, want_experts=True)
        assert e["token"] == r["token"], "step %d" % s
        np.testing.assert_array_equal(e["experts"], r["experts"])
        tok = r["token"]


def test_import_failure_leaves_the_cache_alone(eng, tmp_path):
    eng.reset()
    eng.generate(W.START_TOKEN, 0, 6)
    before = eng.kv_read(1, 0, 6)
    bad = tmp_path / "bad.kv"
    eng.kv_export(bad, 6, 1, SEED)
    data = bytearray(bad.read_bytes())
    data[100] ^= 1
    bad.write_bytes(bytes(data))
    with pytest.raises(RuntimeError, match="accumulated KV snapshot payload mismatch"):
        eng.kv_import(bad, SEED)
    with pytest.raises(RuntimeError, match="accumulated KV snapshot header mismatch"):
        eng.kv_export(bad, 6, 1, SEED) or eng.kv_import(bad, SEED + 1)
    after = eng.kv_read(1, 0, 6)
    for a, b in zip(before, after):
        np.testing.assert_array_equal(a, b)
