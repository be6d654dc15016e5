"""QXKVSNP1 accumulated-KV snapshots (src/qx_format.c:5860-5969) on the host:
the library's SHA-256 against hashlib, the writer byte-for-byte against the
reference's own writer, and the reader against the reference's files and its
error messages.  The device round trips are in test_gpu_snapshot.py."""
import ctypes as C
import hashlib
import os

import numpy as np
import pytest

import qxlib

LAYERS, CTX, KVH, HD = 3, 20, 2, 128
SEED = 7


def kv_arrays(rng):
    k = rng.integers(-127, 128, (LAYERS, CTX, KVH * HD), dtype=np.int8)
    v = rng.integers(-127, 128, (LAYERS, CTX, KVH * HD), dtype=np.int8)
    ks = rng.random((LAYERS, CTX), dtype=np.float32) + 0.01
    vs = rng.random((LAYERS, CTX), dtype=np.float32) + 0.01
    return k, v, ks, vs


def ref_fn(ref, name):
    f = getattr(ref.lib, name)
    P, U32 = C.c_void_p, C.c_uint32
    if name == "qxref_kv_snapshot_write":
        f.argtypes = [C.c_char_p, U32, U32, U32, U32, U32, U32, U32, P, P, P, P, C.c_char_p, C.c_uint64]
    else:
        f.argtypes = [C.c_char_p, U32, U32, U32, U32, U32, P, P, P, P, P, P, C.c_char_p, C.c_uint64]
    return f


def ref_write(ref, path, k, v, ks, vs, positions, next_token, seed=SEED):
    err = qxlib.err_buf()
    ok = ref_fn(ref, "qxref_kv_snapshot_write")(str(path).encode(), LAYERS, positions, CTX, KVH, HD, next_token, seed,
                                                k.ctypes.data, v.ctypes.data, ks.ctypes.data, vs.ctypes.data, err,
                                                len(err))
    assert ok, err.value


def ref_read_message(ref, path, seed=SEED):
    k = np.zeros((LAYERS, CTX, KVH * HD), np.int8)
    v, ks, vs = k.copy(), np.zeros((LAYERS, CTX), np.float32), np.zeros((LAYERS, CTX), np.float32)
    pos, nt = np.zeros(1, np.uint32), np.zeros(1, np.uint32)
    err = qxlib.err_buf()
    ok = ref_fn(ref, "qxref_kv_snapshot_read")(str(path).encode(), LAYERS, CTX, KVH, HD, seed, k.ctypes.data,
                                               v.ctypes.data, ks.ctypes.data, vs.ctypes.data, pos.ctypes.data,
                                               nt.ctypes.data, err, len(err))
    return None if ok else err.value.decode()


@pytest.mark.parametrize("n", [0, 1, 55, 56, 63, 64, 65, 127, 1000, 1 << 20])
def test_sha256_matches_hashlib(n):
    data = np.random.default_rng(n).integers(0, 256, n, dtype=np.uint8).tobytes()
    assert qxlib.sha256(data) == hashlib.sha256(data).digest()


def test_writer_is_byte_identical_to_the_reference(ref, tmp_path):
    k, v, ks, vs = kv_arrays(np.random.default_rng(1))
    for positions in (1, 13, CTX):
        ours, theirs = tmp_path / "ours.kv", tmp_path / "ref.kv"
        qxlib.kv_snapshot_write(ours, k, v, ks, vs, positions, 4242, SEED, KVH, HD)
        ref_write(ref, theirs, k, v, ks, vs, positions, 4242)
        assert ours.read_bytes() == theirs.read_bytes()
        assert ours.stat().st_size == 48 + LAYERS * positions * (2 * KVH * HD + 8) + 32


def test_reader_loads_a_reference_snapshot(ref, tmp_path):
    k, v, ks, vs = kv_arrays(np.random.default_rng(2))
    path = tmp_path / "ref.kv"
    ref_write(ref, path, k, v, ks, vs, 9, 77)
    rk, rv, rks, rvs, pos, nt = qxlib.kv_snapshot_read(path, LAYERS, CTX, KVH, HD, SEED)
    assert (pos, nt) == (9, 77)
    np.testing.assert_array_equal(rk[:, :9], k[:, :9])
    np.testing.assert_array_equal(rv[:, :9], v[:, :9])
    np.testing.assert_array_equal(rks[:, :9], ks[:, :9])
    np.testing.assert_array_equal(rvs[:, :9], vs[:, :9])
    assert not rk[:, 9:].any() and not rks[:, 9:].any()


def corruptions(good):
    b = bytearray(good)
    payload = bytearray(b)
    payload[60] ^= 1                      # a K byte
    digest = bytearray(b)
    digest[-1] ^= 0x80
    version = bytearray(b)
    version[8] = 3
    nan_scale = bytearray(b)
    off = 48 + 2 * KVH * HD                # first K scale
    nan_scale[off:off + 4] = np.array([np.nan], np.float32).tobytes()
    return {"payload byte": bytes(payload), "digest": bytes(digest), "version": bytes(version),
            "trailing byte": bytes(b) + b"\0", "truncated": bytes(b[:-5]), "non-finite scale": bytes(nan_scale)}


def test_reader_rejects_what_the_reference_rejects_with_its_messages(ref, tmp_path):
    k, v, ks, vs = kv_arrays(np.random.default_rng(3))
    good = tmp_path / "good.kv"
    qxlib.kv_snapshot_write(good, k, v, ks, vs, 5, 1, SEED, KVH, HD)
    cases = corruptions(good.read_bytes())
    for name, data in cases.items():
        path = tmp_path / ("bad_%s.kv" % name.replace(" ", "_"))
        path.write_bytes(data)
        want = ref_read_message(ref, path)
        assert want is not None, name
        with pytest.raises(RuntimeError) as e:
            qxlib.kv_snapshot_read(path, LAYERS, CTX, KVH, HD, SEED)
        assert want in str(e.value), (name, want, str(e.value))
    # header fields the reader checks against the engine
    for seed in (SEED + 1,):
        with pytest.raises(RuntimeError, match="accumulated KV snapshot header mismatch"):
            qxlib.kv_snapshot_read(good, LAYERS, CTX, KVH, HD, seed)
    with pytest.raises(RuntimeError, match="accumulated KV snapshot header mismatch"):
        qxlib.kv_snapshot_read(good, LAYERS, CTX + 1, KVH, HD, SEED)
    with pytest.raises(RuntimeError, match="cannot open accumulated KV snapshot input"):
        qxlib.kv_snapshot_read(tmp_path / "missing.kv", LAYERS, CTX, KVH, HD, SEED)
