"""The reference-side binding as a C program:
tests/c/qx_state_loop_b200.c is compiled with gcc against include/qx_cuda.h,
linked to qx-mini-c_b200/libqxcuda.so, and run on a QXF1 file on disk.  Its
greedy tokens must equal the CPU checker's (oracle/qx_oracle.c, pinned to the
reference), and a corrupted file must fail closed with the checksum message.
"""
import json
import os
import subprocess

import pytest

import workloads as W

pytestmark = pytest.mark.gpu
ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def build(tmp_path):
    exe = str(tmp_path / "qx_state_loop_b200")
    pkg = os.path.join(ROOT, "qx-mini-c_b200")
    subprocess.check_call(["gcc", "-std=c11", "-O2", "-Wall", "-Werror", "-I", os.path.join(ROOT, "include"),
                           os.path.join(ROOT, "tests", "c", "qx_state_loop_b200.c"), "-L", pkg, "-lqxcuda",
                           "-Wl,-rpath," + pkg, "-o", exe])
    return exe


def test_c_binding_runs_the_state_loop(mini_image, port, tmp_path):
    exe = build(tmp_path)
    path = str(tmp_path / "mini.qxf")
    mini_image.tofile(path)
    prompt = [W.START_TOKEN, 7, 1999]
    gen = 12
    r = subprocess.run([exe, path, "64", str(gen)] + [str(t) for t in prompt], capture_output=True, text=True,
                       timeout=300)
    assert r.returncode == 0, r.stdout + r.stderr
    out = json.loads(r.stdout)
    assert out["ok"] and out["cuda_profile"]["enabled"] and out["cuda_profile"]["backend"] == "b200-sm100a"
    P = port.open_image(mini_image)
    kv = P.new_kv(64)
    want = []
    tok = None
    for pos, t in enumerate(prompt):
        tok = P.decode_step(t, pos, kv)["token"]
    want.append(tok)
    for s in range(gen - 1):
        tok = P.decode_step(tok, len(prompt) + s, kv)["token"]
        want.append(tok)
    assert out["tokens"] == want


def test_c_binding_fails_closed_on_a_corrupt_file(mini_image, tmp_path):
    exe = build(tmp_path)
    import qximg
    bad = mini_image.copy()
    _, off, size, _, _ = qximg.tensors(bad)["output.weight"]
    bad[off + size // 3] ^= 0x10                 # one byte of the head's data
    path = str(tmp_path / "bad.qxf")
    bad.tofile(path)
    r = subprocess.run([exe, path, "64", "2", str(W.START_TOKEN)], capture_output=True, text=True, timeout=300)
    assert r.returncode == 1
    out = json.loads(r.stdout)
    assert not out["ok"] and "tensor checksum mismatch" in out["error"]
