"""Edits of synthetic QXF1 images for the parity tests.

A QXF1 container is a 272-byte header, a directory of 208-byte entries (name
char[96] @0, dims u64[4] @112, offset u64 @144, byte_size u64 @152, flags =
ggml type u32 @164, checksum u64 @168) and the tensor data (the reference's
include/qx_format.h:56-82).  After a tensor's bytes change its FNV-1a
checksum is recomputed (src/qx_format.c:220-228 defines it), so the edited
image is still a valid container for the reference, the C restatement and the
engine.
"""
import ctypes as C
import struct

import numpy as np

import qxlib


def tensors(img):
    """{name: (entry_offset, data_offset, byte_size, dims, ggml_type)}."""
    hdr = img[:272].tobytes()
    count = struct.unpack_from("<I", hdr, 16)[0]
    diro = struct.unpack_from("<Q", hdr, 24)[0]
    out = {}
    for i in range(count):
        eo = diro + 208 * i
        e = img[eo:eo + 208].tobytes()
        name = e[:96].split(b"\0")[0].decode()
        dims = struct.unpack_from("<4Q", e, 112)
        off, size = struct.unpack_from("<QQ", e, 144)
        out[name] = (eo, off, size, dims, struct.unpack_from("<I", e, 164)[0])
    return out


def data(img, name):
    """Writable uint8 view of a tensor's bytes."""
    _, off, size, _, _ = tensors(img)[name]
    return img[off:off + size]


def reseal(img, names):
    """Recompute the FNV-1a checksum of each named tensor after an edit."""
    lib = qxlib.host()
    lib.qxh_fnv1a64.argtypes = [C.c_void_p, C.c_uint64]
    lib.qxh_fnv1a64.restype = C.c_uint64
    t = tensors(img)
    for name in names:
        eo, off, size, _, _ = t[name]
        view = np.ascontiguousarray(img[off:off + size])
        h = lib.qxh_fnv1a64(view.ctypes.data, size)
        img[eo + 168:eo + 176] = np.frombuffer(struct.pack("<Q", h), np.uint8)
    return img


def tie_image(cfg):
    """A model whose router rows come in triples (rows 3k+1 and 3k+2 repeat
    row 3k in every layer) and whose head rows r and r + V/2 are equal.  Every
    top-8 then holds tied experts, and the 8th slot is always cut inside a
    tied triple (8 = 3 + 3 + 2), so the reference's strict-> scan
    (src/qx_format.c:5272-5285) must keep the lower index; the greedy argmax
    ties between r and r + V/2 go to r (:3723-3730)."""
    img = qxlib.build_image(cfg)
    t = tensors(img)
    edited = []
    for layer in range(cfg.layers):
        name = "blk.%d.ffn_gate_inp.weight" % layer
        rows = data(img, name).view(np.float32).reshape(cfg.experts, cfg.hidden)
        for e in range(0, cfg.experts - 2, 3):
            rows[e + 1] = rows[e]
            rows[e + 2] = rows[e]
        edited.append(name)
    head = data(img, "output.weight")
    row = t["output.weight"][2] // cfg.vocab
    half = cfg.vocab // 2
    hv = head.reshape(cfg.vocab, row)
    hv[half:2 * half] = hv[:half]
    edited.append("output.weight")
    return reseal(img, edited)


def fp16_inf_image(cfg, token):
    """Blocks whose fp16 scale fields have exponent 31 (Inf/NaN bit patterns),
    which the reference reads as +-65504 (src/qx_format.c:1868-1869): the
    Q4_K d / dmin of `token`'s embedding row, the Q6_K d of head rows 5 and 9,
    and the IQ4_XS d of two blocks of layer 0's Q projection."""
    img = qxlib.build_image(cfg)
    t = tensors(img)
    nblk = cfg.hidden // 256
    emb = data(img, "token_embd.weight").reshape(cfg.vocab, nblk * 144)
    emb[token, 0:2] = (0x00, 0x7C)                 # d = +Inf
    emb[token, 144 + 2:144 + 4] = (0x00, 0xFC)     # dmin = -Inf
    emb[token, 144:146] = (0x01, 0x7E)             # d = NaN
    head = data(img, "output.weight").reshape(cfg.vocab, nblk * 210)
    head[5, 208:210] = (0x00, 0x7C)
    head[9, 210 + 208:210 + 210] = (0x00, 0xFE)    # -NaN
    q = data(img, "blk.0.attn_q.weight").reshape(-1, nblk * 136)
    q[3, 0:2] = (0x00, 0x7C)
    q[40, 136:138] = (0x00, 0xFC)
    return reseal(img, ["token_embd.weight", "output.weight", "blk.0.attn_q.weight"])
