"""Host-side logic of expert parallelism, without a GPU: the work split
(qx_cuda_ep_partition), the rank-ordered handle exchange that maps the peers
(qxlib.connect_ep), and option validation before any device work.  The
multi-rank case runs as two gloo processes on the CPU."""
import ctypes as C
import os
import socket

import numpy as np
import pytest
import torch.distributed as dist
import torch.multiprocessing as mp

import qxlib

E, V = 128, 151936


def free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def test_partition_tiles_experts_and_vocabulary():
    for world in range(1, 9):
        parts = [qxlib.ep_partition(E, V, world, r) for r in range(world)]
        assert parts[0][0] == 0 and parts[-1][1] == E
        assert parts[0][2] == 0 and parts[-1][3] == V
        for a, b in zip(parts, parts[1:]):
            assert a[1] == b[0] and a[3] == b[2]           # contiguous, in rank order
        for e0, e1, r0, r1 in parts:
            assert e1 - e0 in (E // world, -(-E // world))  # balanced within one expert
            assert r0 % 32 == 0 and r1 % 32 == 0            # whole 32-row head groups


def test_partition_rejects_bad_arguments():
    with pytest.raises(ValueError):
        qxlib.ep_partition(E, V, 2, 2)
    with pytest.raises(ValueError):
        qxlib.ep_partition(E, V + 16, 2, 0)


class FakeEngine:
    """Stands in for an expert-parallel Engine: a handle that names its rank."""

    def __init__(self, rank):
        self.rank = rank
        self.connected = None

    def ep_handle(self):
        return bytes([self.rank]) * qxlib.Engine.EP_HANDLE_BYTES

    def ep_connect(self, handles):
        self.connected = list(handles)


def _rank_main(rank, world, port, out_dir):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        # every rank derives its own share; together they must tile the model
        parts = [None] * world
        dist.all_gather_object(parts, qxlib.ep_partition(E, V, world, rank))

        def gather(obj):
            got = [None] * world
            dist.all_gather_object(got, obj)
            return got

        eng = FakeEngine(rank)
        qxlib.connect_ep(eng, gather)
        np.save(os.path.join(out_dir, "r%d.npy" % rank),
                np.array([list(p) for p in parts] + [[h[0] for h in eng.connected] + [0] * (4 - world)],
                         dtype=np.int64))
    finally:
        dist.destroy_process_group()


def test_two_gloo_ranks_agree_on_split_and_map_peers_in_rank_order(tmp_path):
    world = 2
    mp.spawn(_rank_main, args=(world, free_port(), str(tmp_path)), nprocs=world, join=True)
    for r in range(world):
        out = np.load(tmp_path / ("r%d.npy" % r))
        assert [tuple(p) for p in out[:world]] == [qxlib.ep_partition(E, V, world, k) for k in range(world)]
        assert list(out[world][:world]) == list(range(world))   # handle of rank k at position k


def test_create_rejects_bad_expert_parallel_options_before_touching_a_device(mini_image):
    h = C.c_void_p()
    err = qxlib.err_buf()
    for rank, world in ((2, 2), (0, 9)):
        opt = qxlib.CudaOptions(device=-1, ctx_tokens=64, ep_rank=rank, ep_world=world)
        ok = qxlib.cuda().qx_cuda_engine_create_from_image(mini_image.ctypes.data, mini_image.nbytes, C.byref(opt),
                                                           C.byref(h), err, len(err))
        assert ok == 0 and err.value == b"invalid expert-parallel rank or world size"
    opt = qxlib.CudaOptions(device=-1, ctx_tokens=64, nccl_comm=1)
    ok = qxlib.cuda().qx_cuda_engine_create_from_image(mini_image.ctypes.data, mini_image.nbytes, C.byref(opt),
                                                       C.byref(h), err, len(err))
    assert ok == 0 and err.value == b"nccl_comm is reserved and must be NULL"


# ---- the split MoE combine -----------------------------------------------------
# The expert-parallel step splits the 8 selected experts of a layer by owner:
# rank r computes the term (float)(w_k * (double)y_k) of every slot k whose
# expert it owns (rows of the down projection y_k, double weights w_k), writes
# it into slot k of every rank's exchange table, and each rank then adds the 8
# slots of a row in rank order in float, as the one-GPU step does
# (src/qx_format.c:5287-5303).  Slot k is written by exactly one rank, so the
# sum is the one-GPU sum bit for bit.

H_C = 64


def _combine_inputs(seed):
    rng = np.random.default_rng(seed)
    sel = rng.choice(E, 8, replace=False)                    # rank order of the top-8
    w = rng.random(8) + 0.01
    w = w / w.sum()                                          # renormalised double weights
    y = rng.standard_normal((8, H_C)).astype(np.float32)     # expert outputs (down rows)
    x = rng.standard_normal(H_C).astype(np.float32)          # residual
    return sel, w, y, x


def _one_gpu_combine(sel, w, y, x):
    moe = np.zeros(H_C, np.float32)
    for k in range(8):
        moe = (moe + (w[k] * y[k].astype(np.float64)).astype(np.float32)).astype(np.float32)
    return (x + moe).astype(np.float32)


def _combine_main(rank, world, port, out_dir):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        e0, e1, _, _ = qxlib.ep_partition(E, V, world, rank)
        for seed in range(20):
            sel, w, y, x = _combine_inputs(seed)
            table = np.zeros((8, H_C), np.float32)           # this rank's contribution to the exchange
            for k in range(8):
                if e0 <= sel[k] < e1:
                    table[k] = (w[k] * y[k].astype(np.float64)).astype(np.float32)
            got = [None] * world
            dist.all_gather_object(got, table)
            owners = np.array([[np.any(t[k] != 0) for k in range(8)] for t in got])
            slots = np.sum(got, axis=0, dtype=np.float64).astype(np.float32)   # one writer per slot: exact
            moe = np.zeros(H_C, np.float32)
            for k in range(8):
                moe = (moe + slots[k]).astype(np.float32)
            np.save(os.path.join(out_dir, "c%d_%d.npy" % (rank, seed)), (x + moe).astype(np.float32))
            np.save(os.path.join(out_dir, "o%d_%d.npy" % (rank, seed)), owners.sum(axis=0))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world", [2, 4])
def test_split_moe_combine_equals_the_one_gpu_combine(tmp_path, world):
    mp.spawn(_combine_main, args=(world, free_port(), str(tmp_path)), nprocs=world, join=True)
    for seed in range(20):
        want = _one_gpu_combine(*_combine_inputs(seed))
        for r in range(world):
            np.testing.assert_array_equal(np.load(tmp_path / ("c%d_%d.npy" % (r, seed))), want)
            assert list(np.load(tmp_path / ("o%d_%d.npy" % (r, seed)))) == [1] * 8   # one writer per slot
