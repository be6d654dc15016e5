"""Expert parallelism on two B200s through the C ABI: each rank computes its
share of the experts and of the head, the ranks exchange MoE terms and head
maxima through mapped peer memory, and the greedy tokens, top-8 experts and
final residual must equal the single-GPU engine's bit for bit.  Needs at least
two GPUs (skipped otherwise); ranks are processes, handles travel over gloo."""
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

import qxlib
import workloads as W

pytestmark = pytest.mark.gpu
STEPS = 40


def free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def model_image(kind):
    if kind == "mini":
        return qxlib.build_image(qxlib.mini_config(7))
    return qxlib.build_image(qxlib.synth_config(7, layers=4))   # full geometry, 4 layers


def run_engine(eng):
    """STEPS greedy tokens with the on-device loop, then stepwise with outputs."""
    eng.reset()
    gen = eng.generate(W.START_TOKEN, 0, STEPS)
    eng.reset()
    tok, experts, resid = W.START_TOKEN, [], None
    for s in range(8):
        r = eng.decode_step(tok, s, want_residual=True, want_experts=True)
        experts.append(r["experts"])
        resid = r["residual"]
        tok = r["token"]
    return gen, np.stack(experts), resid


def _rank_main(rank, world, port, kind, out_dir):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        img = model_image(kind)
        eng = qxlib.Engine(img, ctx=64, device=rank, ep_rank=rank, ep_world=world)

        def gather(obj):
            got = [None] * world
            dist.all_gather_object(got, obj)
            return got

        qxlib.connect_ep(eng, gather)
        gen, experts, resid = run_engine(eng)
        np.savez(os.path.join(out_dir, "ep%d.npz" % rank), gen=gen, experts=experts, resid=resid)
        dist.barrier()
        eng.close()
        if rank == 0:
            single = qxlib.Engine(img, ctx=64, device=0)
            gen, experts, resid = run_engine(single)
            np.savez(os.path.join(out_dir, "single.npz"), gen=gen, experts=experts, resid=resid)
            single.close()
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("kind", ["mini", "full4"])
def test_two_gpu_expert_parallel_matches_one_gpu(kind, tmp_path):
    if torch.cuda.device_count() < 2:
        pytest.skip("expert parallelism needs two GPUs")
    world = 2
    mp.spawn(_rank_main, args=(world, free_port(), kind, str(tmp_path)), nprocs=world, join=True)
    single = np.load(tmp_path / "single.npz")
    assert len(set(single["gen"].tolist())) > 1
    for r in range(world):
        ep = np.load(tmp_path / ("ep%d.npz" % r))
        np.testing.assert_array_equal(ep["gen"], single["gen"], err_msg="tokens, rank %d" % r)
        np.testing.assert_array_equal(ep["experts"], single["experts"], err_msg="experts, rank %d" % r)
        np.testing.assert_array_equal(ep["resid"], single["resid"], err_msg="final residual, rank %d" % r)


def _stall_main(rank, world, port, out_dir):
    """Rank 1 connects but never decodes: rank 0's step must end with the
    bounded-wait error instead of hanging, and its context must stay usable."""
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        img = model_image("mini")
        eng = qxlib.Engine(img, ctx=64, device=rank, ep_rank=rank, ep_world=world)

        def gather(obj):
            got = [None] * world
            dist.all_gather_object(got, obj)
            return got

        qxlib.connect_ep(eng, gather)
        msg = ""
        if rank == 0:
            try:
                eng.decode_step(W.START_TOKEN, 0)
            except RuntimeError as e:
                msg = str(e)
            # the device still works for a single-GPU engine afterwards
            single = qxlib.Engine(img, ctx=64, device=0)
            ok = single.decode_step(W.START_TOKEN, 0)["token"] >= 0
            single.close()
            with open(os.path.join(out_dir, "stall.txt"), "w") as f:
                f.write("%s\n%d\n" % (msg, int(ok)))
        dist.barrier()                     # rank 1 leaves only after rank 0 is done
        eng.close()
    finally:
        dist.destroy_process_group()


def test_a_rank_that_never_steps_fails_the_peer_step_with_a_bounded_wait(tmp_path):
    if torch.cuda.device_count() < 2:
        pytest.skip("expert parallelism needs two GPUs")
    mp.spawn(_stall_main, args=(2, free_port(), str(tmp_path)), nprocs=2, join=True)
    msg, ok = (tmp_path / "stall.txt").read_text().splitlines()
    assert "device grid barrier timed out" in msg
    assert ok == "1"
