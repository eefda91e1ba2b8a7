"""Data parallelism.

CPU (gloo, world size 2): sharding the samples of a batch over ranks, summing the per-rank
gradient sums and dividing by the global sample count reproduces the reference's
accumulation mean over the whole batch (src/ac/train_controls.h:96-100), and the update that
follows is identical on every rank.

GPU (>= 2 devices, NCCL through the library's own communicator): the all-reduced gradients and
the updated adapters are identical on both ranks and equal a one-device run over the union of
the shards.
"""
import os
import socket
import sys

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def _paths():
    for p in (os.path.join(ROOT, "oracle"), os.path.join(ROOT, "audiocraft.cpp_b200"), HERE):
        if p not in sys.path:
            sys.path.insert(0, p)


# ---------------------------------------------------------------------------------------
# CPU: gloo ranks over the oracle

def _cpu_rank(rank, world, port, out):
    _paths()
    import oracle as O
    from fixtures import GOLDEN, load
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    z, c, ad = load(os.path.join(GOLDEN, "dit_small_dora.npz"))
    n = z["t"].shape[0]
    shard = np.arange(rank, n, world)  # samples dealt round-robin
    _, g = O.dit_step(c, z["W"], ad, z["params"], z["clean"][shard], z["noise"][shard], z["hidden"][shard],
                      z["t"][shard], z["uncond"][shard], z["valid"][shard])
    t = torch.from_numpy(g.astype(np.float64))
    dist.all_reduce(t)
    params = z["params"].copy()
    m = np.zeros_like(params)
    v = np.zeros_like(params)
    gsum = t.numpy().astype(np.float32)
    decays = np.ones(params.size, np.uint8)
    O.lib().ora_adamw(params.size, params, m, v, gsum.copy(), decays, n, 1, 1e-3, 0.9, 0.999, 1e-8, 0.01, 1.0)
    out[rank] = (gsum, params)
    dist.barrier()
    dist.destroy_process_group()


def test_sample_sharded_gradients_equal_full_batch_accumulation():
    _paths()
    import oracle as O
    from fixtures import GOLDEN, load
    world, port = 2, _free_port()
    mgr = mp.get_context("spawn").Manager()  # no fork of a process that may hold a CUDA context
    out = mgr.dict()
    mp.spawn(_cpu_rank, args=(world, port, out), nprocs=world, join=True)
    z, c, ad = load(os.path.join(GOLDEN, "dit_small_dora.npz"))
    _, gfull = O.dit_step(c, z["W"], ad, z["params"], z["clean"], z["noise"], z["hidden"], z["t"], z["uncond"],
                          z["valid"])
    g0, p0 = out[0]
    g1, p1 = out[1]
    np.testing.assert_array_equal(g0, g1)
    np.testing.assert_array_equal(p0, p1)
    np.testing.assert_allclose(g0, gfull, rtol=1e-5, atol=1e-7 * np.abs(gfull).max())


# ---------------------------------------------------------------------------------------
# GPU: NCCL all-reduce inside libactrain.so

def _gpu_rank(rank, world, port, out, mode, dora):
    _paths()
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    from datetime import timedelta
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timedelta(seconds=120))
    torch.cuda.set_device(rank)
    import actrain as A
    import dp
    from cases import MfCase
    host = dp.host_group(30.0)
    case = MfCase(seed=31, batch=4, device=rank, dora=dora)
    inputs = MfCase.inputs(case, n=4)              # same rng stream on both ranks: identical batch
    shard = [np.asarray(x)[rank::world] for x in inputs]
    case.ctx.set_timeout(60_000)
    case.ctx.nccl_init(dp.share_nccl_id(host, rank, A.Context.nccl_unique_id), world, rank)
    if mode == "in_step":   # all-reduce inside the step, per-layer buckets (DoRA: one at the end)
        case.ctx.set_grad_sync(4)
        case.ctx.mf_step(*shard)
    else:                   # after the step
        case.ctx.mf_step(*shard)
        case.ctx.allreduce_grads(4)
    g = case.ctx.get_grads()
    case.ctx.optimizer(lr=1e-3, step=1, weight_decay=0.01)
    v, _, _ = case.ctx.get_params()
    if mode == "in_step":   # a second in-step step replays the captured graph with its all-reduce
        for _ in range(2):
            case.ctx.set_grad_sync(4)
            case.ctx.mf_step(*shard)
        g2 = case.ctx.get_grads()
        case.ctx.zero_grads()
    else:
        g2 = None
    ref = None
    if rank == 0:  # one device over the union of the shards
        solo = MfCase(seed=31, batch=4, device=rank, dora=dora)
        solo.ctx.mf_step(*[np.concatenate([np.asarray(x)[r::world] for r in range(world)]) for x in inputs])
        ref = solo.ctx.get_grads()
        solo.ctx.optimizer(lr=1e-3, step=1, weight_decay=0.01)
        ref = (ref, solo.ctx.get_params()[0])
        solo.ctx.close()
    out[rank] = (g, v, ref, g2)
    dp.check_peers(host, 30.0, "teardown")
    case.ctx.close()
    dist.destroy_process_group()


@pytest.mark.gpu
@pytest.mark.skipif(not torch.cuda.is_available() or torch.cuda.device_count() < 2, reason="needs 2 GPUs")
@pytest.mark.parametrize("mode,dora", [("after", False), ("in_step", False), ("in_step", True)],
                         ids=["allreduce-after", "in-step-lora", "in-step-dora"])
def test_nccl_allreduce_matches_single_device(mode, dora):
    world, port = 2, _free_port()
    mgr = mp.get_context("spawn").Manager()  # no fork of a process that may hold a CUDA context
    out = mgr.dict()
    mp.spawn(_gpu_rank, args=(world, port, out, mode, dora), nprocs=world, join=True)
    g0, v0, ref, g20 = out[0]
    g1, v1, _, g21 = out[1]
    np.testing.assert_array_equal(g0, g1)
    np.testing.assert_array_equal(v0, v1)
    gref, vref = ref
    cos = float(np.dot(g0.astype(np.float64), gref) / (np.linalg.norm(g0) * np.linalg.norm(gref)))
    assert cos > 0.99999, cos
    # Adam's first step moves every parameter by about lr * sign(g): where the gradient is ~0
    # the sign is summation-order noise between the two-rank sum and the one-device sum, so
    # those entries may differ by up to 2 lr; every other entry must agree closely.
    big = np.abs(gref) > 1e-3 * np.abs(gref).max()
    np.testing.assert_allclose(v0[big], vref[big], rtol=1e-4, atol=1e-6)
    assert np.abs(v0 - vref).max() <= 2.1e-3
    if g20 is not None:  # two more all-reducing steps (eager, then the captured graph) on both ranks
        np.testing.assert_array_equal(g20, g21)
        assert np.linalg.norm(g20) > 0


def _leaving_rank(rank, world, port, out):
    """Rank 1 leaves between steps (nothing of it in flight); rank 0 learns it on the host, at its
    next peer check, and does not launch the step's all-reduce."""
    _paths()
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    from datetime import timedelta
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timedelta(seconds=60))
    torch.cuda.set_device(rank)
    import actrain as A
    import dp
    from cases import MfCase
    host = dp.host_group(5.0)
    case = MfCase(seed=33, batch=2, device=rank)
    case.ctx.set_timeout(30_000)
    case.ctx.nccl_init(dp.share_nccl_id(host, rank, A.Context.nccl_unique_id), world, rank)
    inputs = case.inputs(n=2)
    case.ctx.set_grad_sync(2 * world)
    case.ctx.mf_step(*inputs)
    case.ctx.optimizer(lr=1e-3, step=1)
    if rank == 1:
        out[1] = "left"
        os._exit(0)
    try:
        dp.check_peers(host, 5.0, "step 2")
        out[0] = "not detected"
    except dp.PeerFailure as e:
        out[0] = "detected: " + str(e)[:100]
    os._exit(0)


@pytest.mark.gpu
@pytest.mark.skipif(not torch.cuda.is_available() or torch.cuda.device_count() < 2, reason="needs 2 GPUs")
def test_rank_leaving_between_steps_is_detected_before_the_next_collective():
    import multiprocessing as mproc
    ctx = mproc.get_context("spawn")
    out = ctx.Manager().dict()
    port = _free_port()
    procs = [ctx.Process(target=_leaving_rank, args=(r, 2, port, out)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(180)
    for p in procs:
        if p.is_alive():
            p.kill()
    assert out.get(1) == "left", dict(out)
    assert str(out.get(0, "")).startswith("detected"), dict(out)
