"""GPU: tensor-parallel AWQ linears over NCCL (one process per GPU), checked against the
single-GPU product.  Needs >= 2 GPUs; skipped otherwise.

Bar: max |tp - single| / max |single| <= 1e-2 (the parity tolerance used everywhere).
"""
from __future__ import annotations

import os
import socket

import numpy as np
import pytest
import torch
import torch.multiprocessing as mp

from oracle import oracle as O

pytestmark = pytest.mark.gpu
TOL = 1e-2
HIDDEN, INTER = 3584, 18944


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _start(procs, world):
    """Start the world-`world` workers with exactly the first `world` GPUs visible to
    them (the ones they use), whatever the box has."""
    vis = os.environ.get("CUDA_VISIBLE_DEVICES")
    devs = vis.split(",") if vis else [str(i) for i in range(torch.cuda.device_count())]
    os.environ["CUDA_VISIBLE_DEVICES"] = ",".join(devs[:world])
    try:
        for p in procs:
            p.start()
    finally:
        if vis is None:
            del os.environ["CUDA_VISIBLE_DEVICES"]
        else:
            os.environ["CUDA_VISIBLE_DEVICES"] = vis


def _collect(q, procs, world, limit_s=240):
    """One result per rank from the workers' queue.  A worker that raises sends its
    traceback instead; a worker that dies or goes silent fails the test within limit_s."""
    import queue
    import time
    got = []
    t0 = time.monotonic()
    while len(got) < world:
        try:
            item = q.get(timeout=5)
        except queue.Empty:
            dead = [p.exitcode for p in procs if p.exitcode not in (None, 0)]
            if dead:
                pytest.fail(f"a TP worker exited with {dead} before sending its result")
            if time.monotonic() - t0 > limit_s:
                pytest.fail(f"TP workers sent {len(got)} of {world} results in {limit_s} s")
            continue
        if isinstance(item, tuple) and item and item[0] == "error":
            pytest.fail(f"TP worker rank {item[1]} raised:\n{item[2]}")
        got.append(item)
    return got


def _layers(seed):
    gu = O.make_awq_layer(HIDDEN, 2 * INTER, 128, seed=seed)
    dn = O.make_awq_layer(INTER, HIDDEN, 128, seed=seed + 1)
    o = O.make_awq_layer(HIDDEN, HIDDEN, 128, seed=seed + 2)
    return gu, dn, o


def _worker(rank, world, port, M, seed, q):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    os.environ.setdefault("NCCL_NVLS_ENABLE", "0")
    import datetime
    import sys
    sys.path.insert(0, os.environ["AWQ_PKG"])
    sys.path.insert(0, os.environ["AWQ_REPO"])
    import torch.distributed as dist
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=60), device_id=dev)
    try:
        from awq_b200 import tp
        gu, dn, o = _layers(seed)
        to = lambda t: tuple(torch.from_numpy(np.ascontiguousarray(a)).to(dev) for a in t)
        x = torch.from_numpy(O.make_x(M, HIDDEN, seed=seed + 3)).to(dev)
        mlp = tp.TensorParallelMLP(tp.AWQWeights(*to(gu)), tp.AWQWeights(*to(dn)), INTER, world, rank)
        y = mlp(x)
        ro = tp.RowParallelAWQ(tp.AWQWeights(*to(o)), world, rank)
        z = ro(x[:, ro.k0:ro.k1].contiguous())
        torch.cuda.synchronize()
        q.put((rank, y.float().cpu().numpy(), z.float().cpu().numpy()))
    except BaseException:
        import traceback
        q.put(("error", rank, traceback.format_exc()))
        raise
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("M", [1, 12, 512])   # decode, small-M tcgen05, prefill kernels
def test_tp_world2_matches_single_gpu(cuda, M):
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    import awq_b200
    from conftest import PKG, REPO
    world, seed = 2, 21
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    env = dict(os.environ, AWQ_PKG=str(PKG), AWQ_REPO=str(REPO))
    os.environ.update(env)
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, M, seed, q)) for r in range(world)]
    _start(procs, world)
    res = {}
    for rank, y, z in _collect(q, procs, world):
        res[rank] = (y, z)
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    # single-GPU reference through the same library
    gu, dn, o = _layers(seed)
    to = lambda t: tuple(torch.from_numpy(np.ascontiguousarray(a)).to(cuda) for a in t)
    x = torch.from_numpy(O.make_x(M, HIDDEN, seed=seed + 3)).to(cuda)
    g = awq_b200.gemm(x, *to(gu), 128)
    h = (torch.nn.functional.silu(g[:, :INTER].float()) * g[:, INTER:].float()).half()
    y_ref = awq_b200.gemm(h, *to(dn), 128).float().cpu().numpy()
    z_ref = awq_b200.gemm(x, *to(o), 128).float().cpu().numpy()
    for rank in range(world):
        y, z = res[rank]
        assert O.max_rel_err(y, y_ref) <= TOL, rank
        assert O.max_rel_err(z, z_ref) <= TOL, rank


def _fused_worker(rank, world, port, Ms, seed, q, chain_M=1):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    os.environ.setdefault("NCCL_NVLS_ENABLE", "0")
    import datetime
    import sys
    sys.path.insert(0, os.environ["AWQ_PKG"])
    sys.path.insert(0, os.environ["AWQ_REPO"])
    import torch.distributed as dist
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=60), device_id=dev)
    comm = None
    try:
        import awq_b200
        from awq_b200 import tp
        comm = awq_b200.TPComm.from_group(HIDDEN)
        gu, dn, o = _layers(seed)
        to = lambda t: tuple(torch.from_numpy(np.ascontiguousarray(a)).to(dev) for a in t)
        ro = tp.RowParallelAWQ(tp.AWQWeights(*to(o)), world, rank, comm=comm)
        rd = tp.RowParallelAWQ(tp.AWQWeights(*to(dn)), world, rank, comm=comm)
        res = {}
        for M in Ms:
            x = torch.from_numpy(O.make_x(M, HIDDEN, seed=seed + 3)).to(dev)
            h = torch.from_numpy(O.make_x(M, INTER, seed=seed + 4)).to(dev)
            assert ro.comm.supported(x[:, ro.k0:ro.k1].contiguous(), ro.w.qweight, HIDDEN)
            z = ro(x[:, ro.k0:ro.k1].contiguous())
            y = rd(h[:, rd.k0:rd.k1].contiguous())
            res[M] = (z.cpu().numpy(), y.cpu().numpy())
        # a chain of fused calls replayed from a CUDA graph: o, then down on o's output
        # (tiled to INTER columns), 3 times, against the same chain run eagerly
        x = torch.from_numpy(O.make_x(chain_M, HIDDEN, seed=seed + 5)).to(dev)

        def chain():
            v = x
            for _ in range(3):
                z = ro(v[:, ro.k0:ro.k1].contiguous())
                hh = z.repeat(1, INTER // HIDDEN + 1)[:, :INTER] * 0.05
                v = rd(hh[:, rd.k0:rd.k1].contiguous())
            return v
        eager = chain()
        s = torch.cuda.Stream()
        s.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(s):
            chain()
        torch.cuda.synchronize()
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, stream=s):
            out = chain()
        for _ in range(3):
            g.replay()
        torch.cuda.synchronize()
        st = awq_b200.device_status()
        q.put((rank, res, eager.cpu().numpy(), out.cpu().numpy(), st))
        del g
    except BaseException:
        import traceback
        q.put(("error", rank, traceback.format_exc()))
        raise
    finally:
        torch.cuda.synchronize()
        if comm is not None:
            dist.barrier()
            comm.close()
        dist.destroy_process_group()


def test_fused_allreduce_world2_matches_single_gpu_and_ranks_agree(cuda):
    """Row-parallel o and down through the fused kernel (product + all-reduce over NVLink
    peer memory) on 2 GPUs: equal to the single-GPU product within the tolerance, and
    bit-identical on both ranks (sum in rank order); a graph-replayed chain of fused
    calls gives the eager chain's bits."""
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    import awq_b200
    from conftest import PKG, REPO
    world, seed, Ms = 2, 31, (1, 4, 16)
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    os.environ.update(AWQ_PKG=str(PKG), AWQ_REPO=str(REPO))
    port = _free_port()
    procs = [ctx.Process(target=_fused_worker, args=(r, world, port, Ms, seed, q)) for r in range(world)]
    _start(procs, world)
    _check_fused(cuda, q, procs, world, Ms, seed)


def _check_fused(cuda, q, procs, world, Ms, seed):
    import awq_b200
    got = {}
    for rank, res, eager, graphed, st in _collect(q, procs, world):
        got[rank] = (res, eager, graphed, st)
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    gu, dn, o = _layers(seed)
    to = lambda t: tuple(torch.from_numpy(np.ascontiguousarray(a)).to(cuda) for a in t)
    for M in Ms:
        x = torch.from_numpy(O.make_x(M, HIDDEN, seed=seed + 3)).to(cuda)
        h = torch.from_numpy(O.make_x(M, INTER, seed=seed + 4)).to(cuda)
        z_ref = awq_b200.gemm(x, *to(o), 128).float().cpu().numpy()
        y_ref = awq_b200.gemm(h, *to(dn), 128).float().cpu().numpy()
        for rank in range(world):
            z, y = got[rank][0][M]
            assert O.max_rel_err(z.astype(np.float32), z_ref) <= TOL, (M, rank)
            assert O.max_rel_err(y.astype(np.float32), y_ref) <= TOL, (M, rank)
        assert np.array_equal(got[0][0][M][0], got[1][0][M][0])
        assert np.array_equal(got[0][0][M][1], got[1][0][M][1])
    for rank in range(world):
        _, eager, graphed, st = got[rank]
        assert st == 0
        assert np.array_equal(eager, graphed)
    assert np.array_equal(got[0][1], got[1][1])


def test_prefill_allreduce_world2_matches_single_gpu_and_ranks_agree(cuda):
    """Row-parallel o and down above 16 tokens on 2 GPUs: each rank's prefill product goes
    into its communicator plane, and the library's all-reduce kernel sums the row slices
    over NVLink (reduce-scatter, then all-gather through the other rank's plane; no
    NCCL).  Equal to the single-GPU product within the tolerance, bit-identical on both
    ranks, ragged slices (M = 17, 100), and a graph-replayed chain of 48-token calls
    gives the eager chain's bits (the call numbers in the flags advance on replay)."""
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    from conftest import PKG, REPO
    world, seed, Ms = 2, 37, (17, 100, 512)
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    os.environ.update(AWQ_PKG=str(PKG), AWQ_REPO=str(REPO))
    port = _free_port()
    procs = [ctx.Process(target=_fused_worker, args=(r, world, port, Ms, seed, q, 48))
             for r in range(world)]
    _start(procs, world)
    _check_fused(cuda, q, procs, world, Ms, seed)


def _recovery_worker(rank, world, port, seed, q):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    os.environ.setdefault("NCCL_NVLS_ENABLE", "0")
    import datetime
    import sys
    sys.path.insert(0, os.environ["AWQ_PKG"])
    sys.path.insert(0, os.environ["AWQ_REPO"])
    import torch.distributed as dist
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=60), device_id=dev)
    comm = None
    try:
        import awq_b200
        from awq_b200 import tp
        comm = awq_b200.TPComm.from_group(HIDDEN)
        comm.set_timeout(0.3)
        _, _, o = _layers(seed)
        to = lambda t: tuple(torch.from_numpy(np.ascontiguousarray(a)).to(dev) for a in t)
        ro = tp.RowParallelAWQ(tp.AWQWeights(*to(o)), world, rank, comm=comm)
        x = torch.from_numpy(O.make_x(1, HIDDEN, seed=seed + 3)).to(dev)
        xl = x[:, ro.k0:ro.k1].contiguous()
        assert ro.fused_for(1)
        if rank == 0:
            ro(xl)            # rank 1 skips this call: rank 0's wait for its tiles runs out
        torch.cuda.synchronize()
        raised = ""
        try:
            comm.check(collective=True)    # both ranks learn of it, not only rank 0
        except awq_b200.AwqError as e:
            raised = str(e)
        comm.reset()                       # collective: barrier, clear, barrier
        z = ro(xl)                         # the next call is correct again
        torch.cuda.synchronize()
        q.put((rank, raised, z.cpu().numpy(), awq_b200.device_status()))
    except BaseException:
        import traceback
        q.put(("error", rank, traceback.format_exc()))
        raise
    finally:
        torch.cuda.synchronize()
        if comm is not None:
            dist.barrier()
            comm.close()
        dist.destroy_process_group()


def test_fused_allreduce_recovers_after_a_skipped_call(cuda):
    """A rank that skips a fused row-parallel call leaves the other rank's wait to run out
    (bounded: status bit 4, no hang).  A collective ``TPComm.check`` raises AwqError on
    both ranks, ``TPComm.reset`` clears both communicators, and the next fused call gives
    the single-GPU product, bit-identical on both ranks."""
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    import awq_b200
    from conftest import PKG, REPO
    world, seed = 2, 41
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    os.environ.update(AWQ_PKG=str(PKG), AWQ_REPO=str(REPO))
    port = _free_port()
    procs = [ctx.Process(target=_recovery_worker, args=(r, world, port, seed, q)) for r in range(world)]
    _start(procs, world)
    got = {rank: (raised, z, st) for rank, raised, z, st in _collect(q, procs, world)}
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    _, _, o = _layers(seed)
    to = lambda t: tuple(torch.from_numpy(np.ascontiguousarray(a)).to(cuda) for a in t)
    x = torch.from_numpy(O.make_x(1, HIDDEN, seed=seed + 3)).to(cuda)
    z_ref = awq_b200.gemm(x, *to(o), 128).float().cpu().numpy()
    for rank in range(world):
        raised, z, st = got[rank]
        assert "timed out waiting for another rank" in raised, (rank, raised)
        assert st == 0
        assert O.max_rel_err(z.astype(np.float32), z_ref) <= TOL, rank
    assert np.array_equal(got[0][1], got[1][1])
