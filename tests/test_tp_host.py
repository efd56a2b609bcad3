"""CPU: host logic of the tensor-parallel wrapper (awq_b200.tp) with `gloo` process groups
of 2, 4 and 8 ranks.  The GEMM is the CPU oracle here (injected through ``gemm=``); on GPUs
the same classes call the sm_100a library and NCCL."""
from __future__ import annotations

import os
import socket
import time

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from oracle import oracle as O


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _cpu_gemm(x, qw, qz, s, gs):
    return O.torch_awq_gemm_f32(x, qw, qz, s, gs).to(torch.float16)


def _layer(K, N, seed, gs=128):
    qw, qz, s = O.make_awq_layer(K, N, gs, seed=seed)
    return torch.from_numpy(qw), torch.from_numpy(qz), torch.from_numpy(s)


def test_bounds_partition_exactly():
    from awq_b200 import tp
    for world in (1, 2, 3, 4, 8):
        for N in (512, 4608, 37888, 3584):
            b = [tp.column_bounds(N, world, r) for r in range(world)]
            assert b[0][0] == 0 and b[-1][1] == N
            assert all(b[i][1] == b[i + 1][0] for i in range(world - 1))
            assert all(lo % 8 == 0 for lo, _ in b)
        for K in (3584, 18944):
            b = [tp.row_bounds(K, 128, world, r) for r in range(world)]
            assert b[0][0] == 0 and b[-1][1] == K
            assert all(lo % 128 == 0 and hi % 128 == 0 for lo, hi in b)
            sizes = [hi - lo for lo, hi in b]
            assert max(sizes) - min(sizes) <= 128
    # Qwen2-7B down at 8 ranks: 148 groups -> 19/18
    assert [tp.row_bounds(18944, 128, 8, r)[1] - tp.row_bounds(18944, 128, 8, r)[0]
            for r in range(8)] == [2432] * 4 + [2304] * 4


def test_fused_column_shards_keep_parts_aligned():
    from awq_b200 import tp
    inter = 512
    qw, qz, s = _layer(256, 2 * inter, seed=3)
    full = O.awq_dequant(qw.numpy(), qz.numpy(), s.numpy())
    for world in (2, 4):
        for r in range(world):
            lo, hi = tp.row_bounds(inter, 128, world, r)
            sqw, sqz, ss = tp.shard_fused_columns(
                qw, qz, s, [inter, inter], world, r, bounds=lambda w, ww, rr: tp.row_bounds(w, 128, ww, rr))
            got = O.awq_dequant(sqw.numpy(), sqz.numpy(), ss.numpy())
            import numpy as np
            want = np.concatenate([full[:, lo:hi], full[:, inter + lo:inter + hi]], axis=1)
            assert np.array_equal(got.view(np.uint16), want.view(np.uint16))


def _worker(rank, world, port, K, inter, hidden, seed, q):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    import datetime
    dist.init_process_group("gloo", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=30))
    try:
        from awq_b200 import tp
        gu = _layer(hidden, 2 * inter, seed)
        dn = _layer(inter, hidden, seed + 1)
        o = _layer(hidden, hidden, seed + 2)
        x = torch.from_numpy(O.make_x(3, hidden, seed=seed + 3))
        mlp = tp.TensorParallelMLP(tp.AWQWeights(*gu), tp.AWQWeights(*dn), inter, world, rank,
                                   gemm=_cpu_gemm)
        y = mlp(x)
        ro = tp.RowParallelAWQ(tp.AWQWeights(*o), world, rank, gemm=_cpu_gemm)
        z = ro(x[:, ro.k0:ro.k1].contiguous())
        q.put((rank, y.float().numpy(), z.float().numpy()))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world,inter,hidden", [
    (2, 512, 256),
    (4, 1024, 384),      # o has 3 groups for 4 ranks: the last rank holds no rows
    (8, 1024, 512),      # one group of the intermediate dimension per rank
])
def test_tp_mlp_and_row_parallel_gloo(world, inter, hidden):
    K, seed = hidden, 11
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, K, inter, hidden, seed, q))
             for r in range(world)]
    for p in procs:
        p.start()
    results = {}
    for _ in range(world):
        rank, y, z = q.get(timeout=120)
        results[rank] = (y, z)
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    # unsharded reference
    gu = _layer(hidden, 2 * inter, seed)
    dn = _layer(inter, hidden, seed + 1)
    o = _layer(hidden, hidden, seed + 2)
    x = torch.from_numpy(O.make_x(3, hidden, seed=seed + 3))
    g = _cpu_gemm(x, *gu, 128)
    h = (torch.nn.functional.silu(g[:, :inter].float()) * g[:, inter:].float()).half()
    y_ref = _cpu_gemm(h, *dn, 128).float().numpy()
    z_ref = _cpu_gemm(x, *o, 128).float().numpy()
    for rank in range(world):
        y, z = results[rank]
        assert O.max_rel_err(y, y_ref) <= 1e-2
        assert O.max_rel_err(z, z_ref) <= 1e-2


def _failing_worker(rank, world, port, q):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    import datetime
    dist.init_process_group("gloo", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=4))
    if rank == 1:
        q.put((rank, "raised"))
        q.close()
        q.join_thread()                    # flush the message before dying
        os._exit(3)                        # a rank that dies between steps
    try:
        from awq_b200 import tp
        o = _layer(256, 128, 5)
        ro = tp.RowParallelAWQ(tp.AWQWeights(*o), world, rank, gemm=_cpu_gemm)
        x = torch.from_numpy(O.make_x(1, 256, seed=1))
        ro(x[:, ro.k0:ro.k1].contiguous())
        q.put((rank, "no error"))
    except Exception as e:                 # the collective must fail, not hang
        q.put((rank, f"error: {type(e).__name__}"))
    q.close()
    q.join_thread()
    os._exit(0)


def test_dead_rank_surfaces_as_error_not_hang():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_failing_worker, args=(r, 2, port, q)) for r in range(2)]
    t0 = time.time()
    for p in procs:
        p.start()
    msgs = dict(q.get(timeout=90) for _ in range(2))
    for p in procs:
        p.join(timeout=30)
    assert msgs[1] == "raised"
    assert msgs[0].startswith("error"), msgs[0]
    assert time.time() - t0 < 90


# ---- attention projections split by whole heads (Qwen2-7B: 28 query heads, 4 kv heads) ----
NQ, NKV, HD = 28, 4, 128


def test_head_shards_partition_and_follow_gqa():
    from awq_b200 import tp
    for world in (1, 2, 3, 4, 7, 8):
        bounds = [tp.head_bounds(NQ, world, r) for r in range(world)]
        assert bounds[0][0] == 0 and bounds[-1][1] == NQ
        assert all(bounds[i][1] == bounds[i + 1][0] for i in range(world - 1))
        for h0, h1 in bounds:
            g0, g1 = tp.kv_head_bounds(NQ, NKV, h0, h1)
            assert {h // (NQ // NKV) for h in range(h0, h1)} == set(range(g0, g1))
    assert [tp.head_bounds(NQ, 8, r)[1] - tp.head_bounds(NQ, 8, r)[0] for r in range(8)] == \
        [4, 4, 4, 4, 3, 3, 3, 3]


def test_qkv_head_shards_are_the_right_columns():
    import numpy as np
    from awq_b200 import tp
    K, N = 256, (NQ + 2 * NKV) * HD
    qw, qz, s = _layer(K, N, seed=41)
    bias = torch.from_numpy(np.random.default_rng(2).uniform(-1, 1, N).astype(np.float16))
    full = O.awq_dequant(qw.numpy(), qz.numpy(), s.numpy())
    qsz, kvsz = NQ * HD, NKV * HD
    for world in (2, 3, 8):
        for r in range(world):
            sh = tp.shard_qkv_by_heads(tp.AWQWeights(qw, qz, s, 128, bias), NQ, NKV, HD, world, r)
            (h0, h1), (g0, g1) = sh.q_heads, sh.kv_heads
            cols = np.r_[h0 * HD:h1 * HD, qsz + g0 * HD:qsz + g1 * HD,
                         qsz + kvsz + g0 * HD:qsz + kvsz + g1 * HD]
            got = O.awq_dequant(sh.weights.qweight.numpy(), sh.weights.qzeros.numpy(),
                                sh.weights.scales.numpy())
            assert np.array_equal(got.view(np.uint16), full[:, cols].view(np.uint16))
            assert torch.equal(sh.weights.bias, bias[torch.from_numpy(cols)])
            assert sh.q_size == (h1 - h0) * HD and sh.kv_size == (g1 - g0) * HD


def _qkv_bias():
    import numpy as np
    return torch.from_numpy(np.random.default_rng(9).uniform(-1, 1, (NQ + 2 * NKV) * HD)
                            .astype(np.float16))


def _attn_worker(rank, world, port, seed, q):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    import datetime
    dist.init_process_group("gloo", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=30))
    try:
        from awq_b200 import tp
        qkv = _layer(256, (NQ + 2 * NKV) * HD, seed)
        o = _layer(NQ * HD, 256, seed + 1)
        x = torch.from_numpy(O.make_x(2, 256, seed=seed + 2))
        attn = torch.from_numpy(O.make_x(2, NQ * HD, seed=seed + 3))   # stands in for attention
        lin = tp.AttentionLinearsTP(tp.AWQWeights(*qkv, 128, _qkv_bias()), tp.AWQWeights(*o), NQ,
                                    NKV, HD, world, rank, gemm=_cpu_gemm)
        qv, kv, vv = lin.project_qkv(x)
        h0, h1 = lin.shard.q_heads
        y = lin.project_o(attn[:, h0 * HD:h1 * HD].contiguous())
        q.put((rank, lin.shard.q_heads, lin.shard.kv_heads, qv.float().numpy(),
               kv.float().numpy(), vv.float().numpy(), y.float().numpy()))
    finally:
        dist.destroy_process_group()


def test_attention_linears_by_heads_gloo_world4():
    world, seed = 4, 51
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_attn_worker, args=(r, world, port, seed, q)) for r in range(world)]
    for p in procs:
        p.start()
    got = [q.get(timeout=120) for _ in range(world)]
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    qkv = _layer(256, (NQ + 2 * NKV) * HD, seed)
    o = _layer(NQ * HD, 256, seed + 1)
    x = torch.from_numpy(O.make_x(2, 256, seed=seed + 2))
    attn = torch.from_numpy(O.make_x(2, NQ * HD, seed=seed + 3))
    full = (_cpu_gemm(x, *qkv, 128) + _qkv_bias()).float().numpy()     # q/k/v carry a bias
    y_ref = _cpu_gemm(attn, *o, 128).float().numpy()
    qsz, kvsz = NQ * HD, NKV * HD
    for rank, (h0, h1), (g0, g1), qv, kv, vv, y in got:
        assert O.max_rel_err(qv, full[:, h0 * HD:h1 * HD]) <= 1e-2
        assert O.max_rel_err(kv, full[:, qsz + g0 * HD:qsz + g1 * HD]) <= 1e-2
        assert O.max_rel_err(vv, full[:, qsz + kvsz + g0 * HD:qsz + kvsz + g1 * HD]) <= 1e-2
        assert O.max_rel_err(y, y_ref) <= 1e-2


# ---- the fused / NCCL choice of a row-parallel call is the same on every rank ----
class _FakeComm:
    """Stands in for awq_b200.TPComm on CPU ranks, with the library's rule in small: up
    to 16 tokens the fused decode kernel, which needs K a multiple of 256 here (so ranks
    whose K differ answer differently on their own); 17 to max_rows tokens the prefill
    product and the all-reduce kernel, which any K takes; beyond that NCCL.  The agreed
    choice must come out the same everywhere."""
    max_rows = 128

    def supported_shape(self, M, N, K, group_size=128):
        if M > 16:
            return K > 0 and M <= self.max_rows
        return K > 0 and K % 256 == 0


def _choice_worker(rank, world, port, K, q):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    import datetime
    dist.init_process_group("gloo", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=30))
    try:
        from awq_b200 import tp
        o = _layer(K, 128, 7)
        ro = tp.RowParallelAWQ(tp.AWQWeights(*o), world, rank, gemm=_cpu_gemm, comm=_FakeComm())
        local = _FakeComm().supported_shape(1, 128, ro.k1 - ro.k0)
        q.put((rank, ro.k1 - ro.k0, local, ro.fused_for(1), ro.fused_for(64),
               ro.fused_for(512)))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world,K,want,want64", [
    (2, 512, True, True),      # 256 rows each: every rank can run the fused kernel
    (2, 384, False, True),     # 256 and 128 rows: rank 1 cannot, so neither does at M = 1
    (4, 384, False, False),    # 3 groups over 4 ranks: the last rank holds no rows
])
def test_row_parallel_fused_choice_agrees_across_ranks(world, K, want, want64):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_choice_worker, args=(r, world, port, K, q)) for r in range(world)]
    for p in procs:
        p.start()
    got = [q.get(timeout=120) for _ in range(world)]
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    assert {g[3] for g in got} == {want}           # M = 1: one decision, the expected one
    assert {g[4] for g in got} == {want64}         # M = 64: product + all-reduce kernel
    assert {g[5] for g in got} == {False}          # M = 512 > max_rows: NCCL
    if not want:
        # at least one rank would have chosen the fused kernel on its own K alone
        assert any(g[2] for g in got) or any(g[1] == 0 for g in got)
