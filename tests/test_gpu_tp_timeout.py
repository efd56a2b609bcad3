"""GPU, one device: the fused row-parallel all-reduce's wait for other ranks is bounded.

A world of 2 is built inside this process (two communicators on one GPU, each opening
the other's buffer); only rank 0 calls, so its wait for rank 1's tiles (M = 1: the fused
decode kernel) or rank 1's partial and row slice (M = 48: the all-reduce kernel after the
prefill product) can never end.
The kernel must give up after the communicator's time-out, set status bit 4 and finish
-- no hang, no fault -- and the library must keep working afterwards.  Nothing runs on
a second device and no kernel waits on another kernel of this GPU.
"""
from __future__ import annotations

import time

import numpy as np
import pytest
import torch

from oracle import oracle as O

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("M", [1, 48])
def test_fused_allreduce_wait_times_out_with_status(cuda, M):
    import awq_b200
    import awq_b200._lib as L
    K, N = 1024, 512
    c0 = awq_b200.TPComm(2, 0, N)
    c1 = awq_b200.TPComm(2, 1, N)
    try:
        c0.open([c0.handle, c1.handle])
        c1.open([c0.handle, c1.handle])
        c0.set_timeout(0.05)
        qw, qz, s = (torch.from_numpy(a).to(cuda) for a in O.make_awq_layer(K, N, 128, seed=4))
        x = torch.from_numpy(O.make_x(M, K, seed=4)).to(cuda)
        assert c0.supported(x, qw, N)
        torch.cuda.synchronize()
        t0 = time.perf_counter()
        awq_b200.gemm_allreduce(x, qw, qz, s, 128, c0)
        torch.cuda.synchronize()
        waited = time.perf_counter() - t0
        assert waited < 10.0
        # the time-out surfaces as an exception from the communicator's check ...
        with pytest.raises(awq_b200.AwqError, match="timed out waiting for another rank"):
            c0.check()
        assert awq_b200.device_status() == 0          # check() read and cleared the word
        # ... and both ranks' communicators go back to their opened state (the collective
        # TPComm.reset puts a barrier of the ranks around this call; here one process
        # holds both ranks)
        lib = L.load()
        for c in (c0, c1):
            L.check(lib.awq_tp_comm_reset(c._ptr))
        assert awq_b200.device_status() == 0
        # the device and the library are fine afterwards
        ref = O.awq_gemm_f32(x.cpu().numpy(), *(a.cpu().numpy() for a in (qw, qz, s)))
        out = awq_b200.gemm(x, qw, qz, s, 128)
        assert O.max_rel_err(out.float().cpu().numpy(), ref) <= 1e-2
        assert awq_b200.device_status() == 0
    finally:
        torch.cuda.synchronize()
        c1.close()
        c0.close()


@pytest.mark.parametrize("M", [3, 40])
def test_world1_communicator_is_a_plain_product(cuda, M):
    import awq_b200
    K, N = 2048, 1024
    c = awq_b200.TPComm(1, 0, N)
    try:
        c.open([c.handle])
        qw, qz, s = (torch.from_numpy(a).to(cuda) for a in O.make_awq_layer(K, N, 128, seed=6))
        x = torch.from_numpy(O.make_x(M, K, seed=6)).to(cuda)
        a = awq_b200.gemm_allreduce(x, qw, qz, s, 128, c)
        b = awq_b200.gemm(x, qw, qz, s, 128)
        torch.cuda.synchronize()
        assert torch.equal(a, b)
    finally:
        torch.cuda.synchronize()
        c.close()
