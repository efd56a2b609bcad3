"""GPU: the allocation-free entry point awq_gemm_f16_noalloc, called through the C ABI.

Who needs it: hosts that cannot allocate device memory where the AWQ product runs --
an engine that plans all device memory up front and forbids library allocations on its
decode loop (cudaMalloc / cudaFree can synchronize the device and stall every stream),
or a plugin interface that hands the library only its input and output buffers.  The
entry point keeps its split-K scratch in a 4 MiB device array inside the library.

Checked here: on two calls in a row, its output matches the existing entry point
awq_gemm_f16 (which takes a caller-allocated workspace) and the CPU oracle (the
reference's dequantize-then-fp32-matmul restated; the two GPU entry points can run
different kernels, so the oracle also guards against a fault they share), each within
the parity tolerance used everywhere else (max |a - b| / max |b| <= 1e-2), and a shape
whose scratch would not fit is rejected with AWQ_ERR_WORKSPACE and a message.  This file
is named so that pytest collects it last.
"""
from __future__ import annotations

import ctypes

import numpy as np
import pytest
import torch

from oracle import oracle as O

pytestmark = pytest.mark.gpu
TOL = 1e-2


def _call_noalloc(lib, x, qw, qz, s, out, gs):
    M, K = x.shape
    N = s.shape[1]
    stream = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    return lib.awq_gemm_f16_noalloc(x.data_ptr(), x.stride(0), qw.data_ptr(), qz.data_ptr(),
                                    s.data_ptr(), out.data_ptr(), out.stride(0), M, N, K, gs,
                                    stream)


def _call_existing(lib, x, qw, qz, s, out, gs):
    M, K = x.shape
    N = s.shape[1]
    need = lib.awq_gemm_workspace_bytes(M, N, K, gs)
    ws = torch.zeros(max(need, 16), dtype=torch.uint8, device=x.device)
    stream = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    return lib.awq_gemm_f16(x.data_ptr(), x.stride(0), qw.data_ptr(), qz.data_ptr(),
                            s.data_ptr(), out.data_ptr(), out.stride(0), M, N, K, gs,
                            ws.data_ptr(), ws.numel(), stream)


@pytest.mark.parametrize("M,K,N,gs", [
    (1, 3584, 3584, 128),      # q/o projection, decode
    (4, 18944, 3584, 128),     # down projection, split-K over a long K
    (16, 3584, 4608, 128),     # fused qkv, 16 tokens
    (5, 384, 136, 128),        # ragged N (scalar loads)
    (40, 512, 256, 64),        # more than one 16-row chunk
])
def test_noalloc_matches_existing_entry_point(cuda, M, K, N, gs):
    import awq_b200._lib as L
    lib = L.load()
    qw, qz, s = O.make_awq_layer(K, N, gs, seed=M + K + N)
    x = O.make_x(M, K, seed=N)
    dx, dqw, dqz, ds = (torch.from_numpy(np.ascontiguousarray(a)).to(cuda) for a in (x, qw, qz, s))
    ref = torch.full((M, N), float("nan"), dtype=torch.float16, device=cuda)
    assert _call_existing(lib, dx, dqw, dqz, ds, ref, gs) == 0, lib.awq_last_error()
    oracle = O.awq_gemm_f32(x, qw, qz, s, gs)
    for _ in range(2):                                   # two calls in a row share the array
        out = torch.full((M, N), float("nan"), dtype=torch.float16, device=cuda)
        rc = _call_noalloc(lib, dx, dqw, dqz, ds, out, gs)
        assert rc == 0, lib.awq_last_error()
        torch.cuda.synchronize()
        assert torch.isfinite(out).all()
        got = out.float().cpu().numpy()
        assert O.max_rel_err(got, ref.float().cpu().numpy()) <= TOL
        assert O.max_rel_err(got, oracle) <= TOL


def test_noalloc_rejects_shape_beyond_its_scratch(cuda):
    import awq_b200._lib as L
    lib = L.load()
    # 16 tokens over K=18944, N=37888: the split-K partials cannot fit in 4 MiB.
    M, K, N, gs = 16, 18944, 37888, 128
    x = torch.zeros((M, K), dtype=torch.float16, device=cuda)
    qw = torch.empty((K, N // 8), dtype=torch.int32, device=cuda)
    qz = torch.empty((K // gs, N // 8), dtype=torch.int32, device=cuda)
    s = torch.empty((K // gs, N), dtype=torch.float16, device=cuda)
    out = torch.empty((M, N), dtype=torch.float16, device=cuda)
    rc = _call_noalloc(lib, x, qw, qz, s, out, gs)
    assert rc == L.AWQ_ERR_WORKSPACE
    assert b"no-alloc" in lib.awq_last_error()
