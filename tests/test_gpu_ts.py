"""GPU parity of the small-M tcgen05 kernel (AWQ_PATH_TS: dequantized weights written into
tensor memory as the MMA's A operand, tokens as its N) against the CPU oracle.

Bar: max |out - ref| / max |ref| <= 1e-2 against the fp32 oracle x.float() @ W.float()
(the W the kernel forms is bit-identical to the reference's, so the only difference is
fp32 summation order and the final fp16 rounding).
"""
from __future__ import annotations

import ctypes

import numpy as np
import pytest
import torch

from oracle import oracle as O

pytestmark = pytest.mark.gpu
TOL = 1e-2


def _dev(cuda, *arrays):
    return [torch.from_numpy(np.ascontiguousarray(a)).to(cuda) for a in arrays]


@pytest.mark.parametrize("M,K,N,gs", [
    (1, 128, 32, 128), (5, 256, 256, 128), (16, 512, 512, 128), (17, 384, 320, 128),
    (33, 1024, 768, 128), (64, 640, 4608, 128), (12, 1024, 544, 256), (3, 768, 1024, 64),
])
def test_ts_small_shapes_vs_oracle(cuda, M, K, N, gs):
    import awq_b200
    qw, qz, s = O.make_awq_layer(K, N, gs, seed=M + N + gs)
    x = O.make_x(M, K, seed=K + M)
    ref = O.awq_gemm_f32(x, qw, qz, s, gs)
    dx, dqw, dqz, ds = _dev(cuda, x, qw, qz, s)
    out = awq_b200.gemm(dx, dqw, dqz, ds, gs, path=awq_b200.AWQ_PATH_TS)
    assert O.max_rel_err(out.float().cpu().numpy(), ref) <= TOL
    assert awq_b200.device_status() == 0


@pytest.mark.parametrize("M,K,N", [
    (16, 3584, 3584),       # o: 14 tiles, split along K
    (8, 18944, 3584),       # down: 14 tiles, split along K
    (16, 3584, 37888),      # gate+up: 148 tiles, no split
    (40, 3584, 4608),       # q/k/v at 32 < M <= 64: 64-token tiles
])
def test_ts_model_shapes(cuda, M, K, N):
    """Checked against the CPU oracle on three 64-column blocks and against an fp32
    product of the exactly dequantized weights everywhere; repeated calls give the same
    bits; without a workspace the kernel runs one CTA per tile with the same result."""
    import awq_b200
    import awq_b200._lib as L
    qw, qz, s = O.make_awq_layer(K, N, 128, seed=M * 7 + N)
    x = O.make_x(M, K, seed=M + 1)
    dx, dqw, dqz, ds = _dev(cuda, x, qw, qz, s)
    a = awq_b200.gemm(dx, dqw, dqz, ds, 128, path=awq_b200.AWQ_PATH_TS)
    b = awq_b200.gemm(dx, dqw, dqz, ds, 128, path=awq_b200.AWQ_PATH_TS)
    torch.cuda.synchronize()
    assert torch.equal(a, b)
    for c0 in (0, (N // 2) // 64 * 64, N - 64):
        ref = O.awq_gemm_f32(x, qw[:, c0 // 8:(c0 + 64) // 8], qz[:, c0 // 8:(c0 + 64) // 8],
                             s[:, c0:c0 + 64], 128)
        assert O.max_rel_err(a[:, c0:c0 + 64].float().cpu().numpy(), ref) <= TOL, c0
    full = dx.float() @ awq_b200.dequant(dqw, dqz, ds, 128).float()
    assert O.max_rel_err(a.float().cpu().numpy(), full.cpu().numpy()) <= TOL
    lib = L.load()
    out = torch.empty((M, N), dtype=torch.float16, device=cuda)
    rc = lib.awq_gemm_f16_ex(dx.data_ptr(), K, dqw.data_ptr(), dqz.data_ptr(), ds.data_ptr(),
                             out.data_ptr(), N, M, N, K, 128, None, 0,
                             ctypes.c_void_p(torch.cuda.current_stream().cuda_stream),
                             awq_b200.AWQ_PATH_TS)
    assert rc == 0, lib.awq_last_error()
    torch.cuda.synchronize()
    assert O.max_rel_err(out.float().cpu().numpy(), full.cpu().numpy()) <= TOL
    assert awq_b200.device_status() == 0


def test_ts_golden(golden, cuda):
    import awq_b200
    ran = 0
    for name, c in golden.items():
        if name == "extreme_scales":
            continue
        x = c["x"].reshape(-1, c["x"].shape[-1])
        dx, dqw, dqz, ds = _dev(cuda, x, c["qweight"], c["qzeros"], c["scales"])
        if x.shape[0] > 64 or not awq_b200.tc_supported(dx, dqw, dqz, ds, c["group_size"]):
            continue                         # M <= 64, N % 32 and group_size % 64 rules
        out = awq_b200.gemm(dx, dqw, dqz, ds, c["group_size"], path=awq_b200.AWQ_PATH_TS)
        ref = c["out_ref_f32"].reshape(out.shape)
        assert O.max_rel_err(out.float().cpu().numpy(), ref) <= TOL, name
        ran += 1
    assert ran > 0


def test_ts_rejects_large_m(cuda):
    import awq_b200
    qw, qz, s = O.make_awq_layer(256, 256, 128, seed=1)
    dx, dqw, dqz, ds = _dev(cuda, O.make_x(65, 256, seed=1), qw, qz, s)
    with pytest.raises(awq_b200.AwqError):
        awq_b200.gemm(dx, dqw, dqz, ds, 128, path=awq_b200.AWQ_PATH_TS)


@pytest.mark.parametrize("M,K,N", [
    (12, 3584, 3584),       # few tiles: split along K, bias added by the reduce kernel
    (16, 512, 37888),       # 148 tiles: one CTA each, bias added in the epilogue
    (9, 3584, 4608),        # q/k/v at the lower end of the range
])
def test_ts_auto_dispatch_and_bias(cuda, M, K, N):
    """AUTO takes the small-M kernel here: its result is bit-identical to the explicit
    path, and the fused bias matches fp32 (x @ W + bias)."""
    import awq_b200
    qw, qz, s = O.make_awq_layer(K, N, 128, seed=M + K)
    x = O.make_x(M, K, seed=N)
    dx, dqw, dqz, ds = _dev(cuda, x, qw, qz, s)
    auto = awq_b200.gemm(dx, dqw, dqz, ds, 128)
    ts = awq_b200.gemm(dx, dqw, dqz, ds, 128, path=awq_b200.AWQ_PATH_TS)
    torch.cuda.synchronize()
    assert torch.equal(auto, ts)
    bias = torch.from_numpy(np.random.default_rng(M).uniform(-2, 2, N).astype(np.float16)).to(cuda)
    ab = awq_b200.gemm(dx, dqw, dqz, ds, 128, bias=bias)
    full = dx.float() @ awq_b200.dequant(dqw, dqz, ds, 128).float() + bias.float()
    assert O.max_rel_err(ab.float().cpu().numpy(), full.cpu().numpy()) <= TOL
    assert awq_b200.device_status() == 0
