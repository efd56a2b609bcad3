"""GPU parity of the tcgen05/TMEM prefill kernel (AWQ_PATH_TC) against the CPU oracle.

Bar: max |out - ref| / max |ref| <= 1e-2 against the fp32 oracle x.float() @ W.float()
(the W the kernel forms is bit-identical to the reference's, so the only difference is
fp32 summation order and the final fp16 rounding).
"""
from __future__ import annotations

import numpy as np
import pytest
import torch

from oracle import oracle as O

pytestmark = pytest.mark.gpu
TOL = 1e-2


def _dev(cuda, *arrays):
    return [torch.from_numpy(np.ascontiguousarray(a)).to(cuda) for a in arrays]


@pytest.mark.parametrize("M,K,N", [
    (17, 256, 256), (64, 128, 32), (128, 256, 512), (129, 384, 320), (256, 512, 256),
    (300, 1024, 768), (513, 640, 4608 // 8 * 8),
])
def test_tc_small_shapes_vs_oracle(cuda, M, K, N):
    import awq_b200
    qw, qz, s = O.make_awq_layer(K, N, 128, seed=M + N)
    x = O.make_x(M, K, seed=K)
    ref = O.awq_gemm_f32(x, qw, qz, s, 128)
    dx, dqw, dqz, ds = _dev(cuda, x, qw, qz, s)
    assert awq_b200.tc_supported(dx, dqw, dqz, ds, 128)
    out = awq_b200.gemm(dx, dqw, dqz, ds, 128, path=awq_b200.AWQ_PATH_TC)
    assert O.max_rel_err(out.float().cpu().numpy(), ref) <= TOL
    assert awq_b200.device_status() == 0


def test_tc_golden(golden, cuda):
    import awq_b200
    for name, c in golden.items():
        if name == "extreme_scales":
            continue
        x = c["x"].reshape(-1, c["x"].shape[-1])
        dx, dqw, dqz, ds = _dev(cuda, x, c["qweight"], c["qzeros"], c["scales"])
        if not awq_b200.tc_supported(dx, dqw, dqz, ds, c["group_size"]):
            continue                         # N % 32 or group_size % 64 rule
        out = awq_b200.gemm(dx, dqw, dqz, ds, c["group_size"], path=awq_b200.AWQ_PATH_TC)
        ref = c["out_ref_f32"].reshape(out.shape)
        assert O.max_rel_err(out.float().cpu().numpy(), ref) <= TOL, name


def test_tc_group_size_256_and_rejects_64(cuda):
    import awq_b200
    K, N, M = 512, 256, 40
    qw, qz, s = O.make_awq_layer(K, N, 256, seed=4)
    x = O.make_x(M, K, seed=5)
    dx, dqw, dqz, ds = _dev(cuda, x, qw, qz, s)
    out = awq_b200.gemm(dx, dqw, dqz, ds, 256, path=awq_b200.AWQ_PATH_TC)
    assert O.max_rel_err(out.float().cpu().numpy(), O.awq_gemm_f32(x, qw, qz, s, 256)) <= TOL
    qw, qz, s = O.make_awq_layer(K, 264, 32, seed=4)          # N % 32 != 0, gs 32
    dqw, dqz, ds = _dev(cuda, qw, qz, s)
    with pytest.raises(awq_b200.AwqError):
        awq_b200.gemm(dx, dqw, dqz, ds, 32, path=awq_b200.AWQ_PATH_TC)
    # AUTO falls back to the decode kernel for such shapes and stays correct
    out = awq_b200.gemm(dx, dqw, dqz, ds, 32)
    assert O.max_rel_err(out.float().cpu().numpy(), O.awq_gemm_f32(x, qw, qz, s, 32)) <= TOL


@pytest.mark.parametrize("K,N", [(3584, 37888), (18944, 3584)])
def test_tc_prefill_2048_full_size(cuda, K, N):
    """M=2048 prefill on gate+up and down.  Three 64-column blocks
    are checked against the CPU oracle over the full K; every element is checked
    against an fp32 GPU matmul of the bit-exact dequantized weights."""
    import awq_b200
    M = 2048
    qw, qz, s = O.make_awq_layer(K, N, 128, seed=K + 3)
    x = O.make_x(M, K, seed=N)
    dx, dqw, dqz, ds = _dev(cuda, x, qw, qz, s)
    out = awq_b200.gemm(dx, dqw, dqz, ds, 128)                # AUTO -> tcgen05
    for c0 in (0, (N // 2) // 64 * 64, N - 64):
        cols = slice(c0, c0 + 64)
        wcols = slice(c0 // 8, (c0 + 64) // 8)
        ref = O.awq_gemm_f32(x, qw[:, wcols], qz[:, wcols], s[:, cols], 128)
        assert O.max_rel_err(out[:, cols].float().cpu().numpy(), ref) <= TOL, c0
    W = awq_b200.dequant(dqw, dqz, ds, 128).float()
    full = dx.float() @ W
    assert O.max_rel_err(out.float().cpu().numpy(), full.cpu().numpy()) <= TOL
    assert awq_b200.device_status() == 0


def test_tc_matches_decode_path(cuda):
    """Both kernels on the same inputs agree within the tolerance."""
    import awq_b200
    K, N, M = 3584, 4608, 96
    qw, qz, s = O.make_awq_layer(K, N, 128, seed=12)
    x = O.make_x(M, K, seed=13)
    dx, dqw, dqz, ds = _dev(cuda, x, qw, qz, s)
    a = awq_b200.gemm(dx, dqw, dqz, ds, 128, path=awq_b200.AWQ_PATH_TC).float()
    b = awq_b200.gemm(dx, dqw, dqz, ds, 128, path=awq_b200.AWQ_PATH_DECODE).float()
    assert O.max_rel_err(a.cpu().numpy(), b.cpu().numpy()) <= TOL
