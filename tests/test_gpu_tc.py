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


@pytest.mark.parametrize("M,K,N", [
    (128, 18944, 3584),     # down shape: 14 tiles -> 10 CTAs per tile along K
    (40, 3584, 3584),       # o shape at small M: 14 tiles -> 7 per tile
    (300, 3584, 4608),      # fused q/k/v at M = 300: 36 tiles of 256 rows -> 4 per tile
])
def test_tc_split_k(cuda, M, K, N):
    """Few output tiles: the tcgen05 kernel splits K over several CTAs per tile, writes
    fp32 partials into the workspace and a reduce kernel sums them in split order.
    Checked against the CPU oracle on three 64-column blocks and against an fp32 product
    of the exactly dequantized weights everywhere; repeated calls give the same bits; the
    bias goes through the reduce kernel; without a workspace the kernel runs unsplit."""
    import ctypes
    import awq_b200
    import awq_b200._lib as L
    qw, qz, s = O.make_awq_layer(K, N, 128, seed=M * 3 + N)
    x = O.make_x(M, K, seed=M)
    dx, dqw, dqz, ds = _dev(cuda, x, qw, qz, s)
    lib = L.load()
    assert lib.awq_gemm_workspace_bytes(M, N, K, 128) > 0      # the split's partials
    a = awq_b200.gemm(dx, dqw, dqz, ds, 128, path=awq_b200.AWQ_PATH_TC)
    b = awq_b200.gemm(dx, dqw, dqz, ds, 128, path=awq_b200.AWQ_PATH_TC)
    torch.cuda.synchronize()
    assert torch.equal(a, b)
    for c0 in (0, (N // 2) // 64 * 64, N - 64):
        ref = O.awq_gemm_f32(x, qw[:, c0 // 8:(c0 + 64) // 8], qz[:, c0 // 8:(c0 + 64) // 8],
                             s[:, c0:c0 + 64], 128)
        assert O.max_rel_err(a[:, c0:c0 + 64].float().cpu().numpy(), ref) <= TOL, c0
    full = dx.float() @ awq_b200.dequant(dqw, dqz, ds, 128).float()
    assert O.max_rel_err(a.float().cpu().numpy(), full.cpu().numpy()) <= TOL
    bias = torch.from_numpy(np.random.default_rng(3).uniform(-1, 1, N).astype(np.float16)).to(cuda)
    ab = awq_b200.gemm(dx, dqw, dqz, ds, 128, bias=bias)
    assert O.max_rel_err(ab.float().cpu().numpy(), (full + bias.float()).cpu().numpy()) <= TOL
    # no workspace: one CTA per tile, same result within the tolerance
    out = torch.empty((M, N), dtype=torch.float16, device=cuda)
    rc = lib.awq_gemm_f16_ex(dx.data_ptr(), K, dqw.data_ptr(), dqz.data_ptr(), ds.data_ptr(),
                             out.data_ptr(), N, M, N, K, 128, None, 0,
                             ctypes.c_void_p(torch.cuda.current_stream().cuda_stream),
                             awq_b200.AWQ_PATH_TC)
    assert rc == 0, lib.awq_last_error()
    torch.cuda.synchronize()
    assert O.max_rel_err(out.float().cpu().numpy(), full.cpu().numpy()) <= TOL
    assert awq_b200.device_status() == 0


@pytest.mark.parametrize("M,K,N", [
    (2048, 18944, 3584),    # down: 8 x 14 = 112 tiles on 148 SMs, shares reach 4 tiles
    (1536, 18944, 3584),    # 6 x 14 = 84 tiles
    (1536, 3584, 3584),     # 84 tiles, 56 K steps: short tails
    (1536, 18944, 4608),    # 6 x 18 = 108 tiles
    (2000, 18944, 3360),    # ragged last row tile and last column tile
])
def test_tc_stream_k(cuda, M, K, N):
    """Output tiles that fill between half and most of one wave (stream-K): one CTA per
    tile runs the tile's first K steps, the other SMs' CTAs share the tiles' last steps;
    each tile, in two or three parts, is summed from fp32 slots by the last CTA to finish
    a part, in slot order.  Checked against an fp32
    product of the exactly dequantized weights and the CPU oracle on three 64-column
    blocks; repeated calls give the same bits (counters reset, fixed summation order); the
    bias is added once; without a workspace the kernel runs one CTA per tile."""
    import ctypes
    import awq_b200
    import awq_b200._lib as L
    qw, qz, s = O.make_awq_layer(K, N, 128, seed=M + K)
    x = O.make_x(M, K, seed=M)
    dx, dqw, dqz, ds = _dev(cuda, x, qw, qz, s)
    lib = L.load()
    assert lib.awq_gemm_workspace_bytes(M, N, K, 128) > 0      # the stream-K slots
    a = awq_b200.gemm(dx, dqw, dqz, ds, 128, path=awq_b200.AWQ_PATH_TC)
    b = awq_b200.gemm(dx, dqw, dqz, ds, 128, path=awq_b200.AWQ_PATH_TC)
    torch.cuda.synchronize()
    assert torch.equal(a, b)
    full = dx.float() @ awq_b200.dequant(dqw, dqz, ds, 128).float()
    assert O.max_rel_err(a.float().cpu().numpy(), full.cpu().numpy()) <= TOL
    rows = slice(0, min(M, 64))
    for c0 in (0, (N // 2) // 64 * 64, N - 64):
        ref = O.awq_gemm_f32(x[rows], qw[:, c0 // 8:(c0 + 64) // 8], qz[:, c0 // 8:(c0 + 64) // 8],
                             s[:, c0:c0 + 64], 128)
        assert O.max_rel_err(a[rows, c0:c0 + 64].float().cpu().numpy(), ref) <= TOL, c0
    bias = torch.from_numpy(np.random.default_rng(5).uniform(-1, 1, N).astype(np.float16)).to(cuda)
    ab = awq_b200.gemm(dx, dqw, dqz, ds, 128, bias=bias)
    assert O.max_rel_err(ab.float().cpu().numpy(), (full + bias.float()).cpu().numpy()) <= TOL
    out = torch.empty((M, N), dtype=torch.float16, device=cuda)
    rc = lib.awq_gemm_f16_ex(dx.data_ptr(), K, dqw.data_ptr(), dqz.data_ptr(), ds.data_ptr(),
                             out.data_ptr(), N, M, N, K, 128, None, 0,
                             ctypes.c_void_p(torch.cuda.current_stream().cuda_stream),
                             awq_b200.AWQ_PATH_TC)
    assert rc == 0, lib.awq_last_error()
    torch.cuda.synchronize()
    assert O.max_rel_err(out.float().cpu().numpy(), full.cpu().numpy()) <= TOL
    assert awq_b200.device_status() == 0


@pytest.mark.parametrize("M,K,N", [
    (1000, 1024, 10016),    # 4 x 40 = 160 tiles of 256 x 256, ragged last row and column tile
    (300, 2048, 37888),     # 2 x 148 = 296 tiles: every CTA takes two
    (100, 512, 40000),      # 128-row tiles: 1 x 157
])
def test_tc_persistent(cuda, M, K, N):
    """More output tiles than SMs: one CTA per SM takes tiles c, c + SMs, ... in turn, the
    next tile's loads overlapping the current tile's epilogue.  Checked against an fp32
    product of the exactly dequantized weights, the CPU oracle on 64-column blocks at both
    ends, with the bias, and bit-equal on a repeated call."""
    import awq_b200
    qw, qz, s = O.make_awq_layer(K, N, 128, seed=M + 7)
    x = O.make_x(M, K, seed=K + 3)
    dx, dqw, dqz, ds = _dev(cuda, x, qw, qz, s)
    sms = torch.cuda.get_device_properties(cuda).multi_processor_count
    bm = 256 if M > 128 else 128
    assert ((M + bm - 1) // bm) * ((N + 255) // 256) > sms
    a = awq_b200.gemm(dx, dqw, dqz, ds, 128, path=awq_b200.AWQ_PATH_TC)
    b = awq_b200.gemm(dx, dqw, dqz, ds, 128, path=awq_b200.AWQ_PATH_TC)
    torch.cuda.synchronize()
    assert torch.equal(a, b)
    full = dx.float() @ awq_b200.dequant(dqw, dqz, ds, 128).float()
    assert O.max_rel_err(a.float().cpu().numpy(), full.cpu().numpy()) <= TOL
    rows = slice(M - min(M, 64), M)
    for c0 in (0, N - 64):
        ref = O.awq_gemm_f32(x[rows], qw[:, c0 // 8:(c0 + 64) // 8], qz[:, c0 // 8:(c0 + 64) // 8],
                             s[:, c0:c0 + 64], 128)
        assert O.max_rel_err(a[rows, c0:c0 + 64].float().cpu().numpy(), ref) <= TOL, c0
    bias = torch.from_numpy(np.random.default_rng(9).uniform(-1, 1, N).astype(np.float16)).to(cuda)
    ab = awq_b200.gemm(dx, dqw, dqz, ds, 128, bias=bias)
    assert O.max_rel_err(ab.float().cpu().numpy(), (full + bias.float()).cpu().numpy()) <= TOL
    assert awq_b200.device_status() == 0
