"""GPU parity of the gate+up product fused with SiLU-mul (``awq_gemm_f16_silu_mul``,
``awq_b200.gemm_silu_mul``, ``kernels.awq_gemm.awq_gemm_silu_mul_forward``).

Two references: the CPU oracle (fp32 product, fp32 silu(g) * u; bar 1e-2 max relative
error) and the reference MLP's own sequence run on this library's product -- fp16
product, halves, fp32 x * sigmoid(x) * y, fp16 (model/qwen2.py:181-194 with
kernels/silu_mul.py:41-64).  The second differs only by the exp implementation: bar 2e-3.
"""
from __future__ import annotations

import numpy as np
import pytest
import torch
import torch.nn.functional as F

from oracle import oracle as O

pytestmark = pytest.mark.gpu
TOL = 1e-2
TOL_SEQ = 2e-3


def _dev(cuda, *arrays):
    return [torch.from_numpy(np.ascontiguousarray(a)).to(cuda) for a in arrays]


def _sequence(awq_b200, dx, dqw, dqz, ds, gs):
    gu = awq_b200.gemm(dx, dqw, dqz, ds, gs)
    half = gu.shape[1] // 2
    return (F.silu(gu[:, :half].float()) * gu[:, half:].float()).half()


@pytest.mark.parametrize("M,K,N", [
    (1, 512, 5120), (3, 512, 5120), (4, 1024, 5120), (5, 512, 5120), (8, 768, 5120),  # pair epilogue
    (12, 512, 5120), (40, 512, 5120), (300, 512, 5120),                             # product + kernel
    (1, 512, 640),            # halves not on a 256-column strip: product + kernel
    (2, 256, 48),             # N / 2 = 24: generic product, scalar SiLU-mul
])
def test_silu_mul_vs_oracle_and_sequence(cuda, M, K, N):
    import awq_b200
    qw, qz, s = O.make_awq_layer(K, N, 128, seed=M + N)
    x = O.make_x(M, K, seed=K + M)
    dx, dqw, dqz, ds = _dev(cuda, x, qw, qz, s)
    h = awq_b200.gemm_silu_mul(dx, dqw, dqz, ds, 128)
    assert h.shape == (M, N // 2)
    ref = O.awq_silu_mul_f32(x, qw, qz, s, 128)
    assert O.max_rel_err(h.float().cpu().numpy(), ref) <= TOL
    seq = _sequence(awq_b200, dx, dqw, dqz, ds, 128)
    assert O.max_rel_err(h.float().cpu().numpy(), seq.float().cpu().numpy()) <= TOL_SEQ
    assert awq_b200.device_status() == 0


@pytest.mark.parametrize("M", [1, 8, 12, 16])
def test_silu_mul_qwen2_gate_up(cuda, M):
    """The real MLP shape (gate+up 3584 x 37888): 74 gate / up strip pairs; repeated calls
    give the same bits (the pair counters are reset), and the product calls that share the
    workspace before and after stay correct."""
    import awq_b200
    K, N = 3584, 37888
    qw, qz, s = O.make_awq_layer(K, N, 128, seed=11 + M)
    x = O.make_x(M, K, seed=12)
    dx, dqw, dqz, ds = _dev(cuda, x, qw, qz, s)
    seq = _sequence(awq_b200, dx, dqw, dqz, ds, 128)
    a = awq_b200.gemm_silu_mul(dx, dqw, dqz, ds, 128)
    b = awq_b200.gemm_silu_mul(dx, dqw, dqz, ds, 128)
    seq2 = _sequence(awq_b200, dx, dqw, dqz, ds, 128)
    torch.cuda.synchronize()
    assert torch.equal(a, b)
    assert torch.equal(seq, seq2)
    assert O.max_rel_err(a.float().cpu().numpy(), seq.float().cpu().numpy()) <= TOL_SEQ
    for c0 in (0, 9472, 18944 - 64):
        cols = np.r_[c0:c0 + 64, 18944 + c0:18944 + c0 + 64]
        ref = O.awq_silu_mul_f32(x, qw[:, cols[::8] // 8], qz[:, cols[::8] // 8], s[:, cols], 128)
        assert O.max_rel_err(a[:, c0:c0 + 64].float().cpu().numpy(), ref) <= TOL, c0
    assert awq_b200.device_status() == 0


def test_silu_mul_forward_shapes_and_graph(cuda):
    """The drop-in function keeps leading dimensions, and a captured CUDA graph replays
    the fused call with the same result."""
    import awq_b200
    from kernels.awq_gemm import awq_gemm_silu_mul_forward
    K, N = 512, 5120
    qw, qz, s = O.make_awq_layer(K, N, 128, seed=5)
    dqw, dqz, ds = _dev(cuda, qw, qz, s)
    x = torch.from_numpy(O.make_x(2, K, seed=6)).to(cuda).view(1, 2, K)
    h = awq_gemm_silu_mul_forward(x, dqw, dqz, ds)
    assert h.shape == (1, 2, N // 2)
    xs = x.clone()
    awq_gemm_silu_mul_forward(xs, dqw, dqz, ds)            # workspace allocated before capture
    torch.cuda.synchronize()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        hg = awq_gemm_silu_mul_forward(xs, dqw, dqz, ds)
    for _ in range(3):
        g.replay()
    torch.cuda.synchronize()
    assert torch.equal(hg, h)
    assert awq_b200.device_status() == 0


def test_silu_mul_small_halves(cuda):
    """Halves of 20 and 4 columns (N = 40, 8): generic product, scalar SiLU-mul."""
    import awq_b200
    for N in (40, 8):
        qw, qz, s = O.make_awq_layer(128, N, 128, seed=N)
        x = O.make_x(3, 128, seed=N)
        dx, dqw, dqz, ds = _dev(cuda, x, qw, qz, s)
        h = awq_b200.gemm_silu_mul(dx, dqw, dqz, ds, 128)
        assert h.shape == (3, N // 2)
        assert O.max_rel_err(h.float().cpu().numpy(), O.awq_silu_mul_f32(x, qw, qz, s)) <= TOL
    assert awq_b200.device_status() == 0


def test_silu_mul_golden(silu_golden, cuda):
    """Against the reference's own MLP sequence (torch_awq_gemm product, halves, interpreted
    _silu_mul_kernel) committed in tests/golden/silu_golden.npz: M = 3 (pair epilogue) and
    M = 12 with halves of 320 columns (product + elementwise kernel)."""
    import awq_b200
    for name in ("mlp_k256_i256_m3", "mlp_k384_i320_m12"):
        c = silu_golden[name]
        gs = int(c["group_size"])
        dx, dqw, dqz, ds = _dev(cuda, c["x"], c["qweight"], c["qzeros"], c["scales"])
        h = awq_b200.gemm_silu_mul(dx, dqw, dqz, ds, gs)
        ref = c["out_bits"].view(np.float16).astype(np.float32)
        assert O.max_rel_err(h.float().cpu().numpy(), ref) <= TOL, name
    assert awq_b200.device_status() == 0


@pytest.mark.parametrize("M,K,N", [
    (40, 1024, 37888),      # 128-row tiles: 1 x 74 tile pairs of 128 gate + 128 up columns
    (300, 512, 37888),      # 256-row tiles: 2 x 74, persistent CTAs
    (1000, 512, 20480),     # 4 x 40, ragged last row tile
])
def test_silu_mul_tcgen05_epilogue(cuda, M, K, N):
    """Above 16 tokens the tcgen05 kernel applies the SiLU-mul in its epilogue (each tile
    holds 128 gate columns and the matching 128 up columns; only [M, N/2] is written):
    against the CPU oracle, the reference MLP's sequence on this library's product, and
    bit-equal on a repeated call."""
    import awq_b200
    qw, qz, s = O.make_awq_layer(K, N, 128, seed=M + 3)
    x = O.make_x(M, K, seed=K + 5)
    dx, dqw, dqz, ds = _dev(cuda, x, qw, qz, s)
    a = awq_b200.gemm_silu_mul(dx, dqw, dqz, ds, 128)
    b = awq_b200.gemm_silu_mul(dx, dqw, dqz, ds, 128)
    torch.cuda.synchronize()
    assert a.shape == (M, N // 2)
    assert torch.equal(a, b)
    assert O.max_rel_err(a.float().cpu().numpy(), O.awq_silu_mul_f32(x, qw, qz, s, 128)) <= TOL
    seq = _sequence(awq_b200, dx, dqw, dqz, ds, 128)
    assert O.max_rel_err(a.float().cpu().numpy(), seq.float().cpu().numpy()) <= TOL_SEQ
    assert awq_b200.device_status() == 0


@pytest.mark.parametrize("M,K,N", [
    (9, 512, 37888),        # 148 CTAs of 16 tokens x (128 gate + 128 up) columns
    (13, 256, 18944),       # 74 CTAs (K too short to split)
    (16, 1024, 20480),      # 80 CTAs, full 16-token tile
])
def test_silu_mul_small_m_tcgen05_epilogue(cuda, M, K, N):
    """From 9 to 16 tokens the small-M tcgen05 kernel applies the SiLU-mul in its
    epilogue when it runs without a K split (the up lanes hand their sums to the gate
    lanes through shared memory): against the CPU oracle, the reference MLP's sequence
    on this library's product, and bit-equal on a repeated call."""
    import awq_b200
    qw, qz, s = O.make_awq_layer(K, N, 128, seed=M + 7)
    x = O.make_x(M, K, seed=K + 9)
    dx, dqw, dqz, ds = _dev(cuda, x, qw, qz, s)
    a = awq_b200.gemm_silu_mul(dx, dqw, dqz, ds, 128)
    b = awq_b200.gemm_silu_mul(dx, dqw, dqz, ds, 128)
    torch.cuda.synchronize()
    assert a.shape == (M, N // 2)
    assert torch.equal(a, b)
    assert O.max_rel_err(a.float().cpu().numpy(), O.awq_silu_mul_f32(x, qw, qz, s, 128)) <= TOL
    seq = _sequence(awq_b200, dx, dqw, dqz, ds, 128)
    assert O.max_rel_err(a.float().cpu().numpy(), seq.float().cpu().numpy()) <= TOL_SEQ
    assert awq_b200.device_status() == 0
