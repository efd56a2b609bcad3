"""GPU parity: the sm_100a kernels (through the C-ABI) against the CPU oracle.

Bars (written out here, checked below):
  * dequantized weights: bit-exact with the reference's fp16 (w - z) * scale
    (NaN payloads aside);
  * outputs: max |out - ref| / max |ref| <= 1e-2 against the fp32 oracle
    x.float() @ W.float(), the tolerance BASELINE.json's north star states.
"""
from __future__ import annotations

import numpy as np
import pytest
import torch

from oracle import oracle as O

pytestmark = pytest.mark.gpu
TOL = 1e-2


def _to_dev(c, dev):
    return (torch.from_numpy(np.ascontiguousarray(c["qweight"])).to(dev),
            torch.from_numpy(np.ascontiguousarray(c["qzeros"])).to(dev),
            torch.from_numpy(np.ascontiguousarray(c["scales"])).to(dev))


def _same_bits(a: np.ndarray, b: np.ndarray) -> bool:
    nan = np.isnan(a.view(np.float16)) & np.isnan(b.view(np.float16))
    return bool(((a.view(np.uint16) == b.view(np.uint16)) | nan).all())


# ------------------------------------------------------------------ dequant -------
def test_dequant_bit_exact_golden(golden, cuda):
    import awq_b200
    for name, c in golden.items():
        qw, qz, s = _to_dev(c, cuda)
        w = awq_b200.dequant(qw, qz, s, c["group_size"]).cpu().numpy()
        assert _same_bits(w, c["w_bits"].view(np.float16)), name


def test_dequant_dropin_writes_out_buf(golden, cuda):
    from kernels import awq_gemm
    c = golden["random_full_range"]
    qw, qz, s = _to_dev(c, cuda)
    buf = torch.full((qw.shape[0], s.shape[1]), float("nan"), dtype=torch.float16, device=cuda)
    r = awq_gemm._dequant_to_fp16(qw, qz, s, buf, c["group_size"])
    assert r is buf
    assert _same_bits(buf.cpu().numpy(), c["w_bits"].view(np.float16))


@pytest.mark.parametrize("K,N", [(3584, 3584), (18944, 3584), (3584, 37888)])
def test_dequant_full_size_sampled_groups(cuda, K, N):
    """Full Qwen2-7B shapes; the CPU oracle checks the first, a middle and the last group."""
    import awq_b200
    rng = np.random.default_rng(K + N)
    qw = rng.integers(-2**31, 2**31, size=(K, N // 8), dtype=np.int64).astype(np.int32)
    qz = rng.integers(-2**31, 2**31, size=(K // 128, N // 8), dtype=np.int64).astype(np.int32)
    s = rng.uniform(0.002, 0.02, size=(K // 128, N)).astype(np.float16)
    w = awq_b200.dequant(*(torch.from_numpy(a).to(cuda) for a in (qw, qz, s)), 128)
    for grp in (0, (K // 128) // 2, K // 128 - 1):
        rows = slice(grp * 128, grp * 128 + 128)
        ref = O.awq_dequant(qw[rows], qz[grp:grp + 1], s[grp:grp + 1], 128)
        assert _same_bits(w[rows].cpu().numpy(), ref), grp


# ------------------------------------------------------------------ GEMM ----------
@pytest.mark.parametrize("path", [0, 1])      # AUTO, DECODE
def test_gemm_golden(golden, cuda, path):
    import awq_b200
    for name, c in golden.items():
        if name == "extreme_scales":
            continue
        qw, qz, s = _to_dev(c, cuda)
        x = torch.from_numpy(c["x"]).to(cuda)
        x2 = x.reshape(-1, x.shape[-1])
        out = awq_b200.gemm(x2, qw, qz, s, c["group_size"], path=path)
        out = out.view(*x.shape[:-1], s.shape[1]).float().cpu().numpy()
        assert O.max_rel_err(out, c["out_ref_f32"]) <= TOL, name
        # and against the reference's own fp16 result
        assert O.max_rel_err(out, c["out_ref_fp16"]) <= TOL, name


def test_dropin_golden_shapes(golden, cuda):
    from kernels import awq_gemm
    for name, c in golden.items():
        if name == "extreme_scales":
            continue
        qw, qz, s = _to_dev(c, cuda)
        x = torch.from_numpy(c["x"]).to(cuda)
        out = awq_gemm.awq_gemm_forward(x, qw, qz, s, c["group_size"])
        assert out.shape == tuple(c["x"].shape[:-1]) + (s.shape[1],), name
        assert out.dtype == torch.float16
        assert O.max_rel_err(out.float().cpu().numpy(), c["out_ref_f32"]) <= TOL, name


SMALL_SHAPES = [  # (M, K, N, gs): ragged N (scalar loads), one group, tiny N, odd M
    (1, 128, 8, 128), (1, 256, 136, 128), (3, 384, 136, 128), (5, 256, 96, 64),
    (7, 512, 264, 128), (8, 1024, 512, 128), (9, 256, 256, 32), (13, 640, 328, 128),
    (16, 1024, 1024, 128), (17, 256, 512, 128), (33, 512, 256, 128), (100, 256, 64, 128),
]


@pytest.mark.parametrize("M,K,N,gs", SMALL_SHAPES)
def test_gemm_small_shapes_vs_oracle(cuda, M, K, N, gs):
    import awq_b200
    qw, qz, s = O.make_awq_layer(K, N, gs, seed=M * 1000 + N)
    x = O.make_x(M, K, seed=M + K)
    ref = O.awq_gemm_f32(x, qw, qz, s, gs)
    dev = [torch.from_numpy(a).to(cuda) for a in (x, qw, qz, s)]
    for path in (0, 1):
        out = awq_b200.gemm(dev[0], dev[1], dev[2], dev[3], gs, path=path)
        assert O.max_rel_err(out.float().cpu().numpy(), ref) <= TOL, (M, K, N, gs, path)


QWEN_SHAPES = {"q_o": (3584, 3584), "k_v": (3584, 512), "qkv": (3584, 4608),
               "gate_up": (3584, 37888), "down": (18944, 3584)}


@pytest.mark.parametrize("M", [1, 4, 16])
@pytest.mark.parametrize("shape", list(QWEN_SHAPES))
def test_gemm_qwen_shapes_vs_oracle_columns(cuda, shape, M):
    """Full decode shapes.  The CPU oracle computes three 64-column blocks (first,
    middle, last) over the whole K; the rest is checked against an fp32 GPU matmul of
    the bit-exact dequantized weights."""
    import awq_b200
    K, N = QWEN_SHAPES[shape]
    qw, qz, s = O.make_awq_layer(K, N, 128, seed=K * 7 + N)
    x = O.make_x(M, K, seed=M)
    dqw, dqz, ds, dx = (torch.from_numpy(a).to(cuda) for a in (qw, qz, s, x))
    out = awq_b200.gemm(dx, dqw, dqz, ds, 128).float()
    for c0 in (0, (N // 2) // 64 * 64, N - 64):
        cols = slice(c0, c0 + 64)
        wcols = slice(c0 // 8, (c0 + 64) // 8)
        ref = O.awq_gemm_f32(x, qw[:, wcols], qz[:, wcols], s[:, cols], 128)
        assert O.max_rel_err(out[:, cols].cpu().numpy(), ref) <= TOL, (shape, M, c0)
    W = awq_b200.dequant(dqw, dqz, ds, 128).float()
    full = dx.float() @ W
    assert O.max_rel_err(out.cpu().numpy(), full.cpu().numpy()) <= TOL


def test_gemm_deterministic_and_counters_reset(cuda):
    """Two calls in a row give identical bits (split-K counters return to zero and
    the reduction order is fixed)."""
    import awq_b200
    K, N = 18944, 3584
    qw, qz, s = O.make_awq_layer(K, N, 128, seed=5)
    x = O.make_x(4, K, seed=9)
    d = [torch.from_numpy(a).to(cuda) for a in (x, qw, qz, s)]
    a = awq_b200.gemm(*d, 128)
    b = awq_b200.gemm(*d, 128)
    torch.cuda.synchronize()
    assert torch.equal(a, b)
    assert awq_b200.device_status() == 0


def test_gemm_linearity_full_size(cuda):
    """out(x1 + x2) == out(x1) + out(x2) within the tolerance (gate+up, M = 16)."""
    import awq_b200
    K, N = 3584, 37888
    g = torch.Generator(device=cuda).manual_seed(3)
    qw = torch.randint(-2**31, 2**31, (K, N // 8), dtype=torch.int64, device=cuda,
                       generator=g).to(torch.int32)
    qz = torch.randint(-2**31, 2**31, (K // 128, N // 8), dtype=torch.int64, device=cuda,
                       generator=g).to(torch.int32)
    s = (torch.rand((K // 128, N), device=cuda, generator=g) * 0.018 + 0.002).half()
    x1 = torch.randn((16, K), device=cuda, generator=g).half()
    x2 = torch.randn((16, K), device=cuda, generator=g).half()
    y12 = awq_b200.gemm((x1.float() + x2.float()).half(), qw, qz, s).float()
    y1 = awq_b200.gemm(x1, qw, qz, s).float()
    y2 = awq_b200.gemm(x2, qw, qz, s).float()
    assert O.max_rel_err((y1 + y2).cpu().numpy(), y12.cpu().numpy()) <= TOL


def test_empty_and_strided_inputs(cuda):
    from kernels import awq_gemm
    K, N = 256, 64
    qw, qz, s = (torch.from_numpy(a).to(cuda) for a in O.make_awq_layer(K, N, 128, seed=2))
    out = awq_gemm.awq_gemm_forward(torch.empty((0, K), dtype=torch.float16, device=cuda),
                                    qw, qz, s)
    assert out.shape == (0, N)
    big = torch.randn((6, 2 * K), device=cuda).half()
    xs = big[:, ::2]                                    # non-contiguous view
    ref = O.awq_gemm_f32(xs.cpu().numpy(), *(a.cpu().numpy() for a in (qw, qz, s)))
    out = awq_gemm.awq_gemm_forward(xs, qw, qz, s)
    assert O.max_rel_err(out.float().cpu().numpy(), ref) <= TOL


def test_errors_on_gpu(cuda):
    from kernels import awq_gemm
    K, N = 256, 64
    qw, qz, s = (torch.from_numpy(a).to(cuda) for a in O.make_awq_layer(K, N, 128, seed=2))
    x = torch.randn((1, K), device=cuda).half()
    with pytest.raises(TypeError):
        awq_gemm.awq_gemm_forward(x.float(), qw, qz, s)
    with pytest.raises(ValueError):
        awq_gemm.awq_gemm_forward(x, qw, qz, s, group_size=96)
    with pytest.raises(ValueError):
        awq_gemm.awq_gemm_forward(torch.randn((1, K + 8), device=cuda).half(), qw, qz, s)


@pytest.mark.parametrize("M", [1, 4, 16])
def test_chained_calls_read_the_previous_output(cuda, M):
    """Six dependent calls back to back on one stream -- each call's activations are the
    previous call's output, with split and unsplit tiles alternating -- give the same
    bits eagerly, replayed from a CUDA graph, and with a device synchronisation between
    the calls.  Under programmatic dependent launch a call starts before the previous
    kernel has finished; this checks that it never reads the activations early and that
    the shared workspace's counters and slots are reused safely."""
    import awq_b200
    dims = [1024, 4096, 1024, 2048, 1024, 4096, 1024]
    layers = [tuple(torch.from_numpy(a).to(cuda)
                    for a in O.make_awq_layer(dims[i], dims[i + 1], 128, seed=60 + i))
              for i in range(len(dims) - 1)]
    x0 = torch.from_numpy(O.make_x(M, dims[0], seed=M)).to(cuda)

    def chain(sync):
        h = x0
        for w in layers:
            h = awq_b200.gemm(h, *w, 128)
            if sync:
                torch.cuda.synchronize()
        return h

    ref = chain(True)
    assert torch.isfinite(ref).all()
    eager = chain(False)
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        chain(False)                                   # workspace for this stream
    torch.cuda.synchronize()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g, stream=s):
        out = chain(False)
    g.replay()
    torch.cuda.synchronize()
    assert torch.equal(eager, ref)
    assert torch.equal(out, ref)
    assert awq_b200.device_status() == 0
    # the chain as a whole against fp32 dequantize-then-matmul, layer by layer
    h = x0.float()
    for w in layers:
        h = (h.half().float() @ awq_b200.dequant(*w, 128).float())
    assert O.max_rel_err(ref.float().cpu().numpy(), h.cpu().numpy()) <= 3 * TOL


@pytest.mark.parametrize("M,K,N,gs", [
    (1, 3584, 4608, 128),     # decode kernel, split tiles (fused q/k/v shape)
    (4, 3584, 4608, 128),     # decode kernel, 4 tokens
    (16, 1024, 1024, 128),    # decode kernel, 8-token chunks
    (1, 512, 37888, 128),     # decode kernel, one CTA per tile
    (5, 384, 136, 128),       # generic decode kernel (ragged N)
    (300, 1024, 1024, 128),   # tcgen05 prefill kernel
])
def test_bias_epilogue(cuda, M, K, N, gs):
    """awq_gemm_bias_forward = product + bias in one kernel (model/qwen2.py:45-46,108-109):
    within the tolerance of the fp32 oracle plus bias, and of the two-step GPU form."""
    import awq_b200
    from kernels import awq_gemm
    qw, qz, s = O.make_awq_layer(K, N, gs, seed=M + N)
    x = O.make_x(M, K, seed=K)
    b = np.random.default_rng(7).uniform(-2, 2, size=N).astype(np.float16)
    ref = O.awq_gemm_f32(x, qw, qz, s, gs) + b.astype(np.float32)
    dx, dqw, dqz, ds, db = (torch.from_numpy(a).to(cuda) for a in (x, qw, qz, s, b))
    out = awq_gemm.awq_gemm_bias_forward(dx, dqw, dqz, ds, db, gs)
    assert out.shape == (M, N) and out.dtype == torch.float16
    assert O.max_rel_err(out.float().cpu().numpy(), ref) <= TOL
    two_step = awq_b200.gemm(dx, dqw, dqz, ds, gs).float() + db.float()
    assert O.max_rel_err(out.float().cpu().numpy(), two_step.cpu().numpy()) <= TOL
    assert awq_b200.device_status() == 0
    with pytest.raises(ValueError):
        awq_gemm.awq_gemm_bias_forward(dx, dqw, dqz, ds, db[:-8], gs)


def test_two_devices_in_one_process(cuda):
    """One process driving two GPUs: every kernel family (decode, small-M, prefill) runs
    on both devices -- their shared-memory limits are raised per device."""
    import awq_b200
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    K, N = 512, 512
    qw, qz, s = O.make_awq_layer(K, N, 128, seed=31)
    for dev_index in (1, 0, 1):
        d = torch.device("cuda", dev_index)
        dqw, dqz, ds = (torch.from_numpy(np.ascontiguousarray(a)).to(d) for a in (qw, qz, s))
        for M in (1, 12, 300):
            x = O.make_x(M, K, seed=M + dev_index)
            with torch.cuda.device(d):
                out = awq_b200.gemm(torch.from_numpy(x).to(d), dqw, dqz, ds, 128)
            assert out.device == d
            assert O.max_rel_err(out.float().cpu().numpy(), O.awq_gemm_f32(x, qw, qz, s)) <= TOL
