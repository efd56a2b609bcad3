"""CPU oracle for the AWQ W4A16 path -- TEST INFRASTRUCTURE ONLY.

Only ``tests/``, ``__graft_entry__.smoke()`` and ``bench.py`` (its cpu_baseline
leg and its ``--impl reference`` arm) may import this module.  It checks the
CUDA library and is never the thing that is measured or shipped: the product
path (``kernels.awq_gemm.awq_gemm_forward`` and the C-ABI) has no CPU fallback.

Everything here restates songqiuyu/Qwen2-7B-Triton_Engine:

* ``awq_unpack`` / ``awq_dequant`` -- ``kernels/awq_gemm.py:36-59``
  (``_dequant_awq_kernel``): element ``e = n % 8`` of a packed int32 sits at
  ``shift = 4 * [0,4,1,5,2,6,3,7][e]``; ``W = (fp16(w) - fp16(z)) * scale`` in
  fp16, with ``scale``/``z`` taken from row ``k // group_size``.  The same
  arithmetic appears vectorised in ``test/compare_benchmark.py:79-92`` and as a
  per-column loop in ``inference/baseline_kernels.py:44-57``.
* ``awq_gemm_f32`` -- the reference's dequantize-then-matmul path
  (``test/compare_benchmark.py:94``, ``kernels/awq_gemm.py:266``) with the
  matmul in fp32 on the host: ``x.float() @ W.float()``.
* ``silu_mul_f16`` -- ``kernels/silu_mul.py:31-38`` (fp16 in, fp32 x * sigmoid(x) * y,
  fp16 out); pinned bit-exact against the reference's interpreted kernel
  (``tests/golden/silu_golden.npz``, made by ``tests/golden/make_golden_silu.py``).
* ``awq_silu_mul_f32`` -- the reference MLP's activation on the fused gate+up product
  (``model/qwen2.py:181-194``: halves sliced out of the product, then
  ``kernels/silu_mul.py:41-64``: ``x * sigmoid(x) * y``), all in fp32.
* ``awq_pack`` -- the inverse packing, used to build synthetic checkpoints in
  the layout ``model/qwen2.py:34-36`` registers (qweight int32 [K, N/8],
  qzeros int32 [K/gs, N/8], scales fp16 [K/gs, N]).

The C restatement in ``awq_oracle.c`` computes the same functions; ``load_c``
builds nothing, it only opens ``oracle/_build/liboracle.so`` made by
``oracle/Makefile``.
"""
from __future__ import annotations

import ctypes
import os
import pathlib

import numpy as np

# Element e of an 8-pack sits at nibble AWQ_ORDER[e] (kernels/awq_gemm.py:5-6,38).
AWQ_ORDER = np.array([0, 4, 1, 5, 2, 6, 3, 7], dtype=np.int64)
AWQ_SHIFTS = AWQ_ORDER * 4

_HERE = pathlib.Path(__file__).resolve().parent
C_LIB_PATH = _HERE / "_build" / "liboracle.so"


def awq_unpack(packed: np.ndarray) -> np.ndarray:
    """int32 [R, C] -> uint8 [R, 8*C]: element n = 8*c + e is nibble AWQ_ORDER[e]."""
    p = np.ascontiguousarray(packed).view(np.uint32).astype(np.uint64)
    vals = (p[:, :, None] >> AWQ_SHIFTS[None, None, :].astype(np.uint64)) & 0xF
    return vals.reshape(p.shape[0], p.shape[1] * 8).astype(np.uint8)


def awq_pack(vals: np.ndarray) -> np.ndarray:
    """uint8 [R, N] with values 0..15 -> int32 [R, N/8] in AWQ nibble order."""
    v = np.asarray(vals).astype(np.uint64)
    r, n = v.shape
    assert n % 8 == 0, "N must be a multiple of 8"
    v = v.reshape(r, n // 8, 8)
    word = np.zeros((r, n // 8), dtype=np.uint64)
    for e in range(8):
        word |= (v[:, :, e] & 0xF) << np.uint64(AWQ_SHIFTS[e])
    return word.astype(np.uint32).view(np.int32)


def check_shapes(qweight, qzeros, scales, group_size):
    """Shape rules of the packed layout (model/qwen2.py:34-36)."""
    K, pn = qweight.shape
    N = scales.shape[1]
    if N != pn * 8:
        raise ValueError(f"scales has N={N} but qweight packs {pn * 8} columns")
    if group_size <= 0 or K % group_size:
        raise ValueError(f"K={K} is not a multiple of group_size={group_size}")
    if qzeros.shape != (K // group_size, pn) or scales.shape != (K // group_size, N):
        raise ValueError("qzeros/scales shapes do not match [K/group_size, ...]")
    return K, N


def awq_dequant(qweight: np.ndarray, qzeros: np.ndarray, scales: np.ndarray,
                group_size: int = 128) -> np.ndarray:
    """fp16 [K, N]: ``(fp16(w) - fp16(z)) * scale`` (kernels/awq_gemm.py:59).

    numpy evaluates an fp16 * fp16 product in fp32 and rounds once to fp16;
    the fp32 product of an integer in [-15, 15] and an fp16 value is exact, so
    this equals an IEEE fp16 multiply (round to nearest even).
    """
    K, N = check_shapes(qweight, qzeros, scales, group_size)
    w = awq_unpack(qweight).astype(np.float16)                        # [K, N]
    z = awq_unpack(qzeros).astype(np.float16)                         # [K/gs, N]
    s = np.asarray(scales, dtype=np.float16)
    diff = (w.reshape(K // group_size, group_size, N) - z[:, None, :])  # exact ints
    with np.errstate(over="ignore", invalid="ignore"):   # inf scales / overflow are data
        out = (diff * s[:, None, :]).astype(np.float16)
    return out.reshape(K, N)


def awq_gemm_f32(x: np.ndarray, qweight, qzeros, scales, group_size: int = 128) -> np.ndarray:
    """fp32 [..., N] = x.float() @ dequant(W).float() (the fp32 host path)."""
    x = np.asarray(x, dtype=np.float16)
    W = awq_dequant(qweight, qzeros, scales, group_size)
    x2 = x.reshape(-1, x.shape[-1]).astype(np.float32)
    out = x2 @ W.astype(np.float32)
    return out.reshape(*x.shape[:-1], W.shape[1])


def silu_mul_f16(gate: np.ndarray, up: np.ndarray) -> np.ndarray:
    """fp16 silu(gate) * up with fp32 arithmetic (kernels/silu_mul.py:31-38: load as fp32,
    x * sigmoid(x) * y, store fp16)."""
    with np.errstate(over="ignore"):
        x = np.asarray(gate, dtype=np.float16).astype(np.float32)
        y = np.asarray(up, dtype=np.float16).astype(np.float32)
        sig = np.float32(1.0) / (np.float32(1.0) + np.exp(-x))
        return (x * sig * y).astype(np.float16)


def awq_silu_mul_f32(x: np.ndarray, qweight, qzeros, scales, group_size: int = 128) -> np.ndarray:
    """fp32 [..., N/2] = silu(P[..., :N/2]) * P[..., N/2:] with P = awq_gemm_f32(x, W)."""
    p = awq_gemm_f32(x, qweight, qzeros, scales, group_size).astype(np.float64)
    half = p.shape[-1] // 2
    g, u = p[..., :half], p[..., half:]
    return (g / (1.0 + np.exp(-g)) * u).astype(np.float32)


def max_rel_err(out: np.ndarray, ref: np.ndarray) -> float:
    """max |out - ref| / max |ref| -- the error measure the parity tests bound."""
    out = np.asarray(out, dtype=np.float64)
    ref = np.asarray(ref, dtype=np.float64)
    denom = float(np.max(np.abs(ref))) if ref.size else 0.0
    if denom == 0.0:
        return float(np.max(np.abs(out))) if out.size else 0.0
    return float(np.max(np.abs(out - ref)) / denom)


# ----------------------------------------------------------------------------------
# Synthetic inputs (distributions of the benchmark configs: x ~ N(0,1); int4 weights
# and zeros uniform 0..15; scales uniform in [0.002, 0.02]; group 128).
# ----------------------------------------------------------------------------------
def make_awq_layer(K: int, N: int, group_size: int = 128, seed: int = 1):
    """Seeded synthetic AWQ layer.  Uniform random 32-bit words give every nibble
    (weight and zero) an independent uniform value in 0..15."""
    rng = np.random.default_rng(seed)
    qw = rng.integers(0, 2**32, size=(K, N // 8), dtype=np.uint32).view(np.int32)
    qz = rng.integers(0, 2**32, size=(K // group_size, N // 8), dtype=np.uint32).view(np.int32)
    s = rng.uniform(0.002, 0.02, size=(K // group_size, N)).astype(np.float16)
    return qw, qz, s


def make_x(M: int, K: int, seed: int = 0) -> np.ndarray:
    rng = np.random.default_rng(seed)
    return rng.standard_normal((M, K)).astype(np.float16)


# ----------------------------------------------------------------------------------
# torch restatement of the same host path, used as the timed CPU baseline (torch's
# CPU matmul uses every thread torch is given).  Mirrors test/compare_benchmark.py:72-95
# with the final matmul in fp32.
# ----------------------------------------------------------------------------------
def torch_awq_gemm_f32(x, qweight, qzeros, scales, group_size: int = 128):
    import torch
    K = qweight.shape[0]
    N = scales.shape[1]
    G = K // group_size
    shifts = torch.as_tensor(AWQ_SHIFTS, dtype=torch.int32).view(1, 1, 8)
    w = ((qweight.view(K, N // 8, 1) >> shifts) & 0xF).reshape(K, N).to(torch.float16)
    z = ((qzeros.view(G, N // 8, 1) >> shifts) & 0xF).reshape(G, N).to(torch.float16)
    W = ((w.view(G, group_size, N) - z.view(G, 1, N)) * scales.view(G, 1, N)).view(K, N)
    x2 = x.reshape(-1, K).float()
    return (x2 @ W.float()).view(*x.shape[:-1], N)


# ----------------------------------------------------------------------------------
# C restatement (awq_oracle.c), loaded through ctypes.
# ----------------------------------------------------------------------------------
_c = None


def load_c():
    """Open the C oracle built by ``make -C oracle``; raises if it was not built."""
    global _c
    if _c is not None:
        return _c
    if not C_LIB_PATH.exists():
        raise FileNotFoundError(f"{C_LIB_PATH} missing: run `make -C oracle`")
    lib = ctypes.CDLL(str(C_LIB_PATH))
    P = ctypes.c_void_p
    I64 = ctypes.c_int64
    lib.oracle_awq_dequant.argtypes = [P, P, P, P, I64, I64, I64]
    lib.oracle_awq_dequant.restype = ctypes.c_int
    lib.oracle_awq_gemm_f32.argtypes = [P, I64, P, P, P, I64, I64, I64, P, P]
    lib.oracle_awq_gemm_f32.restype = ctypes.c_int
    lib.oracle_float_to_half_array.argtypes = [P, P, I64]
    lib.oracle_float_to_half_array.restype = None
    _c = lib
    return lib


def _ptr(a: np.ndarray):
    return a.ctypes.data_as(ctypes.c_void_p)


def c_awq_dequant(qweight, qzeros, scales, group_size: int = 128) -> np.ndarray:
    lib = load_c()
    K, N = check_shapes(qweight, qzeros, scales, group_size)
    qw = np.ascontiguousarray(qweight, dtype=np.int32)
    qz = np.ascontiguousarray(qzeros, dtype=np.int32)
    s = np.ascontiguousarray(scales, dtype=np.float16)
    out = np.empty((K, N), dtype=np.float16)
    rc = lib.oracle_awq_dequant(_ptr(qw), _ptr(qz), _ptr(s), _ptr(out), K, N, group_size)
    if rc:
        raise ValueError("oracle_awq_dequant rejected the shapes")
    return out


def c_awq_gemm_f32(x, qweight, qzeros, scales, group_size: int = 128) -> np.ndarray:
    lib = load_c()
    K, N = check_shapes(qweight, qzeros, scales, group_size)
    x = np.ascontiguousarray(np.asarray(x, dtype=np.float16))
    x2 = x.reshape(-1, K)
    qw = np.ascontiguousarray(qweight, dtype=np.int32)
    qz = np.ascontiguousarray(qzeros, dtype=np.int32)
    s = np.ascontiguousarray(scales, dtype=np.float16)
    out = np.empty((x2.shape[0], N), dtype=np.float32)
    scratch = np.empty((K, N), dtype=np.float16)
    rc = lib.oracle_awq_gemm_f32(_ptr(x2), x2.shape[0], _ptr(qw), _ptr(qz), _ptr(s), K, N,
                                 group_size, _ptr(out), _ptr(scratch))
    if rc:
        raise ValueError("oracle_awq_gemm_f32 rejected the shapes")
    return out.reshape(*x.shape[:-1], N)


def c_float_to_half(a: np.ndarray) -> np.ndarray:
    lib = load_c()
    a = np.ascontiguousarray(a, dtype=np.float32)
    out = np.empty(a.shape, dtype=np.float16)
    lib.oracle_float_to_half_array(_ptr(a), _ptr(out), a.size)
    return out


def cpu_threads() -> int:
    try:
        return len(os.sched_getaffinity(0))
    except AttributeError:  # pragma: no cover
        return os.cpu_count() or 1
