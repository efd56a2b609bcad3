"""Drop-in replacement for songqiuyu/Qwen2-7B-Triton_Engine ``kernels/awq_gemm.py``.

Same module path and names as the reference, so a caller can put this package's
directory first on ``sys.path`` (``import kernels.awq_gemm``) or assign
``kernels.awq_gemm.awq_gemm_forward = <this function>`` the way
``test/compare_benchmark.py:111,120`` swaps implementations.

* ``awq_gemm_forward(x, qweight, qzeros, scales, group_size=128)`` -- reference
  ``kernels/awq_gemm.py:237-284``.  Same signature, same packed layout, same output
  shape ``x.shape[:-1] + (N,)`` with ``N = scales.shape[1]``.  M <= 8 runs the
  sm_100a decode kernel (mma.sync, split-K), 9 <= M <= 16 the small-M tcgen05 kernel
  (weights dequantized into tensor memory); larger M runs the tcgen05/TMEM prefill
  GEMM (split along K when its output tiles cannot fill the GPU) where its CTAs fill at
  least half the GPU or M > 64 (otherwise the decode kernel in 16-token launches).  Differences: inputs are validated up front (TypeError / ValueError), a CPU
  tensor raises instead of running, and no global K*N fp16 buffer is kept.
* ``awq_gemm_bias_forward(x, qweight, qzeros, scales, bias, group_size=128)`` -- not in
  the reference: the product plus the layer's bias in one kernel, for the callers that
  add the bias afterwards (``model/qwen2.py:45-46,108-109``).
* ``awq_gemm_silu_mul_forward(x, qweight, qzeros, scales, group_size=128)`` -- not in the
  reference: silu(gate) * up of the fused gate+up product in one call, replacing
  ``awq_gemm_forward`` + the two ``.contiguous()`` slices + ``silu_mul_forward`` of the
  reference MLP (``model/qwen2.py:181-194``, ``kernels/silu_mul.py:41-64``).  Output
  ``x.shape[:-1] + (N/2,)``.
* ``_dequant_to_fp16(qweight, qzeros, scales, out_buf, group_size=128)`` --
  reference ``kernels/awq_gemm.py:66-87``; writes the bit-identical fp16 weights.
"""
from __future__ import annotations

import torch

import awq_b200

__all__ = ["awq_gemm_forward", "awq_gemm_bias_forward", "awq_gemm_silu_mul_forward",
           "_dequant_to_fp16"]


def _dequant_to_fp16(qweight: torch.Tensor, qzeros: torch.Tensor, scales: torch.Tensor,
                     out_buf: torch.Tensor, group_size: int = 128) -> torch.Tensor:
    """AWQ int4 packed weights -> fp16 dense matrix, written into ``out_buf``."""
    if out_buf.is_contiguous() and out_buf.data_ptr() % 16 == 0:
        return awq_b200.dequant(qweight, qzeros, scales, group_size, out=out_buf)
    out_buf.copy_(awq_b200.dequant(qweight, qzeros, scales, group_size))
    return out_buf


def awq_gemm_forward(x: torch.Tensor, qweight: torch.Tensor, qzeros: torch.Tensor,
                     scales: torch.Tensor, group_size: int = 128) -> torch.Tensor:
    """AWQ W4A16 product: ``x [..., K] fp16 @ W [K, N]`` -> fp16 ``[..., N]``."""
    if awq_b200._ext is not None:                   # the same steps in C++ (awq_b200 docstring)
        return awq_b200._ext.forward(x, qweight, qzeros, scales, int(group_size))
    if not isinstance(x, torch.Tensor):
        raise TypeError("x must be a torch.Tensor")
    if x.dim() < 1:
        raise ValueError("x must have at least one dimension")
    in_shape = x.shape
    x_flat = x.reshape(-1, x.shape[-1])
    N = scales.shape[1]
    out = awq_b200.gemm(x_flat, qweight, qzeros, scales, group_size)
    return out.view(*in_shape[:-1], N)


def awq_gemm_bias_forward(x: torch.Tensor, qweight: torch.Tensor, qzeros: torch.Tensor,
                          scales: torch.Tensor, bias: torch.Tensor,
                          group_size: int = 128) -> torch.Tensor:
    """``awq_gemm_forward(x, ...) + bias`` in one kernel: the bias (fp16 [N]) is added in
    the product's epilogue.  For the reference's biased call sites, which add the bias
    after the product (``model/qwen2.py:45-46``, ``:108-109``).  Not in the reference
    module; the result differs from the two-step form only by its single fp16 rounding."""
    if awq_b200._ext is not None:
        return awq_b200._ext.forward_bias(x, qweight, qzeros, scales, bias, int(group_size))
    if not isinstance(x, torch.Tensor):
        raise TypeError("x must be a torch.Tensor")
    if x.dim() < 1:
        raise ValueError("x must have at least one dimension")
    in_shape = x.shape
    x_flat = x.reshape(-1, x.shape[-1])
    N = scales.shape[1]
    out = awq_b200.gemm(x_flat, qweight, qzeros, scales, group_size, bias=bias)
    return out.view(*in_shape[:-1], N)


def awq_gemm_silu_mul_forward(x: torch.Tensor, qweight: torch.Tensor, qzeros: torch.Tensor,
                              scales: torch.Tensor, group_size: int = 128) -> torch.Tensor:
    """``silu(P[..., :N/2]) * P[..., N/2:]`` for ``P = awq_gemm_forward(x, ...)`` with the
    fused gate+up weights (N = 2 * intermediate): the MLP activation of the reference
    (``model/qwen2.py:181-194``) in one call.  The decode, small-M and prefill kernels
    apply it in their epilogues where the shape allows (every Qwen2-7B gate+up call on one
    GPU), and P is then never written."""
    if awq_b200._ext is not None:
        return awq_b200._ext.forward_silu_mul(x, qweight, qzeros, scales, int(group_size))
    if not isinstance(x, torch.Tensor):
        raise TypeError("x must be a torch.Tensor")
    if x.dim() < 1:
        raise ValueError("x must have at least one dimension")
    in_shape = x.shape
    x_flat = x.reshape(-1, x.shape[-1])
    N = scales.shape[1]
    out = awq_b200.gemm_silu_mul(x_flat, qweight, qzeros, scales, group_size)
    return out.view(*in_shape[:-1], N // 2)
