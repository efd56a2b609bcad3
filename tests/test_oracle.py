"""CPU: the oracle (numpy and C restatements) pinned against the golden fixtures
generated from the reference's own code (tests/golden/make_golden.py)."""
from __future__ import annotations

import numpy as np
import pytest
from hypothesis import given, settings, strategies as st

from oracle import oracle as O


@pytest.fixture(scope="module", autouse=True)
def _build_c_oracle():
    import subprocess
    subprocess.run(["make", "-s", "-C", str(O._HERE)], check=True)


def _same_bits(a: np.ndarray, b: np.ndarray) -> bool:
    a16, b16 = a.view(np.uint16), b.view(np.uint16)
    nan = np.isnan(a.view(np.float16)) & np.isnan(b.view(np.float16))
    return bool(((a16 == b16) | nan).all())


def test_golden_cases_present(golden):
    assert {"kat_nibble_order", "kat_all_f_weights", "kat_all_zero_weights", "random_full_range",
            "ragged_k384_n136", "x3d_2x3", "m16_k512_n256", "group64",
            "extreme_scales"} <= set(golden)


def test_kat_nibble_order_by_hand(golden):
    # every word 0x76543210 holds nibble value j in slot j; element e sits in slot
    # [0,4,1,5,2,6,3,7][e] (kernels/awq_gemm.py:5-6,38), zeros 0, scales 1
    c = golden["kat_nibble_order"]
    w = c["w_bits"].view(np.float16)
    expect = np.tile(np.array([0, 4, 1, 5, 2, 6, 3, 7], np.float16), w.shape[1] // 8)
    assert np.array_equal(w, np.broadcast_to(expect, w.shape))


@pytest.mark.parametrize("impl", ["numpy", "c"])
def test_dequant_bit_exact_vs_reference(golden, impl):
    fn = O.awq_dequant if impl == "numpy" else O.c_awq_dequant
    for name, c in golden.items():
        w = fn(c["qweight"], c["qzeros"], c["scales"], c["group_size"])
        assert _same_bits(w, c["w_bits"].view(np.float16)), name


@pytest.mark.parametrize("impl", ["numpy", "c"])
def test_gemm_f32_vs_reference(golden, impl):
    fn = O.awq_gemm_f32 if impl == "numpy" else O.c_awq_gemm_f32
    for name, c in golden.items():
        if name == "extreme_scales":
            continue
        out = fn(c["x"], c["qweight"], c["qzeros"], c["scales"], c["group_size"])
        assert out.shape == c["out_ref_f32"].shape, name
        assert O.max_rel_err(out, c["out_ref_f32"]) < 1e-5, name


def test_reference_fp16_paths_agree_with_oracle(golden):
    # the reference's own fp16 outputs (torch_awq_gemm and the interpreted Triton
    # kernels) sit within the parity tolerance of the fp32 oracle
    for name, c in golden.items():
        if name == "extreme_scales":
            continue
        ref = O.awq_gemm_f32(c["x"], c["qweight"], c["qzeros"], c["scales"], c["group_size"])
        assert O.max_rel_err(c["out_ref_fp16"], ref) < 1e-2, name
        if "out_ref_triton" in c:
            assert O.max_rel_err(c["out_ref_triton"], ref) < 1e-2, name


def test_pack_unpack_round_trip():
    rng = np.random.default_rng(7)
    v = rng.integers(0, 16, size=(33, 64), dtype=np.uint8)
    assert np.array_equal(O.awq_unpack(O.awq_pack(v)), v)
    words = rng.integers(-2**31, 2**31, size=(5, 9), dtype=np.int64).astype(np.int32)
    assert np.array_equal(O.awq_pack(O.awq_unpack(words)), words)


def test_float_to_half_matches_numpy():
    rng = np.random.default_rng(3)
    f = np.concatenate([
        rng.standard_normal(200000).astype(np.float32) * np.float32(1e-5),
        rng.standard_normal(200000).astype(np.float32) * np.float32(3e4),
        np.array([0.0, -0.0, np.inf, -np.inf, 65504, 65519.99, 65520, 2**-25, 2**-24 * 1.5,
                  2**-14, 2**-14 * (1 - 2**-11)], np.float32)])
    with np.errstate(over="ignore"):
        expect = f.astype(np.float16)
    assert np.array_equal(O.c_float_to_half(f).view(np.uint16), expect.view(np.uint16))


def test_oracle_rejects_bad_shapes():
    qw, qz, s = O.make_awq_layer(256, 64)
    with pytest.raises(ValueError):
        O.awq_dequant(qw, qz, s, group_size=96)
    with pytest.raises(ValueError):
        O.awq_dequant(qw, qz, s[:, :32], group_size=128)


def test_silu_mul_f16_bit_exact_vs_reference(silu_golden):
    # the reference's _silu_mul_kernel (kernels/silu_mul.py:17-38), interpreted on the CPU,
    # over N(0, 3), saturating, overflowing, signed-zero and subnormal inputs
    c = silu_golden["elementwise"]
    out = O.silu_mul_f16(c["g"], c["u"])
    assert _same_bits(out, c["out_bits"].view(np.float16))


def test_silu_mlp_sequence_vs_oracle(silu_golden):
    # the reference MLP's fp16 sequence (product, halves, silu_mul) against the fp32 oracle
    names = [n for n in silu_golden if n.startswith("mlp_")]
    assert len(names) == 2
    for name in names:
        c = silu_golden[name]
        ref = c["out_bits"].view(np.float16).astype(np.float32)
        out = O.awq_silu_mul_f32(c["x"], c["qweight"], c["qzeros"], c["scales"], int(c["group_size"]))
        assert out.shape == ref.shape, name
        assert O.max_rel_err(out, ref) <= 1e-2, name


def _scalar_dequant(qweight, qzeros, scales, group_size, k, n):
    """W[k, n] by the reference's formula, one element at a time in pure Python
    (kernels/awq_gemm.py:36-59): nibble at shift 4 * [0,4,1,5,2,6,3,7][n % 8] of the
    packed words, (fp16(w) - fp16(z)) * scale with one fp16 rounding per operation."""
    shift = 4 * [0, 4, 1, 5, 2, 6, 3, 7][n % 8]
    w = (int(qweight[k, n // 8]) >> shift) & 0xF
    z = (int(qzeros[k // group_size, n // 8]) >> shift) & 0xF
    d = np.float16(np.float16(w) - np.float16(z))
    with np.errstate(over="ignore"):
        return np.float16(d * scales[k // group_size, n])



@settings(max_examples=40, deadline=None)
@given(groups=st.integers(1, 4), gs=st.sampled_from([32, 64, 128]), words=st.integers(1, 6),
       seed=st.integers(0, 2**32 - 1))
def test_three_restatements_agree(groups, gs, words, seed):
    """numpy, C and a scalar pure-Python restatement give the same bits on random shapes,
    full-range packed words and fp16 scales of every magnitude and sign."""
    K, N = groups * gs, 8 * words
    rng = np.random.default_rng(seed)
    qw = rng.integers(-2**31, 2**31, size=(K, N // 8), dtype=np.int64).astype(np.int32)
    qz = rng.integers(-2**31, 2**31, size=(groups, N // 8), dtype=np.int64).astype(np.int32)
    bits = rng.integers(0, 0x7C00, size=(groups, N), dtype=np.int64).astype(np.uint16)
    sign = (rng.integers(0, 2, size=(groups, N)).astype(np.uint16) << 15).astype(np.uint16)
    s = (bits | sign).view(np.float16)
    a = O.awq_dequant(qw, qz, s, gs)
    assert _same_bits(a, O.c_awq_dequant(qw, qz, s, gs))
    for k, n in zip(rng.integers(0, K, 16), rng.integers(0, N, 16)):
        assert _same_bits(np.array([a[k, n]]), np.array([_scalar_dequant(qw, qz, s, gs, k, n)]))
