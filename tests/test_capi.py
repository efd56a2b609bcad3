"""CPU: the C-ABI library loads, exports what include/awq_b200.h declares, and the
host-side checks reject bad input before any device work."""
from __future__ import annotations

import re

import pytest
import torch

from conftest import REPO


def _declared_symbols():
    text = (REPO / "include" / "awq_b200.h").read_text()
    return set(re.findall(r"AWQ_API\s+[\w\s\*]+?\b(awq_\w+)\s*\(", text))


def test_header_declares_expected_api():
    syms = _declared_symbols()
    assert {"awq_dequant_f16", "awq_gemm_f16", "awq_gemm_f16_ex", "awq_gemm_workspace_bytes",
            "awq_workspace_init", "awq_last_error", "awq_device_status", "awq_version",
            "awq_tc_supported"} <= syms


def test_library_exports_every_declared_symbol():
    import awq_b200._lib as L
    lib = L.load()
    for name in _declared_symbols():
        assert hasattr(lib, name), name
    # the binding's signature table covers the whole header
    assert _declared_symbols() <= set(L.SIGNATURES)
    assert lib.awq_version() >= 100


def test_library_is_the_in_tree_build():
    import awq_b200
    assert awq_b200.LIB_PATH.resolve().is_relative_to((REPO / "qwen2-7b-triton_engine_b200").resolve())


def test_invalid_arguments_rejected_without_a_device():
    import awq_b200._lib as L
    lib = L.load()
    # null weights: rejected by validation, before any CUDA call
    rc = lib.awq_gemm_f16(None, 256, None, None, None, None, 64, 1, 64, 256, 128, None, 0, None)
    assert rc == L.AWQ_ERR_INVALID_ARG
    assert b"null" in lib.awq_last_error()
    rc = lib.awq_dequant_f16(16, 16, 16, 16, 256, 60, 128, None)       # N % 8 != 0
    assert rc == L.AWQ_ERR_INVALID_ARG
    rc = lib.awq_dequant_f16(16, 16, 16, 16, 200, 64, 128, None)       # K % gs != 0
    assert rc == L.AWQ_ERR_INVALID_ARG
    rc = lib.awq_dequant_f16(16, 16, 18, 16, 256, 64, 128, None)       # misaligned scales
    assert rc == L.AWQ_ERR_INVALID_ARG


def _layer(K=256, N=64, gs=128, device="cpu"):
    qw = torch.zeros((K, N // 8), dtype=torch.int32, device=device)
    qz = torch.zeros((K // gs, N // 8), dtype=torch.int32, device=device)
    s = torch.ones((K // gs, N), dtype=torch.float16, device=device)
    return qw, qz, s


def test_dropin_refuses_cpu_tensors():
    from kernels import awq_gemm
    qw, qz, s = _layer()
    with pytest.raises(ValueError, match="CUDA only"):
        awq_gemm.awq_gemm_forward(torch.zeros(1, 256, dtype=torch.float16), qw, qz, s)
    with pytest.raises(ValueError, match="CUDA only"):
        awq_gemm._dequant_to_fp16(qw, qz, s, torch.empty(256, 64, dtype=torch.float16))


def test_dropin_signature_matches_reference():
    import inspect
    from kernels import awq_gemm
    sig = inspect.signature(awq_gemm.awq_gemm_forward)
    assert list(sig.parameters) == ["x", "qweight", "qzeros", "scales", "group_size"]
    assert sig.parameters["group_size"].default == 128
    sig = inspect.signature(awq_gemm._dequant_to_fp16)
    assert list(sig.parameters) == ["qweight", "qzeros", "scales", "out_buf", "group_size"]


def test_weight_checks():
    import awq_b200
    qw, qz, s = _layer()
    # shape checks run before the device check only for CUDA tensors; on CPU the
    # device error comes first and is the one a caller sees
    with pytest.raises(ValueError):
        awq_b200.check_weights(qw, qz, s, 128)


def test_new_entry_points_reject_bad_input_without_a_device():
    import awq_b200._lib as L
    lib = L.load()
    # gate+up with SiLU-mul: null weights, then a null workspace, before any CUDA call
    rc = lib.awq_gemm_f16_silu_mul(16, 256, None, None, None, 16, 32, 1, 64, 256, 128, 16, 1 << 20,
                                   None)
    assert rc == L.AWQ_ERR_INVALID_ARG
    rc = lib.awq_gemm_f16_silu_mul(16, 256, 16, 16, 16, 16, 32, 1, 64, 256, 128, None, 0, None)
    assert rc == L.AWQ_ERR_INVALID_ARG
    assert b"workspace" in lib.awq_last_error()
    rc = lib.awq_gemm_f16_silu_mul(16, 256, 16, 16, 16, 16, 16, 1, 64, 256, 128, 16, 1 << 20,
                                   None)                                  # ldo < N / 2
    assert rc == L.AWQ_ERR_INVALID_ARG
    # explicit small-M path: an unknown path number is refused before the device is touched
    rc = lib.awq_gemm_f16_ex(16, 256, 16, 16, 16, 16, 64, 1, 64, 256, 128, None, 0, None, 7)
    assert rc == L.AWQ_ERR_INVALID_ARG
    assert L.AWQ_PATH_TS == 3


def test_silu_dropin_refuses_cpu_tensors_and_keeps_signature():
    import inspect
    from kernels import awq_gemm
    sig = inspect.signature(awq_gemm.awq_gemm_silu_mul_forward)
    assert list(sig.parameters) == ["x", "qweight", "qzeros", "scales", "group_size"]
    qw, qz, s = _layer(N=512)
    with pytest.raises(ValueError, match="CUDA only"):
        awq_gemm.awq_gemm_silu_mul_forward(torch.zeros(1, 256, dtype=torch.float16), qw, qz, s)


def test_header_is_c_and_links_from_a_c_host(tmp_path):
    """The boundary is plain C: a C99 program includes include/awq_b200.h, links the
    in-tree libawq_b200.so and calls entry points that need no device (version, error
    string, argument checks), as a non-Python host would."""
    import shutil
    import subprocess

    import awq_b200
    cc = shutil.which("gcc") or shutil.which("cc")
    if cc is None:
        pytest.skip("no C compiler")
    src = tmp_path / "host.c"
    src.write_text(r"""
#include <stdio.h>
#include "awq_b200.h"
int main(void) {
  int v = awq_version();
  int rc = awq_gemm_f16(0, 256, 0, 0, 0, 0, 64, 1, 64, 256, 128, 0, 0, 0);
  const char* e = awq_last_error();
  int rc2 = awq_gemm_f16_silu_mul(0, 256, 0, 0, 0, 0, 32, 1, 64, 256, 128, 0, 0, 0);
  printf("%d %d %d %s\n", v, rc == AWQ_ERR_INVALID_ARG, rc2 == AWQ_ERR_INVALID_ARG, e ? "msg" : "none");
  return 0;
}
""")
    exe = tmp_path / "host"
    lib = awq_b200.LIB_PATH
    subprocess.run([cc, "-std=c99", "-Wall", "-Werror", "-I", str(REPO / "include"), str(src),
                    "-o", str(exe), "-L", str(lib.parent), "-lawq_b200",
                    f"-Wl,-rpath,{lib.parent}"], check=True)
    out = subprocess.run([str(exe)], check=True, capture_output=True, text=True).stdout.split()
    assert int(out[0]) >= 100 and out[1:] == ["1", "1", "msg"]


@pytest.mark.parametrize("K,N,gs,why", [
    (0, 64, 128, b"positive"),            # empty K
    (256, 0, 128, b"positive"),           # empty N
    (256, 60, 128, b"multiple of 8"),     # N not whole packed words
    (256, 64, 0, b"group_size"),          # no groups
    (256, 64, 12, b"group_size"),         # group not a multiple of 8
    (200, 64, 128, b"multiple of group_size"),
    ((1 << 30) + 128, 64, 128, b"2^30"),  # sizes above the library's index range
])
def test_weight_shape_checks_without_a_device(K, N, gs, why):
    import awq_b200._lib as L
    lib = L.load()
    for rc in (lib.awq_gemm_f16(16, K, 16, 16, 16, 16, N, 1, N, K, gs, None, 0, None),
               lib.awq_dequant_f16(16, 16, 16, 16, K, N, gs, None)):
        assert rc == L.AWQ_ERR_INVALID_ARG
        assert why in lib.awq_last_error()


def test_activation_and_output_checks_without_a_device():
    import awq_b200._lib as L
    lib = L.load()
    ok = (16, 16, 16)                                            # aligned weight pointers
    cases = [
        ((16, 256, *ok, 16, 64, 0, 64, 256, 128), b"M="),        # M = 0
        ((16, 255, *ok, 16, 64, 1, 64, 256, 128), b"ldx"),       # ldx < K
        ((16, 256, *ok, 16, 63, 1, 64, 256, 128), b"ldx"),       # ldo < N
        ((17, 256, *ok, 16, 64, 1, 64, 256, 128), b"aligned"),   # odd x address
        ((16, 256, *ok, None, 64, 1, 64, 256, 128), b"null"),    # no output
    ]
    for args, why in cases:
        assert lib.awq_gemm_f16(*args, None, 0, None) == L.AWQ_ERR_INVALID_ARG, why
        assert why in lib.awq_last_error(), (why, lib.awq_last_error())
    # a bias pointer is required by the biased entry point
    assert lib.awq_gemm_f16_bias(16, 256, *ok, None, 16, 64, 1, 64, 256, 128, None, 0, None) == \
        L.AWQ_ERR_INVALID_ARG
    assert b"bias" in lib.awq_last_error()


def test_communicator_create_rejects_bad_arguments_without_a_device():
    """awq_tp_comm_create_ex validates world, rank, max_n and max_rows before it touches
    CUDA: a bad request fails with AWQ_ERR_INVALID_ARG and leaves no communicator."""
    import ctypes
    import awq_b200._lib as L
    lib = L.load()
    h = ctypes.create_string_buffer(L.AWQ_IPC_HANDLE_BYTES)
    for world, rank, max_n, max_rows in [(0, 0, 256, 0), (9, 0, 256, 0), (2, 2, 256, 0),
                                         (2, 0, 100, 0), (2, 0, 256, -1),
                                         (2, 0, 1 << 16, 1 << 17)]:
        ptr = ctypes.c_void_p(1)
        rc = lib.awq_tp_comm_create_ex(world, rank, max_n, max_rows, h, ctypes.byref(ptr))
        assert rc == L.AWQ_ERR_INVALID_ARG, (world, rank, max_n, max_rows)
        assert ptr.value is None
    assert lib.awq_tp_comm_create_ex(2, 0, 256, 0, None, None) == L.AWQ_ERR_INVALID_ARG
