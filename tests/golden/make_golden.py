"""Generate the golden AWQ fixtures in this folder from the reference's own code.

Run in a container that has the reference checkout (it is not needed on the GPU
box; the tests only read the committed ``awq_golden.npz``):

    python tests/golden/make_golden.py --reference /path/to/Qwen2-7B-Triton_Engine

For every case it runs three implementations that ship with the reference and
requires them to agree bit-for-bit on the dequantized weights:

* ``kernels/awq_gemm.py::_dequant_to_fp16`` (the Triton kernel, lines 14-87),
  executed on the CPU by Triton's interpreter (``TRITON_INTERPRET=1``);
* ``test/compare_benchmark.py::torch_awq_gemm`` (lines 72-95), applied to an
  identity activation so that its output is the dequantized matrix itself;
* ``inference/baseline_kernels.py::awq_gemm_forward`` (lines 36-60), same trick.

It stores the inputs, the dequantized weights (as raw fp16 bits), the
reference's fp16 output ``torch_awq_gemm(x, ...)``, the fp32 output
``x.float() @ W.float()``, and -- where the interpreter can run them -- the
outputs of the reference's Triton GEMM paths (the M<=4 dequant + matmul branch of
``awq_gemm_forward`` and the fused ``_awq_gemm_kernel``).

The reference ships ``__pycache__`` bytecode; this script sets
``sys.pycache_prefix`` so Python compiles the reference's sources itself and
never reads those files.
"""
from __future__ import annotations

import argparse
import ast
import os
import pathlib
import sys
import tempfile

os.environ["TRITON_INTERPRET"] = "1"          # must precede the first triton import
sys.pycache_prefix = tempfile.mkdtemp(prefix="ref_pycache_")

import numpy as np  # noqa: E402
import torch  # noqa: E402

HERE = pathlib.Path(__file__).resolve().parent
REPO = HERE.parent.parent
sys.path.insert(0, str(REPO))
from oracle import oracle as O  # noqa: E402


def _load_function(path: pathlib.Path, name: str, env: dict):
    """Exec one top-level function definition from a reference source file."""
    tree = ast.parse(path.read_text(), filename=str(path))
    for node in tree.body:
        if isinstance(node, ast.FunctionDef) and node.name == name:
            mod = ast.Module(body=[node], type_ignores=[])
            code = compile(mod, str(path), "exec")
            exec(code, env)
            return env[name]
    raise KeyError(f"{name} not found in {path}")


def _cases():
    """(name, M-shape, K, N, group_size, qweight, qzeros, scales, x) tuples."""
    rng = np.random.default_rng(20261201)
    out = []

    def rnd_words(shape):
        return rng.integers(-2**31, 2**31, size=shape, dtype=np.int64).astype(np.int32)

    def x_of(shape):
        return rng.standard_normal(shape).astype(np.float16)

    # 1. hand-checkable nibble pattern: every word 0x76543210 -> elements 0,4,1,5,2,6,3,7
    K, N, gs = 256, 64, 128
    qw = np.full((K, N // 8), 0x76543210, dtype=np.int32)
    qz = np.zeros((K // gs, N // 8), dtype=np.int32)
    s = np.ones((K // gs, N), dtype=np.float16)
    out.append(("kat_nibble_order", (3,), K, N, gs, qw, qz, s, x_of((3, K))))
    # 2. same words used as zeros, weights all 0xF, scale 0.5
    qw = np.full((K, N // 8), -1, dtype=np.int32)
    qz = np.full((K // gs, N // 8), 0x76543210, dtype=np.int32)
    s = np.full((K // gs, N), 0.5, dtype=np.float16)
    out.append(("kat_all_f_weights", (2,), K, N, gs, qw, qz, s, x_of((2, K))))
    # 3. all-zero weights, all-0xF zeros -> W = -15 * s
    qw = np.zeros((K, N // 8), dtype=np.int32)
    qz = np.full((K // gs, N // 8), -1, dtype=np.int32)
    s = rng.uniform(0.002, 0.02, size=(K // gs, N)).astype(np.float16)
    out.append(("kat_all_zero_weights", (1,), K, N, gs, qw, qz, s, x_of((1, K))))
    # 4. full-range random words (negative int32 included), benchmark-style scales
    K, N = 256, 128
    qw, qz = rnd_words((K, N // 8)), rnd_words((K // gs, N // 8))
    s = rng.uniform(0.002, 0.02, size=(K // gs, N)).astype(np.float16)
    out.append(("random_full_range", (3,), K, N, gs, qw, qz, s, x_of((3, K))))
    # 5. ragged: 3 groups, 17 packed columns (N = 136), M = 5
    K, N = 384, 136
    qw, qz = rnd_words((K, N // 8)), rnd_words((K // gs, N // 8))
    s = rng.uniform(0.002, 0.02, size=(K // gs, N)).astype(np.float16)
    out.append(("ragged_k384_n136", (5,), K, N, gs, qw, qz, s, x_of((5, K))))
    # 6. 3-D activation [2, 3, K]
    K, N = 256, 64
    qw, qz = rnd_words((K, N // 8)), rnd_words((K // gs, N // 8))
    s = rng.uniform(0.002, 0.02, size=(K // gs, N)).astype(np.float16)
    out.append(("x3d_2x3", (2, 3), K, N, gs, qw, qz, s, x_of((2, 3, K))))
    # 7. decode-width activation at M = 16
    K, N = 512, 256
    qw, qz = rnd_words((K, N // 8)), rnd_words((K // gs, N // 8))
    s = rng.uniform(0.002, 0.02, size=(K // gs, N)).astype(np.float16)
    out.append(("m16_k512_n256", (16,), K, N, gs, qw, qz, s, x_of((16, K))))
    # 8. group size 64
    K, N, gs64 = 256, 64, 64
    qw, qz = rnd_words((K, N // 8)), rnd_words((K // gs64, N // 8))
    s = rng.uniform(0.002, 0.02, size=(K // gs64, N)).astype(np.float16)
    out.append(("group64", (4,), K, N, gs64, qw, qz, s, x_of((4, K))))
    # 9. extreme scales: fp16 subnormals, large values whose products overflow to inf,
    #    negative scales.  Used for the dequant bit-exactness test only.
    K, N = 256, 64
    qw, qz = rnd_words((K, N // 8)), rnd_words((K // gs, N // 8))
    bits = rng.integers(0, 0x7C00, size=(K // gs, N), dtype=np.int64).astype(np.uint16)
    sign = (rng.integers(0, 2, size=(K // gs, N)).astype(np.uint16) << 15).astype(np.uint16)
    s = (bits | sign).view(np.float16)
    out.append(("extreme_scales", (1,), K, N, gs, qw, qz, s, x_of((1, K))))
    return out


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", default=os.environ.get("AWQ_REFERENCE", ""),
                    help="path of the reference checkout")
    ap.add_argument("--out", default=str(HERE / "awq_golden.npz"))
    args = ap.parse_args()
    ref = pathlib.Path(args.reference)
    if not (ref / "kernels" / "awq_gemm.py").exists():
        sys.exit(f"reference not found at {ref!r}")

    sys.path.insert(0, str(ref))
    import kernels.awq_gemm as ref_awq           # Triton module, interpreted on CPU
    torch_awq_gemm = _load_function(ref / "test" / "compare_benchmark.py", "torch_awq_gemm",
                                    {"torch": torch})
    baseline_awq = _load_function(ref / "inference" / "baseline_kernels.py", "awq_gemm_forward",
                                  {"torch": torch})

    store = {}
    names = []
    for (name, mshape, K, N, gs, qw, qz, s, x) in _cases():
        tqw, tqz, ts = torch.from_numpy(qw), torch.from_numpy(qz), torch.from_numpy(s)
        eye = torch.eye(K, dtype=torch.float16)
        # (a) Triton dequant kernel, interpreted
        w_tri = torch.empty((K, N), dtype=torch.float16)
        ref_awq._dequant_to_fp16(tqw, tqz, ts, w_tri, gs)
        # (b) vectorised torch path on the identity
        w_cmp = torch_awq_gemm(eye, tqw, tqz, ts, gs)
        # (c) per-column torch loop on the identity
        w_base = baseline_awq(eye, tqw, tqz, ts, gs)
        wb = [w.numpy().view(np.uint16) for w in (w_tri, w_cmp, w_base)]
        # The identity trick reads a column of W through a matmul, so a column that
        # holds an inf comes back as NaN (0 * inf) and -0.0 comes back as +0.0 (the
        # sum starts at +0).  Compare the torch paths by value on the all-finite
        # columns; the Triton kernel output is compared bit for bit everywhere.
        col_ok = np.isfinite(w_tri.numpy()).all(axis=0)
        for other in (w_cmp.numpy(), w_base.numpy()):
            if not np.array_equal(w_tri.numpy()[:, col_ok], other[:, col_ok]):
                sys.exit(f"{name}: reference dequant paths disagree")
        w_or = O.awq_dequant(qw, qz, s, gs)
        same = (w_or.view(np.uint16) == wb[0]) | (np.isnan(w_or) & np.isnan(w_tri.numpy()))
        if not same.all():
            sys.exit(f"{name}: numpy oracle disagrees with the reference dequant")

        tx = torch.from_numpy(x)
        out16 = torch_awq_gemm(tx, tqw, tqz, ts, gs).numpy()
        out32 = (tx.reshape(-1, K).float() @ w_tri.float()).reshape(*mshape, N).numpy()
        M = int(np.prod(mshape))
        tri = None
        if name != "extreme_scales":
            if M <= 4:
                tri = ref_awq.awq_gemm_forward(tx, tqw, tqz, ts, gs).numpy()
            else:
                x2 = tx.reshape(-1, K).contiguous()
                o = torch.empty((M, N), dtype=torch.float16)
                BM, BN, BK = 16, 32, 32
                grid = (((M + BM - 1) // BM) * ((N + BN - 1) // BN),)
                ref_awq._awq_gemm_kernel.fn[grid](
                    x2, tqw, tqz, ts, o, M, N, K,
                    x2.stride(0), x2.stride(1), tqw.stride(0), tqw.stride(1),
                    tqz.stride(0), tqz.stride(1), ts.stride(0), ts.stride(1),
                    o.stride(0), o.stride(1), group_size=gs,
                    BLOCK_SIZE_M=BM, BLOCK_SIZE_N=BN, BLOCK_SIZE_K=BK, GROUP_SIZE_M=8)
                tri = o.reshape(*mshape, N).numpy()
        p = name + "/"
        store[p + "x"] = x
        store[p + "qweight"] = qw
        store[p + "qzeros"] = qz
        store[p + "scales"] = s
        store[p + "group_size"] = np.array(gs)
        store[p + "w_bits"] = wb[0]
        store[p + "out_ref_fp16"] = out16
        store[p + "out_ref_f32"] = out32
        if tri is not None:
            store[p + "out_ref_triton"] = tri
        names.append(name)
        print(f"{name}: K={K} N={N} gs={gs} x{tuple(x.shape)} ok")
    store["cases"] = np.array(names)
    np.savez_compressed(args.out, **store)
    print("wrote", args.out)


if __name__ == "__main__":
    main()
