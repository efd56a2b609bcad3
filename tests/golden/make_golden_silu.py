"""Generate the SiLU-mul golden fixture in this folder from the reference's own code.

Run in a container that has the reference checkout (the tests only read the committed
``silu_golden.npz``):

    python tests/golden/make_golden_silu.py --reference /path/to/Qwen2-7B-Triton_Engine

* ``elementwise``: ``kernels/silu_mul.py::_silu_mul_kernel`` (lines 17-38; wrapper
  ``silu_mul_forward`` lines 41-64), executed on the CPU by Triton's interpreter
  (``TRITON_INTERPRET=1``, through the autotuner's JIT function with BLOCK_SIZE=1024), on
  fp16 gate / up vectors that cover N(0, 3) values, large magnitudes (sigmoid saturating
  at 0 and 1), signed zeros, fp16 subnormals and products that overflow fp16.
* ``mlp_*``: the reference MLP's sequence (``model/qwen2.py:181-194``) on an AWQ gate+up
  product: ``test/compare_benchmark.py::torch_awq_gemm`` (lines 72-95, fp16 product),
  the two ``.contiguous()`` halves, then the same interpreted kernel.

The reference ships ``__pycache__`` bytecode; ``sys.pycache_prefix`` makes Python compile
the reference's sources itself and never read those files.
"""
from __future__ import annotations

import argparse
import importlib.util
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
sys.path.insert(0, str(HERE))
from oracle import oracle as O  # noqa: E402
from make_golden import _load_function  # noqa: E402


def _ref_silu_mul(kernel, g: torch.Tensor, u: torch.Tensor) -> torch.Tensor:
    out = torch.empty_like(g)
    n = g.numel()
    kernel.fn[((n + 1023) // 1024,)](g, u, out, n, BLOCK_SIZE=1024)
    return out


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", default=os.environ.get("AWQ_REFERENCE", ""),
                    help="path of the reference checkout")
    ap.add_argument("--out", default=str(HERE / "silu_golden.npz"))
    args = ap.parse_args()
    ref = pathlib.Path(args.reference)
    if not (ref / "kernels" / "silu_mul.py").exists():
        sys.exit(f"reference not found at {ref!r}")
    spec = importlib.util.spec_from_file_location("ref_silu_mul", ref / "kernels" / "silu_mul.py")
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    kernel = mod._silu_mul_kernel
    torch_awq_gemm = _load_function(ref / "test" / "compare_benchmark.py", "torch_awq_gemm",
                                    {"torch": torch})
    rng = np.random.default_rng(20261202)
    store = {}

    # elementwise
    parts = [rng.normal(0, 3, 4096)]
    parts.append(np.array([0.0, -0.0, 1e-7, -1e-7, 6e-8, -6e-8, 11.0, -11.0, 17.0, -17.0,
                           65504.0, -65504.0, 300.0, -300.0, 1.0, -1.0, 88.0, -88.0]))
    parts.append(rng.uniform(-20, 20, 2048))
    g = np.concatenate(parts).astype(np.float16)
    u = np.concatenate([rng.normal(0, 3, 4096),
                        np.array([1.0, 1.0, 1.0, 1.0, 65504.0, -65504.0, 2.0, 2.0, 1e4, 1e4,
                                  2.0, 2.0, 300.0, 300.0, 0.0, -0.0, 1.0, 1.0]),
                        rng.uniform(-20, 20, 2048)]).astype(np.float16)
    out = _ref_silu_mul(kernel, torch.from_numpy(g), torch.from_numpy(u)).numpy()
    store["elementwise/g"] = g
    store["elementwise/u"] = u
    store["elementwise/out_bits"] = out.view(np.uint16)
    mine = O.silu_mul_f16(g, u)
    print(f"elementwise: {np.count_nonzero(mine.view(np.uint16) != out.view(np.uint16))} "
          f"of {g.size} differ from the oracle's silu_mul_f16")

    # the MLP sequence on AWQ products
    for name, M, K, inter, gs in (("mlp_k256_i256_m3", 3, 256, 256, 128),
                                  ("mlp_k384_i320_m12", 12, 384, 320, 128)):
        N = 2 * inter
        qw = rng.integers(-2**31, 2**31, size=(K, N // 8), dtype=np.int64).astype(np.int32)
        qz = rng.integers(-2**31, 2**31, size=(K // gs, N // 8), dtype=np.int64).astype(np.int32)
        s = rng.uniform(0.002, 0.02, size=(K // gs, N)).astype(np.float16)
        x = rng.standard_normal((M, K)).astype(np.float16)
        gu = torch_awq_gemm(torch.from_numpy(x), torch.from_numpy(qw), torch.from_numpy(qz),
                            torch.from_numpy(s), gs)
        gate, up = gu[..., :inter].contiguous(), gu[..., inter:].contiguous()
        h = _ref_silu_mul(kernel, gate, up).numpy()
        for k, v in (("x", x), ("qweight", qw), ("qzeros", qz), ("scales", s),
                     ("group_size", np.array(gs)), ("out_bits", h.view(np.uint16))):
            store[f"{name}/{k}"] = v
        err = O.max_rel_err(h.astype(np.float32), O.awq_silu_mul_f32(x, qw, qz, s, gs))
        print(f"{name}: reference sequence vs fp32 oracle max rel err {err:.2e}")
    np.savez_compressed(args.out, **store)
    print("wrote", args.out)


if __name__ == "__main__":
    main()
