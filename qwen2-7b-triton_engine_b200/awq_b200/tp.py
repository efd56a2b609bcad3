"""Single-box tensor parallelism for the AWQ linears (one process per GPU, NCCL).

The reference runs on one GPU and has no parallelism (inference/engine.py:15,
model/config.py:24).  This module adds the standard Megatron split on top of the
AWQ drop-in, in the packed layout the reference registers (model/qwen2.py:34-36):

* column parallel (q/k/v, gate, up): rank r keeps output columns [n0, n1) -- whole
  packed words, so qweight[:, n0/8:n1/8], qzeros[:, n0/8:n1/8], scales[:, n0:n1].
  No communication.  For the fused gate+up matrix (model/qwen2.py:176-178) gate and
  up are sliced with the same bounds, so SiLU(gate) * up stays local to the rank.
* row parallel (o, down): rank r keeps K rows [k0, k1) in whole quantization groups
  (qweight[k0:k1], qzeros/scales[k0/gs:k1/gs]); groups are dealt out as evenly as
  possible (Qwen2-7B down has 148 groups: 19/18 at 8 ranks).  Each rank's product is
  a partial sum and one all-reduce (sum) of the fp16 [M, N] output finishes it.

* attention by whole heads (``AttentionLinearsTP``): the fused q/k/v columns of the
  rank's query heads and of the key/value heads they read under grouped-query attention
  (model/qwen2.py:131-138), and o's rows of the same query heads, so attention itself
  runs per rank with no exchange until o's all-reduce.

The product runs through ``kernels.awq_gemm.awq_gemm_forward`` (the sm_100a
library); ``gemm=`` lets host-logic tests substitute a CPU function under ``gloo``.
"""
from __future__ import annotations

from dataclasses import dataclass
from typing import Callable, Optional

import torch
import torch.distributed as dist
import torch.nn.functional as F

GemmFn = Callable[[torch.Tensor, torch.Tensor, torch.Tensor, torch.Tensor, int], torch.Tensor]


def _default_gemm() -> GemmFn:
    from kernels.awq_gemm import awq_gemm_forward
    return awq_gemm_forward


def _default_gemm_bias():
    """The library product with the bias added in its epilogue (one kernel)."""
    from kernels.awq_gemm import awq_gemm_bias_forward
    return awq_gemm_bias_forward


def _default_silu_mul():
    """The library's gate+up product with silu(gate) * up in the same call."""
    from kernels.awq_gemm import awq_gemm_silu_mul_forward
    return awq_gemm_silu_mul_forward


def even_split(total: int, parts: int, rank: int) -> tuple[int, int]:
    """[lo, hi) of `rank` when `total` units are dealt as evenly as possible."""
    base, extra = divmod(total, parts)
    lo = rank * base + min(rank, extra)
    return lo, lo + base + (1 if rank < extra else 0)


def column_bounds(N: int, world: int, rank: int) -> tuple[int, int]:
    """Column shard [n0, n1) in whole packed words (multiples of 8 columns)."""
    if N % 8:
        raise ValueError(f"N={N} is not a multiple of 8")
    w0, w1 = even_split(N // 8, world, rank)
    return w0 * 8, w1 * 8


def row_bounds(K: int, group_size: int, world: int, rank: int) -> tuple[int, int]:
    """Row shard [k0, k1) in whole quantization groups."""
    if K % group_size:
        raise ValueError(f"K={K} is not a multiple of group_size={group_size}")
    g0, g1 = even_split(K // group_size, world, rank)
    return g0 * group_size, g1 * group_size


def shard_columns(qweight, qzeros, scales, n0: int, n1: int):
    return (qweight[:, n0 // 8:n1 // 8].contiguous(), qzeros[:, n0 // 8:n1 // 8].contiguous(),
            scales[:, n0:n1].contiguous())


def shard_rows(qweight, qzeros, scales, k0: int, k1: int, group_size: int):
    return (qweight[k0:k1].contiguous(), qzeros[k0 // group_size:k1 // group_size].contiguous(),
            scales[k0 // group_size:k1 // group_size].contiguous())


def shard_fused_columns(qweight, qzeros, scales, parts: list[int], world: int, rank: int,
                        bounds: Optional[Callable[[int, int, int], tuple[int, int]]] = None):
    """Column shard of a matrix that concatenates several projections along N
    (fused gate+up, fused q/k/v): each part is split on its own and the rank's
    slices are concatenated again, so part boundaries survive sharding.
    `bounds(width, world, rank)` gives a part's [lo, hi); default: whole words."""
    bounds = bounds or column_bounds
    out_qw, out_qz, out_s, off = [], [], [], 0
    for width in parts:
        a, b = bounds(width, world, rank)
        qw, qz, s = shard_columns(qweight, qzeros, scales, off + a, off + b)
        out_qw.append(qw), out_qz.append(qz), out_s.append(s)
        off += width
    if off != scales.shape[1]:
        raise ValueError(f"parts {parts} do not add up to N={scales.shape[1]}")
    return torch.cat(out_qw, 1), torch.cat(out_qz, 1), torch.cat(out_s, 1)


@dataclass
class AWQWeights:
    qweight: torch.Tensor
    qzeros: torch.Tensor
    scales: torch.Tensor
    group_size: int = 128
    bias: Optional[torch.Tensor] = None


class ColumnParallelAWQ:
    """Rank's column slice of an AWQ linear (optionally a fused multi-part one)."""

    def __init__(self, full: AWQWeights, world: int, rank: int, parts: Optional[list[int]] = None,
                 gemm: Optional[GemmFn] = None, bounds=None):
        parts = parts or [full.scales.shape[1]]
        bounds = bounds or column_bounds
        self.parts_local = [bounds(p, world, rank)[1] - bounds(p, world, rank)[0] for p in parts]
        qw, qz, s = shard_fused_columns(full.qweight, full.qzeros, full.scales, parts, world, rank,
                                        bounds)
        bias = None
        if full.bias is not None:
            pieces, off = [], 0
            for p in parts:
                a, b = bounds(p, world, rank)
                pieces.append(full.bias[off + a:off + b])
                off += p
            bias = torch.cat(pieces)
        self.w = AWQWeights(qw, qz, s, full.group_size, bias)
        self.gemm = gemm or _default_gemm()
        # the library's product fuses the bias; a substituted product adds it afterwards
        self.gemm_bias = _default_gemm_bias() if gemm is None else None

    def __call__(self, x: torch.Tensor) -> torch.Tensor:
        return _column_forward(self.w, self.gemm, self.gemm_bias, x)


def _column_forward(w: AWQWeights, gemm, gemm_bias, x: torch.Tensor) -> torch.Tensor:
    """x @ W (+ bias) for a column shard: the bias in the product's epilogue with the
    library, after the product with a substituted one (model/qwen2.py:45-46)."""
    N = w.scales.shape[1]
    if N == 0:                                        # more ranks than heads / columns
        return torch.zeros((*x.shape[:-1], 0), dtype=torch.float16, device=x.device)
    if w.bias is not None and gemm_bias is not None:
        return gemm_bias(x, w.qweight, w.qzeros, w.scales, w.bias, w.group_size)
    out = gemm(x, w.qweight, w.qzeros, w.scales, w.group_size)
    if w.bias is not None:
        out = out + w.bias
    return out


class RowParallelAWQ:
    """Rank's K-row slice of an AWQ linear; the partial outputs are all-reduced.

    With ``comm`` (an ``awq_b200.TPComm``) a call the fused kernel supports runs the
    product and the all-reduce in one kernel (``awq_b200.gemm_allreduce``: peer stores
    over NVLink, sum in rank order); other calls use the library product and an NCCL
    all-reduce.  The choice must be the same on every rank -- a rank in the fused kernel
    waits for the others' tiles while a rank in NCCL waits for the others' NCCL call --
    so it is made from quantities every rank knows alike: M, N, the group size and every
    rank's K (gathered once at construction).  A rank without rows makes every rank use
    NCCL.  ``check=True`` reads the device status after each fused call (a
    synchronisation) and raises on a time-out; otherwise call ``comm.check()`` where the
    caller synchronises anyway."""

    def __init__(self, full: AWQWeights, world: int, rank: int, group: Optional[object] = None,
                 gemm: Optional[GemmFn] = None, comm=None,
                 k_bounds: Optional[tuple[int, int]] = None, check: bool = False):
        K = full.qweight.shape[0]
        # default: whole quantization groups dealt evenly; k_bounds: the caller's split
        # (whole attention heads for o, see AttentionLinearsTP), group-aligned
        self.k0, self.k1 = k_bounds if k_bounds is not None else row_bounds(K, full.group_size,
                                                                            world, rank)
        if self.k0 % full.group_size or self.k1 % full.group_size or not 0 <= self.k0 <= self.k1 <= K:
            raise ValueError(f"row bounds [{self.k0}, {self.k1}) are not whole groups of {K}")
        qw, qz, s = shard_rows(full.qweight, full.qzeros, full.scales, self.k0, self.k1,
                               full.group_size)
        self.w = AWQWeights(qw, qz, s, full.group_size, full.bias if rank == 0 else None)
        self.bias = full.bias
        self.group = group
        self.world = world
        self.gemm = gemm or _default_gemm()
        self.comm = comm
        self.check = check
        self.k_all: Optional[list[int]] = None     # every rank's K, rank order
        if comm is not None and world > 1:
            ks = [None] * world
            dist.all_gather_object(ks, self.k1 - self.k0, group=group)
            self.k_all = [int(k) for k in ks]
        self._fused_ok: dict = {}

    def fused_for(self, M: int) -> bool:
        """Whether a call with M activation rows runs the library's all-reduce (the same
        answer on every rank: it depends on M, N, the group size, every rank's K and the
        communicator's capacity only).  Up to 16 tokens that is the fused decode kernel;
        above, the prefill product followed by the all-reduce kernel, up to the
        communicator's ``max_rows``; beyond that, the product and NCCL."""
        if self.comm is None or self.world < 2 or self.k_all is None:
            return False
        ok = self._fused_ok.get(M)
        if ok is None:
            N = self.w.scales.shape[1]
            ok = all(k > 0 and self.comm.supported_shape(M, N, k, self.w.group_size)
                     for k in self.k_all)
            self._fused_ok[M] = ok
        return ok

    def _fused(self, x_local: torch.Tensor) -> Optional[torch.Tensor]:
        import awq_b200
        M = 1
        for d in x_local.shape[:-1]:
            M *= int(d)
        if not self.fused_for(M):
            return None
        x2 = x_local.reshape(M, x_local.shape[-1])
        # the decision assumed a dense, 16-byte aligned x: make it so
        if x2.stride(1) != 1 or x2.data_ptr() % 16 or (x2.stride(0) * 2) % 16 \
                or x2.stride(0) != x2.shape[1]:
            x2 = x2.contiguous().clone()
        N = self.w.scales.shape[1]
        out = awq_b200.gemm_allreduce(x2, self.w.qweight, self.w.qzeros, self.w.scales,
                                      self.w.group_size, self.comm)
        if self.check:
            self.comm.check()
        out = out.view(*x_local.shape[:-1], N)
        return out + self.bias if self.bias is not None else out

    def __call__(self, x_local: torch.Tensor) -> torch.Tensor:
        """x_local holds this rank's K columns [k0, k1) of the activation."""
        fused = self._fused(x_local)
        if fused is not None:
            return fused
        if self.k1 > self.k0:
            out = self.gemm(x_local, self.w.qweight, self.w.qzeros, self.w.scales,
                            self.w.group_size)
        else:                                         # more ranks than groups
            out = torch.zeros((*x_local.shape[:-1], self.w.scales.shape[1]),
                              dtype=torch.float16, device=x_local.device)
        if self.w.bias is not None:
            out = out + self.w.bias
        if self.world > 1:
            dist.all_reduce(out, op=dist.ReduceOp.SUM, group=self.group)
        return out


def head_bounds(num_heads: int, world: int, rank: int) -> tuple[int, int]:
    """[h0, h1) attention heads of `rank`: whole heads dealt as evenly as possible
    (Qwen2-7B's 28 query heads at 8 ranks: 4,4,4,4,3,3,3,3)."""
    return even_split(num_heads, world, rank)


def kv_head_bounds(num_heads: int, num_kv_heads: int, h0: int, h1: int) -> tuple[int, int]:
    """[g0, g1) key/value heads that query heads [h0, h1) read under grouped-query
    attention: query head h uses key/value head h // (num_heads / num_kv_heads)
    (model/qwen2.py:131-138 expands each kv head to its group of query heads)."""
    if num_heads % num_kv_heads:
        raise ValueError(f"{num_heads} query heads do not group over {num_kv_heads} kv heads")
    if h1 <= h0:
        return 0, 0
    g = num_heads // num_kv_heads
    return h0 // g, (h1 - 1) // g + 1


@dataclass
class QKVShard:
    """A rank's slice of the fused q/k/v projection in whole heads: its query heads
    [q_heads) and the key/value heads [kv_heads) they use.  The local fused matrix keeps
    the reference's order -- q columns, then k, then v (model/qwen2.py:81-83) -- so the
    local product splits at q_size and q_size + kv_size as the reference's does
    (:111-113)."""
    q_heads: tuple[int, int]
    kv_heads: tuple[int, int]
    head_dim: int
    weights: AWQWeights

    @property
    def q_size(self) -> int:
        return (self.q_heads[1] - self.q_heads[0]) * self.head_dim

    @property
    def kv_size(self) -> int:
        return (self.kv_heads[1] - self.kv_heads[0]) * self.head_dim


def shard_qkv_by_heads(full: AWQWeights, num_heads: int, num_kv_heads: int, head_dim: int,
                       world: int, rank: int) -> QKVShard:
    """Column shard of the fused q/k/v weights (and bias) by whole heads.  Key/value heads
    shared by the query heads of two ranks are held by both (replicated), so every rank
    can attend over its own query heads without communication."""
    if head_dim % 8:
        raise ValueError(f"head_dim={head_dim} is not a whole number of packed words")
    q_size, kv_size = num_heads * head_dim, num_kv_heads * head_dim
    if full.scales.shape[1] != q_size + 2 * kv_size:
        raise ValueError(f"fused q/k/v has {full.scales.shape[1]} columns, expected "
                         f"{q_size + 2 * kv_size}")
    h0, h1 = head_bounds(num_heads, world, rank)
    g0, g1 = kv_head_bounds(num_heads, num_kv_heads, h0, h1)
    cols = [(h0 * head_dim, h1 * head_dim),
            (q_size + g0 * head_dim, q_size + g1 * head_dim),
            (q_size + kv_size + g0 * head_dim, q_size + kv_size + g1 * head_dim)]
    parts = [shard_columns(full.qweight, full.qzeros, full.scales, a, b) for a, b in cols]
    qw, qz, sc = (torch.cat([p[i] for p in parts], 1) for i in range(3))
    bias = None
    if full.bias is not None:
        bias = torch.cat([full.bias[a:b] for a, b in cols])
    return QKVShard((h0, h1), (g0, g1), head_dim, AWQWeights(qw, qz, sc, full.group_size, bias))


class AttentionLinearsTP:
    """The attention block's two AWQ projections over `world` ranks, split by whole heads
    (the reference runs them on one GPU, model/qwen2.py:81-113,156): the fused q/k/v
    projection column-parallel over the rank's query heads plus the key/value heads they
    use, and o row-parallel over the same query heads' rows, followed by the all-reduce.
    Attention itself (RoPE, cache, softmax) runs on the rank's heads in between."""

    def __init__(self, qkv: AWQWeights, o: AWQWeights, num_heads: int, num_kv_heads: int,
                 head_dim: int, world: int, rank: int, group: Optional[object] = None,
                 gemm: Optional[GemmFn] = None, comm=None, check: bool = False):
        if o.qweight.shape[0] != num_heads * head_dim:
            raise ValueError("o must have K == num_heads * head_dim")
        self.shard = shard_qkv_by_heads(qkv, num_heads, num_kv_heads, head_dim, world, rank)
        h0, h1 = self.shard.q_heads
        self.gemm = gemm or _default_gemm()
        self.gemm_bias = _default_gemm_bias() if gemm is None else None
        self.o = RowParallelAWQ(o, world, rank, group=group, gemm=gemm, comm=comm,
                                k_bounds=(h0 * head_dim, h1 * head_dim), check=check)

    def project_qkv(self, x: torch.Tensor):
        """(q, k, v) of this rank's heads: [..., q_size], [..., kv_size], [..., kv_size]."""
        out = _column_forward(self.shard.weights, self.gemm, self.gemm_bias, x)
        qs, ks = self.shard.q_size, self.shard.kv_size
        return out[..., :qs], out[..., qs:qs + ks], out[..., qs + ks:]

    def project_o(self, attn_local: torch.Tensor) -> torch.Tensor:
        """o of the rank's heads' attention output [..., q_size], summed over the ranks."""
        return self.o(attn_local)


class TensorParallelMLP:
    """Qwen2 MLP (model/qwen2.py:160-197) over `world` ranks: fused gate+up column
    parallel, SiLU(gate) * up local, down row parallel + all-reduce.

    The intermediate dimension is split in whole quantization groups, so a rank's
    gate/up columns [lo, hi) are exactly the K rows of down it holds."""

    def __init__(self, gate_up: AWQWeights, down: AWQWeights, intermediate: int, world: int,
                 rank: int, group: Optional[object] = None, gemm: Optional[GemmFn] = None,
                 comm=None, check: bool = False):
        if down.qweight.shape[0] != intermediate:
            raise ValueError("down must have K == intermediate")
        gs = down.group_size

        def bounds(width, w, r):
            return row_bounds(width, gs, w, r)

        self.gate_up = ColumnParallelAWQ(gate_up, world, rank, parts=[intermediate, intermediate],
                                         gemm=gemm, bounds=bounds)
        self.inter_local = self.gate_up.parts_local[0]
        self.down = RowParallelAWQ(down, world, rank, group=group, gemm=gemm, comm=comm,
                                   check=check)
        assert (self.down.k1 - self.down.k0) == self.inter_local
        # the library computes silu(gate) * up with the product; a substituted product
        # (host-logic tests) goes through the slices below
        self.silu_mul = _default_silu_mul() if gemm is None and gate_up.bias is None else None

    def __call__(self, x: torch.Tensor) -> torch.Tensor:
        if self.silu_mul is not None and self.inter_local > 0:
            w = self.gate_up.w
            h = self.silu_mul(x, w.qweight, w.qzeros, w.scales, w.group_size)
            return self.down(h)
        gu = self.gate_up(x)
        gate, up = gu[..., :self.inter_local], gu[..., self.inter_local:]
        h = (F.silu(gate.float()) * up.float()).to(torch.float16)
        return self.down(h)
