"""awq_b200 -- host side of the sm_100a AWQ W4A16 library.

Thin PyTorch-facing layer over libawq_b200.so: tensor checks, device/stream
selection and the per-(device, stream) split-K workspace.  All compute happens in
the CUDA library; nothing here has a CPU fallback.

Public functions
  dequant(qweight, qzeros, scales, group_size)      -> fp16 [K, N]   (bit-exact W)
  gemm(x2d, qweight, qzeros, scales, group_size, path) -> fp16 [M, N]
  device_status(stream)                              -> status bits of the kernels
The reference-facing drop-in, ``kernels.awq_gemm.awq_gemm_forward``, is built on
``gemm``.

Host glue: a decode step calls the product once per linear layer (112 times per token
of Qwen2-7B), so the per-call host work matters.  When the C++ module ``_awq_ext``
(``build_ext.py``, in ``lib/`` beside the library) is built, ``gemm``, ``gemm_silu_mul``
and the drop-in's functions run their checks, output allocation, stream and workspace
lookup in it; otherwise the same steps run here in Python and call the library through
ctypes.  Both call the same C entry points (include/awq_b200.h) and raise the same
exceptions.  With ``AWQ_B200_LIB`` pointing at another build of the library, only the
ctypes path is used, so that build is the one that runs.
"""
from __future__ import annotations

import ctypes
import threading

import torch

from . import _lib
from ._lib import (AWQ_PATH_AUTO, AWQ_PATH_DECODE, AWQ_PATH_TC, AWQ_PATH_TS, AwqError,  # noqa: F401
                   LIB_PATH)

__all__ = ["dequant", "gemm", "gemm_silu_mul", "gemm_allreduce", "TPComm", "device_status", "workspace_for", "AwqError",
           "AWQ_PATH_AUTO", "AWQ_PATH_DECODE", "AWQ_PATH_TC", "AWQ_PATH_TS", "LIB_PATH"]

_ws_lock = threading.Lock()
_workspaces: dict = {}


def _load_ext():
    """The C++ host glue, or None when it is not built (or another library is forced)."""
    import importlib.util
    import os
    import sysconfig
    default = (_lib.PKG_ROOT / "lib" / "libawq_b200.so").resolve()
    if LIB_PATH.resolve() != default or os.environ.get("AWQ_B200_NO_EXT") == "1":
        return None
    path = _lib.PKG_ROOT / "lib" / ("_awq_ext" + sysconfig.get_config_var("EXT_SUFFIX"))
    if not path.exists():
        return None
    _lib.load()                       # the same libawq_b200.so the module links
    spec = importlib.util.spec_from_file_location("_awq_ext", path)
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    mod.set_error_class(AwqError)
    return mod


_ext = _load_ext()


def _require_cuda(t: torch.Tensor, name: str) -> None:
    if not isinstance(t, torch.Tensor):
        raise TypeError(f"{name} must be a torch.Tensor")
    if t.device.type != "cuda":
        raise ValueError(f"{name} is on {t.device}; the AWQ kernels run on CUDA only "
                         "(no CPU fallback)")


def _dense16(t: torch.Tensor) -> torch.Tensor:
    """Contiguous and 16-byte aligned (copies only when needed)."""
    if not t.is_contiguous():
        t = t.contiguous()
    if t.data_ptr() % 16:
        t = t.clone()
    return t


def check_weights(qweight, qzeros, scales, group_size):
    """Validate the packed layout; returns (K, N).  Mirrors the shapes that
    LinearAWQ registers (model/qwen2.py:34-36); N comes from scales.shape[1] as in
    awq_gemm_forward (kernels/awq_gemm.py:247)."""
    for t, name in ((qweight, "qweight"), (qzeros, "qzeros"), (scales, "scales")):
        _require_cuda(t, name)
        if t.dim() != 2:
            raise ValueError(f"{name} must be 2-D, got shape {tuple(t.shape)}")
    if qweight.dtype != torch.int32 or qzeros.dtype != torch.int32:
        raise TypeError("qweight and qzeros must be int32")
    if scales.dtype != torch.float16:
        raise TypeError("scales must be float16")
    if not (qweight.device == qzeros.device == scales.device):
        raise ValueError("qweight, qzeros and scales must be on one device")
    group_size = int(group_size)
    K = qweight.shape[0]
    N = scales.shape[1]
    if qweight.shape[1] * 8 != N:
        raise ValueError(f"scales.shape[1]={N} but qweight packs {qweight.shape[1] * 8} columns")
    if group_size <= 0 or K % group_size:
        raise ValueError(f"K={K} is not a multiple of group_size={group_size}")
    G = K // group_size
    if tuple(qzeros.shape) != (G, N // 8) or tuple(scales.shape) != (G, N):
        raise ValueError(f"qzeros {tuple(qzeros.shape)} / scales {tuple(scales.shape)} do not "
                         f"match [K/group_size={G}, N/8={N // 8}] / [{G}, {N}]")
    return K, N


def _stream_handle(device: torch.device):
    return ctypes.c_void_p(torch.cuda.current_stream(device).cuda_stream)


class _DeviceGuard:
    """Make `device` current for the ctypes call only when it is not already."""

    def __init__(self, device: torch.device):
        self.idx = device.index if device.index is not None else torch.cuda.current_device()
        self.prev = None

    def __enter__(self):
        cur = torch.cuda.current_device()
        if cur != self.idx:
            self.prev = cur
            torch.cuda.set_device(self.idx)

    def __exit__(self, *exc):
        if self.prev is not None:
            torch.cuda.set_device(self.prev)


def workspace_for(device: torch.device, nbytes: int, stream=None) -> torch.Tensor:
    """Zero-initialised split-K workspace for (device, stream -- default: the current
    one), grown on demand.

    The kernels leave its arrival counters at zero after every call, so it is
    zeroed once per allocation only.  One workspace per stream keeps concurrent
    streams from sharing counters.
    """
    if stream is None:
        stream = torch.cuda.current_stream(device)
    key = (device.index, stream.cuda_stream)
    with _ws_lock:
        ws = _workspaces.get(key)
        if ws is None or ws.numel() < nbytes:
            size = max(nbytes, 1 << 20)
            ws = torch.zeros(size, dtype=torch.uint8, device=device)
            _workspaces[key] = ws
        return ws


# Per-call host work that only depends on the weights' metadata or the shape is cached:
# a decode step issues 112 calls on the same weight tensors.
_checked_lock = threading.Lock()
_checked: dict = {}        # weight metadata -> (K, N) of dense, 16-byte aligned weights
_ws_need: dict = {}        # (device, M, N, K, group_size, silu_mul) -> workspace bytes


def _prepared_weights(qweight, qzeros, scales, group_size):
    """check_weights + _dense16, skipped for weights validated before with the same
    pointers, shapes, strides, dtypes and device (the checks depend on nothing else).
    Returns (K, N, qweight, qzeros, scales)."""
    try:
        key = (qweight.data_ptr(), qzeros.data_ptr(), scales.data_ptr(), qweight.shape,
               qzeros.shape, scales.shape, qweight.stride(), qzeros.stride(), scales.stride(),
               qweight.dtype, qzeros.dtype, scales.dtype, qweight.device, int(group_size))
    except (AttributeError, TypeError, ValueError):
        key = None
    if key is not None:
        hit = _checked.get(key)
        if hit is not None:
            return hit[0], hit[1], qweight, qzeros, scales
    K, N = check_weights(qweight, qzeros, scales, group_size)
    dense = [_dense16(t) for t in (qweight, qzeros, scales)]
    if key is not None and all(d is t for d, t in zip(dense, (qweight, qzeros, scales))):
        with _checked_lock:
            if len(_checked) > 65536:
                _checked.clear()
            _checked[key] = (K, N)
    return (K, N, *dense)


def _workspace_need(lib, dev: torch.device, M: int, N: int, K: int, group_size: int,
                    silu_mul: bool = False) -> int:
    key = (dev.index, M, N, K, group_size, silu_mul)
    need = _ws_need.get(key)
    if need is None:
        fn = lib.awq_gemm_silu_mul_workspace_bytes if silu_mul else lib.awq_gemm_workspace_bytes
        need = int(fn(M, N, K, group_size))
        with _checked_lock:
            if len(_ws_need) > 65536:
                _ws_need.clear()
            _ws_need[key] = need
    return need


def dequant(qweight: torch.Tensor, qzeros: torch.Tensor, scales: torch.Tensor,
            group_size: int = 128, out: torch.Tensor | None = None) -> torch.Tensor:
    """fp16 [K, N] dequantized weights, bit-identical to the reference's
    _dequant_to_fp16 (kernels/awq_gemm.py:66-87)."""
    K, N = check_weights(qweight, qzeros, scales, group_size)
    qweight, qzeros, scales = _dense16(qweight), _dense16(qzeros), _dense16(scales)
    dev = qweight.device
    if out is None:
        out = torch.empty((K, N), dtype=torch.float16, device=dev)
    else:
        _require_cuda(out, "out")
        if out.dtype != torch.float16 or tuple(out.shape) != (K, N) or not out.is_contiguous() \
                or out.data_ptr() % 16:
            raise ValueError("out must be a contiguous, 16-byte aligned fp16 [K, N] tensor")
    lib = _lib.load()
    with _DeviceGuard(dev):
        _lib.check(lib.awq_dequant_f16(qweight.data_ptr(), qzeros.data_ptr(), scales.data_ptr(),
                                       out.data_ptr(), K, N, int(group_size),
                                       _stream_handle(dev)))
    return out


def gemm(x2d: torch.Tensor, qweight: torch.Tensor, qzeros: torch.Tensor, scales: torch.Tensor,
         group_size: int = 128, path: int = AWQ_PATH_AUTO,
         out: torch.Tensor | None = None, bias: torch.Tensor | None = None) -> torch.Tensor:
    """fp16 [M, N] = x2d fp16 [M, K] @ W (+ bias fp16 [N], added in the kernel's
    epilogue before the fp16 rounding) with fp32 accumulation, on the current stream."""
    if _ext is not None:
        return _ext.gemm(x2d, qweight, qzeros, scales, int(group_size), int(path), out, bias)
    K, N, qweight, qzeros, scales = _prepared_weights(qweight, qzeros, scales, group_size)
    if bias is not None:
        _require_cuda(bias, "bias")
        if bias.dtype != torch.float16 or tuple(bias.shape) != (N,):
            raise ValueError(f"bias must be float16 [N={N}], got {bias.dtype} {tuple(bias.shape)}")
        if path != AWQ_PATH_AUTO:
            raise ValueError("the bias epilogue runs on the automatic kernel choice only")
        bias = bias.contiguous()
    _require_cuda(x2d, "x")
    if x2d.dtype != torch.float16:
        raise TypeError(f"x must be float16, got {x2d.dtype}")
    if x2d.dim() != 2 or x2d.shape[1] != K:
        raise ValueError(f"x must be [M, K={K}], got {tuple(x2d.shape)}")
    dev = x2d.device
    if dev != qweight.device:
        raise ValueError("x and the weights must be on one device")
    M = x2d.shape[0]
    if out is None:
        out = torch.empty((M, N), dtype=torch.float16, device=dev)
    if M == 0:
        return out
    if x2d.stride(1) != 1 or x2d.data_ptr() % 16 or (x2d.stride(0) * 2) % 16:
        x2d = x2d.contiguous()
        if x2d.data_ptr() % 16:
            x2d = x2d.clone()
    lib = _lib.load()
    gs = int(group_size)
    with _DeviceGuard(dev):
        stream = torch.cuda.current_stream(dev)
        need = _workspace_need(lib, dev, M, N, K, gs)
        ws = workspace_for(dev, need, stream) if need else None
        if bias is None:
            _lib.check(lib.awq_gemm_f16_ex(
                x2d.data_ptr(), x2d.stride(0), qweight.data_ptr(), qzeros.data_ptr(),
                scales.data_ptr(), out.data_ptr(), out.stride(0), M, N, K, gs,
                ws.data_ptr() if ws is not None else None, ws.numel() if ws is not None else 0,
                stream.cuda_stream, int(path)))
        else:
            _lib.check(lib.awq_gemm_f16_bias(
                x2d.data_ptr(), x2d.stride(0), qweight.data_ptr(), qzeros.data_ptr(),
                scales.data_ptr(), bias.data_ptr(), out.data_ptr(), out.stride(0), M, N, K, gs,
                ws.data_ptr() if ws is not None else None, ws.numel() if ws is not None else 0,
                stream.cuda_stream))
    return out


def gemm_silu_mul(x2d: torch.Tensor, qweight: torch.Tensor, qzeros: torch.Tensor,
                  scales: torch.Tensor, group_size: int = 128,
                  out: torch.Tensor | None = None) -> torch.Tensor:
    """fp16 [M, N/2] = silu(P[:, :N/2]) * P[:, N/2:] for the fused gate+up product
    P = x2d @ W (``awq_gemm_f16_silu_mul``): P's halves rounded to fp16, fp32
    x * sigmoid(x) * y, one fp16 rounding -- the reference MLP's awq_gemm_forward, slices
    and silu_mul_forward (model/qwen2.py:181-194) in one call."""
    if _ext is not None:
        return _ext.gemm_silu_mul(x2d, qweight, qzeros, scales, int(group_size), out)
    K, N, qweight, qzeros, scales = _prepared_weights(qweight, qzeros, scales, group_size)
    if N % 2:
        raise ValueError(f"N={N} is not even: no gate / up halves")
    _require_cuda(x2d, "x")
    if x2d.dtype != torch.float16:
        raise TypeError(f"x must be float16, got {x2d.dtype}")
    if x2d.dim() != 2 or x2d.shape[1] != K:
        raise ValueError(f"x must be [M, K={K}], got {tuple(x2d.shape)}")
    dev = x2d.device
    if dev != qweight.device:
        raise ValueError("x and the weights must be on one device")
    M = x2d.shape[0]
    if out is None:
        out = torch.empty((M, N // 2), dtype=torch.float16, device=dev)
    if M == 0:
        return out
    if x2d.stride(1) != 1 or x2d.data_ptr() % 16 or (x2d.stride(0) * 2) % 16:
        x2d = x2d.contiguous()
        if x2d.data_ptr() % 16:
            x2d = x2d.clone()
    lib = _lib.load()
    gs = int(group_size)
    with _DeviceGuard(dev):
        stream = torch.cuda.current_stream(dev)
        need = _workspace_need(lib, dev, M, N, K, gs, silu_mul=True)
        ws = workspace_for(dev, need, stream)
        _lib.check(lib.awq_gemm_f16_silu_mul(
            x2d.data_ptr(), x2d.stride(0), qweight.data_ptr(), qzeros.data_ptr(),
            scales.data_ptr(), out.data_ptr(), out.stride(0), M, N, K, gs, ws.data_ptr(),
            ws.numel(), stream.cuda_stream))
    return out


class TPComm:
    """This rank's communicator for the fused row-parallel all-reduce
    (``awq_tp_comm_*`` / ``awq_gemm_f16_allreduce`` in include/awq_b200.h): a receive
    buffer on this rank's GPU that every other rank maps through CUDA IPC and writes its
    tile results into over NVLink.

    ``TPComm(world, rank, max_n, max_rows=2048)`` allocates the buffer on the current
    device and exposes ``handle`` (bytes); ``open(handles)`` takes every rank's handle in
    rank order.  ``TPComm.from_group(max_n, group)`` does both with ``torch.distributed``.
    All ranks must then issue the same sequence of ``gemm_allreduce`` calls, one stream
    per communicator.  ``close()`` after the device has finished those calls.  Calls of
    up to 16 tokens run the fused decode kernel; calls of 17 to ``max_rows`` tokens run
    the prefill product into the buffer and the library's all-reduce kernel over NVLink
    (two fp16 planes of ``max_rows x max_n`` per rank; ``max_rows=0`` leaves them out)."""

    def __init__(self, world: int, rank: int, max_n: int, device=None, max_rows: int = 2048):
        self.device = torch.device("cuda", torch.cuda.current_device()) if device is None \
            else torch.device(device)
        self.world, self.rank, self.max_n = int(world), int(rank), int(max_n)
        self.max_rows = int(max_rows)
        lib = _lib.load()
        h = ctypes.create_string_buffer(_lib.AWQ_IPC_HANDLE_BYTES)
        ptr = ctypes.c_void_p()
        with _DeviceGuard(self.device):
            _lib.check(lib.awq_tp_comm_create_ex(self.world, self.rank, self.max_n,
                                                 self.max_rows, h, ctypes.byref(ptr)))
        self._ptr = ptr
        self.handle = h.raw
        self.opened = False

    def open(self, handles) -> None:
        if len(handles) != self.world or any(len(h) != _lib.AWQ_IPC_HANDLE_BYTES for h in handles):
            raise ValueError(f"need {self.world} handles of {_lib.AWQ_IPC_HANDLE_BYTES} bytes")
        buf = ctypes.create_string_buffer(b"".join(handles), len(handles) * _lib.AWQ_IPC_HANDLE_BYTES)
        with _DeviceGuard(self.device):
            _lib.check(_lib.load().awq_tp_comm_open(self._ptr, buf))
        self.opened = True

    @classmethod
    def from_group(cls, max_n: int, group=None, device=None, max_rows: int = 2048) -> "TPComm":
        import torch.distributed as dist
        comm = cls(dist.get_world_size(group), dist.get_rank(group), max_n, device, max_rows)
        got = [None] * comm.world
        dist.all_gather_object(got, (comm.handle, comm.max_n, comm.max_rows), group=group)
        # every rank's buffer must have the same layout: the ranks store into each other's
        if any(g[1:] != (comm.max_n, comm.max_rows) for g in got):
            comm.close()
            raise ValueError(f"ranks disagree on (max_n, max_rows): {[g[1:] for g in got]}")
        comm.open([g[0] for g in got])
        dist.barrier(group=group)
        return comm

    def set_timeout(self, seconds: float) -> None:
        _lib.check(_lib.load().awq_tp_comm_set_timeout(self._ptr, max(1, int(seconds * 1e9))))

    def supported(self, x2d: torch.Tensor, qweight: torch.Tensor, N: int,
                  group_size: int = 128) -> bool:
        if not self.opened:
            return False
        with _DeviceGuard(self.device):
            return bool(_lib.load().awq_allreduce_supported(
                self._ptr, x2d.data_ptr(), x2d.stride(0), qweight.data_ptr(), x2d.shape[0], N,
                qweight.shape[0], int(group_size)))

    def supported_shape(self, M: int, N: int, K: int, group_size: int = 128) -> bool:
        """``supported`` for a dense, 16-byte aligned x [M, K] and qweight [K, N/8]: the
        shape part of the decision alone.  ``awq_allreduce_supported`` only inspects the
        pointers' alignment, so aligned placeholders stand in for them; a caller that
        evaluates this for every rank's K gets the same answer on every rank."""
        if not self.opened or K <= 0 or M <= 0:
            return False
        with _DeviceGuard(self.device):
            return bool(_lib.load().awq_allreduce_supported(
                self._ptr, 256, K, 256, int(M), int(N), int(K), int(group_size)))

    def check(self, group=None, collective: bool = False) -> None:
        """Synchronise the current stream and raise ``AwqError`` if a kernel on this
        device reported an error since the last check: status bit 4 (a fused all-reduce
        gave up waiting for another rank -- that call's output is wrong and every rank
        must ``reset`` the communicator) or bit 1 (a bounded wait inside a kernel ran
        out).  The status word is cleared.  Call it where the caller synchronises anyway
        (after a decode step, before its result is read).

        Only the rank whose wait ran out sees bit 4; a rank that ran ahead may have summed
        a stale tile without waiting.  With ``collective=True`` (every rank calls it, same
        ``group``) the ranks' status bits are combined with one all-reduce, so every rank
        raises together and can take part in ``reset``."""
        st = device_status(self.device)
        if collective:
            import torch.distributed as dist
            bits = torch.tensor([(st >> b) & 1 for b in range(3)], dtype=torch.int32,
                                device=self.device)
            dist.all_reduce(bits, op=dist.ReduceOp.MAX, group=group)
            st = sum(int(v) << b for b, v in enumerate(bits.tolist()))
        if st:
            what = []
            if st & _lib.STATUS_PEER_TIMEOUT:
                what.append("a fused all-reduce timed out waiting for another rank "
                            "(reset the communicator on every rank)")
            if st & _lib.STATUS_BARRIER_TIMEOUT:
                what.append("a bounded wait inside a kernel ran out")
            if st & _lib.STATUS_SHAPE:
                what.append("a kernel rejected its parameters")
            raise AwqError(_lib.AWQ_ERR_DEVICE, f"device status {st}: " + "; ".join(what))

    def reset(self, group=None) -> None:
        """Collective: return every rank's communicator to its freshly opened state (after
        ``check`` raised for a peer time-out).  Every rank must call it; no fused call may
        be in flight.  Barrier, clear this rank's receive buffer and call number, barrier."""
        import torch.distributed as dist
        torch.cuda.synchronize(self.device)
        dist.barrier(group=group)
        with _DeviceGuard(self.device):
            _lib.check(_lib.load().awq_tp_comm_reset(self._ptr))
        dist.barrier(group=group)

    def close(self) -> None:
        if self._ptr is not None:
            with _DeviceGuard(self.device):
                _lib.check(_lib.load().awq_tp_comm_destroy(self._ptr))
            self._ptr = None


def gemm_allreduce(x2d: torch.Tensor, qweight: torch.Tensor, qzeros: torch.Tensor,
                   scales: torch.Tensor, group_size: int, comm: TPComm,
                   out: torch.Tensor | None = None) -> torch.Tensor:
    """Row-parallel product summed over the tensor-parallel ranks in one kernel: every
    rank gets fp16 [M, N] = sum over ranks of x2d_r @ W_r (bit-identical on all ranks).
    Raises AwqError(AWQ_ERR_UNSUPPORTED) when ``comm.supported`` is false."""
    K, N = check_weights(qweight, qzeros, scales, group_size)
    _require_cuda(x2d, "x")
    if x2d.dtype != torch.float16 or x2d.dim() != 2 or x2d.shape[1] != K:
        raise ValueError(f"x must be float16 [M, K={K}], got {x2d.dtype} {tuple(x2d.shape)}")
    M = x2d.shape[0]
    dev = x2d.device
    if out is None:
        out = torch.empty((M, N), dtype=torch.float16, device=dev)
    if M == 0:
        return out
    qweight, qzeros, scales = _dense16(qweight), _dense16(qzeros), _dense16(scales)
    if x2d.stride(1) != 1 or x2d.data_ptr() % 16 or (x2d.stride(0) * 2) % 16:
        x2d = x2d.contiguous()
        if x2d.data_ptr() % 16:
            x2d = x2d.clone()
    lib = _lib.load()
    with _DeviceGuard(dev):
        need = lib.awq_gemm_workspace_bytes(M, N, K, int(group_size))
        ws = workspace_for(dev, need) if need else None
        _lib.check(lib.awq_gemm_f16_allreduce(
            comm._ptr, x2d.data_ptr(), x2d.stride(0), qweight.data_ptr(), qzeros.data_ptr(),
            scales.data_ptr(), out.data_ptr(), out.stride(0), M, N, K, int(group_size),
            ws.data_ptr() if ws is not None else None, ws.numel() if ws is not None else 0,
            _stream_handle(dev)))
    return out


def tc_supported(x2d, qweight, qzeros, scales, group_size: int = 128) -> bool:
    """Whether the tcgen05 prefill kernel accepts this shape and these pointers."""
    lib = _lib.load()
    K, N = qweight.shape[0], scales.shape[1]
    return bool(lib.awq_tc_supported(x2d.data_ptr(), x2d.stride(0), qweight.data_ptr(),
                                     qzeros.data_ptr(), scales.data_ptr(), x2d.shape[0], N, K,
                                     int(group_size)))


def device_status(device=None) -> int:
    """Synchronise the current stream and return (and clear) the kernels' status bits."""
    dev = torch.device("cuda", torch.cuda.current_device()) if device is None \
        else torch.device(device)
    lib = _lib.load()
    st = ctypes.c_int(0)
    with _DeviceGuard(dev):
        rc = lib.awq_device_status(_stream_handle(dev), ctypes.byref(st))
    if rc not in (_lib.AWQ_OK, _lib.AWQ_ERR_DEVICE):
        _lib.check(rc)
    return st.value
