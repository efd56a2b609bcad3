#!/usr/bin/env python
"""Benchmark of the sm_100a AWQ W4A16 product (drop-in for kernels/awq_gemm.py).

Headline metric: AWQ GEMM HBM TB/s at M=1 decode and TFLOP/s at
M=2048 prefill, as fractions of the B200 roofline.

One *step* = one decode token through the AWQ linears of the 28-layer Qwen2-7B stack
at M=1, in the call shapes the reference uses (model/qwen2.py:81-83,104,156,176-186,196):
fused qkv 3584x4608, o 3584x3584, fused gate+up 3584x37888, down 18944x3584.  That is
112 launches and 3.39 GB of packed weights per step -- 27x the 126 MB L2, so every
step streams from HBM (no flush needed).  Weights are random int4 in the AWQ layout
with the benchmark's distributions (synthetic data; no checkpoint exists here).

  value     algorithmic bytes of a step / device time of a step (CUDA events over K
            CUDA-graph replays), TB/s, whole job (max over ranks); tokens_per_s is
            1 / that step time (the linears' decode rate of the 28-layer stack)
  e2e       the same bytes / time of a step made through the public drop-in
            ``awq_gemm_forward``: per step one H2D copy of the step's 112 inputs from
            pinned host memory and one D2H copy of its 112 outputs, inside the timed
            region (wall clock, synchronised); the outputs read back are checked bit for
            bit against the same calls after a synchronous copy (``outputs_checked``)
  roofline  decode kernel achieved GB/s vs MEASURED_PEAKS.json hbm_gbs
  prefill   M=2048 gate+up and down through the tcgen05 kernel: TFLOP/s vs the
            measured bf16 peak (fp16 and bf16 tensor rates are equal)
  cpu_baseline  the reference's dequantize-then-fp32-matmul host path (oracle port,
            torch on every host core) on one layer's 4 linears at M=1

  mlp       BASELINE config 4: the Qwen2-7B MLP block (gate+up with SiLU-mul, down) at
            M = 1, 16 and 512 over the N GPUs (tensor parallel: gate+up by columns, down
            by rows + all-reduce), with the row-parallel down's product alone, with the
            library's all-reduce (M <= 16: one fused kernel; M = 512: product + the
            NVLink all-reduce kernel), and followed by NCCL, per call
  stack     BASELINE config 5: the 28-layer linear stack with RMSNorm and residual adds
            between the linears, a 1024-token prefill and 512 graph-replayed decode
            steps at batch 1, tokens/s over the N GPUs

With torchrun (N > 1) every rank runs the tensor-parallel stack: qkv and gate+up
column-sharded, o and down row-sharded, each row-parallel call's fp16 output summed over
the ranks by the library's all-reduce over NVLink peer memory (decode: fused into the
product kernel; prefill: a separate all-reduce kernel after the product), else NCCL
(strong scaling: the token's total bytes are fixed).
``--impl reference`` times the reference's own CPU path (oracle port) instead.
``--stack`` runs only the config-5 leg (see stack_bench).
"""
from __future__ import annotations

import argparse
import json
import os
import pathlib
import statistics
import subprocess
import sys
import threading
import time

REPO = pathlib.Path(__file__).resolve().parent
sys.path.insert(0, str(REPO / "qwen2-7b-triton_engine_b200"))
sys.path.insert(0, str(REPO))

HIDDEN, INTER, LAYERS, GS = 3584, 18944, 28, 128
# (name, K, N) per layer, in call order
STACK = [("qkv", HIDDEN, 4608), ("o", HIDDEN, HIDDEN), ("gate_up", HIDDEN, 2 * INTER),
         ("down", INTER, HIDDEN)]
SWEEP = {"q_o": (HIDDEN, HIDDEN), "k_v": (HIDDEN, 512), "qkv": (HIDDEN, 4608),
         "gate_up": (HIDDEN, 2 * INTER), "down": (INTER, HIDDEN)}


# DRAM bytes (read + write) of one cold-cache launch of the decode kernel at M=1 on each
# stack shape, from `ncu --metrics dram__bytes_read.sum,dram__bytes_write.sum` (summary and
# command in profiles/gemv_tma_decode_traffic.md).  Per launch of the stack this averages
# to within 1 % of the algorithmic bytes: no re-reads.
NCU_TRAFFIC_M1 = {"qkv": 8639232, "o": 6732544, "gate_up": 70606592 + 321024,
                  "down": 35363840}


def alg_bytes(M, K, N, gs=GS):
    """Algorithmic bytes of one call: packed weights + zeros + scales + x + out."""
    return K * N // 2 + (K // gs) * (N // 8) * 4 + (K // gs) * N * 2 + 2 * M * K + 2 * M * N


def load_peaks():
    p = REPO / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return d["hbm_gbs"], d["bf16_tflops"], d.get("bf16_tflops_sustained"), "measured"
    return 6650.0, 1590.0, 1400.0, "fallback"


# --------------------------------------------------------------------------- clocks --
class ClockSampler:
    """SM clock and clock-event (throttle) reasons sampled through NVML every 10 ms in a
    thread while the timed region runs (read-only queries; no GPU setting is changed).
    The first sample is taken before __enter__ returns, so even a short timed region is
    covered.  Falls back to nvidia-smi when NVML is unavailable."""
    PERIOD_S = 0.01
    # NVML clock-event reason bits
    REASONS = {0x4: "sw_power_cap", 0x8: "hw_slowdown", 0x20: "sw_thermal_slowdown",
               0x40: "hw_thermal_slowdown", 0x80: "hw_power_brake_slowdown"}

    def __init__(self, torch_index: int):
        self.torch_index = torch_index
        self.rows = []            # (sm_mhz, max_mhz, reason bits)
        self.stop = threading.Event()
        self.thread = None
        self.nvml = None
        self.handle = None

    def _open(self):
        import pynvml
        pynvml.nvmlInit()
        handle = None
        try:                                   # match the CUDA device by PCI bus id
            import torch
            pr = torch.cuda.get_device_properties(self.torch_index)
            bus = f"{pr.pci_domain_id:08x}:{pr.pci_bus_id:02x}:{pr.pci_device_id:02x}.0"
            handle = pynvml.nvmlDeviceGetHandleByPciBusId(bus)
        except Exception:
            handle = pynvml.nvmlDeviceGetHandleByIndex(self.torch_index)
        return pynvml, handle

    def _sample(self):
        nv, h = self.nvml, self.handle
        sm = nv.nvmlDeviceGetClockInfo(h, nv.NVML_CLOCK_SM)
        mx = nv.nvmlDeviceGetMaxClockInfo(h, nv.NVML_CLOCK_SM)
        get = getattr(nv, "nvmlDeviceGetCurrentClocksEventReasons", None) or \
            nv.nvmlDeviceGetCurrentClocksThrottleReasons
        self.rows.append((float(sm), float(mx), int(get(h))))

    def _loop(self):
        while not self.stop.wait(self.PERIOD_S):
            try:
                self._sample()
            except Exception:
                return

    def __enter__(self):
        try:
            self.nvml, self.handle = self._open()
            self._sample()
            self.thread = threading.Thread(target=self._loop, daemon=True)
            self.thread.start()
        except Exception:
            self.nvml = None
            self._smi_once()
        return self

    def _smi_once(self):
        try:
            out = subprocess.run(
                ["nvidia-smi", f"--id={self.torch_index}", "--query-gpu=clocks.sm,clocks.max.sm",
                 "--format=csv,noheader,nounits"], capture_output=True, text=True, timeout=10)
            sm, mx = (float(v) for v in out.stdout.strip().split(",")[:2])
            self.rows.append((sm, mx, 0))
        except Exception:
            pass

    def __exit__(self, *exc):
        if self.thread is not None:
            self.stop.set()
            self.thread.join(timeout=5)
            try:
                self._sample()                 # one more, right after the region
            except Exception:
                pass
        elif self.nvml is None:
            self._smi_once()

    def summary(self):
        if not self.rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"]}
        reasons = set()
        for _, _, bits in self.rows:
            for b, nm in self.REASONS.items():
                if bits & b:
                    reasons.add(nm)
        return {"sm_mhz": statistics.median(r[0] for r in self.rows),
                "sm_max_mhz": max(r[1] for r in self.rows),
                "reasons": sorted(reasons), "samples": len(self.rows),
                "source": "nvml" if self.nvml is not None else "nvidia-smi"}


# ------------------------------------------------------------------------ helpers ----
def make_layer_dev(torch, K, N, dev, gen):
    qw = torch.randint(-2**31, 2**31, (K, N // 8), dtype=torch.int64, device=dev,
                       generator=gen).to(torch.int32)
    qz = torch.randint(-2**31, 2**31, (K // GS, N // 8), dtype=torch.int64, device=dev,
                       generator=gen).to(torch.int32)
    s = (torch.rand((K // GS, N), device=dev, generator=gen) * 0.018 + 0.002).half()
    return qw, qz, s


def cpu_baseline(torch, sample_seconds=12.0):
    """Reference host path (oracle port) on one layer's 4 linears at M=1."""
    from oracle import oracle as O
    threads = O.cpu_threads()
    torch.set_num_threads(threads)
    g = torch.Generator().manual_seed(11)
    layers = []
    for _, K, N in STACK:
        qw = torch.randint(-2**31, 2**31, (K, N // 8), dtype=torch.int64, generator=g).to(torch.int32)
        qz = torch.randint(-2**31, 2**31, (K // GS, N // 8), dtype=torch.int64, generator=g).to(torch.int32)
        s = (torch.rand((K // GS, N), generator=g) * 0.018 + 0.002).half()
        x = torch.randn((1, K), generator=g).half()
        layers.append((x, qw, qz, s, alg_bytes(1, K, N)))
    nbytes, secs, reps = 0, 0.0, 0
    O.torch_awq_gemm_f32(*layers[0][:4])                      # warm-up
    t0 = time.perf_counter()
    while True:
        for (x, qw, qz, s, b) in layers:
            O.torch_awq_gemm_f32(x, qw, qz, s)
            nbytes += b
        reps += 1
        secs = time.perf_counter() - t0
        if secs >= sample_seconds or reps >= 50:
            break
    return {"value": nbytes / secs / 1e12, "unit": "TB/s", "cores": threads, "kind": "port",
            "sample": f"{reps} x one Qwen2-7B layer (qkv, o, gate_up, down) at M=1: torch "
                      f"dequant + fp32 matmul on {threads} host threads, {secs:.1f} s"}


# ------------------------------------------------------------------------ our arm ----
_JSON_FD = None    # descriptor of the real stdout once fd 1 is redirected to stderr


def emit_json(obj) -> None:
    """Print the result line on the process's real stdout."""
    line = json.dumps(obj) + "\n"
    if _JSON_FD is None:
        sys.stdout.write(line)
        sys.stdout.flush()
    else:
        sys.stdout.flush()
        os.write(_JSON_FD, line.encode())


def run_ours(args):
    import torch
    import torch.distributed as dist

    import awq_b200
    from awq_b200 import tp
    from kernels import awq_gemm

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        import datetime
        # keep stdout to the one JSON line: anything the communication libraries print on
        # the process's stdout (NCCL's version banner, for one) goes to stderr
        global _JSON_FD
        _JSON_FD = os.dup(1)
        os.dup2(2, 1)
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                device_id=dev)
    hbm_peak, tc_peak, tc_sust, peak_src = load_peaks()
    gen = torch.Generator(device=dev).manual_seed(1234 + rank)

    # ---- weights of the 28-layer stack (this rank's shards) -------------------------
    calls = []          # (K_local, N_local, tensors, reduce?)
    full_bytes = 0
    for _ in range(LAYERS):
        for name, K, N in STACK:
            full_bytes += alg_bytes(1, K, N)
            if world == 1:
                calls.append((name, K, N, make_layer_dev(torch, K, N, dev, gen), False))
            elif name == "qkv":                          # column parallel, whole words
                n0, n1 = tp.column_bounds(N, world, rank)
                calls.append((name, K, n1 - n0, make_layer_dev(torch, K, n1 - n0, dev, gen), False))
            elif name == "gate_up":                      # gate and up split in whole groups
                i0, i1 = tp.row_bounds(INTER, GS, world, rank)
                nl = 2 * (i1 - i0)
                calls.append((name, K, nl, make_layer_dev(torch, K, nl, dev, gen), False))
            else:                                        # row parallel + all-reduce
                k0, k1 = tp.row_bounds(K, GS, world, rank)
                calls.append((name, k1 - k0, N, make_layer_dev(torch, k1 - k0, N, dev, gen), True))
    xs = {}
    for name, K, N, _, _ in calls:
        xs.setdefault(K, torch.randn((1, K), device=dev, generator=gen).half())
    outs = [torch.empty((1, N), dtype=torch.float16, device=dev) for (_, _, N, _, _) in calls]
    ws = awq_b200.workspace_for(dev, max(
        awq_b200._lib.load().awq_gemm_workspace_bytes(1, N, K, GS) for (_, K, N, _, _) in calls))

    lib = awq_b200._lib.load()
    stream = torch.cuda.Stream(device=dev)

    # row-parallel calls (o, down) under tensor parallelism: product and all-reduce in one
    # kernel over NVLink peer memory where the fused kernel runs the shape (decided once,
    # the same on every rank), else the product followed by an NCCL all-reduce
    comm = None
    fused = [False] * len(calls)
    if world > 1:
        comm = awq_b200.TPComm.from_group(max(N for (_, _, N, _, red) in calls if red))
        ok = torch.tensor([1 if red and comm.supported(xs[K], qw, N, GS) else 0
                           for (_, K, N, (qw, _, _), red) in calls], dtype=torch.int32, device=dev)
        dist.all_reduce(ok, op=dist.ReduceOp.MIN)
        fused = [bool(v) for v in ok.tolist()]

    def step():
        h = torch.cuda.current_stream(dev).cuda_stream
        for i, (name, K, N, (qw, qz, s), red) in enumerate(calls):
            x = xs[K]
            if fused[i]:
                rc = lib.awq_gemm_f16_allreduce(comm._ptr, x.data_ptr(), K, qw.data_ptr(),
                                                qz.data_ptr(), s.data_ptr(), outs[i].data_ptr(),
                                                N, 1, N, K, GS, ws.data_ptr(), ws.numel(), h)
            else:
                rc = lib.awq_gemm_f16(x.data_ptr(), K, qw.data_ptr(), qz.data_ptr(), s.data_ptr(),
                                      outs[i].data_ptr(), N, 1, N, K, GS, ws.data_ptr(),
                                      ws.numel(), h)
            if rc:
                awq_b200._lib.check(rc)
            if red and not fused[i]:
                dist.all_reduce(outs[i])

    # warm-up (eager), then capture one step into a CUDA graph
    with torch.cuda.stream(stream):
        for _ in range(max(1, args.warmup)):
            step()
    torch.cuda.synchronize()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph, stream=stream):
        step()
    for _ in range(args.warmup):
        graph.replay()
    torch.cuda.synchronize()

    # ---- timed region: K graph replays ----------------------------------------------
    ev0 = torch.cuda.Event(enable_timing=True)
    ev1 = torch.cuda.Event(enable_timing=True)
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    with ClockSampler(local) as clk:
        with torch.cuda.stream(stream):
            ev0.record(stream)
            for _ in range(args.steps):
                graph.replay()
            ev1.record(stream)
        torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    ms = ev0.elapsed_time(ev1) / args.steps
    if world > 1:
        t = torch.tensor([ms], device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms = float(t.item())
    value = full_bytes / (ms * 1e-3) / 1e12
    del graph
    torch.cuda.synchronize()

    result = None
    if rank == 0:
        local_bytes = sum(alg_bytes(1, K, N) for (_, K, N, _, _) in calls)
        achieved = local_bytes / (ms * 1e-3) / 1e9
        result = {
            "metric": "AWQ GEMM HBM TB/s (M=1 decode) & TFLOPS (M=2048 prefill), % of B200 roofline",
            "value": round(value, 4), "unit": "TB/s", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": round(ms, 5),
            "tokens_per_s": round(1e3 / ms, 1),      # one step = one decode token, 28 layers
            "higher_is_better": True,
            "scaling": "strong" if world > 1 else "weak", "vs_baseline": None, "dtype": "f16",
            "data": "synthetic (seeded random int4 AWQ weights, x ~ N(0,1); no checkpoint)",
            "config": {"workload": "decode M=1 through the AWQ linears of the 28-layer Qwen2-7B "
                                   "stack (qkv 3584x4608, o 3584x3584, gate_up 3584x37888, down "
                                   "18944x3584 per layer; 112 launches, CUDA-graph replay)",
                       "bytes_per_step": full_bytes, "group_size": GS,
                       "l2": "working set 3.39 GB > 126 MB L2 (no flush needed)",
                       "parallelism": f"tp{world}" if world > 1 else "single",
                       "allreduce": (("fused: product and all-reduce in one kernel over NVLink "
                                      "peer memory" if any(fused) else "nccl")
                                     if world > 1 else None)},
            "roofline": {"bound": "hbm", "achieved": round(achieved, 1), "peak": hbm_peak,
                         "unit": "GB/s", "frac": round(achieved / hbm_peak, 4),
                         "peak_source": peak_src,
                         "traffic": (round(sum(NCU_TRAFFIC_M1.values()) / len(NCU_TRAFFIC_M1))
                                     if world == 1 else None),
                         "traffic_note": "bytes per launch averaged over the 4 stack shapes, "
                                         "ncu dram__bytes_read.sum + dram__bytes_write.sum",
                         "alg_bytes_per_launch": round(local_bytes / len(calls)),
                         "kernel": "awq::gemv_tma_kernel<1> (decode: TMA-streamed mma.sync, "
                                   "one CTA per SM, deterministic split-K)"},
            "gpu_launches": args.steps * len(calls),
        }
        result["clocks"] = clk.summary()

    # ---- end to end through the public drop-in, host buffers ------------------------
    # Every step copies that step's inputs (one x per call) from pinned host memory in
    # one H2D copy, makes the 112 calls through the public drop-in on device views of
    # them, and reads every call's output back in one D2H copy (gathered on the device
    # first); the timed region is wall clock around whole steps, synchronised.  The host
    # launches the calls while the copy in runs; moving both copies to a second stream in
    # per-layer chunks, overlapped with the calls, was slower (1.34 vs 1.29 ms per step
    # against 1.10 ms of graph-replayed device time), so the eager launches set the pace.
    x_off = [0]
    for (_, K, _, _, _) in calls:
        x_off.append(x_off[-1] + K)
    hx_all = torch.randn((x_off[-1],)).half().pin_memory()
    dx_all = torch.empty((x_off[-1],), dtype=torch.float16, device=dev)
    dx = [dx_all[x_off[i]:x_off[i + 1]].view(1, -1) for i in range(len(calls))]
    hout_all = torch.empty((sum(N for (_, _, N, _, _) in calls),), dtype=torch.float16).pin_memory()

    def e2e_step():
        dx_all.copy_(hx_all, non_blocking=True)
        ys = []
        for i, (name, K, N, (qw, qz, s), red) in enumerate(calls):
            if fused[i]:
                y = awq_b200.gemm_allreduce(dx[i], qw, qz, s, GS, comm)
            else:
                y = awq_gemm.awq_gemm_forward(dx[i], qw, qz, s, GS)
                if red:
                    dist.all_reduce(y)
            ys.append(y.view(-1))
        hout_all.copy_(torch.cat(ys), non_blocking=True)
        torch.cuda.synchronize()

    def e2e_check():
        """One timed-form step against the same calls made after a synchronous input
        copy: the outputs read back must be the same bits."""
        e2e_step()
        got = hout_all.clone()
        dx_all.copy_(hx_all)
        torch.cuda.synchronize()
        ys = []
        for i, (name, K, N, (qw, qz, s), red) in enumerate(calls):
            if fused[i]:
                y = awq_b200.gemm_allreduce(dx[i], qw, qz, s, GS, comm)
            else:
                y = awq_gemm.awq_gemm_forward(dx[i], qw, qz, s, GS)
                if red:
                    dist.all_reduce(y)
            ys.append(y.view(-1))
        return bool(torch.equal(got, torch.cat(ys).cpu()))
    for _ in range(max(1, args.warmup)):
        e2e_step()
    e2e_steps = max(3, min(args.steps, 20))
    if world > 1:
        dist.barrier()
    t0 = time.perf_counter()
    for _ in range(e2e_steps):
        e2e_step()
    e2e_ms = (time.perf_counter() - t0) * 1e3 / e2e_steps
    e2e_ok = e2e_check()
    if world > 1:
        t = torch.tensor([e2e_ms], device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        e2e_ms = float(t.item())
    if rank == 0:
        result["e2e"] = {"value": round(full_bytes / (e2e_ms * 1e-3) / 1e12, 4), "unit": "TB/s",
                         "ms_per_step": round(e2e_ms, 4), "tokens_per_s": round(1e3 / e2e_ms, 1),
                         "h2d_bytes_per_step": hx_all.numel() * hx_all.element_size(),
                         "d2h_bytes_per_step": hout_all.numel() * hout_all.element_size(),
                         "copies": "one H2D of the step's 112 inputs, one D2H of its 112 outputs",
                         "outputs_checked": e2e_ok,
                         "host_glue": "C++ (_awq_ext)" if awq_b200._ext is not None else "ctypes",
                         "api": "kernels.awq_gemm.awq_gemm_forward (eager, 112 calls"
                                + ((", o and down through awq_b200.gemm_allreduce: product and "
                                    "all-reduce in one kernel)" if all(
                                        f for f, c in zip(fused, calls) if c[4])
                                    else ", NCCL all-reduce after o and down)")
                                   if world > 1 else ")")}
    calls.clear()                                      # the stack's weights: free them
    torch.cuda.empty_cache()
    mlp = mlp_block_bench(torch, awq_b200, dev, world, rank, comm)
    stack = stack_bench(torch, awq_b200, dev, world, rank, comm, args)
    if rank == 0:
        result["mlp"] = mlp
        result["stack"] = stack
    if world == 1:
        result["prefill"] = prefill_bench(torch, awq_b200, dev, tc_peak, peak_src, args)
        result["sweep"] = decode_sweep(torch, lib, awq_b200, dev, hbm_peak)
        result["cpu_baseline"] = cpu_baseline(torch, args.cpu_seconds)
    if world > 1:
        torch.cuda.synchronize()
        dist.barrier()
        if comm is not None:
            comm.close()
        dist.destroy_process_group()
    if rank == 0:
        emit_json(result)


def prefill_bench(torch, awq_b200, dev, tc_peak, peak_src, args):
    """M=2048 gate+up and down through the tcgen05 kernel (or the decode fallback)."""
    M = 2048
    gen = torch.Generator(device=dev).manual_seed(77)
    res = {"metric": "AWQ GEMM TFLOP/s (M=2048 prefill)", "unit": "TFLOP/s"}
    tot_flops, tot_ms = 0, 0.0
    for name, K, N in (("gate_up", HIDDEN, 2 * INTER), ("down", INTER, HIDDEN)):
        qw, qz, s = make_layer_dev(torch, K, N, dev, gen)
        x = torch.randn((M, K), device=dev, generator=gen).half()
        out = torch.empty((M, N), dtype=torch.float16, device=dev)
        tc = awq_b200.tc_supported(x, qw, qz, s, GS)
        path = awq_b200.AWQ_PATH_TC if tc else awq_b200.AWQ_PATH_DECODE
        flush = torch.empty(256 * 1024 * 1024, dtype=torch.uint8, device=dev)
        for _ in range(3):
            awq_b200.gemm(x, qw, qz, s, GS, path=path, out=out)
        reps = 5
        times = []
        for _ in range(reps):
            flush.zero_()                      # evict the 126 MB L2 between launches
            e0 = torch.cuda.Event(enable_timing=True)
            e1 = torch.cuda.Event(enable_timing=True)
            e0.record()
            awq_b200.gemm(x, qw, qz, s, GS, path=path, out=out)
            e1.record()
            torch.cuda.synchronize()
            times.append(e0.elapsed_time(e1))
        ms = statistics.median(times)
        flops = 2 * M * K * N
        tf = flops / (ms * 1e-3) / 1e12
        res[name] = {"K": K, "N": N, "ms": round(ms, 4), "tflops": round(tf, 1),
                     "frac": round(tf / tc_peak, 4),
                     "kernel": "tcgen05" if tc else "decode-fallback"}
        tot_flops += flops
        tot_ms += ms
        del qw, qz, s, x, out, flush
    tf = tot_flops / (tot_ms * 1e-3) / 1e12
    res["value"] = round(tf, 1)
    res["roofline"] = {"bound": "tensor", "achieved": round(tf, 1), "peak": tc_peak,
                       "unit": "TFLOP/s", "frac": round(tf / tc_peak, 4),
                       "peak_source": f"{peak_src} bf16 burst (fp16 rate is equal)"}
    return res


def decode_sweep(torch, lib, awq_b200, dev, hbm_peak):
    """Per-shape decode GB/s at M in {1,4,16}, weights rotated over a > 2x L2 pool."""
    gen = torch.Generator(device=dev).manual_seed(99)
    out = {}
    for name, (K, N) in SWEEP.items():
        per = alg_bytes(1, K, N)
        copies = max(2, int((300 << 20) // per) + 1)           # pool > 2x L2
        pool = [make_layer_dev(torch, K, N, dev, gen) for _ in range(copies)]
        for M in (1, 4, 16):
            x = torch.randn((M, K), device=dev, generator=gen).half()
            o = torch.empty((M, N), dtype=torch.float16, device=dev)
            for w in pool[:2]:
                awq_b200.gemm(x, *w, GS, out=o)
            reps = 200
            e0 = torch.cuda.Event(enable_timing=True)
            e1 = torch.cuda.Event(enable_timing=True)
            g = torch.cuda.CUDAGraph()
            with torch.cuda.graph(g):
                for r in range(copies):
                    awq_b200.gemm(x, *pool[r], GS, out=o)
            g.replay()
            torch.cuda.synchronize()
            nrep = max(1, reps // copies)
            e0.record()
            for _ in range(nrep):
                g.replay()
            e1.record()
            torch.cuda.synchronize()
            us = e0.elapsed_time(e1) * 1e3 / (nrep * copies)
            gbs = alg_bytes(M, K, N) / (us * 1e-6) / 1e9
            out[f"{name}_M{M}"] = {"us": round(us, 2), "GBps": round(gbs, 1),
                                   "frac": round(gbs / hbm_peak, 3),
                                   "kernel": "decode" if M <= 8 else "tcgen05-small"}
            del g
        del pool
    return out


# ------------------------------------------------------------------ reference arm ----
def run_reference(args):
    """The reference's own CPU implementation of the path (dequantize, then fp32 matmul on
    the host cores), on this arm's metric: W untimed and K timed steps, each step a bounded
    sample of the workload -- one Qwen2-7B layer's 4 linears at M=1 (1/28 of a decode
    token).  Rank 0 only; other ranks exit without work."""
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    if rank != 0:
        return
    import torch
    from oracle import oracle as O
    threads = O.cpu_threads()
    torch.set_num_threads(threads)
    g = torch.Generator().manual_seed(11)
    layers = []
    for _, K, N in STACK:
        qw = torch.randint(-2**31, 2**31, (K, N // 8), dtype=torch.int64, generator=g).to(torch.int32)
        qz = torch.randint(-2**31, 2**31, (K // GS, N // 8), dtype=torch.int64, generator=g).to(torch.int32)
        s = (torch.rand((K // GS, N), generator=g) * 0.018 + 0.002).half()
        x = torch.randn((1, K), generator=g).half()
        layers.append((x, qw, qz, s))
    step_bytes = sum(alg_bytes(1, K, N) for (_, K, N) in STACK)

    def step():
        for (x, qw, qz, s) in layers:
            O.torch_awq_gemm_f32(x, qw, qz, s)
    for _ in range(args.warmup):
        step()
    t0 = time.perf_counter()
    for _ in range(args.steps):
        step()
    secs = time.perf_counter() - t0
    value = step_bytes * args.steps / secs / 1e12
    sample = (f"{args.steps} steps of one Qwen2-7B layer (qkv, o, gate_up, down) at M=1: torch "
              f"dequant + fp32 matmul on {threads} host threads, {secs:.1f} s")
    print(json.dumps({
        "impl": "reference",
        "metric": "AWQ GEMM HBM TB/s (M=1 decode) & TFLOPS (M=2048 prefill), % of B200 roofline",
        "value": round(value, 6), "unit": "TB/s", "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": round(secs * 1e3 / args.steps, 3),
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32",
        "data": "synthetic (seeded random int4 AWQ weights, x ~ N(0,1); no checkpoint)",
        "config": {"workload": "decode M=1 through the AWQ linears of the 28-layer Qwen2-7B "
                               "stack (qkv 3584x4608, o 3584x3584, gate_up 3584x37888, down "
                               "18944x3584 per layer); each timed step is one layer's 4 linears",
                   "path": "reference dequantize-then-matmul on host cores (oracle port of "
                           "test/compare_benchmark.py:72-95 with an fp32 matmul)",
                   "group_size": GS},
        "cpu_baseline": {"value": round(value, 6), "unit": "TB/s", "cores": threads,
                         "kind": "port", "sample": sample},
        "e2e": {"value": round(value, 6), "unit": "TB/s", "h2d_bytes_per_step": 0,
                "d2h_bytes_per_step": 0},
    }))


def run_case(args):
    """One kernel on one shape, `--reps` launches (for ncu captures):
    --case decode:<shape>:<M> | prefill:<shape>:<M> | small:<shape>:<M> (tcgen05 small-M
    kernel) | silu:<shape>:<M> (product + SiLU-mul) | dequant:<shape>, shapes from SWEEP."""
    import torch

    import awq_b200
    kind, shape, *rest = args.case.split(":")
    K, N = SWEEP[shape]
    dev = torch.device("cuda", 0)
    gen = torch.Generator(device=dev).manual_seed(5)
    qw, qz, s = make_layer_dev(torch, K, N, dev, gen)
    if kind == "dequant":
        out = torch.empty((K, N), dtype=torch.float16, device=dev)
        for _ in range(args.reps):
            awq_b200.dequant(qw, qz, s, GS, out=out)
    elif kind == "silu":
        M = int(rest[0]) if rest else 1
        x = torch.randn((M, K), device=dev, generator=gen).half()
        out = torch.empty((M, N // 2), dtype=torch.float16, device=dev)
        for _ in range(args.reps):
            awq_b200.gemm_silu_mul(x, qw, qz, s, GS, out=out)
    else:
        M = int(rest[0]) if rest else {"decode": 1, "small": 16}.get(kind, 2048)
        x = torch.randn((M, K), device=dev, generator=gen).half()
        out = torch.empty((M, N), dtype=torch.float16, device=dev)
        path = {"decode": awq_b200.AWQ_PATH_DECODE, "small": awq_b200.AWQ_PATH_TS,
                "prefill": awq_b200.AWQ_PATH_TC}[kind]
        for _ in range(args.reps):
            awq_b200.gemm(x, qw, qz, s, GS, path=path, out=out)
    torch.cuda.synchronize()
    st = awq_b200.device_status()
    print(json.dumps({"case": args.case, "reps": args.reps, "status": st}))


def _max_over_ranks(torch, dev, world, v):
    if world == 1:
        return v
    import torch.distributed as dist
    t = torch.tensor([v], device=dev, dtype=torch.float64)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def _dev_time_ms(torch, dev, world, fn, reps, graph):
    """Device time of one fn() call: `reps` calls, as one CUDA-graph replay or eagerly,
    between CUDA events on the current stream; max over the ranks.  Every rank makes
    the same calls (collectives included)."""
    s = torch.cuda.Stream(device=dev)
    s.wait_stream(torch.cuda.current_stream(dev))
    with torch.cuda.stream(s):
        for _ in range(3):
            fn()
        g = None
        if graph:
            g = torch.cuda.CUDAGraph()
            with torch.cuda.graph(g, stream=s):
                for _ in range(reps):
                    fn()
            g.replay()
        torch.cuda.synchronize(dev)
        if world > 1:
            import torch.distributed as dist
            dist.barrier()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(s)
        if graph:
            g.replay()
        else:
            for _ in range(reps):
                fn()
        e1.record(s)
        torch.cuda.synchronize(dev)
    ms = e0.elapsed_time(e1) / reps
    del g
    return _max_over_ranks(torch, dev, world, ms)


def mlp_block_bench(torch, awq_b200, dev, world, rank, comm):
    """the Qwen2-7B MLP (model/qwen2.py:181-196: gate+up with SiLU-mul,
    then down) at M = 1, 16 and 512 over `world` GPUs through awq_b200.tp.TensorParallelMLP:
    gate+up split by columns in whole groups, down by the matching rows, the down output
    summed over the ranks (up to 16 tokens the fused decode kernel, above the prefill
    product and the library's all-reduce kernel over NVLink; NCCL where neither runs).
    Also, per call, the rank's down product alone, the same product with the library's
    all-reduce (`down_fused_allreduce_us`), and the product followed by an NCCL
    all-reduce of the [M, 3584] fp16 output: the all-reduce's cost is the difference."""
    import torch.distributed as dist

    from awq_b200 import tp
    gen = torch.Generator(device=dev).manual_seed(555)     # the same full weights on every rank
    gu = tp.AWQWeights(*make_layer_dev(torch, HIDDEN, 2 * INTER, dev, gen))
    dn = tp.AWQWeights(*make_layer_dev(torch, INTER, HIDDEN, dev, gen))
    mlp = tp.TensorParallelMLP(gu, dn, INTER, world, rank, comm=comm if world > 1 else None)
    del gu
    wbytes = alg_bytes(1, HIDDEN, 2 * INTER) + alg_bytes(1, INTER, HIDDEN)
    out = {"what": "TensorParallelMLP: gate+up (SiLU-mul fused) and down, all-reduce of the "
                   "down output across the ranks", "n_gpus": world}
    w = mlp.down.w
    for M in (1, 16, 512):
        x = torch.randn((M, HIDDEN), device=dev, generator=gen).half()
        graph = M <= 16                    # decode: replayed from a CUDA graph
        ms = _dev_time_ms(torch, dev, world, lambda: mlp(x), 20, graph)
        h = torch.randn((M, mlp.inter_local), device=dev, generator=gen).half()
        prod_ms = _dev_time_ms(torch, dev, world, lambda: awq_b200.gemm(h, w.qweight, w.qzeros,
                                                                       w.scales, GS), 20, graph)
        row = {"us": round(ms * 1e3, 2), "weight_TBps": round(wbytes / (ms * 1e-3) / 1e12, 3),
               "down_product_us": round(prod_ms * 1e3, 2), "allreduce_bytes": M * HIDDEN * 2}
        if world > 1:
            if mlp.down.fused_for(M):
                f_ms = _dev_time_ms(torch, dev, world, lambda: awq_b200.gemm_allreduce(
                    h, w.qweight, w.qzeros, w.scales, GS, comm), 20, graph)
                row["down_fused_allreduce_us"] = round(f_ms * 1e3, 2)
                row["fused_allreduce_cost_us"] = round((f_ms - prod_ms) * 1e3, 2)

            def prod_nccl():
                y = awq_b200.gemm(h, w.qweight, w.qzeros, w.scales, GS)
                dist.all_reduce(y)
            n_ms = _dev_time_ms(torch, dev, world, prod_nccl, 20, False)
            row["down_nccl_allreduce_us"] = round(n_ms * 1e3, 2)
            row["nccl_allreduce_cost_us"] = round((n_ms - prod_ms) * 1e3, 2)
            row["block_allreduce"] = (("fused decode kernel" if M <= 16 else
                                       "prefill product + NVLink all-reduce kernel")
                                      if mlp.down.fused_for(M) else "nccl")
        out[f"M{M}"] = row
    st = awq_b200.device_status()
    out["device_status"] = st
    del mlp, dn
    torch.cuda.empty_cache()
    return out


def stack_bench(torch, awq_b200, dev, world, rank, comm, args):
    """the 28-layer Qwen2-7B linear stack (fused q/k/v with bias, o,
    gate+up, down per layer; random AWQ weights) with RMSNorm and the residual adds as
    torch ops between the linears, a prefill of `--prefill` tokens, then `--decode` decode
    steps at batch 1, each one CUDA-graph replay of the 28 layers.  Over `world` GPUs the
    attention linears are split by whole heads (AttentionLinearsTP) and the MLP by whole
    groups (TensorParallelMLP), with the all-reduces of o and down.  The drop-in's fused
    calls stand where the reference has two kernels: the q/k/v bias in the product
    (model/qwen2.py:108-109) and SiLU-mul with the gate+up product (:181-194).  Attention
    itself is not part of the linear stack: o reads the rank's query columns of q/k/v in
    its place."""
    from awq_b200 import tp
    gen = torch.Generator(device=dev).manual_seed(4321)     # the same full weights everywhere
    eps = 1e-6
    layers = []
    for _ in range(LAYERS):
        qkv = tp.AWQWeights(*make_layer_dev(torch, HIDDEN, 4608, dev, gen),
                            bias=(torch.randn(4608, device=dev, generator=gen) * 0.1).half())
        o = tp.AWQWeights(*make_layer_dev(torch, HIDDEN, HIDDEN, dev, gen))
        gu = tp.AWQWeights(*make_layer_dev(torch, HIDDEN, 2 * INTER, dev, gen))
        dn = tp.AWQWeights(*make_layer_dev(torch, INTER, HIDDEN, dev, gen))
        attn = tp.AttentionLinearsTP(qkv, o, 28, 4, 128, world, rank, comm=comm)
        mlp = tp.TensorParallelMLP(gu, dn, INTER, world, rank, comm=comm)
        n1 = torch.ones(HIDDEN, dtype=torch.float16, device=dev)
        n2 = torch.ones(HIDDEN, dtype=torch.float16, device=dev)
        layers.append((attn, mlp, n1, n2))
        del qkv, gu

    def rms(h, w):
        hf = h.float()
        return (hf * torch.rsqrt(hf.pow(2).mean(-1, keepdim=True) + eps)).half() * w

    def forward(h):
        for attn, mlp, n1, n2 in layers:
            q, _, _ = attn.project_qkv(rms(h, n1))
            h = h + attn.project_o(q.contiguous())
            h = h + mlp(rms(h, n2))
        return h

    x = (torch.randn((args.prefill, HIDDEN), device=dev, generator=gen) * 0.1).half()
    prefill_ms = _dev_time_ms(torch, dev, world, lambda: forward(x), 1, False)
    tok = (torch.randn((1, HIDDEN), device=dev, generator=gen) * 0.1).half()
    s = torch.cuda.Stream(device=dev)
    s.wait_stream(torch.cuda.current_stream(dev))
    with torch.cuda.stream(s):
        for _ in range(3):
            forward(tok)
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, stream=s):
            nxt = forward(tok)
        g.replay()
        torch.cuda.synchronize(dev)
        if world > 1:
            import torch.distributed as dist
            dist.barrier()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(s)
        for _ in range(args.decode):
            g.replay()
            tok.copy_(nxt)                                   # the step's output feeds the next
        e1.record(s)
        torch.cuda.synchronize(dev)
    decode_ms = _max_over_ranks(torch, dev, world, e0.elapsed_time(e1) / args.decode)
    st = awq_b200.device_status()
    del g
    layers.clear()
    torch.cuda.empty_cache()
    w_bytes = LAYERS * sum(alg_bytes(1, K, N) for _, K, N in STACK)
    return {"metric": "Qwen2-7B AWQ linear stack, batch 1 (config 5)", "n_gpus": world,
            "prefill_tokens": args.prefill, "prefill_ms": round(prefill_ms, 3),
            "prefill_tokens_per_s": round(args.prefill / prefill_ms * 1e3, 1),
            "decode_steps": args.decode, "decode_ms_per_token": round(decode_ms, 4),
            "decode_tokens_per_s": round(1e3 / decode_ms, 1),
            "decode_weight_TBps": round(w_bytes / (decode_ms * 1e-3) / 1e12, 4),
            "between_layers": "torch RMSNorm and residual adds; q/k/v bias and SiLU-mul fused",
            "device_status": st, "data": "synthetic (random int4 AWQ weights, no checkpoint)"}


def run_stack(args):
    """Only the config-5 leg (``--stack``), on one GPU or under torchrun."""
    import torch
    import torch.distributed as dist

    import awq_b200
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    comm = None
    if world > 1:
        import datetime
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=dev)
        comm = awq_b200.TPComm.from_group(HIDDEN)
    res = stack_bench(torch, awq_b200, dev, world, rank, comm, args)
    if world > 1:
        torch.cuda.synchronize()
        dist.barrier()
        comm.close()
        dist.destroy_process_group()
    if rank == 0:
        emit_json(res)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--case", default=None,
                    help="profile one kernel: decode:<shape>:<M>, prefill:<shape>:<M>, dequant:<shape>")
    ap.add_argument("--reps", type=int, default=3)
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=100)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--cpu-seconds", type=float, default=12.0)
    ap.add_argument("--stack", action="store_true",
                    help="config 5: prefill + decode through the 28-layer linear stack (1 GPU)")
    ap.add_argument("--prefill", type=int, default=1024)
    ap.add_argument("--decode", type=int, default=512)
    args = ap.parse_args()
    if args.warmup < 3:
        args.warmup = 3
    if args.case:
        run_case(args)
    elif args.stack:
        run_stack(args)
    elif args.impl == "reference":
        run_reference(args)
    else:
        run_ours(args)


if __name__ == "__main__":
    main()
