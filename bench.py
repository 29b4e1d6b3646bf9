"""Benchmark of the fake-quantization hot path on B200.

Headline (one JSON line on rank 0): fake-quant GB/s on configuration 2 of the baseline --
MXFP4 EVEN fake-quant of the fused gate/up weight [24576, 4096] (values + STE bit mask)
and MXFP4 CEIL fake-quant of the activations [16384, 4096] -- where one step is one pass
of both kernels over inputs already resident in HBM (both larger than the 126 MB L2).
``value`` counts algorithmic bytes (read 2 + write 2 + mask 1/8 B per weight element,
read 2 + write 2 B per activation element) over the max-over-ranks device time.

Also reported: ``e2e`` (the same metric through the public ``qatfactory_b200.quant`` API
from pinned host buffers, copies included), ``roofline`` for the dominant kernel,
``cpu_baseline`` (the CPU oracle on the host cores, a bounded sample), ``clocks`` sampled
during the timed region, per-kernel timings of the other configurations (``kernels``) and the
configuration-5 QAD student step at this GPU count (``qad``: tokens/s, FSDP2 over all ranks).

    python bench.py [--gpus N --steps K --warmup W] [--impl reference]

Multi-GPU (torchrun, one process per GPU): every rank fake-quantizes its own copy of the
workload (row shards of a larger model need no exchange for MXFP4), so scaling is weak.
"""

from __future__ import annotations

import argparse
import gc
import json
import os
import statistics
import subprocess
import sys
import tempfile
import time
from pathlib import Path

import torch
import torch.distributed as dist

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

METRIC = "fake-quant GB/s vs HBM peak; QAD step tokens/s at 1/2/4/8 B200"
UNIT = "GB/s"
W_SHAPE = (24576, 4096)
X_SHAPE = (16384, 4096)


def algorithmic_bytes_config2() -> tuple[int, int]:
    nw = W_SHAPE[0] * W_SHAPE[1]
    nx = X_SHAPE[0] * X_SHAPE[1]
    return nw * 4 + nw // 8, nx * 4


def config2_config(world: int) -> dict:
    """The headline workload, named identically by both arms."""

    return {"workload": "config2: MXFP4 fake-quant of gate/up weight [24576,4096] (EVEN, +STE mask) "
                        "+ activations [16384,4096] (CEIL)", "io_dtype": "bf16",
            "l2": "inputs larger than L2 (201 MB + 134 MB); no flush", "parallelism": f"replicas{world}"}


def reference_formula_rate(world: int, ms_per_step: float) -> dict:
    """The headline step's rate under the reference benchmark's byte count
    (benchmarks/bench_fp4_fake_quant.py:80-82: 2 x tensor bytes + elements x mask bytes, a one-byte
    bool mask for the masked weight QDQ and none for the activations), for continuity with its
    published figures; ``value`` counts the mask as the bits that are written."""

    w_elems = W_SHAPE[0] * W_SHAPE[1]
    x_elems = X_SHAPE[0] * X_SHAPE[1]
    per_step = (2 * 2 * w_elems + w_elems) + 2 * 2 * x_elems
    return {"value": round(world * per_step / (ms_per_step * 1e-3) / 1e9, 2), "unit": "GB/s",
            "bytes_per_step_per_gpu": per_step}


def measured_peaks() -> dict:
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        d["_source"] = "measured"
        return d
    return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "_source": "fallback"}


# ----------------------------------------------------------------------------- clocks
class ClockSampler:
    """nvidia-smi clocks and throttle reasons sampled every 200 ms during a region."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, index: int):
        self.index = index
        self.proc = None
        self.path = None

    def __enter__(self):
        fd, self.path = tempfile.mkstemp(suffix=".csv")
        os.close(fd)
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", "-i", str(self.index), f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                 "-lms", "100", "-f", self.path], stdout=subprocess.DEVNULL, stderr=subprocess.DEVNULL)
            time.sleep(0.3)  # let the first sample land before the loaded window starts
        except OSError:
            self.proc = None
        return self

    def __exit__(self, *exc):
        if self.proc is not None:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()

    def summary(self) -> dict:
        rows = []
        if self.path and Path(self.path).exists():
            for line in Path(self.path).read_text().splitlines():
                parts = [p.strip() for p in line.split(",")]
                if len(parts) >= 9:
                    rows.append(parts)
            os.unlink(self.path)
        if not rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"], "samples": 0}
        def num(v):
            try:
                return float(v)
            except ValueError:
                return None
        sm = [num(r[1]) for r in rows if num(r[1]) is not None]
        smax = max((num(r[2]) for r in rows if num(r[2]) is not None), default=None)
        names = ("hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap")
        reasons = sorted({n for r in rows for n, v in zip(names, r[5:9]) if v.lower() == "active"})
        loaded = [s for s in sm if smax and s >= 0.5 * smax] or sm
        return {"sm_mhz": statistics.median(loaded) if loaded else None, "sm_max_mhz": smax,
                "reasons": reasons, "samples": len(rows),
                "power_w_max": max((num(r[3]) for r in rows if num(r[3]) is not None), default=None)}


# ------------------------------------------------------------------------------ timing
def keep_loaded(fn, seconds: float, stream) -> None:
    """Run ``fn`` back to back for about ``seconds`` (untimed), so the clock sampler sees the
    GPU under the same load just before and just after the timed region."""

    t_end = time.perf_counter() + seconds
    while time.perf_counter() < t_end:
        for _ in range(50):
            fn()
        stream.synchronize()


def time_region(fn, steps: int, stream: torch.cuda.Stream) -> float:
    """Total ms of ``steps`` calls, CUDA events on the launching stream."""

    start = torch.cuda.Event(enable_timing=True)
    end = torch.cuda.Event(enable_timing=True)
    torch.cuda.synchronize()
    start.record(stream)
    for _ in range(steps):
        fn()
    end.record(stream)
    end.synchronize()
    return start.elapsed_time(end)


def time_each_launch(fn, iters: int, stream, flush: torch.Tensor | None) -> float:
    """Average ms of one launch, L2 flushed between launches: a write of the first half of
    ``flush`` (larger than L2), then a read of its second half (also larger than L2), so the
    flush's dirty lines are written back before the timed launch starts rather than during it."""

    total = 0.0
    half = flush.numel() // 2 if flush is not None else 0
    for _ in range(iters):
        if flush is not None:
            flush[:half].zero_()
            flush[half:].sum()
        s = torch.cuda.Event(enable_timing=True)
        e = torch.cuda.Event(enable_timing=True)
        s.record(stream)
        fn()
        e.record(stream)
        e.synchronize()
        total += s.elapsed_time(e)
    return total / iters


def graphed(fn):
    """``fn`` captured once in a CUDA graph (outputs allocated from the graph's pool), so a timed
    replay carries no host-side argument checks or allocations between the flush and the kernel.
    Returns (replay, outputs); keep the outputs alive while replaying."""

    side = torch.cuda.Stream()
    side.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(side):
        for _ in range(2):
            fn()
    torch.cuda.current_stream().wait_stream(side)
    torch.cuda.synchronize()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        outs = fn()
    graph.replay()
    torch.cuda.synchronize()
    return graph.replay, (graph, outs)


def max_over_ranks(v: float, dev) -> float:
    if dist.is_initialized():
        t = torch.tensor([v], dtype=torch.float64, device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())
    return v


def barrier_sync():
    if dist.is_initialized():
        dist.barrier()
    torch.cuda.synchronize()


# ---------------------------------------------------------------------------- CPU side
def cpu_baseline() -> dict:
    """The CPU oracle (plain-C restatement of the reference, OpenMP over all host threads) on
    the whole of configuration 2, median of three passes; beside it the reference's own torch
    CPU functions (``_fake_quantize_mxfp4_torch`` / ``_fake_quantize_mxfp4_activation_torch``
    from ``baseline/_ref``) on a 1/8 row sample, all host threads."""

    import oracle
    from qatfactory_b200 import workloads

    cores = len(os.sched_getaffinity(0))
    oracle.set_num_threads(cores)
    w = workloads.config2_weight()
    x = workloads.config2_activation()
    oracle.mxfp4_qdq_even(w[:64])
    times = []
    for _ in range(3):
        t0 = time.perf_counter()
        oracle.mxfp4_qdq_even(w)
        oracle.mxfp4_qdq_ceil(x)
        times.append(time.perf_counter() - t0)
    dt = statistics.median(times)
    nbytes = w.numel() * 4 + w.numel() // 8 + x.numel() * 4
    line = {"value": round(nbytes / dt / 1e9, 3), "unit": UNIT, "cores": cores, "kind": "port",
            "sample": f"all of configuration 2 (MXFP4 EVEN [24576,4096] + CEIL [16384,4096] bf16), median of 3 "
                      f"passes, {dt:.2f} s per pass"}
    if reference_quant() is not None:
        from qatfactory.quant.formats import mxfp4 as rmx

        torch.set_num_threads(cores)
        ws, xs = w[: W_SHAPE[0] // 8].contiguous(), x[: X_SHAPE[0] // 8].contiguous()
        rmx._fake_quantize_mxfp4_torch(ws[:64])
        rt = []
        for _ in range(3):
            t0 = time.perf_counter()
            rmx._fake_quantize_mxfp4_torch(ws)
            rmx._fake_quantize_mxfp4_activation_torch(xs)
            rt.append(time.perf_counter() - t0)
        rdt = statistics.median(rt)
        rbytes = ws.numel() * 4 + ws.numel() // 8 + xs.numel() * 4
        line["reference_torch"] = {
            "value": round(rbytes / rdt / 1e9, 3), "unit": UNIT, "cores": cores, "kind": "reference",
            "isa": torch.backends.cpu.get_cpu_capability(),
            "sample": f"reference torch CPU functions on rows 1/8 of configuration 2 ([3072,4096] + [2048,4096]), "
                      f"median of 3, {rdt:.2f} s per pass"}
    return line


def run_reference(args) -> None:
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    import oracle
    from qatfactory_b200 import workloads

    cores = len(os.sched_getaffinity(0))
    oracle.set_num_threads(cores)
    # each step is the whole of configuration 2 (about a quarter second on the host's cores)
    w = workloads.config2_weight()
    x = workloads.config2_activation()
    nbytes = w.numel() * 4 + w.numel() // 8 + x.numel() * 4
    for _ in range(args.warmup):
        oracle.mxfp4_qdq_even(w)
        oracle.mxfp4_qdq_ceil(x)
    t0 = time.perf_counter()
    for _ in range(args.steps):
        oracle.mxfp4_qdq_even(w)
        oracle.mxfp4_qdq_ceil(x)
    dt = time.perf_counter() - t0
    value = nbytes * args.steps / dt / 1e9
    sample = ("all of configuration 2 per step: MXFP4 EVEN [24576,4096] + CEIL [16384,4096] bf16, by the plain-C "
              "restatement of the reference's torch functions (OpenMP), in the rank-0 process only")
    emit({
        "impl": "reference", "metric": METRIC, "value": round(value, 3), "unit": UNIT, "n_gpus": args.gpus,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(dt * 1e3 / args.steps, 3),
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "config": config2_config(args.gpus),
        "cpu_baseline": {"value": round(value, 3), "unit": UNIT, "cores": cores, "kind": "port", "sample": sample},
        "e2e": {"value": round(value, 3), "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    })


# ------------------------------------------------------------------------- GPU bench
# FP32 operations per weight of the Q4_K grid-search fake quant (q4_k.py:68-190): prelude
# (squares, weights, extrema, the initial error: 17), 21 trial steps of 17 (scaled offset,
# rounding, clamp, three weighted sums and the trial error), level-2 re-encode and
# reconstruction (10).
Q4K_GRID_OPS_PER_ELEMENT = 17 + 21 * 17 + 10


def fp32_simt_peak_tops(dev, peaks) -> float:
    """SMs x 128 FP32 lanes x the maximum SM clock, in T operations/s."""

    sms = torch.cuda.get_device_properties(dev).multi_processor_count
    return sms * 128 * float(peaks.get("sm_max_mhz", 1965.0)) * 1e6 / 1e12


def kernel_table(dev, stream, flush, peaks) -> dict:
    """Per-launch timings of the other hot-path kernels: each call captured in a CUDA graph and
    replayed with L2 flushed between launches."""

    from qatfactory_b200 import _native, workloads
    from qatfactory_b200.quant import quantize_nvfp4

    hbm = peaks["hbm_gbs"]
    out = {}

    def rec(name, fn, nbytes, iters=10):
        replay, keep = graphed(fn)
        for _ in range(3):
            replay()
        ms = time_each_launch(replay, iters, stream, flush)
        del keep
        gbs = nbytes / (ms * 1e-3) / 1e9
        out[name] = {"us": round(ms * 1e3, 2), "GB/s": round(gbs, 1), "frac": round(gbs / hbm, 3), "bytes": nbytes}

    # configuration 1 is a single 32 MB weight, smaller than L2: its kernels are timed as a
    # back-to-back stream over 8 distinct copies (256 MB, every launch reads cold data), the way
    # a training step quantizes one layer's weights after another; the host's enqueue cost is
    # then hidden behind the GPU instead of inflating each launch
    w1 = workloads.config1_weight().to(dev)
    g1 = workloads.config1_grad().to(dev)
    n1 = w1.numel()
    copies = 8
    ws = [w1.clone() for _ in range(copies)]
    gs = [g1.clone() for _ in range(copies)]
    amaxes = [_native.tensor_amax(w) for w in ws]
    masks = [_native.nvfp4_qdq(w, a)[1] for w, a in zip(ws, amaxes)]

    def rec_stream(name, fn, nbytes, rounds=4):
        # the launches of one round are captured in a CUDA graph so that the host's per-call
        # cost (argument checks, output allocation) stays out of the device time
        for _ in range(2):
            outs = [fn(i) for i in range(copies)]
            del outs
        torch.cuda.synchronize()
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph):
            outs = [fn(i) for i in range(copies)]
        graph.replay()
        torch.cuda.synchronize()
        ms = time_region(graph.replay, rounds, stream) / (rounds * copies)
        del graph, outs
        gbs = nbytes / (ms * 1e-3) / 1e9
        out[name] = {"us": round(ms * 1e3, 2), "GB/s": round(gbs, 1), "frac": round(gbs / hbm, 3), "bytes": nbytes,
                     "timing": f"CUDA graph of {copies} launches on distinct 32 MB copies (cold data each launch)"}

    rec_stream("config1.amax", lambda i: _native.tensor_amax(ws[i], amaxes[i]), n1 * 2)
    rec_stream("config1.nvfp4_qdq", lambda i: _native.nvfp4_qdq(ws[i], amaxes[i]), n1 * 4 + n1 // 8)
    rec_stream("config1.ste_backward", lambda i: _native.ste_backward(gs[i], masks[i]), n1 * 4 + n1 // 8)
    rec_stream("config1.nvfp4_pack", lambda i: _native.nvfp4_pack(ws[i], amaxes[i], recon=False),
               n1 * 2 + n1 // 2 + n1 // 16)
    del w1, g1, ws, gs, masks
    x4 = workloads.config4_inputs()[0].to(dev)
    xa = _native.tensor_amax(x4)
    n4 = x4.numel()
    rec("config4.x_nvfp4_qdq", lambda: _native.nvfp4_qdq(x4, xa), n4 * 4 + n4 // 8)
    rec("config4.x_nvfp4_pack", lambda: _native.nvfp4_pack(x4, xa, recon=False), n4 * 2 + n4 // 2 + n4 // 16)
    del x4
    w2 = workloads.config2_weight().to(dev)
    n2 = w2.numel()
    rec("config2.mxfp4_pack[weight]", lambda: _native.mxfp4_pack(w2, recon=False), n2 * 2 + n2 // 2 + n2 // 32)
    del w2
    layer = workloads.config3_layer(0)
    gate = layer[4][1].to(dev)
    ng = gate.numel()
    rec("config3.q4k_minmax_pack[gate]", lambda: _native.q4k_encode(gate, "minmax", recon=False, mask=False),
        ng * 2 + ng * 144 // 256)
    rec("config3.q4k_minmax_fakequant[gate]", lambda: _native.q4k_encode(gate, "minmax", blocks=False),
        ng * 4 + ng // 8)
    rec("config3.q4k_grid_fakequant[gate]", lambda: _native.q4k_encode(gate, "grid_search", blocks=False),
        ng * 4 + ng // 8, iters=3)
    # the grid search is bound by FP32 arithmetic, not HBM: its algorithmic operation count is
    # Q4K_GRID_OPS_PER_ELEMENT (the 21-step weighted least-squares search of make_qkx2 plus the
    # level-2 re-encode, counted from the reference expressions), against the scalar FP32
    # issue peak of the SMs at their maximum clock
    g = out["config3.q4k_grid_fakequant[gate]"]
    tops = Q4K_GRID_OPS_PER_ELEMENT * ng / (g["us"] * 1e-6) / 1e12
    fp32_peak = fp32_simt_peak_tops(dev, peaks)
    out["config3.q4k_grid_fakequant[gate]"] = {"us": g["us"], "TFLOP/s": round(tops, 2),
                                               "frac": round(tops / fp32_peak, 3),
                                               "peak": f"scalar FP32 SIMT {fp32_peak:.1f} TFLOP/s"}
    blocks = _native.q4k_encode(gate, "minmax", recon=False, mask=False)[0]
    rec("config3.q4k_dequant[gate]", lambda: _native.q4k_dequant(blocks, gate.shape[1]), ng * 144 // 256 + ng * 4)
    return out


FP4_DENSE_NOMINAL_TFLOPS = 9000.0  # B200 dense FP4 tensor rate (nominal; no measured FP4 peak exists)


def cublas_nvfp4_comparator(x, xa, w, wa):
    """A callable running cuBLASLt's block-scaled NVFP4 GEMM (torch._scaled_mm with E2M1
    operands and E4M3 block-16 scales in cuBLAS's 128 x 4 blocked layout) on the codes and scales
    of ``quantize_nvfp4`` for x and w, or None when this torch cannot run it.  Used only as a
    measured comparator for the tcgen05 FP4 GEMM; its result is checked against ours first."""

    from qatfactory_b200 import _native

    def blocked(sc):
        r, c = sc.shape
        b = sc.view(r // 128, 128, c // 4, 4).permute(0, 2, 1, 3)
        return b.reshape(-1, 4, 32, 4).transpose(1, 2).reshape(-1, 32, 16).flatten()

    try:
        px, sxr, _, _ = _native.nvfp4_pack(x, xa, recon=False)
        pw, swr, _, _ = _native.nvfp4_pack(w, wa, recon=False)
        a4, b4 = px.view(torch.float4_e2m1fn_x2), pw.view(torch.float4_e2m1fn_x2)
        sa, sb = blocked(sxr.view(torch.float8_e4m3fn)), blocked(swr.view(torch.float8_e4m3fn))

        def run():
            return torch._scaled_mm(a4, b4.t(), sa, sb, out_dtype=torch.bfloat16)

        cx, sx, _, _ = _native.nvfp4_operand(x, xa, _native.OPERAND_A)
        cw, sw, _, _ = _native.nvfp4_operand(w, wa, _native.OPERAND_B)
        ours = _native.nvfp4_gemm(cx, sx, xa, cw, sw, wa).float()
        theirs = run().float() * ((xa / 2688.0) * (wa / 2688.0))
        if float((theirs - ours).norm() / ours.norm()) > 1e-2:
            return None
        return run
    except (RuntimeError, TypeError, AttributeError, ValueError):
        return None


def w4a4_table(dev, stream, flush, peaks) -> dict:
    """Configuration 4 (NVFP4 W4A4 fused-QKV linear, X [16384,4096], W [6144,4096], dY
    [16384,6144]): the operand quantizers, the block-scaled FP4 forward GEMM and the two BF16
    backward GEMMs, each launch timed alone with L2 flushed, next to cuBLAS BF16 (torch) on the
    same dequantized operands, which is what the reference's F.linear runs."""

    from qatfactory_b200 import _native, workloads

    x, w, dy = (t.to(dev) for t in workloads.config4_inputs())
    m, k = x.shape
    n = w.shape[0]
    xa, wa = _native.tensor_amax(x), _native.tensor_amax(w)
    out = {}

    def timed(fn, iters=10, graph=True):
        keep = None
        if graph:
            fn, keep = graphed(fn)
        for _ in range(3):
            fn()
        ms = time_each_launch(fn, iters, stream, flush)
        del keep
        return ms

    def rec_bytes(name, fn, nbytes):
        ms = timed(fn)
        gbs = nbytes / (ms * 1e-3) / 1e9
        out[name] = {"us": round(ms * 1e3, 2), "GB/s": round(gbs, 1), "frac": round(gbs / peaks["hbm_gbs"], 3),
                     "bytes": nbytes}

    def rec_flops(name, fn, flops, peak, peak_name, graph=True):
        ms = timed(fn, graph=graph)
        tf = flops / (ms * 1e-3) / 1e12
        out[name] = {"us": round(ms * 1e3, 2), "TFLOP/s": round(tf, 1), "frac": round(tf / peak, 3),
                     "peak": f"{peak_name} {peak}"}

    # algorithmic bytes: read BF16; write deq, codes, one scale byte per block and mask bits (the
    # scale layouts store each scale four times, once per TMEM lane quarter: 3/16 B/element more
    # written, a layout choice not counted here)
    per_elt = 2 + 2 + 0.5 + 1 / 16 + 1 / 8
    rec_bytes("config4.x_operand", lambda: _native.nvfp4_operand(x, xa, _native.OPERAND_A), int(m * k * per_elt))
    rec_bytes("config4.w_operand", lambda: _native.nvfp4_operand(w, wa, _native.OPERAND_B), int(n * k * per_elt))
    cx, sx, dxq, mx = _native.nvfp4_operand(x, xa, _native.OPERAND_A)
    cw, sw, dwq, mw = _native.nvfp4_operand(w, wa, _native.OPERAND_B)
    flops = 2.0 * m * n * k
    bf16_peak = peaks["bf16_tflops"]
    rec_flops("config4.fwd_nvfp4_gemm", lambda: _native.nvfp4_gemm(cx, sx, xa, cw, sw, wa), flops,
              FP4_DENSE_NOMINAL_TFLOPS, "nominal dense FP4")
    # the same forward with X quantized inside the FP4 GEMM (one launch; deq and mask for the
    # backward written by its quantizer warps), against the two launches above
    rec_flops("config4.fwd_fused_linear", lambda: _native.nvfp4_linear_fwd(x, xa, cw, sw, wa), flops,
              FP4_DENSE_NOMINAL_TFLOPS, "nominal dense FP4 (activation quantization inside)")
    cub = cublas_nvfp4_comparator(x, xa, w, wa)
    if cub is not None:
        # a measured FP4 comparator: cuBLASLt's block-scaled NVFP4 GEMM (through torch) on the
        # same codes and E4M3 block scales, the tensor scales applied afterwards
        rec_flops("config4.cublas_nvfp4_fwd", cub, flops, FP4_DENSE_NOMINAL_TFLOPS, "nominal dense FP4")
        out["config4.fwd_nvfp4_gemm"]["frac_of_cublas_nvfp4"] = round(
            out["config4.cublas_nvfp4_fwd"]["us"] / out["config4.fwd_nvfp4_gemm"]["us"], 3)
    rec_flops("config4.dgrad_bf16_gemm", lambda: _native.bf16_gemm(dy, _native.K_MAJOR, dwq, _native.MN_MAJOR, mx),
              flops, bf16_peak, "measured bf16")
    rec_flops("config4.wgrad_bf16_gemm", lambda: _native.bf16_gemm(dy, _native.MN_MAJOR, dxq, _native.MN_MAJOR, mw),
              flops, bf16_peak, "measured bf16")
    rec_flops("config4.cublas_bf16_fwd", lambda: torch.nn.functional.linear(dxq, dwq), flops, bf16_peak,
              "measured bf16")
    rec_flops("config4.cublas_bf16_dgrad", lambda: dy @ dwq, flops, bf16_peak, "measured bf16")
    rec_flops("config4.cublas_bf16_wgrad", lambda: dy.T @ dxq, flops, bf16_peak, "measured bf16")
    del cx, sx, dxq, mx, cw, sw, dwq, mw

    # one training step of the layer through the public module (forward + backward), against
    # the reference's formulation of the same step: fake-quantized operands into cuBLAS BF16
    from qatfactory_b200.quant.formats.nvfp4 import (NVFP4Linear, fake_quantize_nvfp4,
                                                      fake_quantize_nvfp4_activation)

    lin = NVFP4Linear.from_linear(torch.nn.Linear(k, n, bias=False, device=dev, dtype=torch.bfloat16))
    with torch.no_grad():
        lin.weight.copy_(w)
    lin._quantize_activations = True
    lin._input_amax_static = xa.clone()
    xg = x.detach().requires_grad_(True)

    def layer_step():
        xg.grad = None
        lin.weight.grad = None
        lin(xg).backward(dy)

    wr = lin.weight.detach().clone().requires_grad_(True)

    def reference_step():
        xg.grad = None
        wr.grad = None
        torch.nn.functional.linear(fake_quantize_nvfp4_activation(xg, xa), fake_quantize_nvfp4(wr)).backward(dy)

    step_flops = 3 * flops
    # whole steps run eagerly (autograd), host work between their launches included
    rec_flops("config4.layer_step_w4a4", layer_step, step_flops, bf16_peak, "measured bf16 (3 GEMMs)", graph=False)
    rec_flops("config4.layer_step_reference_formulation", reference_step, step_flops, bf16_peak,
              "measured bf16 (3 GEMMs)", graph=False)
    err = int(_native.gemm_error_word(dev))
    if err:
        raise RuntimeError(f"tcgen05 GEMM reported error word {err}")
    return out


def mxfp4_w4a4_table(dev, stream, flush, peaks) -> dict:
    """Configuration 2's tensors as an MXFP4 W4A4 linear (X [16384,4096] CEIL, the fused gate/up
    W [24576,4096] EVEN): the MXFP4 operand quantizers, the tcgen05 kind::mxf4 forward GEMM next
    to cuBLASLt's block-scaled MXFP4 GEMM and cuBLAS BF16 on the dequantized operands, and one
    forward + backward of MXFP4Linear against the reference's formulation."""

    from qatfactory_b200 import _native, workloads
    from qatfactory_b200.quant.formats.mxfp4 import MXFP4Linear, fake_quantize_mxfp4, fake_quantize_mxfp4_activation

    x = workloads.config2_activation().to(dev)
    w = workloads.config2_weight().to(dev)
    m, k = x.shape
    n = w.shape[0]
    out = {}

    def timed(fn, iters=10, graph=True):
        keep = None
        if graph:
            fn, keep = graphed(fn)
        for _ in range(3):
            fn()
        ms = time_each_launch(fn, iters, stream, flush)
        del keep
        return ms

    def rec_bytes(name, fn, nbytes):
        ms = timed(fn)
        gbs = nbytes / (ms * 1e-3) / 1e9
        out[name] = {"us": round(ms * 1e3, 2), "GB/s": round(gbs, 1), "frac": round(gbs / peaks["hbm_gbs"], 3),
                     "bytes": nbytes}

    def rec_flops(name, fn, flops, peak, peak_name, graph=True, iters=10):
        ms = timed(fn, iters=iters, graph=graph)
        tf = flops / (ms * 1e-3) / 1e12
        out[name] = {"us": round(ms * 1e3, 2), "TFLOP/s": round(tf, 1), "frac": round(tf / peak, 3),
                     "peak": f"{peak_name} {peak}"}

    A, B = _native.OPERAND_A, _native.OPERAND_B
    # algorithmic bytes: read BF16; write deq, codes, one E8M0 byte per 32 elements (and the
    # weight's mask bits)
    rec_bytes("config2.x_mx_operand", lambda: _native.mxfp4_operand(x, A, _native.MXFP4_CEIL, mask=False),
              int(m * k * (2 + 2 + 0.5 + 1 / 32)))
    rec_bytes("config2.w_mx_operand", lambda: _native.mxfp4_operand(w, B, _native.MXFP4_EVEN),
              int(n * k * (2 + 2 + 0.5 + 1 / 32 + 1 / 8)))
    cx, sx, xq, _ = _native.mxfp4_operand(x, A, _native.MXFP4_CEIL, mask=False)
    cw, sw, wq, mw = _native.mxfp4_operand(w, B, _native.MXFP4_EVEN)
    flops = 2.0 * m * n * k
    bf16_peak = peaks["bf16_tflops"]
    rec_flops("config2.fwd_mxfp4_gemm", lambda: _native.mxfp4_gemm(cx, sx, cw, sw), flops, FP4_DENSE_NOMINAL_TFLOPS,
              "nominal dense FP4")
    # the comparator is cuBLAS BF16 on the dequantized operands, the reference's F.linear
    # (torch's _scaled_mm has no E2M1 x E8M0 block-32 recipe: its block-32 path takes FP8)
    rec_flops("config2.cublas_bf16_fwd", lambda: torch.nn.functional.linear(xq, wq), flops, bf16_peak,
              "measured bf16")
    del cx, sx, xq, cw, sw, wq, mw

    # one forward + backward of the layer through the public module, against the reference's
    # formulation of the same step (its quantizers, here ours bit for bit, into cuBLAS BF16)
    lin = MXFP4Linear.from_linear(torch.nn.Linear(k, n, bias=False, device=dev, dtype=torch.bfloat16))
    with torch.no_grad():
        lin.weight.copy_(w)
    lin._quantize_activations = True
    xg = x.detach().requires_grad_(True)
    dy = workloads.normal((m, n), 1.0, seed=23).to(torch.bfloat16).to(dev)

    def layer_step():
        xg.grad = None
        lin.weight.grad = None
        lin(xg).backward(dy)

    wr = lin.weight.detach().clone().requires_grad_(True)

    def reference_step():
        xg.grad = None
        wr.grad = None
        torch.nn.functional.linear(fake_quantize_mxfp4_activation(xg), fake_quantize_mxfp4(wr)).backward(dy)

    rec_flops("config2.layer_step_mxfp4_w4a4", layer_step, 3 * flops, bf16_peak, "measured bf16 (3 GEMMs)",
              graph=False, iters=5)
    rec_flops("config2.layer_step_reference_formulation", reference_step, 3 * flops, bf16_peak,
              "measured bf16 (3 GEMMs)", graph=False, iters=5)
    err = int(_native.gemm_error_word(dev))
    if err:
        raise RuntimeError(f"tcgen05 GEMM reported error word {err}")
    return out


REF_DIR = ROOT / "baseline" / "_ref"


def reference_quant():
    """The unmodified reference package (``qatfactory.quant``), installed by pip under the
    git-ignored ``baseline/_ref``, or None when it is not installed."""

    if not (REF_DIR / "qatfactory").is_dir():
        return None
    if str(REF_DIR) not in sys.path:
        sys.path.append(str(REF_DIR))
    import qatfactory.quant as rq

    return rq


def time_calls(fn, inputs: list, iters: int, stream) -> float:
    """Average ms of one eager call, cycling over ``inputs`` (distinct tensors whose total size
    exceeds L2, so no call reads data a previous call left in L2); CUDA events on ``stream``."""

    for i in range(3):
        fn(inputs[i % len(inputs)])
    torch.cuda.synchronize()
    start = torch.cuda.Event(enable_timing=True)
    end = torch.cuda.Event(enable_timing=True)
    start.record(stream)
    for i in range(iters):
        fn(inputs[i % len(inputs)])
    end.record(stream)
    end.synchronize()
    return start.elapsed_time(end) / iters


def incumbent_table(dev, stream) -> dict:
    """The reference's own GPU path (its Triton kernels behind its public API, unmodified, from
    ``baseline/_ref``) against this repository's public API on the same tensors and the same
    clock: eager calls back to back, CUDA events, inputs cycling over more than L2.  Each row
    also says whether the two outputs are bit-identical."""

    rq = reference_quant()
    if rq is None:
        return {"unavailable": "reference not installed under baseline/_ref"}
    from qatfactory_b200 import quant as oq
    from qatfactory_b200 import workloads

    out = {}

    def row(name, ours, ref, inputs, nbytes, iters=20, same=None):
        us_o = time_calls(ours, inputs, iters, stream) * 1e3
        us_r = time_calls(ref, inputs, iters, stream) * 1e3
        rec = {"ours_us": round(us_o, 2), "reference_us": round(us_r, 2), "speedup": round(us_r / us_o, 2),
               "ours_GB/s": round(nbytes / us_o / 1e3, 1), "reference_GB/s": round(nbytes / us_r / 1e3, 1)}
        if same is not None:
            rec.update(same)
        out[name] = rec

    def bits_equal(a, b):
        """Ours against the reference's GPU path, element by element: identical bits, or equal
        values that differ only in the sign of a zero (the reference's own tests compare with
        torch.equal, which does not see the sign of zero; this repository matches the
        reference's torch CPU path, sign of zero included), or a count of other differences."""

        a, b = a.contiguous(), b.contiguous()
        ia, ib = a.view(torch.int16), b.view(torch.int16)
        diff = ia != ib
        n = int(diff.sum())
        if n == 0:
            return {"bit_equal": True}
        zero_sign = int((diff & (a == 0) & (b == 0)).sum())
        return {"bit_equal": False, "elements_differ": n, "of_which_signed_zero_only": zero_sign,
                "value_equal": bool(torch.equal(a, b))}

    w2 = workloads.config2_weight().to(dev)
    n2 = w2.numel()
    row("config2.mxfp4_even_qdq[weight]", oq.fake_quantize_mxfp4, rq.fake_quantize_mxfp4, [w2], n2 * 4 + n2 // 8,
        same=bits_equal(oq.fake_quantize_mxfp4(w2), rq.fake_quantize_mxfp4(w2)))
    del w2
    x2 = workloads.config2_activation().to(dev)
    row("config2.mxfp4_ceil_qdq[activations]", oq.fake_quantize_mxfp4_activation, rq.fake_quantize_mxfp4_activation,
        [x2], x2.numel() * 4,
        same=bits_equal(oq.fake_quantize_mxfp4_activation(x2), rq.fake_quantize_mxfp4_activation(x2)))
    del x2
    w1 = workloads.config1_weight().to(dev)
    copies = [w1.clone() for _ in range(8)]  # 8 x 32 MB: cold data on every call
    n1 = w1.numel()
    row("config1.nvfp4_fake_quant[weight, amax+qdq]", oq.fake_quantize_nvfp4, rq.fake_quantize_nvfp4, copies,
        n1 * 2 + n1 * 4 + n1 // 8, iters=40,
        same=bits_equal(oq.fake_quantize_nvfp4(w1), rq.fake_quantize_nvfp4(w1)))
    del w1, copies
    x4, w4, dy4 = (t.to(dev) for t in workloads.config4_inputs())
    xa = x4.float().abs().amax()
    n4 = x4.numel()
    row("config4.nvfp4_activation_qdq[x, static amax]", lambda t: oq.fake_quantize_nvfp4_activation(t, xa),
        lambda t: rq.fake_quantize_nvfp4_activation(t, xa), [x4], n4 * 4 + n4 // 8,
        same=bits_equal(oq.fake_quantize_nvfp4_activation(x4, xa), rq.fake_quantize_nvfp4_activation(x4, xa)))

    # configuration 4 layer step, forward + backward: this repository's NVFP4Linear (W4A4 on the
    # tcgen05 GEMMs) against the reference's own formulation F.linear(fq_act(x), fq(w)) on its
    # Triton quantizers and cuBLAS
    k, n = x4.shape[1], w4.shape[0]
    lin = oq.NVFP4Linear.from_linear(torch.nn.Linear(k, n, bias=False, device=dev, dtype=torch.bfloat16))
    with torch.no_grad():
        lin.weight.copy_(w4)
    lin._quantize_activations = True
    lin._input_amax_static = xa.clone()
    xg = x4.detach().requires_grad_(True)
    wr = w4.detach().clone().requires_grad_(True)

    def ours_step(_):
        xg.grad = None
        lin.weight.grad = None
        lin(xg).backward(dy4)

    def ref_step(_):
        xg.grad = None
        wr.grad = None
        torch.nn.functional.linear(rq.fake_quantize_nvfp4_activation(xg, xa), rq.fake_quantize_nvfp4(wr)).backward(dy4)

    row("config4.layer_step[fwd+bwd]", ours_step, ref_step, [None], 0, iters=10)
    out["config4.layer_step[fwd+bwd]"].pop("ours_GB/s")
    out["config4.layer_step[fwd+bwd]"].pop("reference_GB/s")
    del lin, xg, wr, x4, w4, dy4

    # configuration 2's tensors as an MXFP4 W4A4 layer: MXFP4Linear on the kind::mxf4 GEMM
    # against the reference's own formulation on its Triton MXFP4 quantizers and cuBLAS
    x2 = workloads.config2_activation().to(dev)
    w2 = workloads.config2_weight().to(dev)
    dy2 = workloads.normal((x2.shape[0], w2.shape[0]), 1.0, seed=23).to(torch.bfloat16).to(dev)
    lin2 = oq.MXFP4Linear.from_linear(torch.nn.Linear(w2.shape[1], w2.shape[0], bias=False, device=dev,
                                                      dtype=torch.bfloat16))
    with torch.no_grad():
        lin2.weight.copy_(w2)
    lin2._quantize_activations = True
    xg2 = x2.detach().requires_grad_(True)
    wr2 = w2.detach().clone().requires_grad_(True)

    def ours_mx_step(_):
        xg2.grad = None
        lin2.weight.grad = None
        lin2(xg2).backward(dy2)

    def ref_mx_step(_):
        xg2.grad = None
        wr2.grad = None
        torch.nn.functional.linear(rq.fake_quantize_mxfp4_activation(xg2), rq.fake_quantize_mxfp4(wr2)).backward(dy2)

    row("config2.mxfp4_layer_step[fwd+bwd]", ours_mx_step, ref_mx_step, [None], 0, iters=5)
    out["config2.mxfp4_layer_step[fwd+bwd]"].pop("ours_GB/s")
    out["config2.mxfp4_layer_step[fwd+bwd]"].pop("reference_GB/s")
    del lin2, xg2, wr2, x2, w2, dy2

    layer = workloads.config3_layer(0)
    gate_up = [layer[4][1].to(dev), layer[5][1].to(dev)]  # 2 x 100 MB
    del layer
    ng = gate_up[0].numel()
    rb, ob = rq.quantize_q4_k(gate_up[0], method="minmax"), oq.quantize_q4_k(gate_up[0], method="minmax")
    row("config3.q4k_minmax_pack[gate/up]", lambda t: oq.quantize_q4_k(t, method="minmax"),
        lambda t: rq.quantize_q4_k(t, method="minmax"), gate_up, ng * 2 + ng * 144 // 256 + ng * 2, iters=6,
        same={"blocks_" + k: v for k, v in
              bits_equal(ob.packed_weight.view(torch.int16), rb.packed_weight.view(torch.int16)).items()})
    del rb, ob
    row("config3.q4k_minmax_fake_quant[gate/up]", lambda t: oq.fake_quantize_q4_k(t, method="minmax"),
        lambda t: rq.fake_quantize_q4_k(t, method="minmax"), gate_up, ng * 4 + ng // 8, iters=10,
        same=bits_equal(oq.fake_quantize_q4_k(gate_up[0], method="minmax"),
                        rq.fake_quantize_q4_k(gate_up[0], method="minmax")))
    yo = oq.fake_quantize_q4_k(gate_up[0], method="grid_search")
    yr = rq.fake_quantize_q4_k(gate_up[0], method="grid_search")
    agree = float((yo.view(torch.int16) == yr.view(torch.int16)).float().mean())
    del yo, yr
    row("config3.q4k_grid_fake_quant[gate/up]", lambda t: oq.fake_quantize_q4_k(t, method="grid_search"),
        lambda t: rq.fake_quantize_q4_k(t, method="grid_search"), gate_up, ng * 4 + ng // 8, iters=4,
        same={"weights_equal_frac": round(agree, 6)})
    del gate_up
    torch.cuda.empty_cache()
    return out


def run_ncu_workload() -> None:
    """Each hot kernel twice on the benchmark tensors, untimed: the workload the committed ncu
    summaries under profiles/ were captured from (a few hundred MB on one GPU)."""

    from qatfactory_b200 import _native, workloads

    dev = torch.device("cuda", 0)
    w2 = workloads.config2_weight().to(dev)
    x2 = workloads.config2_activation().to(dev)
    x4 = workloads.config4_inputs()[0].to(dev)
    gate = workloads.config3_layer(0)[4][1].to(dev)
    xa = _native.tensor_amax(x4)
    for _ in range(2):
        _native.mxfp4_qdq_even(w2)
        _native.mxfp4_qdq_ceil(x2)
        _native.nvfp4_qdq(x4, xa)
        _native.q4k_encode(gate, "minmax", recon=False, mask=False)
        _native.q4k_encode(gate, "minmax", blocks=False)
        _native.tensor_amax(x4)
        _native.mxfp4_pack(w2, recon=False)
        _native.nvfp4_pack(x4, xa, recon=False)
    blocks = _native.q4k_encode(gate, "minmax", recon=False, mask=False)[0]
    experts = w2.view(24, 1024, 4096)  # the fused gate/up weight read as 24 expert slices
    for _ in range(2):
        _native.q4k_dequant(blocks, gate.shape[1])
        _native.tensor_amax_batched(experts)
    # configuration 4 (W4A4): operand passes, FP4 forward GEMM, BF16 backward GEMMs, once each
    w4, dy4 = (t.to(dev) for t in workloads.config4_inputs()[1:])
    wa = _native.tensor_amax(w4)
    cx, sx, xq, mx = _native.nvfp4_operand(x4, xa, _native.OPERAND_A)
    cw, sw, wq, mw = _native.nvfp4_operand(w4, wa, _native.OPERAND_B)
    _native.nvfp4_gemm(cx, sx, xa, cw, sw, wa)
    _native.nvfp4_linear_fwd(x4, xa, cw, sw, wa)
    _native.bf16_gemm(dy4, _native.K_MAJOR, wq, _native.MN_MAJOR, mx)
    _native.bf16_gemm(dy4, _native.MN_MAJOR, xq, _native.MN_MAJOR, mw)  # split-K tail + reduce
    # MXFP4 W4A4 at configuration 2: both operand passes and the kind::mxf4 GEMM (CTA pairs)
    cx2, sx2, _, _ = _native.mxfp4_operand(x2, _native.OPERAND_A, _native.MXFP4_CEIL, mask=False)
    cw2, sw2, _, _ = _native.mxfp4_operand(w2, _native.OPERAND_B, _native.MXFP4_EVEN)
    _native.mxfp4_gemm(cx2, sx2, cw2, sw2)
    del cx2, sx2, cw2, sw2
    # quantize-before-gather: the shadow QDQ of an FP32 latent shard (config-4 W as FP32)
    latent = w4.float()
    shadow = torch.empty_like(latent)
    smask = torch.empty(_native.mask_nbytes(latent.numel()), dtype=torch.uint8, device=dev)
    _native.nvfp4_qdq_shadow(latent, wa, shadow, smask)
    torch.cuda.synchronize()
    print("ncu workload done", file=sys.stderr, flush=True)


def shard_tensors(sizes: list[int], world: int) -> list[list[int]]:
    """Whole tensors to ranks, largest first onto the least-loaded rank (elements balanced);
    a Q4_K block never spans two rows, so a tensor's encoding is independent of the others'."""

    loads = [0] * world
    owned: list[list[int]] = [[] for _ in range(world)]
    for i in sorted(range(len(sizes)), key=lambda j: (-sizes[j], j)):
        r = min(range(world), key=lambda q: (loads[q], q))
        owned[r].append(i)
        loads[r] += sizes[i]
    return owned


def config3_stack_sharded(args, world: int, rank: int, dev, stream, peaks) -> dict:
    """Configuration 3 as configured, split across the ranks (strong scaling): the Q4_K minmax
    encode + pack of every linear of the 36-layer Qwen3-8B stack (252 tensors, 6.95 G weights,
    13.9 GB BF16 in, 3.9 GB of block_q4_K out), each rank encoding its share of whole tensors.
    One step = every tensor once; time = max over ranks of the device time; value = the stack's
    algorithmic bytes over that time.  Inputs are drawn on the device (N(0, 0.02), seeded per
    tensor): the timing does not depend on the bits, and the bits are pinned by the tests."""

    from qatfactory_b200 import _native, workloads

    shapes = [(o, i) for _ in range(workloads.QWEN3_8B_LAYERS) for _, o, i in workloads.QWEN3_8B_LINEARS]
    sizes = [o * i for o, i in shapes]
    mine = shard_tensors(sizes, world)[rank]
    g = torch.Generator(device=dev)
    ws = []
    for idx in mine:
        g.manual_seed(5 + idx)
        ws.append(torch.randn(shapes[idx], generator=g, device=dev, dtype=torch.float32).mul_(0.02).to(torch.bfloat16))
    outs = [torch.empty((w.shape[0], w.shape[1] // 256 * 144), dtype=torch.uint8, device=dev) for w in ws]
    lib = _native.load_library()
    s = stream.cuda_stream

    def step():
        for w, o in zip(ws, outs):
            st = lib.qatf_q4k_encode(w.data_ptr(), 2, w.shape[0], w.shape[1], w.shape[1], 1, None, None,
                                     o.data_ptr(), s)
            if st != 0:
                raise RuntimeError(f"qatf_q4k_encode failed with status {st}")

    step()
    barrier_sync()
    k = 3
    ms = max_over_ranks(time_region(step, k, stream), dev) / k
    barrier_sync()
    total_elems = sum(sizes)
    nbytes = total_elems * 2 + total_elems * 144 // 256
    gbs = nbytes / (ms * 1e-3) / 1e9
    res = {"workload": "config3: Q4_K minmax encode + pack of all 36 layers x 7 linears of Qwen3-8B "
                       "(252 tensors, 13.9 GB BF16 -> 3.9 GB block_q4_K), whole tensors split across ranks",
           "scaling": "strong", "n_gpus": world, "ms": round(ms, 3), "GB/s": round(gbs, 1),
           "frac_of_hbm_per_gpu": round(gbs / (world * peaks["hbm_gbs"]), 3),
           "tensors_per_rank": [len(x) for x in shard_tensors(sizes, world)],
           "elements_max_rank_over_mean": round(max(sum(sizes[i] for i in x) for x in shard_tensors(sizes, world))
                                                / (total_elems / world), 4),
           "launches_per_rank_per_step": len(mine)}
    del ws, outs
    torch.cuda.empty_cache()
    return res


def qad_measure(args, world: int, rank: int, dev, peaks: dict) -> dict:
    """Configuration 5: the NVFP4 W4A16 QAD student step (Qwen3-8B architecture, random init,
    seq 4096, micro-batch 1 per GPU, FSDP2 over all ranks).  Tokens/s = 4096 * world per step
    over the max-over-ranks device time of ``qad_steps`` steps after ``warmup`` steps."""

    from qatfactory_b200 import _native, qad_step

    seq = 4096
    cfg = qad_step.qwen3_config(num_hidden_layers=args.qad_layers) if args.qad_layers else qad_step.qwen3_config()
    t0 = time.perf_counter()
    # quantize before the gather only where there is a gather to shard (at one GPU it saves the
    # recompute's QDQ but masks FP32 gradients instead of BF16 ones: measured even, +28 GB)
    quantized_gather = args.qad_gather == "quantized" or (args.qad_gather == "auto" and world > 1)
    step = qad_step.QADStep(cfg, dev, quantized_gather=quantized_gather)
    build_s = time.perf_counter() - t0
    stream = torch.cuda.current_stream(dev)
    k = args.qad_steps
    host = [qad_step.synthetic_tokens(cfg.vocab_size, seq, rank, i, "cpu").pin_memory()
            for i in range(args.warmup + 2 * k)]
    losses = []
    for i in range(args.warmup):
        losses.append(float(step(host[i].to(dev, non_blocking=True))))
    resident = [t.to(dev) for t in host[args.warmup:args.warmup + k]]
    barrier_sync()
    launches0 = _native.launch_count()
    with ClockSampler(int(os.environ.get("LOCAL_RANK", "0"))) as clocks:
        barrier_sync()
        start = torch.cuda.Event(enable_timing=True)
        end = torch.cuda.Event(enable_timing=True)
        start.record(stream)
        out = [step(t) for t in resident]
        end.record(stream)
        end.synchronize()
        ms = start.elapsed_time(end)
        barrier_sync()
    launches = _native.launch_count() - launches0
    losses += [float(v) for v in out]
    ms = max_over_ranks(ms, dev) / k

    # end to end: token ids from pinned host memory each step, the loss read back each step
    barrier_sync()
    start = torch.cuda.Event(enable_timing=True)
    end = torch.cuda.Event(enable_timing=True)
    start.record(stream)
    for t in host[args.warmup + k:]:
        losses.append(float(step(t.to(dev, non_blocking=True))))
    end.record(stream)
    end.synchronize()
    ms_e2e = max_over_ranks(start.elapsed_time(end), dev) / k
    barrier_sync()

    flops = qad_step.step_flops(cfg, seq)
    achieved = flops / (ms * 1e-3) / 1e12
    peak = peaks.get("bf16_tflops_sustained") or peaks["bf16_tflops"]
    result = {
        "metric": "QAD student step tokens/s", "value": round(world * seq / (ms * 1e-3), 1), "unit": "tokens/s",
        "n_gpus": world, "steps": k, "warmup": args.warmup, "ms_per_step": round(ms, 2),
        "higher_is_better": True, "scaling": "weak", "dtype": "bf16", "data": "synthetic",
        "config": {"workload": "config5: NVFP4 W4A16 QAD student step, forward KL to a frozen BF16 teacher, AdamW "
                               "on FP32 latent masters, gradient checkpointing",
                   "model": f"Qwen3-8B architecture, {cfg.num_hidden_layers} layers, random init N(0,0.02)",
                   "global_batch": world, "seq_len": seq, "micro_batch_per_gpu": 1, "parallelism": f"fsdp2x{world}",
                   "weight_gather": ("quantized: each rank fake-quantizes its FP32 latent shards once per optimizer "
                                     "step and FSDP2 gathers the quantized weights (same results bit for bit)"
                                     if quantized_gather else
                                     "latent: FSDP2 gathers the BF16 latents and every forward and recompute "
                                     "fake-quantizes the gathered weight (the reference's data flow)"),
                   "l2": "weights and activations far larger than L2; no flush"},
        "roofline": {"bound": "tensor", "achieved": round(achieved, 1), "peak": peak, "unit": "TFLOP/s",
                     "frac": round(achieved / peak, 3), "traffic": None,
                     "kernel": "whole step (per GPU): algorithmic matmul FLOPs / step time",
                     "flops_per_step_per_gpu": flops,
                     "peak_source": f"{peaks['_source']} (bf16_tflops_sustained)"},
        "e2e": {"value": round(world * seq / (ms_e2e * 1e-3), 1), "unit": "tokens/s",
                "h2d_bytes_per_step": seq * 8, "d2h_bytes_per_step": 4, "ms_per_step": round(ms_e2e, 2)},
        "gpu_launches": launches, "clocks": clocks.summary(),
        "loss_first_last": [round(losses[0], 6), round(losses[-1], 6)],
        "max_memory_gb": round(torch.cuda.max_memory_allocated(dev) / 1e9, 1), "build_s": round(build_s, 1),
    }
    if quantized_gather and world > 1 and not args.no_qad_compare:
        result["gather_comparison"] = qad_gather_comparison(args, cfg, step, resident, dev, stream)
    del step, resident, out
    gc.collect()  # the modules and their amax groups refer to each other
    torch.cuda.empty_cache()
    if not args.no_qad_reference and reference_quant() is not None:
        result["reference"] = qad_variant_measure(
            args, cfg, host, dev, stream, ms, dict(impl="reference", ref_path=REF_DIR),
            "reference modules (qatfactory.quant NVFP4Linear + Triton, kd_loss.distill_loss) in this harness")
    del host
    return result


def qad_gather_comparison(args, cfg, quantized_step, tokens, dev, stream, rounds: int = 6) -> dict:
    """The quantized gather against the reference's data flow on this repository's kernels (the
    gathered BF16 latent fake-quantized in every forward and recompute), both steps resident at
    once and timed in alternating rounds (the order flips every round), so that clock and power
    drift over the run falls on both alike; medians of the per-round device times, max over
    ranks."""

    from qatfactory_b200 import qad_step

    latent_step = qad_step.QADStep(cfg, dev)
    steps = {"quantized": quantized_step, "latent": latent_step}
    k = min(3, len(tokens))
    for t in tokens[:k]:  # warm the second step's allocations and kernels
        latent_step(t)
    times = {name: [] for name in steps}
    for r in range(rounds):
        order = ("quantized", "latent") if r % 2 == 0 else ("latent", "quantized")
        for name in order:
            barrier_sync()
            start = torch.cuda.Event(enable_timing=True)
            end = torch.cuda.Event(enable_timing=True)
            start.record(stream)
            for t in tokens[:k]:
                steps[name](t)
            end.record(stream)
            end.synchronize()
            times[name].append(max_over_ranks(start.elapsed_time(end), dev) / k)
    del latent_step, steps
    gc.collect()
    torch.cuda.empty_cache()
    med = {name: statistics.median(v) for name, v in times.items()}
    return {"method": f"both steps resident, {rounds} alternating rounds of {k} steps, median ms per step",
            "quantized_ms": round(med["quantized"], 2), "latent_ms": round(med["latent"], 2),
            "speedup_of_quantized": round(med["latent"] / med["quantized"], 4),
            "rounds_ms": {name: [round(x, 1) for x in v] for name, v in times.items()}}


def qad_variant_measure(args, cfg, host, dev, stream, ms_ours: float, step_kwargs: dict, label: str) -> dict:
    """The same QAD step in the same FSDP2 harness built with ``step_kwargs``: the reference's
    own modules (unmodified ``qatfactory.quant`` NVFP4Linear with its Triton quantizers,
    ``apply_fake_quant``, ``refresh_nvfp4_weight_amax`` and
    ``qatfactory.distill.kd_loss.distill_loss``, from ``baseline/_ref``), or this repository's
    kernels with the other weight-gather form; on the same token ids, timed the same way (max
    over ranks)."""

    from qatfactory_b200 import _native, qad_step

    torch.cuda.reset_peak_memory_stats(dev)
    t0 = time.perf_counter()
    step = qad_step.QADStep(cfg, dev, **step_kwargs)
    build_s = time.perf_counter() - t0
    k = args.qad_steps
    for i in range(args.warmup):
        step(host[i].to(dev, non_blocking=True))
    resident = [t.to(dev) for t in host[args.warmup:args.warmup + k]]
    barrier_sync()
    launches0 = _native.launch_count()
    start = torch.cuda.Event(enable_timing=True)
    end = torch.cuda.Event(enable_timing=True)
    start.record(stream)
    out = [step(t) for t in resident]
    end.record(stream)
    end.synchronize()
    ms = max_over_ranks(start.elapsed_time(end), dev) / k
    barrier_sync()
    world = dist.get_world_size() if dist.is_initialized() else 1
    res = {"impl": label,
           "ms_per_step": round(ms, 2), "value": round(world * 4096 / (ms * 1e-3), 1), "unit": "tokens/s",
           "speedup_of_ours": round(ms / ms_ours, 3), "loss_last": round(float(out[-1]), 6),
           "gpu_launches_of_this_repository": _native.launch_count() - launches0,
           "max_memory_gb": round(torch.cuda.max_memory_allocated(dev) / 1e9, 1), "build_s": round(build_s, 1)}
    del step, resident, out
    gc.collect()  # the modules and their amax groups refer to each other
    torch.cuda.empty_cache()
    return res


def run_qad_only(args) -> None:
    from qatfactory_b200 import qad_step

    rank, world, local = qad_step.ensure_process_group()
    dev = torch.device("cuda", local)
    result = qad_measure(args, world, rank, dev, measured_peaks())
    if rank == 0:
        emit(result)
    dist.barrier()
    dist.destroy_process_group()


def run_b200(args) -> None:
    from qatfactory_b200 import _native, workloads
    from qatfactory_b200.quant import fake_quantize_mxfp4, fake_quantize_mxfp4_activation

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        from datetime import timedelta

        dist.init_process_group("nccl", timeout=timedelta(seconds=120), device_id=dev)
    peaks = measured_peaks()
    stream = torch.cuda.current_stream(dev)

    w = workloads.config2_weight().to(dev)
    x = workloads.config2_activation().to(dev)
    bw, bx = algorithmic_bytes_config2()

    def step():
        _native.mxfp4_qdq_even(w)
        _native.mxfp4_qdq_ceil(x)

    for _ in range(args.warmup):
        step()
    barrier_sync()
    with ClockSampler(local) as clocks:
        keep_loaded(step, 0.7, stream)
        barrier_sync()
        launches0 = _native.launch_count()
        ms = time_region(step, args.steps, stream)
        launches = _native.launch_count() - launches0
        barrier_sync()
        keep_loaded(step, 0.7, stream)
    ms = max_over_ranks(ms, dev)
    ms_per_step = ms / args.steps
    value = world * (bw + bx) / (ms_per_step * 1e-3) / 1e9

    # dominant kernel roofline (each kernel timed alone, back to back; inputs exceed L2)
    ms_w = time_region(lambda: _native.mxfp4_qdq_even(w), args.steps, stream) / args.steps
    ms_x = time_region(lambda: _native.mxfp4_qdq_ceil(x), args.steps, stream) / args.steps
    dom_name, dom_bytes, dom_ms = ("mxfp4_qdq_even", bw, ms_w) if ms_w >= ms_x else ("mxfp4_qdq_ceil", bx, ms_x)
    achieved = dom_bytes / (dom_ms * 1e-3) / 1e9
    traffic = None
    tf = ROOT / "profiles" / "traffic.json"
    if tf.exists():
        traffic = json.loads(tf.read_text()).get(dom_name)
    roofline = {"bound": "hbm", "achieved": round(achieved, 1), "peak": peaks["hbm_gbs"], "unit": "GB/s",
                "frac": round(achieved / peaks["hbm_gbs"], 3), "traffic": traffic, "kernel": dom_name,
                "peak_source": f"{peaks['_source']} (hbm_gbs)",
                "other": {"mxfp4_qdq_even_us": round(ms_w * 1e3, 1), "mxfp4_qdq_ceil_us": round(ms_x * 1e3, 1)}}

    # end to end through the public API, pinned host buffers, copies inside the region
    w_h = w.cpu().pin_memory()
    x_h = x.cpu().pin_memory()
    out_w = torch.empty(W_SHAPE, dtype=torch.bfloat16).pin_memory()
    out_x = torch.empty(X_SHAPE, dtype=torch.bfloat16).pin_memory()
    del w, x

    from qatfactory_b200.host_stream import stream_jobs

    def e2e_step():
        # host tensors streamed through the public quantizers in row chunks, both tensors in
        # one pipeline: the two PCIe directions and the kernels overlap (results identical to
        # whole-tensor calls)
        stream_jobs([(fake_quantize_mxfp4, w_h, out_w), (fake_quantize_mxfp4_activation, x_h, out_x)], dev)

    e2e_steps = max(1, min(args.steps, 5))
    for _ in range(2):
        e2e_step()
    # host-side PCIe and memory traffic of other jobs on the machine can slow a window (one run
    # saw rounds of 27.9, 7.4 and 10.1 ms): the median of five timed rounds of e2e_steps steps
    # each (all five reported)
    rounds = []
    for _ in range(5):
        barrier_sync()
        rounds.append(max_over_ranks(time_region(e2e_step, e2e_steps, stream), dev) / e2e_steps)
    barrier_sync()
    ms_e2e = statistics.median(rounds)
    e2e = {"value": round(world * (bw + bx) / (ms_e2e * 1e-3) / 1e9, 2), "unit": UNIT,
           "h2d_bytes_per_step": w_h.numel() * 2 + x_h.numel() * 2,
           "d2h_bytes_per_step": out_w.numel() * 2 + out_x.numel() * 2, "ms_per_step": round(ms_e2e, 3),
           "rounds_ms_per_step": [round(r, 3) for r in rounds], "steps_per_round": e2e_steps}
    del w_h, x_h, out_w, out_x

    kernels, incumbents = {}, None
    if rank == 0 and world == 1 and not args.no_kernel_table:  # a single-GPU characterisation
        flush = torch.zeros(2 * 256 * 1024 * 1024 // 4, dtype=torch.float32, device=dev)
        kernels = kernel_table(dev, stream, flush, peaks)
        kernels.update(w4a4_table(dev, stream, flush, peaks))
        kernels.update(mxfp4_w4a4_table(dev, stream, flush, peaks))
        del flush
        torch.cuda.empty_cache()
        incumbents = incumbent_table(dev, stream)
    cpu = cpu_baseline() if (rank == 0 and world == 1 and not args.no_cpu) else None
    torch.cuda.empty_cache()
    strong = None if args.no_strong else config3_stack_sharded(args, world, rank, dev, stream, peaks)
    qad = None
    if not args.no_qad:
        from qatfactory_b200 import qad_step

        torch.cuda.empty_cache()
        qad_step.ensure_process_group()  # FSDP2 needs a process group, also at one GPU
        qad = qad_measure(args, world, rank, dev, peaks)

    if rank == 0:
        line = {
            "metric": METRIC, "value": round(value, 2), "unit": UNIT, "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": round(ms_per_step, 4), "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
            "config": config2_config(world),
            "roofline": roofline, "cpu_baseline": cpu, "e2e": e2e, "gpu_launches": launches,
            "value_reference_formula": reference_formula_rate(world, ms_per_step),
            "clocks": {**clocks.summary(), "window": "samples every 100 ms over ~0.7 s of identical untimed load "
                                                          "before and after the timed region, and during it"},
            "kernels_fields": ["us", "GB/s or TFLOP/s", "fraction of the measured peak (HBM for GB/s)"],
            "kernels": compact_kernels(kernels), "incumbents": incumbents,
            "sharded_workloads": "strong (configuration 3 stack split across the ranks, time to completion) and "
                                 "qad (FSDP2 over all ranks); value above is per-rank replicas",
            "strong": strong, "qad": qad,
        }
        emit(line)
    if dist.is_initialized():
        dist.barrier()
        dist.destroy_process_group()


def compact_kernels(kernels: dict) -> dict:
    """Each kernel-table entry as [us, rate, frac] so the whole line stays short."""

    out = {}
    for name, v in kernels.items():
        rate = v.get("GB/s", v.get("TFLOP/s"))
        out[name] = [v["us"], rate, v["frac"]]
        if "frac_of_cublas_nvfp4" in v:  # cuBLAS time / ours on the same FP4 operands
            out[name].append({"of_cublas_nvfp4": v["frac_of_cublas_nvfp4"]})
    return out


RESULT = sys.stdout


def emit(line: dict) -> None:
    """The one JSON line of this run, on the process's original standard output."""

    RESULT.write(json.dumps(line) + "\n")
    RESULT.flush()


def main() -> None:
    global RESULT
    # Library banners (NCCL prints its version on file descriptor 1) go to stderr, so standard
    # output carries exactly one JSON line.
    sys.stdout.flush()
    RESULT = os.fdopen(os.dup(1), "w")
    os.dup2(2, 1)
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=("b200", "reference"), default="b200")
    ap.add_argument("--no-cpu", action="store_true", help="skip the CPU-baseline sample")
    ap.add_argument("--no-kernel-table", action="store_true", help="skip the per-kernel table")
    ap.add_argument("--ncu-workload", action="store_true", help="run the untimed profiling workload and exit")
    ap.add_argument("--qad", action="store_true", help="measure only the configuration-5 QAD step")
    ap.add_argument("--no-qad", action="store_true", help="skip the configuration-5 QAD step")
    ap.add_argument("--no-strong", action="store_true", help="skip the sharded configuration-3 stack")
    ap.add_argument("--no-qad-reference", action="store_true",
                    help="skip the QAD step on the reference's own modules (baseline/_ref)")
    ap.add_argument("--incumbents", action="store_true",
                    help="only the table against the reference's own GPU path (one GPU)")
    ap.add_argument("--qad-steps", type=int, default=5, help="timed QAD steps")
    ap.add_argument("--qad-layers", type=int, default=0, help="decoder layers (0 = the full 36)")
    ap.add_argument("--qad-gather", choices=("auto", "quantized", "latent"), default="auto",
                    help="FSDP2 weight gather of the QAD step: quantized shards, or the BF16 latents quantized "
                         "after the gather in every forward; auto = quantized on more than one GPU")
    ap.add_argument("--no-qad-compare", action="store_true",
                    help="skip the interleaved comparison of the two gather forms (more than one GPU)")
    args = ap.parse_args()
    args.warmup = max(3, args.warmup)  # the timing rules require at least 3 warm-up steps
    if args.ncu_workload:
        run_ncu_workload()
    elif args.incumbents:
        torch.cuda.set_device(0)
        dev = torch.device("cuda", 0)
        emit({"incumbents": incumbent_table(dev, torch.cuda.current_stream(dev))})
    elif args.qad:
        run_qad_only(args)
    elif args.impl == "reference":
        run_reference(args)
    else:
        run_b200(args)


if __name__ == "__main__":
    main()
