"""Benchmark of the FP8 DiT hot path on B200 (one JSON line on rank 0).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl qik|reference]
    torchrun --nproc-per-node N bench.py --gpus N ...           (N > 1)

Workload ("DiT FFN pair on 1 B200"): per GPU, M = 4352
token rows x 3072 -> 12288 (GELU-tanh) -> 3072, both linears FP8 per-tensor with
static e4m3 weights (N(0, 0.02) init) and dynamic per-tensor activation scales,
the hidden activation re-quantized between them, bf16 output.  Activations are
N(0,1) with 8 outlier channels x20 (synthetic; no dataset is involved).

A step is one FFN pair over one batch.  ``value`` = FLOPs (2*M*N*K summed over both
linears and all ranks) / device time of the K timed steps (CUDA events on the
launching stream, max over ranks); L2 is flushed between steps, outside the timed
events: a 256 MiB write, then a 256 MiB read of a second buffer, so the write's dirty
lines are written back during the flush and not during the next timed kernel.  ``e2e`` is the same metric through the public API
with every step's input copied from pinned host memory and its output copied back
inside the timed region: the serving form (qik.host_pipeline.HostPipeline, the copies
of neighbouring steps overlapping this step's kernels) as the value, the form with
copy in, kernels and copy out back to back beside it as ``e2e.serial``.  ``roofline`` covers the dominant kernel (the tcgen05 FP8
GEMM): algorithmic FLOPs per launch / its average CUDA-event duration.

Multi-GPU: token-row shards, one process per GPU, no collective on the data path
(weak scaling).  ``--impl reference`` times the reference's arithmetic (fp8
quantize + dequantized-fp32 matmuls, restated in PyTorch) on the host CPU cores
on a bounded row sample of the same workload.
"""
from __future__ import annotations

import argparse
import json
import os
import shutil
import statistics
import subprocess
import sys
import tempfile
import time
from pathlib import Path

import torch

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT / "qwen-image-kernel_b200"))
sys.path.insert(0, str(ROOT))

METRIC = "FP8 linear TFLOPS/GPU & % dense-FP8 peak at DiT shapes; DiT-block ms @1024px"
M_ROWS, K_IN, HIDDEN = 4352, 3072, 12288
FLOPS_PER_LINEAR = 2.0 * M_ROWS * K_IN * HIDDEN
FLOPS_PER_STEP = 2 * FLOPS_PER_LINEAR
NOMINAL_FP8_TFLOPS = 4500.0


def peaks() -> dict:
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return {"fp8_tflops": 2.0 * float(d["bf16_tflops_sustained"]),
                "fp8_tflops_burst": 2.0 * float(d["bf16_tflops"]), "hbm_gbs": float(d["hbm_gbs"]),
                "source": "measured (MEASURED_PEAKS.json)"}
    return {"fp8_tflops": 2.0 * 1400.0, "fp8_tflops_burst": 2.0 * 1590.0, "hbm_gbs": 6650.0,
            "source": "fallback: 2 x 1.40 PFLOP/s sustained bf16, 2 x 1.59 burst, 6.65 TB/s"}


def fp8_peak_cublaslt(device: torch.device, iters: int = 10) -> float:
    """Dense FP8 tensor-core peak measured on this GPU: the best of `iters` back-to-back
    torch._scaled_mm (cuBLASLt, the reference's call, fp8.py:87) at 8192^3 in e4m3,
    bf16 out, per-tensor scales (a burst figure: each launch timed alone)."""
    n = 8192
    g = torch.Generator(device=device).manual_seed(3)
    a = torch.randn(n, n, device=device, generator=g).to(torch.float8_e4m3fn)
    b = torch.randn(n, n, device=device, generator=g).to(torch.float8_e4m3fn)
    one = torch.ones((), device=device)
    fn = lambda: torch._scaled_mm(a, b.t(), scale_a=one, scale_b=one, out_dtype=torch.bfloat16)  # noqa: E731
    for _ in range(3):
        fn()
    stream = torch.cuda.current_stream(device)
    evs = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(iters)]
    torch.cuda._sleep(int(2e7))
    for e0, e1 in evs:
        e0.record(stream)
        fn()
        e1.record(stream)
    torch.cuda.synchronize(device)
    best = min(e0.elapsed_time(e1) for e0, e1 in evs)
    return 2.0 * n ** 3 / (best / 1e3) / 1e12


class L2Flush:
    """The cache flush between timed launches: a 256 MiB write (more than the 126 MB L2,
    so nothing of the previous launch stays cached) followed by a 256 MiB read of a
    second buffer, which writes the first buffer's dirty lines back to HBM here rather
    than during the next timed kernel's reads."""

    def __init__(self, device: torch.device):
        n = 256 * 1024 * 1024 // 4
        self.w = torch.empty(n, dtype=torch.float32, device=device)
        self.r = torch.zeros(n, dtype=torch.float32, device=device)
        self.sink = torch.empty((), dtype=torch.float32, device=device)

    def __call__(self, i: int = 0) -> None:
        self.w.fill_(float(i))
        torch.sum(self.r, dim=0, out=self.sink)


# DRAM traffic of the FP8 GEMM inside the FFN step: dram__bytes_read.sum +
# dram__bytes_write.sum per launch, the mean of GEMM1 and GEMM2 of one configs[1]
# step, from `ncu --set full --clock-control none -k regex:fp8_gemm -s 2 -c 2
# python bench.py --steps 3 --warmup 3 --no-extras` (the algorithmic bytes are 158.1 MB
# for GEMM1 and 117.9 MB for GEMM2).
GEMM_DRAM_BYTES_PER_LAUNCH = 140240512
GEMM_TRAFFIC_SOURCE = ("ncu capture (dram__bytes_read.sum + dram__bytes_write.sum, mean of the step's two GEMM "
                       "launches): ncu --set full --clock-control none -k regex:fp8_gemm -s 2 -c 2 "
                       "python bench.py --steps 3 --warmup 3 --no-extras")


def bench_config(world: int) -> dict:
    """The workload both arms run (identical for the qik and the reference arm)."""
    return {"workload": "configs[1] DiT FFN pair: M=4352 x 3072 -> 12288 (GELU-tanh) -> 3072, FP8 per-tensor, "
                        "dynamic activation re-quantization, bf16 out",
            "rows_per_gpu": M_ROWS, "global_rows": M_ROWS * world,
            "l2": "flushed between timed steps, outside the timed events: 256 MiB write, then a 256 MiB read of "
                  "a second buffer (the write's dirty lines go back to HBM during the flush)",
            "parallelism": f"dp{world}: token-row shards, no data-path collective"}


# ------------------------------------------------------------------------------ inputs
def make_inputs(seed: int, device: torch.device):
    g = torch.Generator(device="cpu").manual_seed(seed)
    x = torch.randn(M_ROWS, K_IN, generator=g)
    x[:, :8] *= 20.0
    x = x.to(torch.bfloat16)
    w1 = (torch.randn(HIDDEN, K_IN, generator=g) * 0.02).to(torch.bfloat16)
    w2 = (torch.randn(K_IN, HIDDEN, generator=g) * 0.02).to(torch.bfloat16)
    return x, w1, w2


# ------------------------------------------------------------------------------ clocks
class ClockSampler:
    """nvidia-smi clocks/throttle sampling during the timed region."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int):
        self.idx = gpu_index
        self.proc = None
        self.path = None

    def __enter__(self):
        if shutil.which("nvidia-smi") is None:
            return self
        fd, self.path = tempfile.mkstemp(suffix=".csv")
        os.close(fd)
        self.fh = open(self.path, "w")
        self.proc = subprocess.Popen(["nvidia-smi", "-i", str(self.idx), f"--query-gpu={self.FIELDS}",
                                      "--format=csv,noheader,nounits", "-lms", "50"],
                                     stdout=self.fh, stderr=subprocess.DEVNULL)
        time.sleep(0.3)
        return self

    def __exit__(self, *a):
        if self.proc is not None:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()
            self.fh.close()

    def summary(self) -> dict:
        if not self.path or not os.path.exists(self.path):
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        rows = []
        for line in open(self.path):
            parts = [p.strip() for p in line.split(",")]
            if len(parts) < 9:
                continue
            try:
                rows.append((float(parts[1]), float(parts[2]), parts[5:9]))
            except ValueError:
                continue
        os.unlink(self.path)
        if not rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["no samples"]}
        smax = max(r[1] for r in rows)
        load = [r for r in rows if r[0] >= 0.5 * smax] or rows
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for r in rows for i, v in enumerate(r[2]) if v.lower() == "active"})
        return {"sm_mhz": statistics.median(r[0] for r in load), "sm_max_mhz": smax, "reasons": reasons,
                "samples": len(rows)}


# ------------------------------------------------------------------------------ qik arm
def run_qik(args, rank: int, world: int, device: torch.device) -> dict | None:
    from qik import fp8 as F
    from qik import _lib as L

    x_cpu, w1, w2 = make_inputs(1234 + rank, device)
    up = F.FP8Linear(K_IN, HIDDEN).to(device)
    down = F.FP8Linear(HIDDEN, K_IN).to(device)
    for lin, w in ((up, w1), (down, w2)):
        wq, sw = F.quantize_weight_tensorwise(w.to(device))
        lin.weight.copy_(wq)
        lin.weight_scale.copy_(sw)
    x = x_cpu.to(device)
    flush = L2Flush(device)
    stream = torch.cuda.current_stream(device)

    lib = L.load()
    ws = torch.empty(lib.qik_fp8_ffn_workspace_bytes(M_ROWS, K_IN, HIDDEN), dtype=torch.uint8, device=device)

    def step(xin: torch.Tensor):
        # the public FP8 FFN path: one chain of four kernels (qik_fp8_ffn)
        return F.fp8_ffn_gelu(xin, up, down, workspace=ws)

    def step_split(xin: torch.Tensor, ev):
        # the same computation launch by launch, with events around each GEMM
        x2 = xin.reshape(-1, K_IN)
        xq, sx = F.quantize_tensorwise(x2)
        amax = torch.zeros(1, dtype=torch.int32, device=device)
        ev[0].record(stream)
        h = F.fp8_gemm(xq, sx, up.weight, up.weight_scale, up.bias, epilogue=L.EPI_GELU_TANH, amax_out=amax)
        ev[1].record(stream)
        hq, sh = F.quantize_from_amax(h, amax)
        ev[2].record(stream)
        y = F.fp8_gemm(hq, sh, down.weight, down.weight_scale, down.bias)
        ev[3].record(stream)
        return y

    launches_per_step = 4  # single-pass quantizer, gemm (GELU+amax), pack, gemm
    clk = ClockSampler(device.index if device.index is not None else 0).__enter__()
    for _ in range(args.warmup):
        step(x)
    torch.cuda.synchronize(device)

    def barrier():
        if world > 1:
            torch.distributed.barrier()
        torch.cuda.synchronize(device)

    # ---- device-resident timed region
    ev_step = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
               for _ in range(args.steps)]
    barrier()
    # a GPU-side sleep ahead of the timed steps lets the host queue all of them, so
    # no host launch latency appears inside the device-timed events
    torch.cuda._sleep(int(2e7))
    for i in range(args.steps):
        flush(i)
        ev_step[i][0].record(stream)
        step(x)
        ev_step[i][1].record(stream)
    barrier()
    clk.__exit__(None, None, None)
    clocks = clk.summary()
    clocks["window"] = "sampled every 50 ms from before the warm-up to the end of the timed steps"
    t_steps = sum(a.elapsed_time(b) for a, b in ev_step) / 1e3            # seconds

    # ---- per-launch GEMM durations (roofline): the same step launch by launch
    ev_k = [[torch.cuda.Event(enable_timing=True) for _ in range(4)] for _ in range(args.steps)]
    torch.cuda._sleep(int(1e8))  # ~50 ms head start: the host queues every split step
    for i in range(args.steps):
        flush(i)
        step_split(x, ev_k[i])
    barrier()
    torch.cuda.synchronize(device)
    # median per GEMM shape, then their mean: one interval that caught a host stall
    # (the queue running dry) cannot move the roofline
    t1 = sorted(ev[0].elapsed_time(ev[1]) for ev in ev_k)
    t2 = sorted(ev[2].elapsed_time(ev[3]) for ev in ev_k)
    gemm_ms = 0.5 * (t1[len(t1) // 2] + t2[len(t2) // 2])

    # ---- end-to-end through the public API with host buffers
    # (a) serving form: qik.host_pipeline.HostPipeline, the next batch's host->device copy
    # and the previous batch's device->host copy overlap this batch's kernels; timed from
    # before the first copy in to the end of the last copy out, every step's copies inside
    from qik.host_pipeline import HostPipeline
    x_host = x_cpu.pin_memory()
    y_hosts = [torch.empty(M_ROWS, K_IN, dtype=torch.bfloat16).pin_memory() for _ in range(2)]
    pipe = HostPipeline(lambda xd, yd: F.fp8_ffn_gelu(xd, up, down, workspace=ws, out=yd),
                        (M_ROWS, K_IN), (M_ROWS, K_IN), device=device, depth=2)
    for i in range(3):
        pipe.submit(x_host, y_hosts[i % 2])
    pipe.synchronize()
    barrier()
    e2e_start = torch.cuda.Event(enable_timing=True)
    torch.cuda._sleep(int(2e7))
    e2e_start.record(stream)
    pipe.h2d_stream.wait_event(e2e_start)
    for i in range(args.steps):
        flush(i)  # L2 flush on the compute stream, inside the timed span
        e2e_end = pipe.submit(x_host, y_hosts[i % 2])
    pipe.synchronize()
    barrier()
    t_e2e = e2e_start.elapsed_time(e2e_end) / 1e3
    # (b) one batch at a time on one stream: copy in, kernels, copy out (events around each)
    y_host = y_hosts[0]
    e2e_ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
              for _ in range(args.steps)]
    torch.cuda._sleep(int(2e7))
    for i in range(args.steps):
        flush(i)
        e2e_ev[i][0].record(stream)
        xd = x_host.to(device, non_blocking=True)
        y_host.copy_(F.fp8_ffn_gelu(xd, up, down, workspace=ws), non_blocking=True)
        e2e_ev[i][1].record(stream)
    barrier()
    t_e2e_serial = sum(a.elapsed_time(b) for a, b in e2e_ev) / 1e3

    parity = ffn_parity(x_cpu, up, down, step(x)) if rank == 0 else {}
    ext = extras(device, flush) if (rank == 0 and not args.no_extras) else None
    tp = tp_stack(device, rank, world, flush) if not args.no_extras else None
    sweep_n = row_shard_sweep(device, rank, world, flush) if not args.no_extras else None
    fp8_peak = fp8_peak_cublaslt(device)
    status = L.device_status(device)
    t = torch.tensor([t_steps, t_e2e, t_e2e_serial, gemm_ms, float(status)], dtype=torch.float64, device=device)
    if world > 1:
        torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX)
    t_steps, t_e2e, t_e2e_serial, gemm_ms, status = t.tolist()
    if rank != 0:
        return None

    pk = peaks()
    # the GEMM is timed launch by launch (a burst), so the roofline compares it with burst
    # peaks: the larger of cuBLASLt's own FP8 GEMM measured above and 2 x the measured
    # burst bf16 rate
    peak = max(fp8_peak, pk["fp8_tflops_burst"])
    peak_source = (f"max of cuBLASLt FP8 8192^3 measured in this run ({fp8_peak:.1f} TF/s, burst) and 2 x "
                   f"bf16 burst from {pk['source']} ({pk['fp8_tflops_burst']:.1f} TF/s)")
    total_flops = FLOPS_PER_STEP * args.steps * world
    value = total_flops / t_steps / 1e12
    achieved = FLOPS_PER_LINEAR / (gemm_ms / 1e3) / 1e12
    out = {
        "metric": METRIC,
        "value": round(value, 2),
        "unit": "TFLOP/s",
        "n_gpus": world,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": round(t_steps / args.steps * 1e3, 4),
        "higher_is_better": True,
        "scaling": "weak",
        "vs_baseline": None,
        "dtype": "e4m3 x e4m3 -> fp32 accumulate, bf16 out",
        "data": "synthetic: N(0,1) activations with 8 outlier channels x20, N(0,0.02) random-init weights",
        "config": bench_config(world),
        "per_gpu_tflops": round(value / world, 2),
        "pct_dense_fp8_peak": round(100.0 * value / world / peak, 1),
        "pct_nominal_fp8_4500": round(100.0 * value / world / NOMINAL_FP8_TFLOPS, 1),
        "e2e": {"value": round(total_flops / t_e2e / 1e12, 2), "unit": "TFLOP/s",
                "h2d_bytes_per_step": M_ROWS * K_IN * 2, "d2h_bytes_per_step": M_ROWS * K_IN * 2,
                "ms_per_step": round(t_e2e / args.steps * 1e3, 4),
                "api": "qik.host_pipeline.HostPipeline over qik.fp8.fp8_ffn_gelu (C ABI qik_fp8_ffn): pinned "
                       "host input copied in and bf16 result copied out every step, the copies of "
                       "neighbouring steps overlapping this step's kernels (depth 2); timed from before "
                       "the first copy in to the end of the last copy out",
                "serial": {"value": round(total_flops / t_e2e_serial / 1e12, 2),
                           "ms_per_step": round(t_e2e_serial / args.steps * 1e3, 4),
                           "form": "copy in, kernels, copy out back to back on one stream"}},
        "roofline": {"kernel": "qik::fp8_gemm_kernel (tcgen05 kind::f8f6f4)", "bound": "tensor",
                     "achieved": round(achieved, 1), "peak": round(peak, 1), "unit": "TFLOP/s",
                     "frac": round(achieved / peak, 3), "traffic": GEMM_DRAM_BYTES_PER_LAUNCH,
                     "traffic_source": GEMM_TRAFFIC_SOURCE, "peak_source": peak_source,
                     "frac_vs_2x_bf16_burst": round(achieved / pk["fp8_tflops_burst"], 3),
                     "frac_vs_cublaslt_fp8": round(achieved / fp8_peak, 3),
                     "avg_launch_ms": round(gemm_ms, 4), "flops_per_launch": FLOPS_PER_LINEAR},
        "parity": parity,
        "gpu_launches": launches_per_step * args.steps * 3,
        "gpu_launches_note": "qik kernels inside the timed regions (device-resident steps + pipelined and serial e2e steps: "
                             "single-pass quantizer of x, GEMM+GELU+amax, pack, GEMM per step, the last three "
                             "chained with programmatic dependent launch; one 1040-byte memset per step clears the "
                             "quantizer's barrier word and the chain's counters); the L2 flush (fill + sum) is "
                             "torch's; GEMM launch times for the "
                             "roofline come from a second pass that runs the step launch by launch with events (median per GEMM)",
        "device_status": int(status),
        "clocks": clocks,
    }
    if ext is not None:
        out["extras"] = ext
    if tp is not None:
        out.setdefault("extras", {})["tp_stack_4block_1024px"] = tp
        if "parity" in tp:
            out["parity"]["tp_peer_vs_nccl"] = tp.pop("parity")
    if sweep_n is not None:
        out.setdefault("extras", {})["cfg5_row_shard_sweep"] = sweep_n
    if world == 1:
        out["cpu_baseline"] = cpu_baseline(args)
    return out


# ------------------------------------------------------------------------------ extras
def _time_ms(fn, iters: int, flush: L2Flush, stream) -> float:
    evs = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(iters)]
    torch.cuda._sleep(int(2e7))
    for i in range(iters):
        flush(i)
        evs[i][0].record(stream)
        fn()
        evs[i][1].record(stream)
    torch.cuda.synchronize()
    return sum(a.elapsed_time(b) for a, b in evs) / iters


def fused_ops_cases(device: torch.device, x: torch.Tensor, mod: torch.Tensor) -> dict:
    """The fused elementwise ops at the t2i block shapes (B = 2, S = 4352, width 3072,
    24 heads of 128, MLP 12288): {name: (callable, algorithmic bytes)}.  Algorithmic
    bytes: every input element read once and every output element written once (bf16;
    e4m3 codes for the layer norm that emits its FP8 linear's input), the modulation
    rows and RoPE tables (L2-resident, shared by all rows) excluded."""
    from qik.triton_fused import (fused_gate_residual, fused_layer_norm_modulate, fused_layer_norm_modulate_e4m3,
                                  fused_rms_norm_rope, fused_swiglu)
    B, S, K = x.shape
    H, D = 24, 128
    g = torch.Generator(device=device).manual_seed(11)
    qkv = torch.randn(B, S, 3 * H * D, device=device, generator=g).to(torch.bfloat16)
    q = qkv.unflatten(-1, (3 * H, D)).chunk(3, dim=-2)[0]
    wn = torch.ones(D, device=device)
    freqs = torch.polar(torch.ones(S, D // 2, device=device), torch.rand(S, D // 2, device=device, generator=g))
    f = torch.randn_like(x)
    gu = torch.randn(B * S, 2 * 12288, device=device, generator=g).to(torch.bfloat16)
    gate, up = gu.chunk(2, dim=-1)
    amax = torch.zeros(1, dtype=torch.int32, device=device)
    n_x = x.numel()
    return {
        "layer_norm_modulate": (lambda: fused_layer_norm_modulate(x, mod, 0, mod.stride(0), None, 1e-6, amax), 4 * n_x),
        "layer_norm_modulate_e4m3": (lambda: fused_layer_norm_modulate_e4m3(x, mod, 0, mod.stride(0), None, 1e-6),
                                     3 * n_x),
        "rms_norm_rope_q": (lambda: fused_rms_norm_rope(q, wn, freqs, 1e-6), 4 * q.numel()),
        "gate_residual": (lambda: fused_gate_residual(x, f, mod, K, None), 6 * n_x),
        "swiglu_12288": (lambda: fused_swiglu(gate, up, amax), 6 * gate.numel()),
    }


def fused_ops(device: torch.device, flush: L2Flush, iters: int, x: torch.Tensor, mod: torch.Tensor) -> dict:
    """HBM roofline of the four fused elementwise kernels at the t2i block shapes
    (fused_ops_cases), L2 flushed between launches."""
    stream = torch.cuda.current_stream(device)
    hbm = peaks()["hbm_gbs"]
    res = {}
    for name, (fn, nbytes) in fused_ops_cases(device, x, mod).items():
        for _ in range(3):
            fn()
        ms = _time_ms(fn, iters, flush, stream)
        gbs = nbytes / ms / 1e6
        res[name] = {"us": round(ms * 1e3, 1), "gbs": round(gbs, 1), "frac_hbm": round(gbs / hbm, 3),
                     "bytes": nbytes}
    return res


def attention_cfg4_cases(device: torch.device, g: torch.Generator) -> dict:
    """BASELINE config 4 attention, synthetic inputs: the prefill form (256 text rows
    with L = q, 2304 cond rows with L = 2559, 4096 target rows with L = 6655) and the
    decode form (4096 target queries over the e4m3-V slab of 2560 keys + 4096 fresh).
    Returns {name: (callable, flops)}."""
    from qik.kv_cache import ContiguousKVCache
    from qik.triton_attention import block_causal_flash_attention as attn
    H, D = 24, 128
    S = 6656
    q, k, v = (torch.randn(1, S, H, D, device=device, generator=g, dtype=torch.bfloat16) for _ in range(3))
    Lp = torch.arange(S, dtype=torch.int32, device=device)
    Lp[256:2560] = 2559
    Lp[2560:] = S - 1
    fl_p = 4.0 * D * H * float((Lp.long() + 1).sum())
    P, T = 2560, 4096
    kp, vp = (torch.randn(1, P, H, D, device=device, generator=g, dtype=torch.bfloat16) for _ in range(2))
    cache = ContiguousKVCache(1, 1, P, H, D, v_fp8=True, device=device)
    cache.get_layer(0).store(kp, vp)
    ck, cv, vs = cache.get_layer(0).views()
    qd, kn, vn = (torch.randn(1, T, H, D, device=device, generator=g, dtype=torch.bfloat16) for _ in range(3))
    Ld = torch.full((T,), P + T - 1, dtype=torch.int32, device=device)
    fl_d = 4.0 * D * H * T * (P + T)
    return {"attention_cfg4_prefill": (lambda: attn(q, k, v, Lp, None), fl_p),
            "attention_cfg4_decode_fp8_slab": (lambda: attn(qd, kn, vn, Ld, None, ck, cv, vs, uniform_full=True),
                                               fl_d)}


def dit_block_case(device: torch.device, g: torch.Generator) -> dict:
    """DiT block @1024 px, CFG batch 2: M = 2 x 4352, the whole block --
    timestep modulation linear (M = 2), LayerNorm + modulate emitting the QKV linear's
    e4m3 input, fused QKV, per-head RMSNorm + RoPE of q and k, block-causal attention
    (256 text causal + 4096 image; its amax feeds the out-proj quantizer), out-proj, gated
    residual, LayerNorm + modulate emitting the FFN's e4m3 input, FFN (GELU-tanh,
    BASELINE configs[2]) and the second gated residual; random-init FP8 weights,
    synthetic activations."""
    from qik import fp8 as F
    from qik.triton_attention import block_causal_flash_attention as attn
    from qik.triton_fused import fused_gate_residual, fused_layer_norm_modulate_e4m3, fused_rms_norm_rope
    H, D = 24, 128
    B2, S2 = 2, 4352
    M, K = B2 * S2, 3072
    lin = {}
    for name, (n_out, n_in) in {"qkv": (9216, 3072), "out": (3072, 3072), "up": (12288, 3072),
                                "down": (3072, 12288), "mod": (18432, 3072)}.items():
        f = F.FP8Linear(n_in, n_out).to(device)
        wq, sw = F.quantize_weight_tensorwise(torch.randn(n_out, n_in, device=device, generator=g) * 0.02)
        f.weight.copy_(wq)
        f.weight_scale.copy_(sw)
        lin[name] = f
    x = torch.randn(B2, S2, K, device=device, generator=g).to(torch.bfloat16)
    temb = torch.randn(B2, K, device=device, generator=g).to(torch.bfloat16)
    wn = torch.ones(D, device=device)
    inv = 1.0 / (10000 ** (torch.arange(0, D, 2, device=device).float() / D))
    freqs = torch.polar(torch.ones(S2, D // 2, device=device),
                        torch.outer(torch.arange(S2, device=device).float(), inv))
    Lt = torch.arange(S2, dtype=torch.int32, device=device)
    Lt[256:] = S2 - 1
    amax = torch.zeros(1, dtype=torch.int32, device=device)

    def block():
        mod = lin["mod"](temb) * 0.05  # [B, 6 x 3072]: scale / gate rows of the two sub-blocks
        amax.zero_()
        hq, hs = fused_layer_norm_modulate_e4m3(x, mod, 0, mod.stride(0), None, 1e-6)
        qkv = lin["qkv"].forward_e4m3(hq, hs).unflatten(-1, (3 * H, D))
        q, k, v = qkv.chunk(3, dim=-2)
        q = fused_rms_norm_rope(q, wn, freqs, 1e-6)
        k = fused_rms_norm_rope(k, wn, freqs, 1e-6)
        o = attn(q, k, v, Lt, None, amax_out=amax)
        h = fused_gate_residual(x, lin["out"].forward_from_amax(o.flatten(2, 3), amax), mod, K, None)
        hq2, hs2 = fused_layer_norm_modulate_e4m3(h, mod, 2 * K, mod.stride(0), None, 1e-6)
        f2 = F.fp8_ffn_gelu(hq2.reshape(M, K), lin["up"], lin["down"], x_scale=hs2).view(B2, S2, K)
        return fused_gate_residual(h, f2, mod, 3 * K, None)

    lin_fl = 2.0 * M * K * (9216 + 3072 + 12288) + 2.0 * M * 12288 * K + 2.0 * B2 * K * 18432
    at_fl = 4.0 * D * H * B2 * float((Lt.long() + 1).sum())
    return {"block": block, "linear_flops": lin_fl, "attention_flops": at_fl, "x": x,
            "mod": lambda: lin["mod"](temb)}


class _Attention(torch.nn.Module):
    """Stand-in for the diffusers attention module with the attributes the processor
    reads (processors.py:50-126): heads, fused_qkv, norm_q / norm_k (weight, eps),
    to_out[0 / 1], and the processor call."""

    def __init__(self, heads, fused_qkv, to_out, wq, wk):
        super().__init__()
        self.heads = heads
        self.fused_qkv = fused_qkv
        self.norm_q = torch.nn.RMSNorm(wq.numel(), eps=1e-6, device=wq.device)
        self.norm_k = torch.nn.RMSNorm(wk.numel(), eps=1e-6, device=wk.device)
        with torch.no_grad():
            self.norm_q.weight.copy_(wq)
            self.norm_k.weight.copy_(wk)
        self.to_out = torch.nn.ModuleList([to_out, torch.nn.Identity()])
        self.processor = None

    def set_processor(self, p):
        self.processor = p

    def forward(self, hidden_states, **kw):
        return self.processor(self, hidden_states, **kw)


def dit_block_product_case(device: torch.device, g: torch.Generator) -> dict:
    """The DiT block @1024 px, CFG batch 2 (M = 2 x 4352), through the product API:
    qik.processors.QwenImage21KernelBlock.forward over stand-in submodules with the
    reference's names -- fused QKV 3072 -> 9216, 24 heads of 128 with RMSNorm + RoPE,
    block-causal prefill attention (256 causal text rows + 4096 image rows), out-proj
    3072 -> 3072, the SwiGLU MLP of the reference block (processors.py:180-187) with its
    fused up projection at BASELINE's 3072 -> 12288 (gate and up halves of 6144) and
    6144 -> 3072 down, the two LayerNorm + modulate and gated residuals -- preceded by the
    timestep-modulation FP8 linear (M = 2, 3072 -> 18432) whose first 4 x 3072 columns
    are the block's modulation rows.  Random-init FP8 weights, synthetic activations."""
    from qik import fp8 as F
    from qik.processors import QwenImage21KernelBlock, QwenImage21KernelProcessor
    H, D, K, B2, S2, HALF = 24, 128, 3072, 2, 4352, 6144

    def lin(n_out, n_in):
        f = F.FP8Linear(n_in, n_out).to(device)
        wq, sw = F.quantize_weight_tensorwise(torch.randn(n_out, n_in, device=device, generator=g) * 0.02)
        f.weight.copy_(wq)
        f.weight_scale.copy_(sw)
        return f

    attn = _Attention(H, lin(3 * K, K), lin(K, K), torch.ones(D, device=device), torch.ones(D, device=device))
    attn.set_processor(QwenImage21KernelProcessor())
    shell = torch.nn.Module()
    shell.img_norm1 = torch.nn.LayerNorm(K, elementwise_affine=False, eps=1e-6)
    shell.img_norm2 = torch.nn.LayerNorm(K, elementwise_affine=False, eps=1e-6)
    shell.attn = attn
    shell.img_mlp = torch.nn.Module()
    shell.img_mlp.fused_up = lin(2 * HALF, K)
    shell.img_mlp.out = lin(K, HALF)
    block = QwenImage21KernelBlock(shell)
    mod_lin = lin(6 * K, K)
    x = torch.randn(B2, S2, K, device=device, generator=g).to(torch.bfloat16)
    temb = torch.randn(B2, K, device=device, generator=g).to(torch.bfloat16)
    inv = 1.0 / (10000 ** (torch.arange(0, D, 2, device=device).float() / D))
    freqs = torch.polar(torch.ones(S2, D // 2, device=device),
                        torch.outer(torch.arange(S2, device=device).float(), inv))
    segments = [(0, 256, True)]

    def run():
        mod = mod_lin(temb)[:, :4 * K]
        return block(x, mod, rotary_emb=freqs, segments=segments)

    M = B2 * S2
    Lt = torch.arange(S2, dtype=torch.int64)
    Lt[256:] = S2 - 1
    lin_fl = 2.0 * M * K * (3 * K + K + 2 * HALF) + 2.0 * M * HALF * K + 2.0 * B2 * K * 6 * K
    at_fl = 4.0 * D * H * B2 * float((Lt + 1).sum())
    return {"block": run, "linear_flops": lin_fl, "attention_flops": at_fl}


PROFILE_CASES = ("attention_cfg4_prefill", "attention_cfg4_decode_fp8_slab", "dit_block_1024px_cfg2",
                 "dit_block_1024px_cfg2_gelu_ffn", "fused_ops_t2i", "modulation_linear", "quantizer_4352",
                 "quantizer_9472", "quantizer_16384", "gemm_256x3072", "gemm_256x12288")


def profile_case(device: torch.device, name: str) -> None:
    """Runs one workload three times (the launches an ncu capture selects from); for
    fused_ops_t2i each of the fused ops three times, for modulation_linear and gemm_<M>x<N>
    the FP8 linear and for quantizer_<M> the activation quantizer three times, an L2 flush
    before every launch."""
    g = torch.Generator(device=device).manual_seed(7)
    if name.startswith("quantizer_"):
        # the dynamic activation quantizer (qik_quantize_act) on M x 3072 bf16 rows
        from qik import fp8 as F
        x = torch.randn(int(name.split("_")[1]), 3072, device=device, generator=g).to(torch.bfloat16)
        flush = L2Flush(device)
        for r in range(3):
            flush(r)
            F.quantize_tensorwise(x)
    elif name.startswith("gemm_"):
        # a configs[4] FP8 linear (K = 3072) at skinny M, default tile configuration
        from qik import fp8 as F
        M, N = (int(v) for v in name.split("_")[1].split("x"))
        wq, sw = F.quantize_weight_tensorwise(torch.randn(N, 3072, device=device, generator=g) * 0.02)
        xq, sx = F.quantize_tensorwise(torch.randn(M, 3072, device=device, generator=g).to(torch.bfloat16))
        flush = L2Flush(device)
        for r in range(3):
            flush(r)
            F.fp8_gemm(xq, sx, wq, sw)
    elif name == "modulation_linear":
        # the DiT block's timestep-modulation FP8 linear: M = 2 (CFG batch) x 3072 -> 18432
        from qik import fp8 as F
        wq, sw = F.quantize_weight_tensorwise(torch.randn(18432, 3072, device=device, generator=g) * 0.02)
        xq, sx = F.quantize_tensorwise(torch.randn(2, 3072, device=device, generator=g).to(torch.bfloat16))
        flush = L2Flush(device)
        for r in range(3):
            flush(r)
            F.fp8_gemm(xq, sx, wq, sw)
    elif name == "fused_ops_t2i":
        x = torch.randn(2, 4352, 3072, device=device, generator=g).to(torch.bfloat16)
        mod = (torch.randn(2, 6 * 3072, device=device, generator=g) * 0.05).to(torch.bfloat16)
        flush = L2Flush(device)
        for i, (fn, _) in enumerate(fused_ops_cases(device, x, mod).values()):
            for r in range(3):
                flush(3 * i + r)
                fn()
    else:
        if name == "dit_block_1024px_cfg2":
            fn = dit_block_product_case(device, g)["block"]
        elif name == "dit_block_1024px_cfg2_gelu_ffn":
            fn = dit_block_case(device, g)["block"]
        else:
            fn = attention_cfg4_cases(device, g)[name][0]
        for _ in range(3):
            fn()
    torch.cuda.synchronize(device)
    from qik import _lib as L
    print(json.dumps({"profile_case": name, "runs": 3, "device_status": L.device_status(device)}), flush=True)


def extras(device: torch.device, flush: L2Flush, iters: int = 10) -> dict:
    """Attention at BASELINE config 4 and the DiT-block time at 1024 px (configs[2] +
    the t2i attention), each on synthetic inputs with the BASELINE shapes."""
    from qik import _lib as L
    stream = torch.cuda.current_stream(device)
    g = torch.Generator(device=device).manual_seed(7)
    out = {}
    for name, (fn, fl) in attention_cfg4_cases(device, g).items():
        for _ in range(3):
            fn()
        ms = _time_ms(fn, iters, flush, stream)
        out[name] = {"ms": round(ms, 4), "tflops": round(fl / ms / 1e9, 1), "gflop": round(fl / 1e9, 1)}
    prod = dit_block_product_case(device, g)
    for _ in range(3):
        prod["block"]()
    ms = _time_ms(prod["block"], iters, flush, stream)
    lin_fl, at_fl = prod["linear_flops"], prod["attention_flops"]
    out["dit_block_1024px_cfg2"] = {
        "ms": round(ms, 4), "tflops": round((lin_fl + at_fl) / ms / 1e9, 1),
        "linear_gflop": round(lin_fl / 1e9, 1), "attention_gflop": round(at_fl / 1e9, 1),
        "api": "qik.processors.QwenImage21KernelBlock.forward (+ the timestep-modulation FP8Linear)",
        "includes": "modulation GEMV (M=2, 3072->18432), 2x LayerNorm+modulate (each emitting its FP8 linear's "
                    "e4m3 input), fused QKV 3072->9216, "
                    "RMSNorm+RoPE (q, k), block-causal attention, out-proj, SwiGLU MLP (fused up 3072->12288 with "
                    "the SwiGLU in its GEMM epilogue, down 6144->3072), 2x gated residual"}
    case = dit_block_case(device, g)
    block = case["block"]
    for _ in range(3):
        block()
    ms = _time_ms(block, iters, flush, stream)
    lin_fl, at_fl = case["linear_flops"], case["attention_flops"]
    out["dit_block_1024px_cfg2_gelu_ffn"] = {
        "ms": round(ms, 4), "tflops": round((lin_fl + at_fl) / ms / 1e9, 1),
        "linear_gflop": round(lin_fl / 1e9, 1), "attention_gflop": round(at_fl / 1e9, 1),
        "api": "the same kernels composed by hand with BASELINE configs[2]'s FFN (3072->12288 GELU-tanh->3072, "
               "qik.fp8.fp8_ffn_gelu)",
        "includes": "modulation GEMV, 2x LayerNorm+modulate, RMSNorm+RoPE (q, k), attention, 4 FP8 linears "
                    "(GELU FFN), 2x gated residual"}
    out["fused_ops_t2i"] = fused_ops(device, flush, iters, case["x"], mod=case["mod"]())
    out["device_status"] = L.device_status(device)
    return out


def tp_stack(device: torch.device, rank: int, world: int, flush: L2Flush, iters: int = 5) -> dict:
    """BASELINE configs[4]'s layer-stack case: 4 DiT blocks at 1024 px, CFG batch 2
    (M = 8704), tensor parallel over `world` GPUs -- QKV by heads and FFN-up column-
    parallel, attention on local heads, out-proj and FFN-down row-parallel with a
    4-byte amax all-reduce(MAX) and the partial products summed as the library's
    comm="auto" does: over NVLink peer memory by the GEMM's own epilogue on 2 ranks, by
    an fp32 NCCL all-reduce(SUM) on more (both forms timed beside it).  Strong scaling:
    the total work is fixed.  Time = max over ranks."""
    from qik import fp8 as F
    from qik import parallel as PX
    H, D, K, HID, B, S = 24, 128, 3072, 12288, 2, 4352
    g = torch.Generator(device=device).manual_seed(11)
    fulls = []
    for _ in range(4):
        full = {}
        for name, (n, kk) in {"qkv": (3 * H * D, K), "out": (K, H * D), "up": (HID, K), "down": (K, HID)}.items():
            w = torch.randn(n, kk, device=device, generator=g) * 0.02
            full[name] = (*F.quantize_weight_tensorwise(w), None)
        fulls.append(full)
    x = torch.randn(B * S, K, device=device, generator=g).to(torch.bfloat16)
    Lt = torch.arange(S, dtype=torch.int32, device=device)
    Lt[256:] = S - 1

    M = B * S
    lo_sp, hi_sp = rank * (M // world), (rank + 1) * (M // world)
    x_local = x[lo_sp:hi_sp].contiguous()

    def make_stack(blocks, sp: bool):
        def stack():
            if sp:  # sequence parallel: this rank's rows between the blocks
                h, amax = x_local, None
                for blk in blocks:
                    h, amax = blk.forward_sp(h, B, S, Lt, amax)
                return h
            h = x
            for blk in blocks:
                h = blk(h, B, S, Lt)
            return h
        return stack

    def timed(chunks: int, comm: str = "nccl", sp: bool = False) -> float:
        """Mean ms per 4-block stack (max over ranks) with `chunks` row blocks per
        row-parallel GEMM / all-reduce (1 = one all-reduce after the whole GEMM), or with
        the row-parallel sums over NVLink peer memory fused with the GEMM (comm="peer"),
        or sequence parallel (sp: reduce-scatter + e4m3 all-gather over NCCL)."""
        blocks = [PX.TPBlock.from_full(full, H, D, rank, world, chunks=chunks, comm=comm, sequence_parallel=sp)
                  for full in fulls]
        stack = make_stack(blocks, sp)

        stream = torch.cuda.current_stream(device)
        for _ in range(2):
            stack()
        torch.cuda.synchronize(device)
        if world > 1:
            torch.distributed.barrier()
        evs = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(iters)]
        torch.cuda._sleep(int(2e7))
        for i in range(iters):
            flush(i)
            evs[i][0].record(stream)
            stack()
            evs[i][1].record(stream)
        torch.cuda.synchronize(device)
        t = torch.tensor([sum(a.elapsed_time(b) for a, b in evs) / iters], dtype=torch.float64, device=device)
        if world > 1:
            torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX)
            torch.distributed.barrier()  # no rank still writes into a peer's workspace
        for blk in blocks:
            for lin in (blk.out, blk.down):
                for red in lin._peer.values():
                    if red:
                        red.close()
        return float(t.item())

    def stack_output(comm: str, sp: bool = False, n_blocks: int = 4) -> torch.Tensor:
        blocks = [PX.TPBlock.from_full(full, H, D, rank, world, chunks=1, comm=comm, sequence_parallel=sp)
                  for full in fulls[:n_blocks]]
        h = make_stack(blocks, sp)().clone()
        torch.cuda.synchronize(device)
        if world > 1:
            torch.distributed.barrier()
        for blk in blocks:
            for lin in (blk.out, blk.down):
                for red in lin._peer.values():
                    if red:
                        red.close()
        return h

    parity = None
    if world > 1:
        # the same stack with the row-parallel sums over peer memory and by NCCL's
        # all-reduce: on 2 ranks both add two fp32 terms, so they must agree bit for bit
        y_peer, y_nccl = stack_output("peer"), stack_output("nccl")
        y_sp = stack_output("nccl", sp=True)
        y_nccl_rows = y_nccl[lo_sp:hi_sp]
        def relf(a, b):
            return ((a.float() - b.float()).norm() / b.float().norm().clamp_min(1e-30)).item()

        same = torch.tensor([1.0 if torch.equal(y_peer, y_nccl) else 0.0,
                             (y_peer.float() - y_nccl.float()).abs().max().item(), relf(y_peer, y_nccl),
                             1.0 if torch.equal(y_sp, y_nccl_rows) else 0.0,
                             (y_sp.float() - y_nccl_rows.float()).abs().max().item(), relf(y_sp, y_nccl_rows),
                             y_nccl.float().abs().max().item()], dtype=torch.float64, device=device)
        ops = (torch.distributed.ReduceOp.MIN, torch.distributed.ReduceOp.MAX, torch.distributed.ReduceOp.MAX) * 2
        for i, op in enumerate(ops + (torch.distributed.ReduceOp.MAX,)):
            torch.distributed.all_reduce(same[i:i + 1], op=op)
        parity = {"bit_identical_all_ranks": bool(same[0].item() == 1.0), "max_abs_diff": float(same[1].item()),
                  "relF": float(same[2].item()), "max_abs_output": float(same[6].item()),
                  "expected": "bit-identical on 2 ranks (two-term fp32 sums commute); on more ranks NCCL's "
                              "summation order differs from the rank-order sum in the last bits, and every "
                              "later FP8 linear re-quantizes with a dynamic per-tensor scale over a stack "
                              "with no normalisation, so after 4 blocks the forms can differ well beyond "
                              "rounding (relF 0.07-0.09 measured on 4 and 8 ranks); one block of every "
                              "form is gated against the single-GPU block below",
                  "sequence_parallel_vs_allreduce": {
                      "bit_identical_all_ranks": bool(same[3].item() == 1.0), "max_abs_diff": float(same[4].item()),
                      "relF": float(same[5].item()),
                      "compared": "each rank's rows of the 4-block stack output, sequence parallel vs the "
                                  "NCCL all-reduce form"}}
        # one block of every form against the single-GPU block, computed by rank 0 alone
        # (a group of one rank: no collective) and broadcast
        g0 = torch.distributed.new_group([0])
        if rank == 0:
            ref1 = PX.TPBlock.from_full(fulls[0], H, D, 0, 1, group=g0)(x, B, S, Lt).contiguous()
        else:
            ref1 = torch.empty(M, K, dtype=torch.bfloat16, device=device)
        torch.distributed.broadcast(ref1, src=0)
        one = torch.tensor([relf(stack_output("peer", n_blocks=1), ref1),
                            relf(stack_output("nccl", n_blocks=1), ref1),
                            relf(stack_output("nccl", sp=True, n_blocks=1), ref1[lo_sp:hi_sp])],
                           dtype=torch.float64, device=device)
        torch.distributed.all_reduce(one, op=torch.distributed.ReduceOp.MAX)
        parity["one_block_vs_single_gpu_relF"] = {
            "peer": float(one[0].item()), "nccl_allreduce": float(one[1].item()),
            "sequence_parallel": float(one[2].item()), "gate": 5e-3,
            "pass": bool(one.max().item() <= 5e-3)}
    ms_peer = timed(1, "peer")
    ms_nccl = timed(1, "nccl") if world > 1 else ms_peer
    ms_overlap = timed(4, "nccl") if world > 1 else ms_peer
    ms_sp = timed(1, "nccl", sp=True) if world > 1 else ms_peer
    ms = ms_peer if world <= 2 else ms_nccl  # comm="auto", the library default
    lin = 2.0 * M * K * (3 * H * D + K + HID) + 2.0 * M * HID * K
    att = 4.0 * D * H * B * float((Lt.long() + 1).sum())
    total = 4 * (lin + att)
    res = {"ms": round(ms, 4), "tflops_total": round(total / ms / 1e9, 1),
            "tflops_per_gpu": round(total / ms / 1e9 / world, 1), "n_gpus": world, "scaling": "strong",
            "form": ("one GPU" if world == 1 else
                     "comm='auto' = peer: row-parallel GEMM epilogue stores fp32 tiles into the owner rank's "
                     "memory over NVLink (CUDA IPC), owner sums its rows and stores bf16 rows into every rank "
                     "(qik_fp8_gemm_scatter + qik_tp_reduce_gather + qik_tp_wait)" if world == 2 else
                     "comm='auto' = nccl: fp32 all-reduce(SUM) of the partial products (faster than the "
                     "peer-memory form from 4 ranks)"),
            "ms_peer_reduction": round(ms_peer, 4),
            "ms_nccl_allreduce": round(ms_nccl, 4),
            "ms_nccl_overlapped_4_blocks": round(ms_overlap, 4),
            "ms_sequence_parallel": round(ms_sp, 4),
            "sequence_parallel_form": "activations kept as row shards between the linears: reduce-scatter of "
                                      "the fp32 partial products, bias + bf16 on the rank's rows, e4m3 rows "
                                      "all-gathered (global scale by a 4-byte all-reduce MAX) before each "
                                      "column-parallel GEMM" if world > 1 else "n/a",
            "overlapped_form": "row-parallel GEMMs in 4 row blocks, each block's all-reduce on a side stream "
                               "under the next block's GEMM (slower here: NCCL's kernels take SMs from the "
                               "persistent GEMM)" if world > 1 else "n/a",
            "collectives_per_stack": "8 x row reductions of fp32 [8704, 3072] partial products "
                                     "+ 8 x all-reduce(MAX) 4 bytes (NCCL)" if world > 1 else "none"}
    if parity is not None:
        res["parity"] = parity
    return res


def row_shard_sweep(device: torch.device, rank: int, world: int, flush: L2Flush, iters: int = 10) -> list:
    """BASELINE configs[4] at this world size: the FP8 linear at K = 3072 for N in
    {3072, 9216, 12288, 18432} and M in {256, 1024, 4352, 9472, 16384}, the M token rows
    split across the ranks (rank r takes M // world rows, one more for r < M % world;
    strong scaling), no collective on the data path: each rank quantizes its rows and
    runs the GEMM.  Time per shape = max over ranks of the mean CUDA-event time of one
    launch; TFLOP/s = 2 M N K / that time."""
    from qik import fp8 as F
    stream = torch.cuda.current_stream(device)
    g = torch.Generator(device=device).manual_seed(5 + rank)
    K = 3072
    rows = []
    for N in (3072, 9216, 12288, 18432):
        wq, sw = F.quantize_weight_tensorwise(torch.randn(N, K, device=device, generator=g) * 0.02)
        for M in (256, 1024, 4352, 9472, 16384):
            m_r = M // world + (1 if rank < M % world else 0)
            x = torch.randn(m_r, K, device=device, generator=g).to(torch.bfloat16)
            xq, sx = F.quantize_tensorwise(x)
            fn = lambda: F.fp8_gemm(xq, sx, wq, sw)  # noqa: E731
            for _ in range(3):
                fn()
            t = torch.tensor([_time_ms(fn, iters, flush, stream)], dtype=torch.float64, device=device)
            if world > 1:
                torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX)
            ms = float(t.item())
            rows.append({"M": M, "N": N, "rows_per_rank": M // world, "ms": round(ms, 4),
                         "tflops_total": round(2.0 * M * N * K / ms / 1e9, 1)})
    return rows


# ------------------------------------------------------------------------------ CPU arm
def cpu_ffn_reference(x: torch.Tensor, w1q, s1, w2q, s2) -> torch.Tensor:
    """The reference's arithmetic on CPU tensors, in PyTorch: dynamic per-tensor e4m3
    quantization (fp8.py:24-53), dequantized fp32 matmul (the fp32-accumulated path
    of fp8.py:87), bf16 output, GELU-tanh, re-quantization, second matmul."""
    def quant(a):
        s = (a.abs().amax().float() / 448.0).clamp_min(1e-12)
        return (a.float() * (1.0 / s)).to(torch.float8_e4m3fn), s

    xq, sx = quant(x)
    y1 = ((xq.float() * sx) @ (w1q.float() * s1).t()).to(torch.bfloat16)
    h = torch.nn.functional.gelu(y1.float(), approximate="tanh").to(torch.bfloat16)
    hq, sh = quant(h)
    return ((hq.float() * sh) @ (w2q.float() * s2).t()).to(torch.bfloat16)


def _cpu_weights():
    x, w1, w2 = make_inputs(4321, torch.device("cpu"))

    def wquant(w):
        s = (w.abs().amax().float() / 448.0).clamp_min(1e-12)
        return (w.float() / s).clamp(-448, 448).to(torch.float8_e4m3fn), s

    return x, wquant(w1), wquant(w2)


def cpu_baseline(args, budget_s: float = 12.0) -> dict:
    """The reference's arithmetic timed on the host cores (all of them) on the whole
    configs[1] workload: FFN pair over all 4352 rows per repetition, as many repetitions
    as fit in `budget_s` (at least one)."""
    threads = os.cpu_count() or 1
    torch.set_num_threads(threads)
    x, (w1q, s1), (w2q, s2) = _cpu_weights()
    cpu_ffn_reference(x[:64], w1q, s1, w2q, s2)                          # warm-up
    reps, t0 = 0, time.perf_counter()
    while True:
        cpu_ffn_reference(x, w1q, s1, w2q, s2)
        reps += 1
        el = time.perf_counter() - t0
        if el >= budget_s or reps >= 50:
            break
    flops = FLOPS_PER_STEP * reps
    return {"value": round(flops / el / 1e12, 4), "unit": "TFLOP/s", "cores": threads, "kind": "port",
            "sample": f"{reps} x FFN pair on all {M_ROWS} rows (configs[1], same shapes and weights), {el:.1f} s "
                      f"wall, PyTorch CPU fp32 dequant matmuls"}


def ffn_parity(x_cpu: torch.Tensor, up, down, y_chain: torch.Tensor) -> dict:
    """The checker leg: this rank's configs[1] step checked stage by stage against the
    CPU oracle (oracle/, the tests' checker) on the step's own intermediates -- the input
    quantizer (bytes and scale bit-exact), GEMM1 + GELU-tanh on the product's e4m3 x
    (relF), the hidden activation's pack (bit-exact), GEMM2 on the product's e4m3 h
    (relF) -- and the fused chain's output against the same step launched stage by stage
    (bit-identical)."""
    import numpy as np
    from oracle import oracle as O
    from qik import _lib as L
    from qik import fp8 as F
    dev = y_chain.device
    x = x_cpu.to(dev)
    xq, sx = F.quantize_tensorwise(x)
    amax = torch.zeros(1, dtype=torch.int32, device=dev)
    h = F.fp8_gemm(xq, sx, up.weight, up.weight_scale, up.bias, epilogue=L.EPI_GELU_TANH, amax_out=amax)
    hq, sh = F.quantize_from_amax(h, amax)
    y = F.fp8_gemm(hq, sh, down.weight, down.weight_scale, down.bias)
    torch.cuda.synchronize(dev)
    torch.set_num_threads(os.cpu_count() or 1)
    q_ref, s_ref = O.quantize_act(x_cpu, O.SCALE_CUDA)
    x_exact = bool(np.array_equal(xq.cpu().view(torch.uint8).numpy(), q_ref)
                   and np.float32(s_ref) == np.float32(sx.item()))
    h_ref = O.gelu_tanh(O.fp8_linear(xq.cpu(), float(sx.item()), up.weight.cpu(),
                                     float(up.weight_scale.item())).to(torch.bfloat16))
    r1 = O.relf(h.cpu(), h_ref)
    hq_ref, sh_ref = O.quantize_act(h.cpu(), O.SCALE_CUDA)
    h_exact = bool(np.array_equal(hq.cpu().view(torch.uint8).numpy(), hq_ref)
                   and np.float32(sh_ref) == np.float32(sh.item()))
    y_ref = O.fp8_linear(hq.cpu(), float(sh.item()), down.weight.cpu(), float(down.weight_scale.item()))
    r2 = O.relf(y.cpu(), y_ref)
    ident = bool(torch.equal(y, y_chain))
    ok = x_exact and h_exact and r1 <= 5e-3 and r2 <= 5e-3 and ident
    return {"x_quant_bit_exact": x_exact, "gemm1_gelu_relF": float(f"{r1:.3e}"), "h_pack_bit_exact": h_exact,
            "gemm2_relF": float(f"{r2:.3e}"), "chain_vs_stages_bit_identical": ident,
            "rows_checked": int(x_cpu.shape[0]), "gate": "quantizers bit-exact, relF <= 5e-3 per GEMM stage",
            "pass": ok}


def run_reference(args, rank: int, world: int) -> dict | None:
    """--impl reference: the reference's arithmetic (cpu_ffn_reference) on the host cores,
    every step one FFN pair over the whole configs[1] workload (all 4352 rows), W untimed
    warm-up steps then K timed ones; rank 0 alone runs it."""
    if rank != 0:
        return None
    threads = os.cpu_count() or 1
    torch.set_num_threads(threads)
    x, (w1q, s1), (w2q, s2) = _cpu_weights()
    for _ in range(args.warmup):
        cpu_ffn_reference(x, w1q, s1, w2q, s2)
    t0 = time.perf_counter()
    for _ in range(args.steps):
        cpu_ffn_reference(x, w1q, s1, w2q, s2)
    el = time.perf_counter() - t0
    value = round(FLOPS_PER_STEP * args.steps / el / 1e12, 4)
    cb = {"value": value, "unit": "TFLOP/s", "cores": threads, "kind": "port",
          "sample": f"{args.steps} timed x FFN pair on all {M_ROWS} rows after {args.warmup} warm-up steps, "
                    f"{el:.1f} s wall, PyTorch CPU fp32 dequant matmuls"}
    return {"metric": METRIC, "value": value, "unit": "TFLOP/s", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": round(el / args.steps * 1e3, 2), "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "e4m3 quantize + fp32 dequant matmul (CPU)",
            "data": "synthetic: N(0,1) activations with 8 outlier channels x20, N(0,0.02) random-init weights",
            "config": bench_config(world),
            "impl": "reference", "cpu_baseline": cb,
            "e2e": {"value": value, "unit": "TFLOP/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}


def sweep(device: torch.device, iters: int = 20, tiles: bool = False) -> list[dict]:
    """the FP8 linear at K = 3072 over N x M, qik's tcgen05 GEMM
    next to cuBLASLt (torch._scaled_mm, the reference's call, fp8.py:87-88) on the same
    e4m3 operands and scales, and the dynamic activation quantizer at each M
    (3 algorithmic bytes per element).  One JSON line per shape.  With ``tiles`` every
    GEMM tile configuration is also timed forced (qik_fp8_gemm_tiled), and the FFN's
    second GEMM (4352 x 3072, K = 12288) is added."""
    from qik import fp8 as F
    stream = torch.cuda.current_stream(device)
    flush = L2Flush(device)
    pk = peaks()
    g = torch.Generator(device=device).manual_seed(5)
    K = 3072
    rows = []
    from qik import _lib as L
    tile_names = {L.GEMM_TILE_PAIR_256: "pair256", L.GEMM_TILE_SINGLE_256: "single256",
                  L.GEMM_TILE_SINGLE_128: "single128", L.GEMM_TILE_SINGLE_64: "single64"}
    shapes = [(M, N, K) for N in (3072, 9216, 12288, 18432) for M in (256, 1024, 4352, 9472, 16384)]
    if tiles:
        shapes.append((4352, 3072, 12288))
    weights = {}
    for M, N, Kx in shapes:
        if (N, Kx) not in weights:
            weights[(N, Kx)] = F.quantize_weight_tensorwise(torch.randn(N, Kx, device=device, generator=g) * 0.02)
        wq, sw = weights[(N, Kx)]
        K = Kx
        x = torch.randn(M, K, device=device, generator=g).to(torch.bfloat16)
        xq, sx = F.quantize_tensorwise(x)
        runs = {"qik": lambda: F.fp8_gemm(xq, sx, wq, sw),
                "cublaslt": lambda: torch._scaled_mm(xq, wq.t(), scale_a=sx, scale_b=sw,
                                                     out_dtype=torch.bfloat16)}
        if tiles:
            for c, name in tile_names.items():
                runs[name] = (lambda c=c: F.fp8_gemm(xq, sx, wq, sw, tile_cfg=c))
        row = {"M": M, "N": N, "K": K, "gflop": round(2.0 * M * N * K / 1e9, 2)}
        for name, fn in runs.items():
            for _ in range(3):
                fn()
            ms = _time_ms(fn, iters, flush, stream)
            row[f"{name}_us"] = round(ms * 1e3, 2)
            row[f"{name}_tflops"] = round(2.0 * M * N * K / ms / 1e9, 1)
        row["qik_vs_cublaslt"] = round(row["cublaslt_us"] / row["qik_us"], 3)
        row["qik_frac_fp8_peak"] = round(row["qik_tflops"] / pk["fp8_tflops_burst"], 3)
        if N == 3072 and K == 3072:
            fn = lambda: F.quantize_tensorwise(x)  # noqa: E731
            for _ in range(3):
                fn()
            ms = _time_ms(fn, iters, flush, stream)
            row["quantizer_us"] = round(ms * 1e3, 2)
            row["quantizer_gbs"] = round(3.0 * M * K / ms / 1e6, 1)
            row["quantizer_frac_hbm"] = round(row["quantizer_gbs"] / pk["hbm_gbs"], 3)
        rows.append(row)
    return rows


def load_reference_gpu_modules() -> dict:
    """The reference's own leaf modules (fp8.py with its Triton cast kernel,
    triton_attention.py with _qwen21_attn_fwd) from the copy of its package under
    baseline/_ref, loaded by file path under a synthetic package (its __init__ needs
    the diffusers runtime).  Used only by --reference-bars."""
    import importlib.util
    import types
    ref_dir = ROOT / "baseline" / "_ref" / "qwen_image_kernel"
    if not (ref_dir / "fp8.py").exists():
        raise SystemExit(f"--reference-bars needs the reference package under {ref_dir}")
    pkg = types.ModuleType("qwen_image_kernel")
    pkg.__path__ = [str(ref_dir)]
    sys.modules["qwen_image_kernel"] = pkg
    mods = {}
    for name in ("fp8", "triton_attention"):
        spec = importlib.util.spec_from_file_location(f"qwen_image_kernel.{name}", ref_dir / f"{name}.py")
        m = importlib.util.module_from_spec(spec)
        sys.modules[f"qwen_image_kernel.{name}"] = m
        spec.loader.exec_module(m)
        mods[name] = m
    return mods


def reference_bars(device: torch.device) -> dict:
    """The reference's own GPU kernels on this B200 beside qik's, same inputs (the bars
    of the reference's paths that run here): quantize_tensorwise (aten amax + the
    Triton _scale_cast_fp8_kernel, fp8.py:24-53) at configs[4] row counts, with the
    bytes and scale compared, and block_causal_flash_attention (Triton
    _qwen21_attn_fwd recompiled for sm_100, triton_attention.py:35-260) at config 4 in
    both forms.  CUDA events, L2 flushed between launches."""
    from qik import fp8 as F
    from qik.kv_cache import ContiguousKVCache
    from qik.triton_attention import block_causal_flash_attention as qattn
    import triton
    mods = load_reference_gpu_modules()
    rattn = mods["triton_attention"].block_causal_flash_attention
    flush = L2Flush(device)
    st = torch.cuda.current_stream(device)
    res = {"triton": triton.__version__}
    for M in (4352, 9472, 16384):
        x = torch.randn(M, 3072, device=device).to(torch.bfloat16)
        for nm, fn in (("reference", lambda: mods["fp8"].quantize_tensorwise(x)), ("qik", lambda: F.quantize_tensorwise(x))):
            for _ in range(3):
                fn()
            ms = _time_ms(fn, 20, flush, st)
            res[f"quantizer_{M}_{nm}_us"] = round(ms * 1e3, 2)
            res[f"quantizer_{M}_{nm}_gbs"] = round(3 * M * 3072 / ms / 1e6, 1)
        qr, sr = mods["fp8"].quantize_tensorwise(x)
        qq, sq = F.quantize_tensorwise(x)
        res[f"quantizer_{M}_bytes_and_scale_equal"] = bool(torch.equal(qr.view(torch.uint8), qq.view(torch.uint8))
                                                           and torch.equal(sr.reshape(-1), sq.reshape(-1)))
    g = torch.Generator(device=device).manual_seed(9)
    H, D, S = 24, 128, 6656
    q, k, v = (torch.randn(1, S, H, D, device=device, generator=g, dtype=torch.bfloat16) for _ in range(3))
    Lp = torch.arange(S, dtype=torch.int32, device=device)
    Lp[256:2560] = 2559
    Lp[2560:] = S - 1
    fl_p = 4.0 * D * H * float((Lp.long() + 1).sum())
    P, T = 2560, 4096
    kp, vp = (torch.randn(1, P, H, D, device=device, generator=g, dtype=torch.bfloat16) for _ in range(2))
    cache = ContiguousKVCache(1, 1, P, H, D, v_fp8=True, device=device)
    cache.get_layer(0).store(kp, vp)
    ck, cv, vs = cache.get_layer(0).views()
    qd, kn, vn = (torch.randn(1, T, H, D, device=device, generator=g, dtype=torch.bfloat16) for _ in range(3))
    Ld = torch.full((T,), P + T - 1, dtype=torch.int32, device=device)
    fl_d = 4.0 * D * H * T * (P + T)
    forms = {"attention_cfg4_prefill": ((q, k, v, Lp, None), {}, fl_p),
             "attention_cfg4_decode_fp8_slab": ((qd, kn, vn, Ld, None, ck, cv, vs), {"uniform_full": True}, fl_d)}
    for name, (a, kw, fl) in forms.items():
        for nm, fn in (("reference", lambda: rattn(*a, **kw)), ("qik", lambda: qattn(*a, **kw))):
            for _ in range(3):
                fn()
            ms = _time_ms(fn, 10, flush, st)
            res[f"{name}_{nm}_ms"] = round(ms, 4)
            res[f"{name}_{nm}_tflops"] = round(fl / ms / 1e9, 1)
        o_r, o_q = rattn(*a, **kw).float(), qattn(*a, **kw).float()
        res[f"{name}_relF_qik_vs_reference"] = float(f"{((o_q - o_r).norm() / o_r.norm()).item():.3e}")
    return res


def main() -> int:
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=["qik", "reference"], default="qik")
    ap.add_argument("--no-extras", action="store_true", help="skip the attention / DiT-block measurements")
    ap.add_argument("--sweep", action="store_true",
                    help="print the configs[4] GEMM / quantizer sweep (one JSON line per shape) instead of the bench")
    ap.add_argument("--sweep-tiles", action="store_true",
                    help="--sweep with every GEMM tile configuration forced beside the default")
    ap.add_argument("--reference-bars", action="store_true",
                    help="time the reference's own GPU kernels (from the copy under baseline/_ref) beside qik's")
    ap.add_argument("--profile-case", choices=PROFILE_CASES,
                    help="run one extras workload three times and exit (the launches an ncu capture selects from)")
    args = ap.parse_args()
    if args.warmup < 3:
        args.warmup = 3

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if args.impl == "reference":
        res = run_reference(args, rank, world)
        if res is not None:
            print(json.dumps(res), flush=True)
        return 0

    device = torch.device("cuda", local)
    torch.cuda.set_device(device)
    if args.profile_case:
        profile_case(device, args.profile_case)
        return 0
    if args.reference_bars:
        print(json.dumps(reference_bars(device)), flush=True)
        return 0
    if args.sweep or args.sweep_tiles:
        for row in sweep(device, tiles=args.sweep_tiles):
            print(json.dumps(row), flush=True)
        return 0
    if world > 1:
        import datetime
        torch.distributed.init_process_group("nccl", device_id=device, timeout=datetime.timedelta(seconds=120))
    try:
        res = run_qik(args, rank, world, device)
    finally:
        if world > 1:
            torch.distributed.destroy_process_group()
    if res is not None:
        print(json.dumps(res), flush=True)
    return 0


if __name__ == "__main__":
    sys.exit(main())
