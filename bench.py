#!/usr/bin/env python3
"""bench.py — GEMM TFLOPS at 8192^3 on B200 (fp16 headline, fp8 alongside), and the
config-5 column split across the GPUs of the box.

Metric: "GEMM TFLOPS fp16 & fp8 at 8192^3 per B200 and 8-GPU box;
% of dense tensor peak". One step = one GEMM launch over resident inputs.

  python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
  python bench.py --mode sweep|profile|power ...        (measurement helpers, below)

Our arm (default, --mode headline):
  * value: C[8192, 8192*N] = A[8192,8192] . B[8192*N,8192]^T split column-wise, one
    8192 x 8192 C slab per GPU (A replicated, B row slab per GPU), fp16 in, fp32
    accumulate, fp16 out, through the C ABI (b200_gemm), inputs resident in HBM
    (256 MiB per GPU, above the 126 MB L2, so no flush between steps). Per-GPU work
    is fixed as N grows ("scaling": "weak"); value = total flops / max-over-ranks time.
    At N = 1 this is BASELINE's 8192^3 fp16 configuration.
  * fp8 (e4m3, per-tensor scales, bf16 out) at 8192^3 per GPU, measured the same way;
    cuBLASLt (torch.matmul / torch._scaled_mm) on the same shapes as a reference column.
  * pct_of_dense_peak: kernel TFLOPS / (SMs x max SM clock x 8192 FLOP/clk/SM), the
    dense peak read from the device; roofline.frac: the same against the measured
    cuBLAS bf16 peak in MEASURED_PEAKS.json.
  * e2e: the same metric through the public API with host buffers: A uploaded once
    per node (rank 0) and broadcast to the other GPUs over NVLink (NCCL), each GPU's
    B slab uploaded by its rank, b200_gemm, C slab downloaded, every step, pipelined
    over streams with double-buffered device operands.
  * strong_split: BASELINE config 5, e4m3 M=16384, N=65536, K=8192 (per-tensor scales,
    bf16 C) with N split evenly across the N GPUs ("scaling": strong, total work
    fixed): whole-box TFLOPS = total flops / max-over-ranks time. For N > 1 the
    all-gather of C is timed separately: NCCL all-gather + re-layout to M x N, and the
    fused GEMM + all-gather (b200_gemm_allgather: the epilogue stores every C tile into
    every GPU's M x N buffer over NVLink), checked bit-identical; and its own e2e
    (A uploaded once and broadcast, B slab up, C slab down per step).
  * cpu_baseline: the reference's host GEMM loop (oracle port) on a bounded row band
    of the same fp16 problem, on this host's cores (rank 0, N = 1 only).

Reference arm (--impl reference): the reference's CPU GEMM (oracle port of
src/05_gemm/gemm_ws.cu:258-265, verbatim loop order, all host threads) timed on
row bands of the same 8192^3 fp16 problem; rank 0 only.

Measurement helpers (single GPU; the committed profiles/ summaries cite them):
  --mode profile  <f16|e4m3> <ours|cublas> [variant] [size] [tile_n] [group_m]: three warm-up
                  launches, then one inside cudaProfilerStart/Stop for
                  `ncu --profile-from-start off`.
  --mode power    <f16|bf16|e4m3> <config>...: sustained TFLOPS, energy per GEMM (NVML
                  total-energy counter), board power and SM clock under the power cap,
                  configurations interleaved in rounds; a config is `cublas` or
                  `<variant>[:tile_n[:group_m]][@ENV=V,...]` (environment set before each
                  call, read by experimental builds only).
  --mode sweep    [--dtypes f16,e4m3] [--shapes MxNxK,...] [config...]: launch time of
                  every pair schedule and tile width (or of the configs given) and of
                  cuBLASLt per shape (CUDA events, median of --steps launches), plus the
                  library's AUTO choice.
"""
from __future__ import annotations

import argparse
import ctypes as C
import importlib.util
import json
import os
import statistics
import sys
import threading
import time
from pathlib import Path

ROOT = Path(__file__).resolve().parent
M = N = K = 8192
FLOPS_8192 = 2.0 * M * N * K
# BASELINE config 5, multi-GPU shape: N split across the GPUs
M5, N5, K5 = 16384, 65536, 8192
FLOPS_5 = 2.0 * M5 * N5 * K5


def load_pkg():
    if "hopper_lab_b200" in sys.modules:
        return sys.modules["hopper_lab_b200"]
    spec = importlib.util.spec_from_file_location("hopper_lab_b200",
                                                  ROOT / "hopper-lab_b200" / "__init__.py")
    mod = importlib.util.module_from_spec(spec)
    sys.modules["hopper_lab_b200"] = mod
    spec.loader.exec_module(mod)
    return mod


def load_multigpu():
    spec = importlib.util.spec_from_file_location("b200_multigpu", ROOT / "hopper-lab_b200" / "multigpu.py")
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


def measured_peaks():
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return {"bf16": d.get("bf16_tflops"), "bf16_sustained": d.get("bf16_tflops_sustained"),
                "hbm": d.get("hbm_gbs"), "source": "measured"}
    return {"bf16": 1590.0, "bf16_sustained": 1400.0, "hbm": 6650.0, "source": "fallback"}


def profile_traffic(kind: str):
    """DRAM bytes (read + write) per launch of the dominant kernel, from a line
    `traffic[<kind>] = <bytes>` in a committed ncu summary under profiles/, or None."""
    import re

    pat = re.compile(r"^traffic\[" + re.escape(kind) + r"\]\s*=\s*(\d+)", re.M)
    for f in sorted((ROOT / "profiles").glob("*.md")):
        m = pat.search(f.read_text())
        if m:
            return int(m.group(1))
    return None


class ClockSampler:
    """Samples SM clock and throttle reasons through NVML while the timed region runs."""

    REASONS = {
        0x1: "gpu_idle", 0x2: "applications_clocks_setting", 0x4: "sw_power_cap",
        0x8: "hw_slowdown", 0x10: "sync_boost", 0x20: "sw_thermal_slowdown",
        0x40: "hw_thermal_slowdown", 0x80: "hw_power_brake_slowdown",
        0x100: "display_clock_setting",
    }

    def __init__(self, index: int, period: float = 0.01):
        self.samples, self.reasons, self.max_mhz = [], 0, None
        self.period, self._stop = period, threading.Event()
        self.ok = False
        try:
            import pynvml

            pynvml.nvmlInit()
            self.nv = pynvml
            self.h = pynvml.nvmlDeviceGetHandleByIndex(index)
            self.max_mhz = pynvml.nvmlDeviceGetMaxClockInfo(self.h, pynvml.NVML_CLOCK_SM)
            self.ok = True
        except Exception:
            self.ok = False

    def _loop(self):
        while not self._stop.is_set():
            try:
                self.samples.append(self.nv.nvmlDeviceGetClockInfo(self.h, self.nv.NVML_CLOCK_SM))
                self.reasons |= self.nv.nvmlDeviceGetCurrentClocksEventReasons(self.h)
            except Exception:
                pass
            time.sleep(self.period)

    def __enter__(self):
        if self.ok:
            self.t = threading.Thread(target=self._loop, daemon=True)
            self.t.start()
        return self

    def __exit__(self, *exc):
        if self.ok:
            self._stop.set()
            self.t.join()

    def summary(self):
        if not self.ok:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvml_unavailable"]}
        names = [n for bit, n in self.REASONS.items() if self.reasons & bit and n != "gpu_idle"]
        return {"sm_mhz": statistics.median(self.samples) if self.samples else None,
                "sm_max_mhz": self.max_mhz, "reasons": names, "samples": len(self.samples)}


def dense_peak(torch, dev_index: int, max_mhz):
    """Dense f16/bf16 peak from the device: SMs x max SM clock x 8192 FLOP/clk/SM (the
    tcgen05 rate peak_tcgen05 measures; e4m3 is twice that)."""
    sms = torch.cuda.get_device_properties(dev_index).multi_processor_count
    mhz = max_mhz or 1965
    return {"tflops": round(sms * mhz * 1e6 * 8192 / 1e12, 1),
            "from": f"{sms} SMs x {mhz} MHz (max SM clock) x 8192 FLOP/clk/SM"}


def dist_env():
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    return rank, world, local


def timed_loop(torch, fn, steps: int, warmup: int, stream):
    """W warm-up calls, then K timed calls bracketed by synchronize; CUDA events on
    the launching stream, one pair per launch. Returns (total_ms, per_launch_ms list)."""
    for _ in range(warmup):
        fn()
    torch.cuda.synchronize()
    ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
          for _ in range(steps)]
    t0 = torch.cuda.Event(enable_timing=True)
    t1 = torch.cuda.Event(enable_timing=True)
    with torch.cuda.stream(stream):
        t0.record(stream)
        for s, e in ev:
            s.record(stream)
            fn()
            e.record(stream)
        t1.record(stream)
    torch.cuda.synchronize()
    per = [s.elapsed_time(e) for s, e in ev]
    return t0.elapsed_time(t1), per


def launch_stats(per):
    """Min / median / mean of the per-launch event times of one rank (ms)."""
    return {"min": round(min(per), 5), "median": round(statistics.median(per), 5),
            "mean": round(statistics.fmean(per), 5)}


def e4m3_rows(torch, rows, cols, gen, dev, chunk=4096):
    """Seeded uniform[-1,1] fp32 values quantised to e4m3 with the per-tensor scale
    amax/448 (amax of uniform[-1,1] taken as 1), generated in row chunks so that the
    fp32 staging stays small. Returns (q [rows, cols] float8_e4m3fn, scale fp32[1])."""
    q = torch.empty((rows, cols), dtype=torch.float8_e4m3fn, device=dev)
    for r in range(0, rows, chunk):
        n = min(chunk, rows - r)
        q[r:r + n] = ((torch.rand((n, cols), generator=gen, device=dev) * 2 - 1) * 448.0).to(torch.float8_e4m3fn)
    return q, torch.full((1,), 1.0 / 448.0, dtype=torch.float32, device=dev)


class Pipe:
    """Pipelined end-to-end steps through the public API, one GPU's share of an
    N-column split GEMM: A (replicated) is uploaded by rank 0 from pinned host memory
    and broadcast over NVLink to every rank (NCCL), each rank uploads its B slab,
    runs b200_gemm and downloads its C slab. Copies, broadcast, GEMM and download run
    on their own streams with two sets of device buffers, so step i+1's uploads and
    step i-1's download overlap step i's GEMM. Host buffers hold raw element bytes
    (uint8 for e4m3); `ab_dtype` is the element type the GEMM sees."""

    def __init__(self, torch, b200, dist, world, rank, dev, ha, hb, a_shape, ab_dtype, c_shape, c_dtype,
                 gemm_kw):
        self.t, self.b200, self.dist = torch, b200, dist
        self.world, self.rank, self.dev = world, rank, dev
        self.ha, self.hb = ha, hb  # pinned host; ha is None on ranks other than 0
        self.ab = ab_dtype
        self.hc = [torch.empty(c_shape, dtype=c_dtype).pin_memory() for _ in range(2)]
        self.da = [torch.empty(a_shape, dtype=hb.dtype, device=dev) for _ in range(2)]
        self.db = [torch.empty(hb.shape, dtype=hb.dtype, device=dev) for _ in range(2)]
        self.dc = [torch.empty(c_shape, dtype=c_dtype, device=dev) for _ in range(2)]
        self.s_up = torch.cuda.Stream(dev)
        self.s_down = torch.cuda.Stream(dev)
        self.stream = torch.cuda.current_stream(dev)
        self.kw = gemm_kw

    def run(self, steps):
        torch, dist = self.t, self.dist
        ev = lambda: torch.cuda.Event()  # noqa: E731
        up_done, gemm_done, down_done = [ev(), ev()], [ev(), ev()], [ev(), ev()]
        t0 = torch.cuda.Event(enable_timing=True)
        t1 = torch.cuda.Event(enable_timing=True)
        st = self.stream
        t0.record(st)
        self.s_up.wait_event(t0)
        self.s_down.wait_event(t0)
        for i in range(steps):
            k = i % 2
            with torch.cuda.stream(self.s_up):
                if i >= 2:
                    self.s_up.wait_event(gemm_done[k])  # buffers k free: GEMM i-2 read them
                if self.rank == 0:
                    self.da[k].copy_(self.ha, non_blocking=True)
                if self.world > 1:
                    # NCCL runs on its own stream, ordered after s_up's work so far; the
                    # blocking call makes s_up wait for the broadcast
                    dist.broadcast(self.da[k].view(torch.uint8), src=0)
                self.db[k].copy_(self.hb, non_blocking=True)
                up_done[k].record(self.s_up)
            st.wait_event(up_done[k])
            if i >= 2:
                st.wait_event(down_done[k])  # C buffer k free: step i-2 downloaded
            self.b200.gemm(self.da[k].view(self.ab), self.db[k].view(self.ab), self.dc[k],
                           stream=st.cuda_stream, **self.kw)
            gemm_done[k].record(st)
            with torch.cuda.stream(self.s_down):
                self.s_down.wait_event(gemm_done[k])
                self.hc[k].copy_(self.dc[k], non_blocking=True)
                down_done[k].record(self.s_down)
        st.wait_event(down_done[(steps - 1) % 2])
        if steps >= 2:
            st.wait_event(down_done[(steps - 2) % 2])
        st.wait_event(up_done[(steps - 1) % 2])
        t1.record(st)
        torch.cuda.synchronize()
        return t0.elapsed_time(t1)


def max_over_ranks(torch, dist, world, dev, ms):
    t = torch.tensor([ms], device=dev, dtype=torch.float64)
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def run_ours(args):
    import torch
    import torch.distributed as dist

    rank, world, local = dist_env()
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    b200 = load_pkg()
    mg = load_multigpu()
    if world > 1:
        from datetime import timedelta

        dist.init_process_group("nccl", timeout=timedelta(seconds=120), device_id=dev)

    def barrier():
        if world > 1:
            dist.barrier(device_ids=[local])
        torch.cuda.synchronize()

    stream = torch.cuda.current_stream(dev)
    handle = stream.cuda_stream

    # ------------------ headline: fp16, one 8192 x 8192 x 8192 C slab per GPU ------------------
    # A is the same on every GPU (the replicated operand of the column split), B is
    # this GPU's row slab; uniform[-1,1] like the reference's make_random_vector,
    # generated on the device (the parity tests use the reference's exact host
    # generator; this only sets the workload's values)
    gen_a = torch.Generator(device=dev)
    gen_a.manual_seed(605)
    gen_b = torch.Generator(device=dev)
    gen_b.manual_seed(606 + rank)
    a = (torch.rand((M, K), generator=gen_a, device=dev) * 2 - 1).to(torch.float16)
    b = (torch.rand((N, K), generator=gen_b, device=dev) * 2 - 1).to(torch.float16)
    c = torch.empty((M, N), dtype=torch.float16, device=dev)

    gemm_args = b200.make_args(a, b, c, variant=args.variant, tile_n=args.tile_n)
    variant_used, tile_used = b200.pick_config(gemm_args)

    def step():
        rc = b200.gemm_raw(gemm_args, handle)
        if rc != 0:
            raise b200.B200Error(rc, "b200_gemm")

    cublas = {}

    def cublas_column(fn, key):
        """cuBLASLt on the same shape, same warm-up and step count, run just before our
        timed region (so a power-capped GPU penalises our arm, not cuBLAS's)."""
        if args.no_cublas:
            return
        try:
            barrier()
            _, pc = timed_loop(torch, fn, args.steps, args.warmup, stream)
            cublas[key] = round(FLOPS_8192 / (statistics.fmean(pc) * 1e-3) / 1e12, 2)
        except Exception as e:  # keep the bench line even if the library call is unavailable
            cublas[key + "_error"] = str(e)[:120]

    cublas_column(lambda: torch.matmul(a, b.t(), out=c), "fp16_tflops")
    barrier()
    with ClockSampler(local) as clk:
        total_ms, per = timed_loop(torch, step, args.steps, args.warmup, stream)
    barrier()
    rc, bits = b200.status(handle)
    if rc != 0:
        raise RuntimeError(f"device status {bits:#x}")
    max_ms = max_over_ranks(torch, dist, world, dev, total_ms)
    ms_per_step = max_ms / args.steps
    value = FLOPS_8192 * world * args.steps / (max_ms * 1e-3) / 1e12
    kernel_tflops = FLOPS_8192 / (statistics.fmean(per) * 1e-3) / 1e12

    # ---------------- fp8 e4m3 8192^3 per GPU, per-tensor scales, bf16 out ----------------
    x32 = torch.rand((M, K), generator=gen_a, device=dev) * 2 - 1
    qa, sa = b200.quantize_e4m3(x32.contiguous())
    x32 = torch.rand((N, K), generator=gen_b, device=dev) * 2 - 1
    qb, sb = b200.quantize_e4m3(x32.contiguous())
    del x32
    c8 = torch.empty((M, N), dtype=torch.bfloat16, device=dev)
    fp8_args = b200.make_args(qa.view(M, K), qb.view(N, K), c8, scale_a=sa, scale_b=sb,
                              variant=args.variant, tile_n=args.tile_n)

    def step8():
        rc = b200.gemm_raw(fp8_args, handle)
        if rc != 0:
            raise b200.B200Error(rc, "b200_gemm fp8")

    cublas_column(lambda: torch._scaled_mm(qa.view(M, K), qb.view(N, K).t(), scale_a=sa, scale_b=sb,
                                           out_dtype=torch.bfloat16), "fp8_tflops")
    barrier()
    with ClockSampler(local) as clk8:
        total8, per8 = timed_loop(torch, step8, args.steps, args.warmup, stream)
    barrier()
    fp8_value = FLOPS_8192 * world * args.steps / (max_over_ranks(torch, dist, world, dev, total8) * 1e-3) / 1e12
    fp8_kernel = FLOPS_8192 / (statistics.fmean(per8) * 1e-3) / 1e12
    del qa, qb, c8
    if cublas:
        cublas["note"] = "torch.matmul / torch._scaled_mm (cuBLASLt), same steps, run before ours"

    # ---------------- e2e: host buffers through the public API ----------------
    ha = a.cpu().pin_memory() if rank == 0 else None
    hb = b.cpu().pin_memory()
    pipe = Pipe(torch, b200, dist, world, rank, dev, ha, hb, (M, K), torch.float16, (M, N), torch.float16,
                {"variant": args.variant, "tile_n": args.tile_n})
    e2e_steps = max(3, min(args.steps, 20))
    barrier()
    pipe.run(2)  # warm-up: first touch of the pinned buffers, streams and NCCL
    barrier()
    e2e_total = pipe.run(e2e_steps)
    barrier()
    # the last step's result arrived on the host and equals the device-resident run
    if not torch.equal(pipe.hc[(e2e_steps - 1) % 2][:4, :8].to(dev), c[:4, :8]):
        raise RuntimeError("e2e result differs from the device-resident run")
    e2e_value = FLOPS_8192 * world * e2e_steps / (max_over_ranks(torch, dist, world, dev, e2e_total) * 1e-3) / 1e12
    h2d_job = M * K * 2 + world * N * K * 2
    d2h_job = world * M * N * 2
    del pipe, ha, hb

    # ---------------- config 5: e4m3 16384 x 65536 x 8192, N split across the GPUs ----------------
    strong = None
    if not args.no_strong:
        strong = strong_split(torch, dist, b200, mg, args, rank, world, local, dev, barrier)

    # ---------------- CPU baseline (rank 0, N = 1 only) ----------------
    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu:
        cpu = cpu_baseline(a, b, budget_s=args.cpu_budget)

    peaks = measured_peaks()
    # Denominator: the sustained cuBLAS figure when the power cap throttled the clock
    # during our timed region (a long run of back-to-back launches, like the sustained
    # measurement), else the burst figure; both fractions are reported.
    capped = "sw_power_cap" in (clk.summary().get("reasons") or [])
    burst = peaks["bf16"]
    peak = peaks["bf16_sustained"] if capped and peaks.get("bf16_sustained") else burst
    peak_kind = (f"bf16 dense cuBLAS {'sustained' if peak != burst else 'burst'} ({peaks['source']})"
                 + ("; sw_power_cap active in the timed region" if capped else ""))
    dpk = dense_peak(torch, local, clk.max_mhz)
    result = {
        "metric": "GEMM TFLOPS fp16 & fp8 at 8192^3 per B200 and 8-GPU box; % of dense tensor peak",
        "value": round(value, 2),
        "unit": "TFLOPS",
        "n_gpus": world,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": round(ms_per_step, 5),
        "higher_is_better": True,
        "scaling": "weak",
        "vs_baseline": None,
        "dtype": "f16",
        "data": "synthetic uniform[-1,1] (device-generated), random values, no dataset",
        "config": {"workload": "gemm_tn_f16_8192x8192x8192_per_gpu", "M": M, "N": N * world, "K": K,
                   "n_per_gpu": N, "ab_dtype": "f16", "c_dtype": "f16", "variant": variant_used,
                   "tile_n": tile_used,
                   "parallelism": f"N-column shards x{world} (A replicated, B row slabs), no data-path collective",
                   "l2": "inputs 256 MiB per GPU > 126 MB L2; no flush"},
        "pct_of_dense_peak": round(kernel_tflops / dpk["tflops"], 4),
        "dense_peak": dpk,
        "roofline": {"bound": "tensor", "achieved": round(kernel_tflops, 2), "peak": peak,
                     "unit": "TFLOP/s", "frac": round(kernel_tflops / peak, 4) if peak else None,
                     "peak_kind": peak_kind, "peak_burst": burst,
                     "frac_burst": round(kernel_tflops / burst, 4) if burst else None,
                     "traffic": profile_traffic("f16_8192"),
                     "algorithmic_bytes": 3 * M * N * 2},
        "fp8": {"value": round(fp8_value, 2), "unit": "TFLOPS", "kernel_tflops": round(fp8_kernel, 2),
                "pct_of_dense_peak": round(fp8_kernel / (2 * dpk["tflops"]), 4),
                "frac": round(fp8_kernel / (2 * peak), 4) if peak else None,
                "peak_kind": "2 x the bf16 figures (the e4m3 dense rate is twice bf16)",
                "config": "e4m3 8192^3 per GPU, per-tensor scales amax/448, bf16 C",
                "traffic": profile_traffic("e4m3_8192"), "clocks": clk8.summary(),
                "launch_ms": launch_stats(per8)},
        "cublaslt": cublas,
        "e2e": {"value": round(e2e_value, 2), "unit": "TFLOPS",
                "h2d_bytes_per_step": h2d_job, "d2h_bytes_per_step": d2h_job,
                "steps": e2e_steps,
                "path": "pinned host -> device -> b200_gemm -> pinned host C every step; A uploaded once "
                        "per node and NCCL-broadcast over NVLink, B slab and C slab per GPU; bytes are "
                        "whole-job totals per step"},
        "launch_ms": launch_stats(per),
        "gpu_launches": args.steps,
        "gpu_launches_note": "fp16 timed region; the fp8 and config-5 regions add their own",
        "clocks": clk.summary(),
        "cpu_baseline": cpu,
    }
    if strong is not None:
        result["strong_split"] = strong  # last key: short enough to survive a tail of the line
    if rank == 0:
        print(json.dumps(result), flush=True)
    if world > 1:
        dist.barrier(device_ids=[local])
        dist.destroy_process_group()


def strong_split(torch, dist, b200, mg, args, rank, world, local, dev, barrier):
    """e4m3 C[16384, 65536] = A[16384, 8192] . B[65536, 8192]^T, N split
    evenly across the GPUs (rank g computes C[:, n0:n1] from all of A and B[n0:n1]).
    Whole-box TFLOPS = total flops / max-over-ranks time. N > 1: the all-gather of C,
    timed separately (NCCL all-gather + re-layout), and the fused GEMM + all-gather."""
    stream = torch.cuda.current_stream(dev)
    handle = stream.cuda_stream
    n0, n1 = mg.shard_columns(N5, world, rank)
    ng = n1 - n0
    gen_a = torch.Generator(device=dev)
    gen_a.manual_seed(907)
    gen_b = torch.Generator(device=dev)
    gen_b.manual_seed(908 + rank)
    qa, sa = e4m3_rows(torch, M5, K5, gen_a, dev)
    qb, sb = e4m3_rows(torch, ng, K5, gen_b, dev)
    c5 = torch.empty((M5, ng), dtype=torch.bfloat16, device=dev)
    args5 = b200.make_args(qa, qb, c5, scale_a=sa, scale_b=sb)
    v5, tn5 = b200.pick_config(args5)

    def step5():
        rc = b200.gemm_raw(args5, handle)
        if rc != 0:
            raise b200.B200Error(rc, "b200_gemm config 5")

    steps = max(3, min(args.steps, 20))
    barrier()
    total, per = timed_loop(torch, step5, steps, args.warmup, stream)
    barrier()
    rc, bits = b200.status(handle)
    if rc != 0:
        raise RuntimeError(f"device status {bits:#x} (config 5)")
    ms = max_over_ranks(torch, dist, world, dev, total) / steps
    out = {"value": round(FLOPS_5 / (ms * 1e-3) / 1e12, 1), "unit": "TFLOPS", "n_gpus": world,
           "scaling": "strong", "ms_per_step": round(ms, 4),
           "shape": f"e4m3 {M5}x{N5}x{K5} split N, {ng} columns per GPU", "variant": f"{v5}:{tn5}"}

    if world > 1 and not args.no_gather:
        # (1) NCCL all-gather of the C slabs and re-layout to M x N, timed alone
        gathered = torch.empty((world, M5, ng), dtype=torch.bfloat16, device=dev)
        full = torch.empty((M5, N5), dtype=torch.bfloat16, device=dev)

        def gather_step():
            dist.all_gather_into_tensor(gathered, c5)
            full.view(M5, world, ng).copy_(gathered.permute(1, 0, 2))

        gc = mg.GatheredC(M5, N5, torch.bfloat16, dev)

        def fused_step():
            gc.gemm(b200, qa, qb, c5, scale_a=sa, scale_b=sb, stream=handle)
            gc.sync()

        def timed_max(fn, reps):
            barrier()
            t, _ = timed_loop(torch, fn, reps, 2, stream)
            barrier()
            return max_over_ranks(torch, dist, world, dev, t) / reps

        reps = max(3, min(args.steps, 10))
        nccl_ms = timed_max(gather_step, reps)
        fused_ms = timed_max(fused_step, reps)
        rc, bits = b200.status(handle)
        barrier()
        same = torch.equal(gc.buf, full)
        flag = torch.tensor([0 if (same and rc == 0) else 1], device=dev)
        dist.all_reduce(flag, op=dist.ReduceOp.MAX)
        out["gather"] = {"gemm_ms": round(ms, 4), "nccl_allgather_relayout_ms": round(nccl_ms, 4),
                         "sequential_ms": round(ms + nccl_ms, 4), "fused_ms": round(fused_ms, 4),
                         "fused_mode": "multicast" if gc.multicast else "peers",
                         "fused_equals_nccl": int(flag.item()) == 0,
                         "bytes_in_per_gpu": M5 * (N5 - ng) * 2}
        del gathered, full, gc

    if not args.no_e2e:
        # e2e of the split: A uploaded once (rank 0) and broadcast, B slab up, C slab down
        ha = qa.view(torch.uint8).cpu().pin_memory() if rank == 0 else None
        hb = qb.view(torch.uint8).cpu().pin_memory()
        pipe = Pipe(torch, b200, dist, world, rank, dev, ha, hb, (M5, K5), torch.float8_e4m3fn, (M5, ng),
                    torch.bfloat16, {"scale_a": sa, "scale_b": sb})
        e_steps = max(3, min(args.steps, 8))
        barrier()
        pipe.run(2)
        barrier()
        et = pipe.run(e_steps)
        barrier()
        ems = max_over_ranks(torch, dist, world, dev, et) / e_steps
        out["e2e"] = {"value": round(FLOPS_5 / (ems * 1e-3) / 1e12, 1), "unit": "TFLOPS",
                      "h2d_bytes_per_step": M5 * K5 + N5 * K5, "d2h_bytes_per_step": M5 * N5 * 2}
        del pipe, ha, hb
    del qa, qb, c5
    torch.cuda.empty_cache()
    return out


def cpu_baseline(a, b, budget_s: float = 8.0):
    """The reference's host GEMM loop (oracle port, naive m-n-k order), all host
    threads, on a row band of the same fp16 8192^3 problem. Band height is
    calibrated so the measurement stays within ~budget_s seconds."""
    import oracle as O

    threads = os.cpu_count() or 1
    A = a.float().cpu().numpy()
    B = b.float().cpu().numpy()
    rows = max(threads, 8)
    t = time.perf_counter()
    O.gemm_tn(A, B, rows=(0, rows), threads=threads, naive=True)
    dt = time.perf_counter() - t
    scale = max(1, int(budget_s / max(dt, 1e-3)))
    rows2 = min(M, rows * scale)
    t = time.perf_counter()
    O.gemm_tn(A, B, rows=(0, rows2), threads=threads, naive=True)
    dt2 = time.perf_counter() - t
    tflops = 2.0 * rows2 * N * K / dt2 / 1e12
    return {"value": round(tflops, 6), "unit": "TFLOPS", "cores": threads, "kind": "port",
            "sample": f"rows [0,{rows2}) of fp16 8192x8192x8192 (all {N} columns, full K), "
                      f"{dt2:.2f} s; reference loop order, fp32 sequential-k"}


def run_reference(args):
    rank, world, local = dist_env()
    if rank != 0:
        return
    import numpy as np

    import oracle as O

    threads = os.cpu_count() or 1
    # the reference's inputs for its 8192^3 fp16 runs: seeds 605/606 (gemm_ws.cu:318-321)
    a = O.f16_bits_to_f32(O.f32_to_f16_bits(O.uniform(605, M * K))).reshape(M, K)
    b = O.f16_bits_to_f32(O.f32_to_f16_bits(O.uniform(606, N * K))).reshape(N, K)
    # calibrate the band so W+K steps finish in ~args.cpu_budget * 6 seconds
    rows = max(threads, 8)
    t = time.perf_counter()
    O.gemm_tn(a, b, rows=(0, rows), threads=threads, naive=True)
    dt = time.perf_counter() - t
    per_step_budget = max(0.05, (args.cpu_budget * 6) / max(1, args.steps + args.warmup))
    rows = int(max(1, min(M, rows * per_step_budget / max(dt, 1e-4))))
    rng = np.random.default_rng(0)
    for _ in range(args.warmup):
        r0 = int(rng.integers(0, M - rows + 1))
        O.gemm_tn(a, b, rows=(r0, r0 + rows), threads=threads, naive=True)
    t = time.perf_counter()
    for _ in range(args.steps):
        r0 = int(rng.integers(0, M - rows + 1))
        O.gemm_tn(a, b, rows=(r0, r0 + rows), threads=threads, naive=True)
    dt = time.perf_counter() - t
    tflops = 2.0 * rows * N * K * args.steps / dt / 1e12
    sample = (f"{args.steps} steps x rows band of {rows} of fp16 8192^3 (all {N} columns, "
              f"full K), seeds 605/606")
    out = {
        "metric": "GEMM TFLOPS fp16 & fp8 at 8192^3 per B200 and 8-GPU box; % of dense tensor peak",
        "impl": "reference",
        "value": round(tflops, 6),
        "unit": "TFLOPS",
        "n_gpus": world,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": round(dt / args.steps * 1e3, 3),
        "higher_is_better": True,
        "scaling": "weak",
        "vs_baseline": None,
        "dtype": "f16",
        "data": "reference seeded inputs (mt19937 uniform[-1,1], seeds 605/606)",
        "config": {"workload": "gemm_tn_f16_8192x8192x8192_per_gpu", "M": M, "N": N, "K": K,
                   "impl": "reference host GEMM loop (oracle port), row-parallel threads"},
        "cpu_baseline": {"value": round(tflops, 6), "unit": "TFLOPS", "cores": threads,
                         "kind": "port", "sample": sample},
        "e2e": {"value": round(tflops, 6), "unit": "TFLOPS", "h2d_bytes_per_step": 0,
                "d2h_bytes_per_step": 0},
        "gpu_launches": 0,
    }
    print(json.dumps(out), flush=True)


# ------------------------------------------------------------------ measurement helpers
def _inputs(torch, b200, dt, M_, N_, K_, seed=0):
    g = torch.Generator(device="cuda")
    g.manual_seed(seed)
    if dt == "e4m3":
        a, sa = e4m3_rows(torch, M_, K_, g, "cuda")
        b, sb = e4m3_rows(torch, N_, K_, g, "cuda")
        c = torch.empty((M_, N_), dtype=torch.bfloat16, device="cuda")

        def cublas():
            torch._scaled_mm(a, b.t(), scale_a=sa, scale_b=sb, out_dtype=torch.bfloat16)
    else:
        tdt = torch.float16 if dt == "f16" else torch.bfloat16
        a = (torch.rand((M_, K_), generator=g, device="cuda") * 2 - 1).to(tdt)
        b = (torch.rand((N_, K_), generator=g, device="cuda") * 2 - 1).to(tdt)
        c = torch.empty((M_, N_), dtype=tdt, device="cuda")
        sa = sb = None

        def cublas():
            torch.matmul(a, b.t(), out=c)
    return a, b, c, sa, sb, cublas


def _parse_size(size: str):
    dims = [int(v) for v in size.split("x")]
    if len(dims) == 1:
        return dims[0], dims[0], dims[0]
    if len(dims) == 2:  # MxK, N = M
        return dims[0], dims[0], dims[1]
    return tuple(dims)


def mode_profile(opt):
    """One launch inside cudaProfilerStart/Stop after three warm-up launches."""
    import torch

    b200 = load_pkg()
    p = opt.rest
    dt, who = p[0], p[1]
    variant = p[2] if len(p) > 2 else "auto"
    M_, N_, K_ = _parse_size(p[3] if len(p) > 3 else "8192")
    tile_n = int(p[4]) if len(p) > 4 else 0
    group_m = int(p[5]) if len(p) > 5 else 0
    torch.cuda.set_device(0)
    a, b, c, sa, sb, cublas = _inputs(torch, b200, dt, M_, N_, K_)

    def run():
        if who == "ours":
            b200.gemm(a, b, c, scale_a=sa, scale_b=sb, variant=variant, tile_n=tile_n, group_m=group_m)
        else:
            cublas()

    for _ in range(3):
        run()
    torch.cuda.synchronize()
    torch.cuda.profiler.start()
    run()
    torch.cuda.synchronize()
    torch.cuda.profiler.stop()
    rc, bits = b200.status()
    assert rc == 0, hex(bits)
    print("ok", dt, who, variant, f"{M_}x{N_}x{K_}", tile_n)


def _config_fn(b200, L, a, b, c, sa, sb, cf, stream):
    """One launch of configuration `variant[:tile_n[:group_m]][@K=V,...]` (the environment
    is set before each call, for experimental builds that read settings from it)."""
    spec, _, env = cf.partition("@")
    parts = spec.split(":")
    args = b200.make_args(a, b, c, scale_a=sa, scale_b=sb, variant=parts[0],
                          tile_n=int(parts[1]) if len(parts) > 1 else 0,
                          group_m=int(parts[2]) if len(parts) > 2 else 0)

    def ours():
        for kv in filter(None, env.split(",")):
            key, _, val = kv.partition("=")
            os.environ[key] = val
        rc = L.b200_gemm(C.byref(args), C.c_void_p(stream))
        if rc != 0:
            raise RuntimeError(b200.strerror(rc))

    return ours


def mode_power(opt):
    """Sustained TFLOPS, energy per GEMM, board power and SM clock under the power cap,
    configurations interleaved in rounds (slow thermal drift hits all of them alike)."""
    import pynvml
    import torch

    b200 = load_pkg()
    L = b200.lib()
    dt, configs = opt.rest[0], opt.rest[1:]
    pynvml.nvmlInit()
    h = pynvml.nvmlDeviceGetHandleByIndex(torch.cuda.current_device())
    M_, N_, K_ = _parse_size(opt.shape) if opt.shape else (opt.size,) * 3
    a, b, c, sa, sb, cublas = _inputs(torch, b200, dt, M_, N_, K_)
    stream = torch.cuda.current_stream().cuda_stream
    fns = {}
    for cf in configs:
        if cf == "cublas":
            fns[cf] = cublas
            continue
        fns[cf] = _config_fn(b200, L, a, b, c, sa, sb, cf, stream)
    flop = 2.0 * M_ * N_ * K_
    res = {k: [] for k in fns}
    for r in range(opt.rounds):
        for name, f in fns.items():
            for _ in range(10):
                f()
            torch.cuda.synchronize()
            t0, k = time.time(), 0
            while time.time() - t0 < 0.3:
                for _ in range(10):
                    f()
                k += 10
                torch.cuda.synchronize()
            iters = max(30, int(k * opt.secs / (time.time() - t0)))
            e0 = pynvml.nvmlDeviceGetTotalEnergyConsumption(h)
            ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            clocks = []
            ev0.record()
            for i in range(iters):
                f()
                if i % 100 == 50:
                    clocks.append(pynvml.nvmlDeviceGetClockInfo(h, pynvml.NVML_CLOCK_SM))
            ev1.record()
            torch.cuda.synchronize()
            e1 = pynvml.nvmlDeviceGetTotalEnergyConsumption(h)  # mJ
            ms = ev0.elapsed_time(ev1)
            row = (flop * iters / ms / 1e9, (e1 - e0) / iters, (e1 - e0) / ms,
                   statistics.median(clocks) if clocks else 0)
            res[name].append(row)
            print(f"round {r} {dt} {name:14s} {row[0]:7.1f} TFLOPS {row[1]:7.1f} mJ/GEMM "
                  f"{row[2]:6.0f} W {row[3]:5.0f} MHz", flush=True)
    print(f"median over {opt.rounds} rounds, {dt} {M_}x{N_}x{K_}:")
    for name, v in res.items():
        med = [statistics.median(x[i] for x in v) for i in range(4)]
        print(f"  {name:14s} {med[0]:7.1f} TFLOPS {med[1]:7.1f} mJ/GEMM {med[2]:6.0f} W {med[3]:5.0f} MHz")


SWEEP_SHAPES = ["256x16384x8192", "512x1024x8192", "1024x1024x8192", "1024x1024x16384",
                "2048x1024x4096", "2048x1024x8192", "1024x4096x8192", "2048x2048x2048",
                "2048x2048x8192", "4096x4096x4096", "8192x8192x1024", "8192x8192x8192"]
SWEEP_CONFIGS = ["2cta:128", "2cta:256", "2cta_clc:128", "2cta_clc:256", "2cta_clc:512",
                 "2cta_streamk:128", "2cta_streamk:256", "persistent:256"]


def mode_sweep(opt):
    """Median launch time of each schedule / tile width and cuBLASLt per shape."""
    import torch

    b200 = load_pkg()
    L = b200.lib()
    torch.cuda.set_device(0)
    stream = torch.cuda.current_stream().cuda_stream
    shapes = opt.shapes.split(",") if opt.shapes else SWEEP_SHAPES
    for dt in opt.dtypes.split(","):
        for size in shapes:
            M_, N_, K_ = _parse_size(size)
            a, b, c, sa, sb, cublas = _inputs(torch, b200, dt, M_, N_, K_)
            flop = 2.0 * M_ * N_ * K_
            row = {"dtype": dt, "shape": size}
            auto = b200.make_args(a, b, c, scale_a=sa, scale_b=sb)
            row["pick"] = "%s:%d" % b200.pick_config(auto)
            # untimed spin-up (~50 ms of launches) so that the first configuration timed
            # does not run while the SM clock is still rising from idle
            t_end = time.perf_counter() + 0.05
            while time.perf_counter() < t_end:
                for _ in range(20):
                    L.b200_gemm(C.byref(auto), C.c_void_p(stream))
                torch.cuda.synchronize()
            for cf in ["auto", "cublas"] + (opt.rest or SWEEP_CONFIGS):
                fn = cublas if cf == "cublas" else _config_fn(b200, L, a, b, c, sa, sb, cf, stream)
                try:
                    _, per = timed_loop(torch, fn, opt.steps, opt.warmup, torch.cuda.current_stream())
                    row[cf] = round(flop / (statistics.median(per) * 1e-3) / 1e12, 1)
                except RuntimeError as e:
                    row[cf] = str(e)[:40]
            rc, bits = b200.status()
            row["status"] = rc
            print(json.dumps(row), flush=True)
            del a, b, c
            torch.cuda.empty_cache()


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--mode", choices=["headline", "profile", "power", "sweep"], default="headline")
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=200)
    ap.add_argument("--warmup", type=int, default=20)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--variant", default="auto")
    ap.add_argument("--tile-n", type=int, default=0, help="0 (library default), 128, 256 or 512")
    ap.add_argument("--no-cpu", action="store_true")
    ap.add_argument("--no-cublas", action="store_true")
    ap.add_argument("--no-strong", action="store_true", help="skip the config-5 split")
    ap.add_argument("--no-gather", action="store_true", help="skip the config-5 all-gather timings")
    ap.add_argument("--no-e2e", action="store_true", help="skip the config-5 e2e")
    ap.add_argument("--cpu-budget", type=float, default=8.0)
    # measurement helpers
    ap.add_argument("--size", type=int, default=8192, help="power: M = N = K")
    ap.add_argument("--secs", type=float, default=1.5, help="power: seconds per configuration and round")
    ap.add_argument("--rounds", type=int, default=3, help="power: rounds")
    ap.add_argument("--shape", default="", help="power: MxNxK instead of --size cubed")
    ap.add_argument("--dtypes", default="f16,e4m3", help="sweep: element types")
    ap.add_argument("--shapes", default="", help="sweep: comma-separated MxNxK list")
    ap.add_argument("rest", nargs="*", help="profile / power positional arguments")
    args = ap.parse_intermixed_args()
    if args.warmup < 3:
        args.warmup = 3
    if args.mode == "profile":
        return mode_profile(args)
    if args.mode == "power":
        return mode_power(args)
    if args.mode == "sweep":
        return mode_sweep(args)
    if args.impl == "reference":
        run_reference(args)
    else:
        run_ours(args)


if __name__ == "__main__":
    main()
