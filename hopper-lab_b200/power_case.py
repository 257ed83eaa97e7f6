"""Sustained throughput, energy per GEMM and SM clock of GEMM configurations under the
B200's 1 kW power cap, read from NVML's total-energy counter.

Under the cap the clock settles where board power meets the limit, so two kernels with
the same tensor-pipe efficiency differ in throughput by how much energy each spends per
GEMM outside the tensor cores (L2 and DRAM traffic above all). This script makes that
visible: every configuration runs back-to-back launches for a fixed time, in rounds
that interleave the configurations (so slow thermal drift hits all of them alike), and
reports the median over rounds of TFLOPS, mJ per GEMM, average board power and SM clock.

    python hopper-lab_b200/power_case.py f16 cublas 2cta 2cta:256 2cta_share
    python hopper-lab_b200/power_case.py e4m3 cublas 2cta 2cta:512 --secs 1.5 --rounds 3

A configuration is `cublas` (torch.matmul / torch._scaled_mm) or `<variant>[:tile_n[:group_m]]`
of this library. Profiling helper: cuBLAS is called on purpose, as the reference column.
"""
from __future__ import annotations

import argparse
import ctypes as C
import importlib.util
import statistics
import time
from pathlib import Path

HERE = Path(__file__).resolve().parent


def _lib():
    spec = importlib.util.spec_from_file_location("hopper_lab_b200", HERE / "__init__.py")
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


def main() -> int:
    ap = argparse.ArgumentParser(description=__doc__.splitlines()[0])
    ap.add_argument("dtype", choices=["f16", "bf16", "e4m3"])
    ap.add_argument("configs", nargs="+")
    ap.add_argument("--size", type=int, default=8192, help="M = N = K")
    ap.add_argument("--secs", type=float, default=1.5, help="timed seconds per configuration and round")
    ap.add_argument("--rounds", type=int, default=3)
    opt = ap.parse_args()

    import pynvml
    import torch

    b200 = _lib()
    L = b200.lib()
    pynvml.nvmlInit()
    dev = torch.cuda.current_device()
    h = pynvml.nvmlDeviceGetHandleByIndex(dev)
    g = torch.Generator(device="cuda")
    g.manual_seed(0)
    n = opt.size
    if opt.dtype == "e4m3":
        a = (torch.rand((n, n), generator=g, device="cuda") * 2 - 1).to(torch.float8_e4m3fn)
        b = (torch.rand((n, n), generator=g, device="cuda") * 2 - 1).to(torch.float8_e4m3fn)
        c = torch.empty((n, n), dtype=torch.bfloat16, device="cuda")
        sa = torch.ones(1, device="cuda")
        sb = torch.ones(1, device="cuda")

        def cublas():
            torch._scaled_mm(a, b.t(), scale_a=sa, scale_b=sb, out_dtype=torch.bfloat16)
    else:
        tdt = torch.float16 if opt.dtype == "f16" else torch.bfloat16
        a = (torch.rand((n, n), generator=g, device="cuda") * 2 - 1).to(tdt)
        b = (torch.rand((n, n), generator=g, device="cuda") * 2 - 1).to(tdt)
        c = torch.empty((n, n), dtype=tdt, device="cuda")
        sa = sb = None

        def cublas():
            torch.matmul(a, b.t(), out=c)

    stream = torch.cuda.current_stream().cuda_stream
    fns = {}
    for cf in opt.configs:
        if cf == "cublas":
            fns[cf] = cublas
            continue
        parts = cf.split(":")
        args = b200.make_args(a, b, c, scale_a=sa, scale_b=sb, variant=parts[0],
                              tile_n=int(parts[1]) if len(parts) > 1 else 0,
                              group_m=int(parts[2]) if len(parts) > 2 else 0)

        def ours(args=args):
            rc = L.b200_gemm(C.byref(args), C.c_void_p(stream))
            if rc != 0:
                raise RuntimeError(b200.strerror(rc))

        fns[cf] = ours

    flop = 2.0 * n * n * n
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
            print(f"round {r} {opt.dtype} {name:14s} {row[0]:7.1f} TFLOPS {row[1]:7.1f} mJ/GEMM "
                  f"{row[2]:6.0f} W {row[3]:5.0f} MHz", flush=True)
    print(f"median over {opt.rounds} rounds, {opt.dtype} {n}^3:")
    for name, v in res.items():
        med = [statistics.median(x[i] for x in v) for i in range(4)]
        print(f"  {name:14s} {med[0]:7.1f} TFLOPS {med[1]:7.1f} mJ/GEMM {med[2]:6.0f} W {med[3]:5.0f} MHz")
    return 0


if __name__ == "__main__":
    raise SystemExit(main())
