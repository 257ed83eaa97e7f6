"""b200_gemm_noalloc — the GEMM entry point for callers that cannot allocate.

Some callers cannot let a library call cudaMalloc: frameworks whose pool allocator
must own every device allocation, processes whose device footprint is fixed after
start-up, and paths that must not take the allocator's locks. b200_gemm_noalloc
runs the same kernels as b200_gemm with the kernel's scratch (its status word) in
a static device array. These tests call it through the C ABI twice in a row and
check each output against the CPU oracle and against b200_gemm's output, within
the GEMM tests' tolerances; they also check what it refuses (stream-K, whose
workspace the static array cannot hold), that AUTO steers clear of stream-K, and
that a bounded-wait failure is reported by one call and cleared by the next.

The file is named so that pytest collects it last: a run that stops at the first
failure has run every other test before it. Each test sets up what it needs, so
the file also passes on its own in a fresh process.
"""
from __future__ import annotations

import ctypes as C

import numpy as np
import pytest

from gemm_check import TOL_16, TOL_E4M3, compare, make_inputs, reference, to_device

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def noalloc_fn(b200):
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    fn = b200.lib().b200_gemm_noalloc
    fn.argtypes = [C.POINTER(b200.GemmArgs), C.c_void_p, C.c_int]
    fn.restype = C.c_int
    return fn


CASES = [
    # (ab dtype, out dtype, M, N, K, variant, tile_n, scaled)
    ("bf16", "bf16", 512, 768, 1024, "2cta", 0, False),
    ("f16", "f16", 300, 520, 200, "persistent", 0, False),
    ("e4m3", "bf16", 1024, 1024, 2048, "2cta", 512, True),
    ("f16", "f16", 2048, 1024, 1024, "2cta_clc", 128, False),
    # AUTO on a nearly empty pair wave with long K: b200_gemm picks stream-K, the
    # allocation-free entry point a schedule without a workspace
    ("f16", "f16", 512, 1024, 8192, "auto", 0, False),
]


@pytest.mark.parametrize("ab,out,M,N,K,variant,tile_n,scaled", CASES)
def test_noalloc_matches_oracle_and_b200_gemm_on_two_calls(b200, oracle, noalloc_fn, ab, out, M, N, K,
                                                           variant, tile_n, scaled):
    torch.cuda.set_device(0)
    inp = make_inputs(oracle, M, N, K, ab, 71 + M, 72 + N, scaled=scaled)
    a, b, sa, sb = to_device(inp, torch)
    odt = {"bf16": torch.bfloat16, "f16": torch.float16}[out]
    stream = torch.cuda.current_stream().cuda_stream

    outs = []
    for call in range(2):
        c = torch.full((M, N), float("nan"), dtype=odt, device="cuda")
        args = b200.make_args(a, b, c, scale_a=sa, scale_b=sb, variant=variant, tile_n=tile_n)
        rc = noalloc_fn(C.byref(args), C.c_void_p(stream), 1)
        assert rc == 0, f"call {call}: {b200.strerror(rc)}"
        outs.append(c.float().cpu().numpy())

    ref = reference(oracle, inp)
    lib_out = b200.gemm(a, b, out_dtype=out, scale_a=sa, scale_b=sb, variant=variant, tile_n=tile_n)
    torch.cuda.synchronize()
    lib_out = lib_out.float().cpu().numpy()
    tol = TOL_E4M3 if ab == "e4m3" else TOL_16
    for call, got in enumerate(outs):
        ok, info = compare(got, ref, tol)
        assert ok, ("oracle", call, info)
        ok, info = compare(got, lib_out, tol)
        assert ok, ("b200_gemm", call, info)
    assert np.array_equal(outs[0], outs[1])


def test_noalloc_auto_avoids_streamk(b200, noalloc_fn):
    """For a shape where b200_gemm's AUTO takes stream-K, an explicit stream-K request
    to the allocation-free entry point returns B200_ERR_SCRATCH_LIMIT, and its AUTO
    resolves to a schedule without a workspace (the result is checked above)."""
    M, N, K = 512, 1024, 8192
    a = torch.zeros((M, K), dtype=torch.float16, device="cuda")
    b = torch.zeros((N, K), dtype=torch.float16, device="cuda")
    c = torch.empty((M, N), dtype=torch.float16, device="cuda")
    args = b200.make_args(a, b, c)
    assert b200.pick_config(args)[0] == "2cta_streamk"
    sk = b200.make_args(a, b, c, variant="2cta_streamk")
    assert noalloc_fn(C.byref(sk), None, 1) == b200.ERR_SCRATCH_LIMIT


def test_noalloc_reports_a_timeout_and_the_next_call_clears_it(b200, oracle, noalloc_fn):
    """fault_inject = 1: the producer issues no loads, so a 10 ms bounded wait gives up;
    the call (check_status = 1) returns B200_ERR_DEVICE_TIMEOUT. The next call clears the
    shared status word first, returns 0 and computes the right result."""
    M, N, K = 256, 512, 384
    inp = make_inputs(oracle, M, N, K, "f16", 81, 82)
    a, b, _, _ = to_device(inp, torch)
    stream = torch.cuda.current_stream().cuda_stream
    c = torch.zeros((M, N), dtype=torch.float16, device="cuda")
    bad = b200.make_args(a, b, c, variant="2cta", fault_inject=1, wait_limit_ns=10_000_000)
    assert noalloc_fn(C.byref(bad), C.c_void_p(stream), 1) == b200.ERR_DEVICE_TIMEOUT
    good = b200.make_args(a, b, c, variant="2cta")
    assert noalloc_fn(C.byref(good), C.c_void_p(stream), 1) == 0
    ok, info = compare(c.float().cpu().numpy(), reference(oracle, inp), TOL_16)
    assert ok, info


def test_noalloc_validates_like_b200_gemm(b200, noalloc_fn):
    args = b200.GemmArgs()
    args.ab_dtype, args.c_dtype = 7, b200.DT_BF16
    assert noalloc_fn(C.byref(args), None, 0) == b200.ERR_INVALID_ARG
