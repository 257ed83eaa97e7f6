"""b200_gemm_noalloc — the GEMM entry point for callers that cannot allocate.

Some callers cannot let a library call cudaMalloc: frameworks whose pool allocator
must own every device allocation, processes whose device footprint is fixed after
start-up, and paths that must not take the allocator's locks. b200_gemm_noalloc
runs the same kernels as b200_gemm with the kernel's scratch (its status word) in
a static device array. These tests call it through the C ABI twice in a row and
check each output against b200_gemm's, within the GEMM tests' tolerances.

The no-alloc calls come first, so that in a fresh process they run before
anything else has set the library up on the device. This file is named to be
collected last.
"""
from __future__ import annotations

import ctypes as C

import numpy as np
import pytest

from gemm_check import TOL_16, TOL_E4M3, compare

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
    # AUTO on a nearly empty pair wave with long K: b200_gemm picks stream-K, the
    # allocation-free entry point the static pair schedule (no workspace)
    ("f16", "f16", 1024, 1024, 8192, "auto", 0, False),
]


@pytest.mark.parametrize("ab,out,M,N,K,variant,tile_n,scaled", CASES)
def test_noalloc_matches_b200_gemm_on_two_calls(b200, noalloc_fn, ab, out, M, N, K, variant,
                                                tile_n, scaled):
    torch.cuda.set_device(0)
    g = torch.Generator(device="cuda")
    g.manual_seed(M * 7 + N)
    tdt = {"bf16": torch.bfloat16, "f16": torch.float16}
    odt = {"bf16": torch.bfloat16, "f16": torch.float16}[out]
    if ab == "e4m3":
        a = (torch.rand((M, K), generator=g, device="cuda") * 2 - 1).to(torch.float8_e4m3fn)
        b = (torch.rand((N, K), generator=g, device="cuda") * 2 - 1).to(torch.float8_e4m3fn)
    else:
        a = (torch.rand((M, K), generator=g, device="cuda") * 2 - 1).to(tdt[ab])
        b = (torch.rand((N, K), generator=g, device="cuda") * 2 - 1).to(tdt[ab])
    sa = torch.tensor([0.5], device="cuda") if scaled else None
    sb = torch.tensor([0.25], device="cuda") if scaled else None
    stream = torch.cuda.current_stream().cuda_stream

    outs = []
    for call in range(2):
        c = torch.full((M, N), float("nan"), dtype=odt, device="cuda")
        args = b200.make_args(a, b, c, scale_a=sa, scale_b=sb, variant=variant, tile_n=tile_n)
        rc = noalloc_fn(C.byref(args), C.c_void_p(stream), 1)
        assert rc == 0, f"call {call}: {b200.strerror(rc)}"
        outs.append(c.float().cpu().numpy())

    ref = b200.gemm(a, b, out_dtype=out, scale_a=sa, scale_b=sb, variant=variant, tile_n=tile_n)
    torch.cuda.synchronize()
    ref = ref.float().cpu().numpy()
    tol = TOL_E4M3 if ab == "e4m3" else TOL_16
    for call, got in enumerate(outs):
        ok, info = compare(got, ref, tol)
        assert ok, (call, info)
    assert np.array_equal(outs[0], outs[1])


def test_noalloc_validates_like_b200_gemm(b200, noalloc_fn):
    args = b200.GemmArgs()
    args.ab_dtype, args.c_dtype = 7, b200.DT_BF16
    assert noalloc_fn(C.byref(args), None, 0) == b200.ERR_INVALID_ARG
