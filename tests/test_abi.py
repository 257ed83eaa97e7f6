"""The C ABI boundary without a GPU: the library loads, exports every function
include/b200gemm.h declares, the ctypes mirror matches the C struct layout, and
argument validation returns the documented codes before any device work."""
import ctypes as C
import re
import subprocess
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]
HEADER = ROOT / "include" / "b200gemm.h"


def declared_functions():
    text = HEADER.read_text()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"^\s*(?:int|void|const char\*)\s+(b200_\w+)\s*\(", text, flags=re.M)))


def test_header_declares_the_python_export_list(b200):
    assert declared_functions() == sorted(b200.EXPORTS)


def test_library_exports_every_declared_symbol(b200):
    L = b200.lib()
    for name in declared_functions():
        assert hasattr(L, name), name
    out = subprocess.run(["nm", "-D", "--defined-only", str(b200.LIB_PATH)], capture_output=True,
                         text=True, check=True).stdout
    syms = {line.split()[-1] for line in out.splitlines() if line.strip()}
    for name in declared_functions():
        assert name in syms, name


def test_library_is_built_for_sm100a_only(b200):
    # the nvcc command lines of the build carry only the sm_100a target
    import importlib.util

    spec = importlib.util.spec_from_file_location("b200_build", ROOT / "hopper-lab_b200" / "build.py")
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    assert mod.ARCH == ["-gencode", "arch=compute_100a,code=sm_100a"]
    assert all("sm_90" not in f and "compute_90" not in f for f in mod.NVFLAGS)


def test_struct_layout_matches_c(b200, tmp_path):
    prog = tmp_path / "layout.c"
    fields = [f for f, _ in b200.GemmArgs._fields_]
    body = "\n".join(f'  printf("{f} %zu\\n", offsetof(B200GemmArgs, {f}));' for f in fields)
    prog.write_text(f"""#include <stddef.h>
#include <stdio.h>
#include "b200gemm.h"
int main(void) {{
{body}
  printf("sizeof %zu\\n", sizeof(B200GemmArgs));
  return 0;
}}
""")
    exe = tmp_path / "layout"
    subprocess.run(["gcc", "-std=c99", f"-I{ROOT / 'include'}", str(prog), "-o", str(exe)], check=True)
    out = subprocess.run([str(exe)], capture_output=True, text=True, check=True).stdout.split()
    got = dict(zip(out[0::2], map(int, out[1::2])))
    for f in fields:
        assert got[f] == getattr(b200.GemmArgs, f).offset, f
    assert got["sizeof"] == C.sizeof(b200.GemmArgs)


def test_abi_version_and_strerror(b200):
    L = b200.lib()
    assert L.b200_gemm_abi_version() == 4
    for code in (0, -1, -2, -3, -4, -5, -6, -7, -8, -9):
        assert b200.strerror(code)
    assert "unknown" in b200.strerror(-99)


def test_variant_info(b200):
    for v in ("1cta", "persistent", "clc"):
        info = b200.variant_info(v)
        assert info["tile_m"] == 128 and info["tile_n"] == 256
        assert info["max_stages"] == 4
    for v in ("2cta", "2cta_clc"):
        info = b200.variant_info(v, b200.DT_E4M3)
        assert info["tile_m"] == 256 and info["tile_n"] == 256 and info["max_stages"] == 3
    for v in ("2cta", "2cta_clc"):
        info = b200.variant_info(v, b200.DT_BF16, tile_n=512)
        assert info["tile_m"] == 256 and info["tile_n"] == 512 and info["max_stages"] == 4
    for v in ("2cta", "2cta_clc", "2cta_streamk"):
        # 256x128 pair tiles: four K atoms per stage, 96 KB, two stages
        info = b200.variant_info(v, b200.DT_E4M3, tile_n=128)
        assert info["tile_m"] == 256 and info["tile_n"] == 128 and info["max_stages"] == 2
    info = b200.variant_info("2cta_streamk", b200.DT_F16)
    assert info["tile_m"] == 256 and info["tile_n"] == 256 and info["max_stages"] == 3
    with pytest.raises(b200.B200Error):
        b200.variant_info("2cta_streamk", tile_n=512)  # stream-K uses one MMA width
    with pytest.raises(b200.B200Error):
        b200.variant_info(7)  # the former B-sharing variant is gone
    for v in ("persistent", "1cta", "clc"):
        for tn in (128, 512):
            with pytest.raises(b200.B200Error):
                b200.variant_info(v, tile_n=tn)  # narrow and wide tiles are pair-only
    with pytest.raises(b200.B200Error):
        b200.variant_info("2cta", tile_n=384)
    with pytest.raises(b200.B200Error):
        b200.variant_info(0)  # AUTO has no fixed shape
    with pytest.raises(b200.B200Error):
        b200.variant_info("1cta", b200.DT_F32)  # f32 is an output type only


def _args(b200, **kw):
    a = b200.GemmArgs()
    a.ab_dtype, a.c_dtype = b200.DT_F16, b200.DT_F16
    a.M, a.N, a.K = 256, 256, 256
    a.lda, a.ldb, a.ldc = 256, 256, 256
    a.A, a.B, a.C = 0x10000, 0x20000, 0x30000
    for k, v in kw.items():
        setattr(a, k, v)
    return a


@pytest.mark.parametrize("kw,code", [
    ({"ab_dtype": 7}, -1),
    ({"ab_dtype": 3}, -1),            # f32 inputs are not a GEMM input type
    ({"c_dtype": 2}, -1),             # e4m3 output not supported
    ({"variant": 9}, -1),
    ({"variant": 7}, -1),             # no variant 7 since ABI 4
    ({"M": -1}, -2),
    ({"K": -5}, -2),
    ({"N": 1 << 31}, -2),
    ({"lda": 128}, -2),               # lda < K
    ({"ldc": 100}, -2),               # ldc < N
    ({"A": 0x10008}, -3),             # A not 16-byte aligned
    ({"C": 0x30004}, -3),
    ({"lda": 260}, -3),               # 520-byte rows: not a 16-byte multiple
    ({"ldc": 257, "N": 257}, -3),
    ({"A": 0}, -1),
    ({"C": 0}, -1),
    ({"group_m": -1}, -1),
    ({"stages": -2}, -1),
    ({"scale_a": 0x40002}, -3),
    ({"tile_n": 384}, -1),
    ({"reserved": 1}, -1),
])
def test_validation_codes(b200, kw, code):
    assert b200.gemm_raw(_args(b200, **kw), 0) == code


def test_empty_problem_is_a_no_op(b200):
    # M == 0 or N == 0 returns before touching the device
    assert b200.gemm_raw(_args(b200, M=0, A=0, B=0, C=0), 0) == 0
    assert b200.gemm_raw(_args(b200, N=0, A=0, B=0, C=0), 0) == 0


def test_valid_args_without_gpu_report_cuda_error(b200):
    import torch

    if torch.cuda.is_available():
        pytest.skip("GPU present")
    assert b200.gemm_raw(_args(b200), 0) == b200.ERR_CUDA


def test_python_wrapper_checks_shapes(b200):
    import torch

    a = torch.empty((4, 8), dtype=torch.float16)
    b = torch.empty((3, 9), dtype=torch.float16)
    c = torch.empty((4, 3), dtype=torch.float16)
    with pytest.raises(ValueError):
        b200.make_args(a, b, c)
    with pytest.raises(TypeError):
        b200.make_args(a, torch.empty((3, 8), dtype=torch.bfloat16), c)
    with pytest.raises(ValueError):
        b200.make_args(a.t(), b, c)


def test_product_path_has_no_oracle_or_fallback():
    """The library and its Python mirror never reach into oracle/ or a CPU GEMM."""
    pkg = ROOT / "hopper-lab_b200"
    product = list(pkg.rglob("*.py")) + list(pkg.rglob("*.cu")) + list(pkg.rglob("*.cuh"))
    for f in product:
        text = f.read_text()
        assert "import oracle" not in text and "oracle/" not in text.replace("oracle/_ref", ""), f
        assert "torch.matmul" not in text, f


def test_noalloc_refuses_streamk_without_touching_the_device(b200):
    """Stream-K needs a partial-tile workspace that the static array cannot hold;
    the allocation-free entry point refuses it before any CUDA call."""
    fn = b200.lib().b200_gemm_noalloc
    fn.argtypes = [C.POINTER(b200.GemmArgs), C.c_void_p, C.c_int]
    fn.restype = C.c_int
    a = _args(b200, variant=b200.VARIANTS["2cta_streamk"])
    assert fn(C.byref(a), None, 0) == b200.ERR_SCRATCH_LIMIT


def test_allgather_entry_point_validates_without_a_gpu(b200):
    """b200_gemm_allgather checks its gather arguments before any CUDA call."""
    L = b200.lib()
    a = _args(b200)
    dst = C.c_void_p(0x40000)
    assert L.b200_gemm_allgather(C.byref(a), None, 1, 0, 512, 0, None) == b200.ERR_INVALID_ARG
    assert L.b200_gemm_allgather(C.byref(a), dst, 3, 0, 512, 0, None) == b200.ERR_INVALID_ARG
    assert L.b200_gemm_allgather(C.byref(a), dst, 2, 0, 512, 0, None) == b200.ERR_INVALID_ARG
    assert L.b200_gemm_allgather(C.byref(a), dst, 1, 0, 248, 0, None) == b200.ERR_SHAPE      # ldg < N
    assert L.b200_gemm_allgather(C.byref(a), dst, 1, 0, 512, 264, None) == b200.ERR_SHAPE    # past ldg
    assert L.b200_gemm_allgather(C.byref(a), dst, 1, 0, 520, 4, None) == b200.ERR_ALIGN      # 8-byte col
    assert L.b200_gemm_allgather(C.byref(a), C.c_void_p(0x40008), 1, 0, 512, 0, None) == b200.ERR_ALIGN
    k0 = _args(b200, K=0)
    assert L.b200_gemm_allgather(C.byref(k0), dst, 1, 0, 512, 0, None) == b200.ERR_SHAPE


def test_plan_validates_without_a_gpu(b200):
    """b200_gemm_plan_create checks its arguments before touching the device."""
    L = b200.lib()
    h = C.c_void_p()
    assert L.b200_gemm_plan_create(C.byref(_args(b200)), None) == b200.ERR_INVALID_ARG
    assert L.b200_gemm_plan_create(C.byref(_args(b200, ab_dtype=7)), C.byref(h)) == b200.ERR_INVALID_ARG
    assert not h.value
    assert L.b200_gemm_plan_create(C.byref(_args(b200, A=0x10001)), C.byref(h)) == b200.ERR_ALIGN
    assert L.b200_gemm_plan_launch(None, None) == b200.ERR_INVALID_ARG
    L.b200_gemm_plan_destroy(None)  # a null plan is accepted, like free(NULL)
