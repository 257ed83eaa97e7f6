"""hopper-lab_b200 — Python host mirror of the B200 GEMM C ABI (include/b200gemm.h).

The reference drives each GEMM experiment through
``dispatch(stages, flag, tmap_a, tmap_b, tmap_d, D, M, N, K[, group_m])``
(src/05_gemm/gemm_ws.cu:214-235, src/08_persistent/gemm_fp8_persist.cu:244-270),
which exits the process on any error. Here the same knobs (stages, group_m,
epilogue/variant) are arguments of :func:`gemm`, which calls ``b200_gemm`` in
``lib/libb200gemm.so`` through ctypes on torch-owned device memory and raises
:class:`B200Error` with the library's code instead of exiting.

There is no CPU fallback: if the shared library is missing, :func:`lib` raises.
The directory name contains a hyphen, so load it with
``importlib`` (see ``__graft_entry__.py``) or add the repository root to a
loader of your own; it registers itself as ``hopper_lab_b200``.
"""
from __future__ import annotations

import ctypes as C
import os
from pathlib import Path

PKG = Path(__file__).resolve().parent
# The in-tree build; B200GEMM_LIB names another build of the same ABI (e.g. one made
# with different compile-time options) to load instead.
LIB_PATH = Path(os.environ.get("B200GEMM_LIB") or PKG / "lib" / "libb200gemm.so")

DT_F16, DT_BF16, DT_E4M3, DT_F32 = 0, 1, 2, 3
VARIANTS = {"auto": 0, "1cta": 1, "2cta": 2, "persistent": 3, "clc": 4, "2cta_clc": 5,
            "2cta_streamk": 6}
VARIANT_NAMES = {v: k for k, v in VARIANTS.items()}

OK = 0
ERR_INVALID_ARG = -1
ERR_SHAPE = -2
ERR_ALIGN = -3
ERR_TMAP = -4
ERR_LAUNCH = -5
ERR_DEVICE_TIMEOUT = -6
ERR_UNSUPPORTED = -7
ERR_CUDA = -8
ERR_SCRATCH_LIMIT = -9

# Symbols declared in include/b200gemm.h (tests check the library exports them all).
EXPORTS = [
    "b200_gemm",
    "b200_gemm_strerror",
    "b200_gemm_status",
    "b200_gemm_variant_info",
    "b200_gemm_pick_variant",
    "b200_gemm_pick_config",
    "b200_quantize_e4m3",
    "b200_gemm_abi_version",
    "b200_gemm_noalloc",
    "b200_gemm_allgather",
    "b200_gemm_plan_create",
    "b200_gemm_plan_launch",
    "b200_gemm_plan_destroy",
]
GATHER_MULTICAST, GATHER_PEERS = 1, 2


class GemmArgs(C.Structure):
    """Mirror of ``B200GemmArgs`` (include/b200gemm.h)."""

    _fields_ = [
        ("ab_dtype", C.c_int32),
        ("c_dtype", C.c_int32),
        ("M", C.c_int64),
        ("N", C.c_int64),
        ("K", C.c_int64),
        ("lda", C.c_int64),
        ("ldb", C.c_int64),
        ("ldc", C.c_int64),
        ("A", C.c_void_p),
        ("B", C.c_void_p),
        ("C", C.c_void_p),
        ("scale_a", C.c_void_p),
        ("scale_b", C.c_void_p),
        ("variant", C.c_int32),
        ("group_m", C.c_int32),
        ("stages", C.c_int32),
        ("fault_inject", C.c_int32),
        ("wait_limit_ns", C.c_uint64),
        ("tile_n", C.c_int32),
        ("reserved", C.c_int32),
    ]


class B200Error(RuntimeError):
    def __init__(self, code: int, what: str = ""):
        self.code = code
        msg = strerror(code)
        super().__init__(f"{what}: {msg} ({code})" if what else f"{msg} ({code})")


_LIB = None


def lib():
    """Load libb200gemm.so (raises if it was not built — there is no fallback)."""
    global _LIB
    if _LIB is None:
        if not LIB_PATH.exists():
            raise RuntimeError(
                f"{LIB_PATH} is missing: build it with `python hopper-lab_b200/build.py` "
                "(there is no CPU fallback)")
        L = C.CDLL(str(LIB_PATH))
        L.b200_gemm.argtypes = [C.POINTER(GemmArgs), C.c_void_p]
        L.b200_gemm.restype = C.c_int
        L.b200_gemm_strerror.argtypes = [C.c_int]
        L.b200_gemm_strerror.restype = C.c_char_p
        L.b200_gemm_status.argtypes = [C.c_void_p, C.c_int, C.POINTER(C.c_uint32)]
        L.b200_gemm_status.restype = C.c_int
        L.b200_gemm_variant_info.argtypes = [C.c_int32, C.c_int32] + [C.POINTER(C.c_int32)] * 4
        L.b200_gemm_variant_info.restype = C.c_int
        L.b200_gemm_pick_variant.argtypes = [C.POINTER(GemmArgs)]
        L.b200_gemm_pick_variant.restype = C.c_int
        L.b200_gemm_pick_config.argtypes = [C.POINTER(GemmArgs), C.POINTER(C.c_int32),
                                            C.POINTER(C.c_int32)]
        L.b200_gemm_pick_config.restype = C.c_int
        L.b200_quantize_e4m3.argtypes = [C.c_void_p, C.c_int64, C.c_void_p, C.c_void_p, C.c_void_p]
        L.b200_quantize_e4m3.restype = C.c_int
        L.b200_gemm_abi_version.argtypes = []
        L.b200_gemm_abi_version.restype = C.c_int
        L.b200_gemm_allgather.argtypes = [C.POINTER(GemmArgs), C.c_void_p, C.c_int32, C.c_int32,
                                          C.c_int64, C.c_int64, C.c_void_p]
        L.b200_gemm_allgather.restype = C.c_int
        L.b200_gemm_plan_create.argtypes = [C.POINTER(GemmArgs), C.POINTER(C.c_void_p)]
        L.b200_gemm_plan_create.restype = C.c_int
        L.b200_gemm_plan_launch.argtypes = [C.c_void_p, C.c_void_p]
        L.b200_gemm_plan_launch.restype = C.c_int
        L.b200_gemm_plan_destroy.argtypes = [C.c_void_p]
        L.b200_gemm_plan_destroy.restype = None
        _LIB = L
    return _LIB


def strerror(code: int) -> str:
    try:
        return lib().b200_gemm_strerror(code).decode()
    except Exception:  # library missing: still produce a message
        return f"error {code}"


def variant_info(variant: str | int, ab_dtype: int = DT_F16, tile_n: int = 0):
    v = VARIANTS[variant] if isinstance(variant, str) else int(variant)
    out = [C.c_int32() for _ in range(4)]
    out[1].value = tile_n
    rc = lib().b200_gemm_variant_info(v, ab_dtype, *[C.byref(o) for o in out])
    if rc != OK:
        raise B200Error(rc, "variant_info")
    return {"tile_m": out[0].value, "tile_n": out[1].value, "max_stages": out[2].value,
            "default_stages": out[3].value}


# ---------------------------------------------------------------------------- torch glue
def _torch():
    import torch  # noqa: WPS433 — torch is plumbing (device memory, streams) only

    return torch


def _dt_of(t) -> int:
    torch = _torch()
    if t.dtype == torch.float16:
        return DT_F16
    if t.dtype == torch.bfloat16:
        return DT_BF16
    if t.dtype in (torch.float8_e4m3fn, torch.uint8):
        return DT_E4M3
    if t.dtype == torch.float32:
        return DT_F32
    raise TypeError(f"unsupported dtype {t.dtype}")


def _torch_dtype(dt: int):
    torch = _torch()
    return {DT_F16: torch.float16, DT_BF16: torch.bfloat16, DT_F32: torch.float32,
            DT_E4M3: torch.float8_e4m3fn}[dt]


def _dtype_code(name) -> int:
    if isinstance(name, int):
        return name
    return {"f16": DT_F16, "fp16": DT_F16, "float16": DT_F16, "bf16": DT_BF16,
            "bfloat16": DT_BF16, "e4m3": DT_E4M3, "fp8": DT_E4M3, "f32": DT_F32,
            "fp32": DT_F32, "float32": DT_F32}[name]


def _stream_handle(stream) -> int:
    torch = _torch()
    if stream is None:
        return torch.cuda.current_stream().cuda_stream
    if isinstance(stream, int):
        return stream
    return stream.cuda_stream


def make_args(a, b, c, *, scale_a=None, scale_b=None, variant="auto", group_m=0, stages=0,
              wait_limit_ns=0, fault_inject=0, tile_n=0) -> GemmArgs:
    """Fill B200GemmArgs from 2-D torch tensors (row-major, unit column stride)."""
    for name, t in (("A", a), ("B", b), ("C", c)):
        if t.dim() != 2 or (t.numel() > 0 and t.stride(1) != 1):
            raise ValueError(f"{name} must be a 2-D row-major tensor with unit column stride")
    M, K = a.shape
    N, K2 = b.shape
    if K != K2 or tuple(c.shape) != (M, N):
        raise ValueError(f"shape mismatch: A {tuple(a.shape)}, B {tuple(b.shape)}, C {tuple(c.shape)}")
    args = GemmArgs()
    args.ab_dtype = _dt_of(a)
    if _dt_of(b) != args.ab_dtype:
        raise TypeError("A and B must have the same element type")
    args.c_dtype = _dt_of(c)
    args.M, args.N, args.K = M, N, K
    args.lda = a.stride(0) if M > 1 else max(K, 1)
    args.ldb = b.stride(0) if N > 1 else max(K, 1)
    args.ldc = c.stride(0) if M > 1 else max(N, 1)
    args.A, args.B, args.C = a.data_ptr(), b.data_ptr(), c.data_ptr()
    args.scale_a = scale_a.data_ptr() if scale_a is not None else None
    args.scale_b = scale_b.data_ptr() if scale_b is not None else None
    args.variant = VARIANTS[variant] if isinstance(variant, str) else int(variant)
    args.group_m = group_m
    args.stages = stages
    args.fault_inject = fault_inject
    args.wait_limit_ns = wait_limit_ns
    args.tile_n = tile_n
    return args


def gemm(a, b, c=None, *, out_dtype="bf16", scale_a=None, scale_b=None, variant="auto",
         group_m: int = 0, stages: int = 0, wait_limit_ns: int = 0, fault_inject: int = 0,
         tile_n: int = 0, stream=None):
    """C = scale_a * scale_b * A . B^T on the GPU (A: M x K, B: N x K, both row-major).

    A/B: torch.float16 | torch.bfloat16 | torch.float8_e4m3fn (or uint8 bits).
    C is allocated with ``out_dtype`` when not given. scale_a/scale_b are 1-element
    fp32 device tensors (or None). Returns C. Raises B200Error on any failure.
    """
    torch = _torch()
    if c is None:
        c = torch.empty((a.shape[0], b.shape[0]), dtype=_torch_dtype(_dtype_code(out_dtype)),
                        device=a.device)
    args = make_args(a, b, c, scale_a=scale_a, scale_b=scale_b, variant=variant, group_m=group_m,
                     stages=stages, wait_limit_ns=wait_limit_ns, fault_inject=fault_inject,
                     tile_n=tile_n)
    rc = lib().b200_gemm(C.byref(args), C.c_void_p(_stream_handle(stream)))
    if rc != OK:
        raise B200Error(rc, "b200_gemm")
    return c


def gemm_allgather(a, b, c, dst: int, mode: int, npeers: int, ldg: int, col_off: int, *,
                   scale_a=None, scale_b=None, variant="auto", tile_n: int = 0, stream=None):
    """b200_gemm_allgather: C = scale_a*scale_b*A.B^T on this GPU, and every C tile also
    stored at G[row*ldg + col_off + col] on every GPU of the node. `dst` is the multicast
    address of G (mode GATHER_MULTICAST) or the device address of an array of `npeers`
    peer base addresses (GATHER_PEERS). The caller synchronises the GPUs before reading G."""
    args = make_args(a, b, c, scale_a=scale_a, scale_b=scale_b, variant=variant, tile_n=tile_n)
    rc = lib().b200_gemm_allgather(C.byref(args), C.c_void_p(dst), mode, npeers, ldg, col_off,
                                   C.c_void_p(_stream_handle(stream)))
    if rc != OK:
        raise B200Error(rc, "b200_gemm_allgather")
    return c


class Plan:
    """b200_gemm_plan_*: a GEMM resolved once (variant, tensor maps, kernel parameters)
    on fixed buffers; `launch()` only launches. Keeps references to the tensors so the
    buffers outlive the plan."""

    def __init__(self, a, b, c, **kw):
        self._h = None
        self._keep = (a, b, c, kw.get("scale_a"), kw.get("scale_b"))
        args = make_args(a, b, c, **kw)
        h = C.c_void_p()
        rc = lib().b200_gemm_plan_create(C.byref(args), C.byref(h))
        if rc != OK:
            raise B200Error(rc, "b200_gemm_plan_create")
        self._h = h

    def launch(self, stream=None):
        rc = lib().b200_gemm_plan_launch(self._h, C.c_void_p(_stream_handle(stream)))
        if rc != OK:
            raise B200Error(rc, "b200_gemm_plan_launch")

    def close(self):
        if self._h:
            lib().b200_gemm_plan_destroy(self._h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


def gemm_raw(args: GemmArgs, stream=None) -> int:
    """Call b200_gemm with a prepared argument block; returns the raw code."""
    return lib().b200_gemm(C.byref(args), C.c_void_p(_stream_handle(stream)))


def pick_variant(a, b, c) -> str:
    args = make_args(a, b, c)
    v = lib().b200_gemm_pick_variant(C.byref(args))
    if v < 0:
        raise B200Error(v, "pick_variant")
    return VARIANT_NAMES[v]


def pick_config(args: GemmArgs) -> tuple[str, int]:
    """(variant name, tile width) that b200_gemm launches for a prepared argument block."""
    v, tn = C.c_int32(), C.c_int32()
    rc = lib().b200_gemm_pick_config(C.byref(args), C.byref(v), C.byref(tn))
    if rc != OK:
        raise B200Error(rc, "pick_config")
    return VARIANT_NAMES[v.value], tn.value


def status(stream=None, clear: bool = True):
    """(code, bits): B200_OK or B200_ERR_DEVICE_TIMEOUT with the raw device bits."""
    bits = C.c_uint32()
    rc = lib().b200_gemm_status(C.c_void_p(_stream_handle(stream)), 1 if clear else 0,
                                C.byref(bits))
    return rc, bits.value


def quantize_e4m3(x, q=None, scale=None, stream=None):
    """Device per-tensor quantiser: returns (q float8_e4m3fn, scale fp32[1])."""
    torch = _torch()
    if x.dtype != torch.float32 or not x.is_contiguous():
        raise ValueError("x must be a contiguous float32 tensor")
    if q is None:
        q = torch.empty(x.shape, dtype=torch.float8_e4m3fn, device=x.device)
    if scale is None:
        scale = torch.empty(1, dtype=torch.float32, device=x.device)
    rc = lib().b200_quantize_e4m3(C.c_void_p(x.data_ptr()), x.numel(), C.c_void_p(q.data_ptr()),
                                  C.c_void_p(scale.data_ptr()),
                                  C.c_void_p(_stream_handle(stream)))
    if rc != OK:
        raise B200Error(rc, "b200_quantize_e4m3")
    return q, scale
