"""CPU oracle for the B200 GEMM path — TEST INFRASTRUCTURE ONLY.

Only ``tests/``, ``__graft_entry__.smoke()`` and ``bench.py``'s CPU legs
(``cpu_baseline`` and ``--impl reference``) may import this package, and only
as the checker or the timed CPU baseline; the product library never links it.

``lib()`` loads ``oracle/_build/liboracle.so`` (the C restatement in
``gemm_oracle.c``, see its header for the reference lines each function
follows). ``ref_lib()`` loads ``oracle/_ref/libhopperref.so`` — the
reference's own host headers compiled by ``oracle/Makefile`` — when it was
built (it needs the reference tree at build time).
"""
from __future__ import annotations

import ctypes as C
import os
import subprocess
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
_LIB = None
_REF = None


class Report(C.Structure):
    _fields_ = [
        ("n", C.c_int64),
        ("mismatches", C.c_int64),
        ("max_abs_err", C.c_double),
        ("max_rel_err", C.c_double),
    ]


def build() -> None:
    subprocess.run(["make", "-s", "-C", str(HERE), "all"], check=True)


def build_ref() -> None:
    subprocess.run(["make", "-s", "-C", str(HERE), "ref"], check=True)


def _fp(a: np.ndarray, t):
    return a.ctypes.data_as(C.POINTER(t))


def lib():
    global _LIB
    if _LIB is None:
        so = HERE / "_build" / "liboracle.so"
        if not so.exists():
            build()
        L = C.CDLL(str(so))
        f32p, u16p, u8p = C.POINTER(C.c_float), C.POINTER(C.c_uint16), C.POINTER(C.c_uint8)
        L.oracle_uniform.argtypes = [C.c_uint32, C.c_int64, C.c_float, C.c_float, f32p]
        L.oracle_normal.argtypes = [C.c_uint32, C.c_int64, C.c_float, C.c_float, f32p]
        for name, src, dst in [
            ("oracle_f32_to_f16", f32p, u16p),
            ("oracle_f16_to_f32", u16p, f32p),
            ("oracle_f32_to_bf16", f32p, u16p),
            ("oracle_bf16_to_f32", u16p, f32p),
            ("oracle_f32_to_e4m3", f32p, u8p),
            ("oracle_e4m3_to_f32", u8p, f32p),
        ]:
            getattr(L, name).argtypes = [src, C.c_int64, dst]
        L.oracle_quantize_e4m3_scaled.argtypes = [f32p, C.c_int64, u8p]
        L.oracle_quantize_e4m3_scaled.restype = C.c_float
        L.oracle_gemm_tn.argtypes = [f32p, f32p, C.c_int64, C.c_int64, C.c_int64, C.c_int64,
                                     C.c_int64, f32p, C.c_int64, C.c_int, C.c_int]
        L.oracle_gemm_tn.restype = C.c_int
        L.oracle_check_close.argtypes = [f32p, f32p, C.c_int64, C.c_double, C.c_double,
                                         C.POINTER(Report)]
        L.oracle_check_close.restype = C.c_int
        _LIB = L
    return _LIB


def ref_lib():
    """The reference's own host code (None when oracle/_ref was not built)."""
    global _REF
    if _REF is None:
        so = HERE / "_ref" / "libhopperref.so"
        if not so.exists():
            return None
        L = C.CDLL(str(so))
        f32p, u16p, u8p = C.POINTER(C.c_float), C.POINTER(C.c_uint16), C.POINTER(C.c_uint8)
        L.ref_make_random_vector.argtypes = [C.c_uint32, C.c_int64, C.c_float, C.c_float, f32p]
        L.ref_normal.argtypes = [C.c_uint32, C.c_int64, C.c_float, C.c_float, f32p]
        L.ref_f32_to_f16.argtypes = [f32p, C.c_int64, u16p]
        L.ref_f32_to_bf16.argtypes = [f32p, C.c_int64, u16p]
        L.ref_f32_to_e4m3.argtypes = [f32p, C.c_int64, u8p]
        L.ref_e4m3_to_f32.argtypes = [u8p, C.c_int64, f32p]
        L.ref_f16_to_f32.argtypes = [u16p, C.c_int64, f32p]
        L.ref_gemm_loop_f16.argtypes = [u16p, u16p, C.c_int64, C.c_int64, C.c_int64, f32p]
        L.ref_gemm_loop_e4m3.argtypes = [u8p, u8p, C.c_int64, C.c_int64, C.c_int64, f32p]
        L.ref_check_close.argtypes = [f32p, f32p, C.c_int64, C.c_double, C.c_double,
                                      C.POINTER(C.c_int64), C.POINTER(C.c_double),
                                      C.POINTER(C.c_double)]
        L.ref_check_close.restype = C.c_int
        _REF = L
    return _REF


# ----------------------------------------------------------------------------- inputs
def uniform(seed: int, n: int, lo: float = -1.0, hi: float = 1.0) -> np.ndarray:
    """make_random_vector(n, seed, lo, hi) (include/common/tensor.h:12-20)."""
    out = np.empty(n, np.float32)
    lib().oracle_uniform(seed, n, lo, hi, _fp(out, C.c_float))
    return out


def normal(seed: int, n: int, mean: float = 0.0, std: float = 1.0) -> np.ndarray:
    """std::normal_distribution<float>(mean, std) over std::mt19937(seed)."""
    out = np.empty(n, np.float32)
    lib().oracle_normal(seed, n, mean, std, _fp(out, C.c_float))
    return out


def _cvt(name, x, out_dtype, in_ct, out_ct):
    x = np.ascontiguousarray(x)
    out = np.empty(x.shape, out_dtype)
    getattr(lib(), name)(_fp(x, in_ct), x.size, _fp(out, out_ct))
    return out


def f32_to_f16_bits(x):
    return _cvt("oracle_f32_to_f16", np.asarray(x, np.float32), np.uint16, C.c_float, C.c_uint16)


def f16_bits_to_f32(x):
    return _cvt("oracle_f16_to_f32", np.asarray(x, np.uint16), np.float32, C.c_uint16, C.c_float)


def f32_to_bf16_bits(x):
    return _cvt("oracle_f32_to_bf16", np.asarray(x, np.float32), np.uint16, C.c_float, C.c_uint16)


def bf16_bits_to_f32(x):
    return _cvt("oracle_bf16_to_f32", np.asarray(x, np.uint16), np.float32, C.c_uint16, C.c_float)


def f32_to_e4m3_bits(x):
    return _cvt("oracle_f32_to_e4m3", np.asarray(x, np.float32), np.uint8, C.c_float, C.c_uint8)


def e4m3_bits_to_f32(x):
    return _cvt("oracle_e4m3_to_f32", np.asarray(x, np.uint8), np.float32, C.c_uint8, C.c_float)


def quantize_e4m3_scaled(x: np.ndarray):
    """scale = amax/448 (1 if amax == 0); q = e4m3(x / scale). Returns (q_bits, scale)."""
    x = np.ascontiguousarray(x, np.float32)
    q = np.empty(x.shape, np.uint8)
    s = lib().oracle_quantize_e4m3_scaled(_fp(x, C.c_float), x.size, _fp(q, C.c_uint8))
    return q, np.float32(s)


def to_bits(x: np.ndarray, dtype: str) -> np.ndarray:
    if dtype == "f16":
        return f32_to_f16_bits(x)
    if dtype == "bf16":
        return f32_to_bf16_bits(x)
    if dtype == "e4m3":
        return f32_to_e4m3_bits(x)
    raise ValueError(dtype)


def from_bits(b: np.ndarray, dtype: str) -> np.ndarray:
    if dtype == "f16":
        return f16_bits_to_f32(b)
    if dtype == "bf16":
        return bf16_bits_to_f32(b)
    if dtype == "e4m3":
        return e4m3_bits_to_f32(b)
    raise ValueError(dtype)


# ------------------------------------------------------------------------------- GEMM
def gemm_tn(A: np.ndarray, B: np.ndarray, rows=None, threads: int | None = None,
            naive: bool = False) -> np.ndarray:
    """Reference host GEMM (src/05_gemm/gemm_ws.cu:258-265): C = A . B^T in fp32,
    sequential in k. A: M x K, B: N x K (fp32 values of the narrow inputs).
    rows=(r0, r1) computes only that band and returns (r1-r0) x N."""
    A = np.ascontiguousarray(A, np.float32)
    B = np.ascontiguousarray(B, np.float32)
    M, K = A.shape
    N, K2 = B.shape
    assert K == K2
    r0, r1 = (0, M) if rows is None else rows
    out = np.empty((r1 - r0, N), np.float32)
    if threads is None:
        threads = os.cpu_count() or 1
    # The C routine indexes C by absolute row; hand it a base pointer shifted back.
    base = out.ctypes.data - r0 * N * 4
    rc = lib().oracle_gemm_tn(_fp(A, C.c_float), _fp(B, C.c_float), M, N, K, r0, r1,
                              C.cast(C.c_void_p(base), C.POINTER(C.c_float)), N, threads,
                              1 if naive else 0)
    if rc != 0:
        raise RuntimeError(f"oracle_gemm_tn failed: {rc}")
    return out


def check_close(got: np.ndarray, ref: np.ndarray, rtol: float, atol: float) -> Report:
    """check_close (include/common/checker.h:30-55); NaNs do not count, as there."""
    got = np.ascontiguousarray(got, np.float32).ravel()
    ref = np.ascontiguousarray(ref, np.float32).ravel()
    r = Report()
    lib().oracle_check_close(_fp(got, C.c_float), _fp(ref, C.c_float), got.size, rtol, atol,
                             C.byref(r))
    return r
