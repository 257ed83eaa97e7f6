"""Generate tests/golden/golden.json from the REFERENCE's own host code.

Run in a tree where oracle/_ref/libhopperref.so was built (``make -C oracle ref``
compiles the reference's include/common/tensor.h and checker.h and the CUDA
headers' __half / __nv_bfloat16 / __nv_fp8_e4m3 conversions). The fixtures are
hashes and short excerpts of the reference's outputs on its own seeded inputs:

- make_random_vector(n, seed, -1, 1) for the seeds of every GEMM CHECK block and
  BASELINE config (src/05_gemm/gemm_ws.cu:247-321, src/07_fp8/gemm_fp8.cu:235-236,
  src/08_persistent/gemm_fp8_persist.cu:289-290, gemm_fp8_bn128.cu:325-326);
- std::normal_distribution<float>(0, 0.1) for the bf16 config's seeds 605/606;
- fp32 -> fp16 / bf16 / e4m3 conversions on edge values and a seeded sweep of bit
  patterns;
- the reference's host GEMM loop on its fp16 CHECK (512x512x256, seeds 601/602)
  and fp8 CHECK (512x512x256, seeds 901/902) inputs;
- check_close on crafted vectors.

Usage: python tests/golden/make_golden.py   (writes tests/golden/golden.json)
"""
import ctypes as C
import hashlib
import json
import sys
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parents[2]
sys.path.insert(0, str(ROOT))
import oracle as O  # noqa: E402

F32P, U16P, U8P = C.POINTER(C.c_float), C.POINTER(C.c_uint16), C.POINTER(C.c_uint8)
SEEDS = [601, 602, 603, 604, 605, 606, 901, 902, 903, 904, 905, 906, 907, 908, 1001, 1002,
         1003, 1004, 2001, 2002]
N_VEC = 1 << 16

EDGE = [0.0, -0.0, 1.0, -1.0, 0.5, 1e-8, -1e-8, 2.0 ** -10, 2.0 ** -9 * 1.5, 2.0 ** -24,
        2.0 ** -25, 3.0 * 2.0 ** -26, 448.0, 449.0, 464.0, 470.0, 480.0, 1e6, -1e6, 65504.0,
        65519.0, 65520.0, 3.3895314e38, float("inf"), float("-inf"), 0.1, -0.3, 1.0 / 3.0,
        239.9, 240.0, 247.99, 248.0, 0.001953125, 0.0009765625, 5.9604645e-08]


def sha(a: np.ndarray) -> str:
    return hashlib.sha256(np.ascontiguousarray(a).tobytes()).hexdigest()


def sweep_bits() -> np.ndarray:
    rng = np.random.default_rng(12345)
    return rng.integers(0, 2 ** 32, size=1 << 20, dtype=np.uint64).astype(np.uint32).view(np.float32)


def main():
    R = O.ref_lib()
    if R is None:
        raise SystemExit("oracle/_ref/libhopperref.so is missing: run `make -C oracle ref` with the reference tree present")
    out = {"generator": "tests/golden/make_golden.py (reference headers via oracle/_ref)", "n_vec": N_VEC}

    uni = {}
    for s in SEEDS:
        v = np.empty(N_VEC, np.float32)
        R.ref_make_random_vector(s, N_VEC, -1.0, 1.0, v.ctypes.data_as(F32P))
        uni[str(s)] = {"sha256": sha(v), "head": [float(x) for x in v[:8]]}
    out["uniform_m1_1"] = uni

    nrm = {}
    for s in (605, 606):
        v = np.empty(N_VEC, np.float32)
        R.ref_normal(s, N_VEC, 0.0, 0.1, v.ctypes.data_as(F32P))
        nrm[str(s)] = {"sha256": sha(v), "head": [float(x) for x in v[:8]]}
    out["normal_0_0.1"] = nrm

    def conv(fn, x, dt, ct):
        y = np.empty(x.shape, dt)
        getattr(R, fn)(x.ctypes.data_as(F32P), x.size, y.ctypes.data_as(C.POINTER(ct)))
        return y

    edge = np.array(EDGE, np.float32)
    sw = sweep_bits()
    out["edge_values"] = [float(x) for x in edge]
    out["edge_f16"] = conv("ref_f32_to_f16", edge, np.uint16, C.c_uint16).tolist()
    out["edge_bf16"] = conv("ref_f32_to_bf16", edge, np.uint16, C.c_uint16).tolist()
    out["edge_e4m3"] = conv("ref_f32_to_e4m3", edge, np.uint8, C.c_uint8).tolist()
    out["sweep_f16_sha256"] = sha(conv("ref_f32_to_f16", sw, np.uint16, C.c_uint16))
    out["sweep_bf16_sha256"] = sha(conv("ref_f32_to_bf16", sw, np.uint16, C.c_uint16))
    out["sweep_e4m3_sha256"] = sha(conv("ref_f32_to_e4m3", sw, np.uint8, C.c_uint8))
    allq = np.arange(256, dtype=np.uint8)
    dq = np.empty(256, np.float32)
    R.ref_e4m3_to_f32(allq.ctypes.data_as(U8P), 256, dq.ctypes.data_as(F32P))
    out["e4m3_decode_sha256"] = sha(dq)

    # the reference's fp16 CHECK: 512x512x256, seeds 601/602 (gemm_ws.cu:246-265)
    M, N, K = 512, 512, 256
    a = np.empty(M * K, np.float32)
    b = np.empty(N * K, np.float32)
    R.ref_make_random_vector(601, M * K, -1.0, 1.0, a.ctypes.data_as(F32P))
    R.ref_make_random_vector(602, N * K, -1.0, 1.0, b.ctypes.data_as(F32P))
    ah = conv("ref_f32_to_f16", a, np.uint16, C.c_uint16)
    bh = conv("ref_f32_to_f16", b, np.uint16, C.c_uint16)
    ref = np.empty(M * N, np.float32)
    R.ref_gemm_loop_f16(ah.ctypes.data_as(U16P), bh.ctypes.data_as(U16P), M, N, K, ref.ctypes.data_as(F32P))
    out["gemm_f16_512x512x256_s601_602"] = {"sha256": sha(ref), "c00": float(ref[0]),
                                            "c_last": float(ref[-1]),
                                            "fro": float(np.linalg.norm(ref.astype(np.float64)))}
    # the reference's fp8 CHECK: 512x512x256, seeds 901/902 (gemm_fp8.cu:234-253)
    R.ref_make_random_vector(901, M * K, -1.0, 1.0, a.ctypes.data_as(F32P))
    R.ref_make_random_vector(902, N * K, -1.0, 1.0, b.ctypes.data_as(F32P))
    aq = conv("ref_f32_to_e4m3", a, np.uint8, C.c_uint8)
    bq = conv("ref_f32_to_e4m3", b, np.uint8, C.c_uint8)
    R.ref_gemm_loop_e4m3(aq.ctypes.data_as(U8P), bq.ctypes.data_as(U8P), M, N, K, ref.ctypes.data_as(F32P))
    out["gemm_e4m3_512x512x256_s901_902"] = {"sha256": sha(ref), "c00": float(ref[0]),
                                             "c_last": float(ref[-1]),
                                             "fro": float(np.linalg.norm(ref.astype(np.float64)))}

    # check_close on crafted vectors (checker.h:30-55)
    g = np.array([1.0, 2.0, 3.001, 4.1, -5.0, 0.0, 1e-7], np.float32)
    e = np.array([1.0, 2.0005, 3.0, 4.0, -5.0, 1e-9, 0.0], np.float32)
    cases = []
    for rtol, atol in [(1e-3, 1e-3), (1e-2, 0.0), (0.0, 0.2), (3e-2, 3e-2)]:
        mm = C.c_int64()
        ma = C.c_double()
        mr = C.c_double()
        p = R.ref_check_close(g.ctypes.data_as(F32P), e.ctypes.data_as(F32P), g.size, rtol, atol,
                              C.byref(mm), C.byref(ma), C.byref(mr))
        cases.append({"rtol": rtol, "atol": atol, "pass": int(p), "mismatches": mm.value,
                      "max_abs": ma.value, "max_rel": mr.value})
    out["check_close"] = {"got": g.tolist(), "ref": e.tolist(), "cases": cases}

    path = ROOT / "tests" / "golden" / "golden.json"
    path.write_text(json.dumps(out, indent=1) + "\n")
    print("wrote", path)


if __name__ == "__main__":
    main()
