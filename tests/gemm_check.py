"""Helpers shared by the GPU parity tests: seeded inputs from the oracle, a GPU
run through the C ABI, and the comparison against the oracle's host GEMM.

Tolerances
- f16/bf16 inputs: relative error <= 1e-2, checked two ways:
  norm-wise ||C - R||_F / ||R||_F <= 1e-2, and element-wise
  |C - R| <= 1e-2 * rms(R) + 1e-2 * |R|.
- fp32 output on the reference's own CHECK cases: the reference's tolerances,
  rtol = atol = 1e-3 for fp16 (src/05_gemm/gemm_ws.cu:272) and 3e-2 for e4m3
  (src/07_fp8/gemm_fp8.cu:260).
- e4m3 with per-tensor scales, bf16 output: the reference's 3e-2, element-wise
  with atol = 3e-2 * rms(R), plus the same 3e-2 norm-wise.
"""
from __future__ import annotations

import numpy as np

TOL_16 = 1e-2
TOL_E4M3 = 3e-2


_CACHE: dict = {}


def make_inputs(oracle, M, N, K, dtype, seed_a, seed_b, dist="uniform", scaled=False):
    """Seeded host inputs as the reference builds them (tensor.h:12-20), cast to
    `dtype`. Returns dict with bit arrays, fp32 views of the narrow values, scales.
    The last few input sets are cached (big shapes repeat across variants)."""
    key = (M, N, K, dtype, seed_a, seed_b, dist, scaled)
    if key in _CACHE:
        return _CACHE[key]
    if len(_CACHE) >= 3:
        _CACHE.pop(next(iter(_CACHE)))
    _CACHE[key] = _make_inputs(oracle, M, N, K, dtype, seed_a, seed_b, dist, scaled)
    return _CACHE[key]


def _make_inputs(oracle, M, N, K, dtype, seed_a, seed_b, dist, scaled):
    if dist == "uniform":
        a32 = oracle.uniform(seed_a, M * K)
        b32 = oracle.uniform(seed_b, N * K)
    else:  # normal(0,1)*0.1 for the bf16 config
        a32 = oracle.normal(seed_a, M * K, 0.0, 0.1)
        b32 = oracle.normal(seed_b, N * K, 0.0, 0.1)
    sa = sb = np.float32(1.0)
    if dtype == "e4m3" and scaled:
        qa, sa = oracle.quantize_e4m3_scaled(a32)
        qb, sb = oracle.quantize_e4m3_scaled(b32)
    else:
        qa = oracle.to_bits(a32, dtype)
        qb = oracle.to_bits(b32, dtype)
    return {
        "M": M, "N": N, "K": K, "dtype": dtype,
        "a_bits": qa.reshape(M, K), "b_bits": qb.reshape(N, K),
        "a_val": oracle.from_bits(qa, dtype).reshape(M, K),
        "b_val": oracle.from_bits(qb, dtype).reshape(N, K),
        "sa": np.float32(sa), "sb": np.float32(sb), "scaled": scaled,
    }


def to_device(inp, torch):
    dt = {"f16": torch.float16, "bf16": torch.bfloat16, "e4m3": torch.float8_e4m3fn}[inp["dtype"]]
    a = torch.from_numpy(np.ascontiguousarray(inp["a_bits"])).cuda().view(dt)
    b = torch.from_numpy(np.ascontiguousarray(inp["b_bits"])).cuda().view(dt)
    sa = sb = None
    if inp["scaled"]:
        sa = torch.tensor([float(inp["sa"])], dtype=torch.float32, device="cuda")
        sb = torch.tensor([float(inp["sb"])], dtype=torch.float32, device="cuda")
    return a, b, sa, sb


def reference(oracle, inp, rows=None):
    """Oracle C (or a band of rows), including the per-tensor scale product."""
    r = oracle.gemm_tn(inp["a_val"], inp["b_val"], rows=rows)
    if inp["scaled"]:
        s = np.float32(inp["sa"]) * np.float32(inp["sb"])
        r = (r * s).astype(np.float32)
    return r


def reference_cols(oracle, inp, cols):
    """Oracle C restricted to the columns [c0, c1): all M rows of that column slab."""
    c0, c1 = cols
    r = oracle.gemm_tn(inp["a_val"], inp["b_val"][c0:c1])
    if inp["scaled"]:
        s = np.float32(inp["sa"]) * np.float32(inp["sb"])
        r = (r * s).astype(np.float32)
    return r


def check_big(oracle, inp, got, tol, seed, rows=256, band=32, slab=256):
    """Big-shape parity: `rows` seeded rows (bands of `band` rows, the first and last
    band included) against all N columns, plus every row of one seeded `slab`-column
    slab of C. Returns a list of failures (empty when everything matches)."""
    M, N = inp["M"], inp["N"]
    fails = []
    for r0, r1 in sample_bands(M, seed, bands=max(1, rows // band - 2), rows=band):
        ok, info = compare(got[r0:r1], reference(oracle, inp, rows=(r0, r1)), tol)
        if not ok:
            fails.append(("rows", r0, r1, info))
    rng = np.random.default_rng(seed + 1)
    c0 = int(rng.integers(0, max(1, (N - slab) // 16 + 1))) * 16 if N > slab else 0
    c1 = min(N, c0 + slab)
    ok, info = compare(got[:, c0:c1], reference_cols(oracle, inp, (c0, c1)), tol)
    if not ok:
        fails.append(("cols", c0, c1, info))
    return fails


def sample_bands(M, seed, bands=4, rows=64):
    """Seeded row bands [r0, r0+rows) spread over M, for big-shape checks."""
    rng = np.random.default_rng(seed)
    if M <= bands * rows:
        return [(0, M)]
    starts = sorted(rng.choice(M // rows, size=bands, replace=False) * rows)
    out = [(0, rows)] + [(int(s), int(s) + rows) for s in starts if s != 0]
    out.append((M - rows, M))
    return sorted(set(out))


def compare(got: np.ndarray, ref: np.ndarray, tol: float, atol_rms: bool = True, rtol=None):
    """Returns (ok, info). got/ref fp32 arrays of the same shape."""
    got = got.astype(np.float32)
    ref = ref.astype(np.float32)
    if not np.all(np.isfinite(got)):
        return False, {"nonfinite": int((~np.isfinite(got)).sum())}
    diff = np.abs(got.astype(np.float64) - ref.astype(np.float64))
    rn = float(np.sqrt(np.mean(ref.astype(np.float64) ** 2)))
    norm_rel = float(np.linalg.norm(diff) / max(np.linalg.norm(ref.astype(np.float64)), 1e-30))
    atol = tol * rn if atol_rms else tol
    rt = tol if rtol is None else rtol
    bad = int((diff > atol + rt * np.abs(ref)).sum())
    info = {"norm_rel": norm_rel, "max_abs": float(diff.max()) if diff.size else 0.0,
            "mismatch": bad, "n": int(diff.size), "rms_ref": rn}
    ok = bad == 0 and (norm_rel <= tol or not atol_rms)
    return ok, info


def out_to_f32(c, torch):
    return c.float().cpu().numpy()
