"""numpy restatement of the reference's tensor-parallel RMSNorm (test oracle).

Two functions, both taking every rank's slice at once:

``allreduce_path`` follows the reference's AllReduce path,
bench_rmsnorm_tp.py:16-22 (identical to test_rmsnorm_tp.py:15-26):
    variance_k = mean over the local slice of x_k.pow(2)   (:18; the square is
                 rounded to x's dtype, the mean accumulates in fp32)
    variance   = (sum_k variance_k) / tp                    (:19-21, all_reduce SUM)
    y_k        = x_k * rsqrt(variance + eps) * w_k          (:22, fp32 result)

``fused_path`` follows the reference's fused kernel, csrc/rmsnorm_tp.cu:
    s_k        = sum of fp32 squares of the local slice     (:72-96)
    S          = s_0 + ... + s_{tp-1}                       (:143-151)
    inv        = rsqrt(S / hidden + eps)                    (:156-157)
    y_k        = (x_k * inv) * w_k                          (:162-170)
which is what the CUDA kernels of this repository compute (in bf16/fp16 too).

``residual_add`` / ``allreduce_path_residual`` / ``fused_path_residual`` cover
the fused residual add, which the reference does not have: the updated residual
is z_k = (x_k + r_k).to(dtype) (an fp32 add rounded once, as torch computes
``x + r`` for bf16/fp16), and the norm is either path above applied to z_k.

``linear_rs_norm_path`` covers the fused row-parallel linear: each rank's
partial product rounded to the dtype (what an NCCL reduce-scatter in that dtype
is given), summed over ranks per column block in rank order, rounded, then the
AllReduce path above (with the residual add when given).

Arrays: fp32 values are np.float32; bf16 values are carried as np.uint16 bit
patterns; fp16 values as np.float16. Sums are taken in float64 and rounded to
fp32 once, which is within an ulp or two of torch's fp32 reductions.
"""
from __future__ import annotations

from typing import List, Sequence

import numpy as np

DTYPES = ("f32", "bf16", "f16")


def bf16_bits_to_f32(bits: np.ndarray) -> np.ndarray:
    """bf16 bit patterns (uint16) -> float32 (exact)."""
    return (np.asarray(bits, dtype=np.uint16).astype(np.uint32) << 16).view(np.float32)


def f32_to_bf16_bits(x: np.ndarray) -> np.ndarray:
    """float32 -> bf16 bit patterns, round to nearest even; NaN stays a quiet NaN."""
    u = np.asarray(x, dtype=np.float32).view(np.uint32)
    rounded = ((u + (np.uint32(0x7FFF) + ((u >> 16) & np.uint32(1)))) >> 16).astype(np.uint16)
    nan = np.isnan(np.asarray(x, dtype=np.float32))
    return np.where(nan, ((u >> 16) | np.uint32(0x40)).astype(np.uint16), rounded)


def to_f32(dtype: str, a: np.ndarray) -> np.ndarray:
    """Stored array of `dtype` -> float32 values."""
    if dtype == "f32":
        return np.asarray(a, dtype=np.float32)
    if dtype == "bf16":
        return bf16_bits_to_f32(a)
    if dtype == "f16":
        return np.asarray(a, dtype=np.float16).astype(np.float32)
    raise ValueError(f"unknown dtype {dtype}")


def from_f32(dtype: str, a: np.ndarray) -> np.ndarray:
    """float32 values -> stored array of `dtype` (round to nearest even)."""
    a = np.asarray(a, dtype=np.float32)
    if dtype == "f32":
        return a
    if dtype == "bf16":
        return f32_to_bf16_bits(a)
    if dtype == "f16":
        return a.astype(np.float16)
    raise ValueError(f"unknown dtype {dtype}")


def round_to(dtype: str, a: np.ndarray) -> np.ndarray:
    """Round float32 values to the grid of `dtype`, returned as float32."""
    return to_f32(dtype, from_f32(dtype, a))


def _rsqrt_f32(v: np.ndarray) -> np.ndarray:
    with np.errstate(divide="ignore", invalid="ignore"):
        return (1.0 / np.sqrt(np.asarray(v, dtype=np.float64))).astype(np.float32)


def allreduce_path(xs: Sequence[np.ndarray], ws: Sequence[np.ndarray], eps: float,
                   dtype: str) -> List[np.ndarray]:
    """Reference AllReduce TP RMSNorm (bench_rmsnorm_tp.py:16-22) over all ranks.

    Returns each rank's fp32 output (the reference returns fp32 for bf16/fp16
    inputs because x * rsqrt(fp32) promotes); round with ``from_f32`` to compare
    with an output in x's dtype.
    """
    tp = len(xs)
    variances = []
    for x in xs:
        xf = to_f32(dtype, x)
        with np.errstate(over="ignore"):
            sq = round_to(dtype, xf * xf)                        # x.pow(2) in x.dtype (:18)
        hl = xf.shape[-1]
        mean = (sq.astype(np.float64).sum(axis=-1, keepdims=True) / hl).astype(np.float32)
        variances.append(mean)                                   # mean(dtype=float32) (:18)
    total = variances[0].copy()
    for v in variances[1:]:
        total = (total + v).astype(np.float32)                   # all_reduce SUM (:20)
    variance = (total / np.float32(tp)).astype(np.float32) if tp > 1 else total   # (:21)
    inv = _rsqrt_f32((variance + np.float32(eps)).astype(np.float32))            # (:22)
    outs = []
    for x, w in zip(xs, ws):
        xf = to_f32(dtype, x)
        wf = to_f32(dtype, w)
        outs.append(((xf * inv).astype(np.float32) * wf).astype(np.float32))    # (:22)
    return outs


def partial_sums(x: np.ndarray, dtype: str) -> np.ndarray:
    """Per-row fp32 sum of squares of one rank's slice (rmsnorm_tp.cu:72-96)."""
    xf = to_f32(dtype, x).astype(np.float64)
    return (xf * xf).sum(axis=-1).astype(np.float32)


def fused_path(xs: Sequence[np.ndarray], ws: Sequence[np.ndarray], eps: float,
               dtype: str) -> List[np.ndarray]:
    """Reference fused-kernel formula (rmsnorm_tp.cu:143-170), any dtype, fp32 math.

    Returns each rank's fp32 output before the final rounding to x's dtype.
    """
    tp = len(xs)
    hidden = xs[0].shape[-1] * tp                                # total_hidden (__init__.py:101)
    S = partial_sums(xs[0], dtype)
    for x in xs[1:]:
        S = (S + partial_sums(x, dtype)).astype(np.float32)      # rank order (:145-148)
    var = (S / np.float32(hidden)).astype(np.float32)            # (:156)
    inv = _rsqrt_f32((var + np.float32(eps)).astype(np.float32))[..., None]   # (:157)
    outs = []
    for x, w in zip(xs, ws):
        xf = to_f32(dtype, x)
        wf = to_f32(dtype, w)
        outs.append(((xf * inv).astype(np.float32) * wf).astype(np.float32))  # (:166-169)
    return outs


def residual_add(x: np.ndarray, r: np.ndarray, dtype: str) -> np.ndarray:
    """z = (x + r) rounded once to `dtype`, in the stored representation of `dtype`."""
    with np.errstate(over="ignore", invalid="ignore"):
        return from_f32(dtype, (to_f32(dtype, x) + to_f32(dtype, r)).astype(np.float32))


def allreduce_path_residual(xs: Sequence[np.ndarray], rs: Sequence[np.ndarray],
                            ws: Sequence[np.ndarray], eps: float, dtype: str):
    """(outputs, updated residuals): the AllReduce path on z_k = x_k + r_k."""
    zs = [residual_add(x, r, dtype) for x, r in zip(xs, rs)]
    return allreduce_path(zs, ws, eps, dtype), zs


def fused_path_residual(xs: Sequence[np.ndarray], rs: Sequence[np.ndarray],
                        ws: Sequence[np.ndarray], eps: float, dtype: str):
    """(outputs, updated residuals): the fused-kernel formula on z_k = x_k + r_k."""
    zs = [residual_add(x, r, dtype) for x, r in zip(xs, rs)]
    return fused_path(zs, ws, eps, dtype), zs


def linear_partials(as_: Sequence[np.ndarray], lws: Sequence[np.ndarray],
                    dtype: str) -> List[np.ndarray]:
    """Rank r's partial product of a row-parallel linear, a_r @ lw_r^T, accumulated
    in float64, rounded to fp32 and then to `dtype` (what the rank sends)."""
    outs = []
    for a, w in zip(as_, lws):
        p = to_f32(dtype, a).astype(np.float64) @ to_f32(dtype, w).astype(np.float64).T
        outs.append(round_to(dtype, p.astype(np.float32)))
    return outs


def linear_reduce_scatter(partials: Sequence[np.ndarray], dtype: str) -> List[np.ndarray]:
    """Reduce-scatter by column block: rank o gets the rank-order fp32 sum of every
    rank's columns [o * hl, (o + 1) * hl), rounded to `dtype` (stored representation)."""
    tp = len(partials)
    hl = partials[0].shape[1] // tp
    xs = []
    for o in range(tp):
        acc = np.zeros((partials[0].shape[0], hl), dtype=np.float32)
        for p in partials:
            acc = (acc + p[:, o * hl:(o + 1) * hl]).astype(np.float32)
        xs.append(from_f32(dtype, acc))
    return xs


def linear_rs_norm_path(as_: Sequence[np.ndarray], lws: Sequence[np.ndarray],
                        gammas: Sequence[np.ndarray], eps: float, dtype: str,
                        residuals: Sequence[np.ndarray] = None):
    """Row-parallel linear -> reduce-scatter -> (residual add) -> the reference's
    AllReduce TP RMSNorm (bench_rmsnorm_tp.py:16-22), the unfused pipeline a
    Megatron-style block runs. Returns (every rank's fp32 output, every rank's
    normalised input z in `dtype`'s stored representation)."""
    xs = linear_reduce_scatter(linear_partials(as_, lws, dtype), dtype)
    if residuals is not None:
        return allreduce_path_residual(xs, residuals, gammas, eps, dtype)
    return allreduce_path(xs, gammas, eps, dtype), xs


def backward_path(xs: Sequence[np.ndarray], dys: Sequence[np.ndarray], ws: Sequence[np.ndarray],
                  eps: float, dtype: str):
    """Gradients of the TP RMSNorm (the reference is forward-only; this is the
    derivative of its formula, bench_rmsnorm_tp.py:16-22, in float64):
    with g = dy * w, S = sum over ranks of sum(x^2), D = sum over ranks of sum(g * x),
    inv = 1 / sqrt(S / hidden + eps):
        dx_k = inv * g_k - x_k * inv^3 * D / hidden,   dw_k = sum over rows of dy_k * x_k * inv.
    Returns (dxs, dws) as float32 values (before rounding to x's dtype)."""
    tp = len(xs)
    hidden = xs[0].shape[-1] * tp
    X = [to_f32(dtype, x).astype(np.float64) for x in xs]
    DY = [to_f32(dtype, d).astype(np.float64) for d in dys]
    W = [to_f32(dtype, w).astype(np.float64) for w in ws]
    S = sum((x * x).sum(axis=-1) for x in X)[..., None]
    D = sum((dy * w * x).sum(axis=-1) for x, dy, w in zip(X, DY, W))[..., None]
    inv = 1.0 / np.sqrt(S / hidden + eps)
    dxs = [(inv * dy * w - x * inv ** 3 * D / hidden).astype(np.float32)
           for x, dy, w in zip(X, DY, W)]
    dws = [(dy * x * inv).sum(axis=0).astype(np.float32) for x, dy in zip(X, DY)]
    return dxs, dws


def dw_magnitude(xs: Sequence[np.ndarray], dys: Sequence[np.ndarray], eps: float,
                 dtype: str) -> List[np.ndarray]:
    """Per rank and column, sum over rows of |dy * x * inv|: the scale of the
    rounding error of any fp32 summation of dw (a sum over rows whose result can be
    much smaller than its terms)."""
    tp = len(xs)
    hidden = xs[0].shape[-1] * tp
    X = [to_f32(dtype, x).astype(np.float64) for x in xs]
    S = sum((x * x).sum(axis=-1) for x in X)[..., None]
    inv = 1.0 / np.sqrt(S / hidden + eps)
    return [np.abs(to_f32(dtype, dy).astype(np.float64) * x * inv).sum(axis=0)
            for x, dy in zip(X, dys)]


# Backward tolerances: the fp32 kernels accumulate S, D and dw in fp32 in another
# order than the float64 oracle, and dx subtracts two terms of similar size. For
# dw, a sum over rows, the absolute tolerance also grows with the sum of the
# magnitudes of its terms (`scale`, from dw_magnitude): 32 fp32 units of it, above
# the typical error of the kernels' two-level summation (per-CTA partials of a
# few rows, then at most 296 partials).
BACKWARD_TOLERANCE = {
    "f32": dict(rtol=1e-4, atol=1e-5),
    "bf16": dict(rtol=1.6e-2, atol=2e-2),
    "f16": dict(rtol=1.6e-2, atol=2e-2),
}
FP32_UNIT = 2.0 ** -24


def compare_backward(dtype: str, got_f32: np.ndarray, want_f32: np.ndarray,
                     scale: np.ndarray = None) -> dict:
    """``compare`` with the backward tolerances (``scale``: see dw_magnitude)."""
    tol = BACKWARD_TOLERANCE[dtype]
    got = np.asarray(got_f32, dtype=np.float64)
    want = np.asarray(want_f32, dtype=np.float64)
    diff = np.abs(got - want)
    atol = tol["atol"] if scale is None else np.maximum(tol["atol"], 32 * FP32_UNIT * scale)
    bad = (diff > atol + tol["rtol"] * np.abs(want)) | (np.isnan(got) != np.isnan(want))
    return {"ok": not bool(bad.any()), "max_abs": float(np.nanmax(diff)) if diff.size else 0.0,
            "bad": int(bad.sum())}


# Tolerances of the parity bar: fp32 relative 1e-5; bf16/fp16 one ulp of the
# output type (atol 1e-2, rtol 1.6e-2).
TOLERANCE = {
    "f32": dict(rtol=1e-5, atol=1e-6),
    "bf16": dict(rtol=1.6e-2, atol=1e-2),
    "f16": dict(rtol=1.6e-2, atol=1e-2),
}


def compare(dtype: str, got_f32: np.ndarray, want_f32: np.ndarray) -> dict:
    """Compare two outputs (float32 arrays) against the tolerance of `dtype`.

    Returns {"ok", "max_abs", "max_rel", "bad"} where ``bad`` counts elements
    outside ``atol + rtol * |want|`` (NaN mismatches included).
    """
    tol = TOLERANCE[dtype]
    got = np.asarray(got_f32, dtype=np.float64)
    want = np.asarray(want_f32, dtype=np.float64)
    diff = np.abs(got - want)
    nan_mismatch = np.isnan(got) != np.isnan(want)
    both_nan = np.isnan(got) & np.isnan(want)
    diff = np.where(both_nan, 0.0, diff)
    bad = (diff > tol["atol"] + tol["rtol"] * np.abs(want)) | nan_mismatch
    rel = diff / np.maximum(np.abs(want), 1e-30)
    return {
        "ok": not bool(bad.any()),
        "max_abs": float(np.nanmax(diff)) if diff.size else 0.0,
        "max_rel": float(np.nanmax(np.where(np.abs(want) > 1e-3, rel, 0.0))) if diff.size else 0.0,
        "bad": int(bad.sum()),
    }
