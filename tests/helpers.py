"""Comparison helpers shared by the parity tests.

Tolerances follow PyFlame's own executor-vs-CPU harness
(tests/backend/rocm/test_rocm_operations.cpp:66-103: |gpu - cpu| <= atol +
rtol*|cpu|, rtol 1e-5, atol 1e-6) and the bar the CUDA executor is held to:
elementwise and reductions within 1e-5 relative, fp32 contractions through
3xTF32 within 1e-4, bf16 contractions within 2e-2.  Reductions and
normalised outputs use a condition-aware absolute term: for a sum the error
budget scales with the sum of |terms|, for LayerNorm/softmax/GEMM rows with
the row's RMS.
"""
import numpy as np

RTOL_EW = 1e-5
ATOL_EW = 1e-6
RTOL_GEMM_TF32X3 = 1e-4
RTOL_GEMM_BF16 = 2e-2


def bitexact(a, b):
    a, b = np.asarray(a), np.asarray(b)
    assert a.shape == b.shape, (a.shape, b.shape)
    same = (a == b) | (np.isnan(a) & np.isnan(b))
    bad = np.argwhere(~same)
    assert bad.size == 0, f"{len(bad)} mismatches, first at {bad[0]}: {a[tuple(bad[0])]} vs {b[tuple(bad[0])]}"


def close(gpu, ref, rtol=RTOL_EW, atol=ATOL_EW, what=""):
    gpu, ref = np.asarray(gpu, np.float64), np.asarray(ref, np.float64)
    assert gpu.shape == ref.shape, (gpu.shape, ref.shape)
    nan_ok = np.isnan(gpu) == np.isnan(ref)
    assert nan_ok.all(), f"{what}: NaN pattern differs"
    inf_g, inf_r = np.isinf(gpu), np.isinf(ref)
    assert (inf_g == inf_r).all() and (gpu[inf_g] == ref[inf_r]).all(), f"{what}: inf pattern differs"
    fin = np.isfinite(ref)
    diff = np.abs(gpu - ref)
    tol = atol + rtol * np.abs(ref)
    tol = np.broadcast_to(tol, diff.shape)
    bad = fin & (diff > tol)
    if bad.any():
        i = tuple(np.argwhere(bad)[0])
        raise AssertionError(f"{what}: {bad.sum()} of {bad.size} outside tolerance; first {i}: gpu={gpu[i]} "
                             f"ref={ref[i]} diff={diff[i]} tol={tol[i]}")


def row_rms(x, axis=-1):
    x = np.asarray(x, np.float64)
    return np.sqrt(np.mean(x * x, axis=axis, keepdims=True)) + 1e-30


def close_rows(gpu, ref, rtol, what=""):
    """|gpu - ref| <= rtol*|ref| + rtol*rms(row of ref)."""
    close(gpu, ref, rtol=rtol, atol=rtol * row_rms(ref), what=what)


def close_sum(gpu, ref, abs_terms_sum, rtol=RTOL_EW, what=""):
    """Reductions: |gpu - ref| <= rtol * sum(|terms|)."""
    close(gpu, ref, rtol=0.0, atol=rtol * np.asarray(abs_terms_sum) + 1e-30, what=what)
