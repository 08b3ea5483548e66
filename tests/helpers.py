"""Comparison helpers shared by the parity tests."""
import numpy as np


def matmul_rel_err(got, ref) -> float:
    """Max relative error of a matmul result: max |got - ref| / max |ref|."""
    got = np.asarray(got, np.float64)
    ref = np.asarray(ref, np.float64)
    scale = max(float(np.max(np.abs(ref))) if ref.size else 0.0, 1e-30)
    return float(np.max(np.abs(got - ref))) / scale if ref.size else 0.0


def assert_matmul_close(got, ref, absdot=None, tol=1e-3, elem_tol=1e-4):
    """The north-star gate: max relative error <= 1e-3 (F32 accumulate).
    With `absdot` (= |W| @ |x|, the sum of |terms| per output) each element
    must also agree within elem_tol * absdot + 1e-6, i.e. reorder error."""
    got = np.asarray(got)
    ref = np.asarray(ref)
    assert got.shape == ref.shape, (got.shape, ref.shape)
    assert np.all(np.isfinite(got)), "non-finite device output"
    err = matmul_rel_err(got, ref)
    assert err <= tol, f"max relative error {err:.3e} > {tol}"
    if absdot is not None:
        bound = elem_tol * np.asarray(absdot, np.float64) + 1e-6
        diff = np.abs(got.astype(np.float64) - ref.astype(np.float64))
        bad = diff > bound
        assert not bad.any(), f"{int(bad.sum())} elements beyond reorder bound; worst {float(diff.max()):.3e}"


def bits(a):
    return np.ascontiguousarray(a, np.float32).view(np.uint32)
