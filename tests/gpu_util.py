"""Helpers for the GPU parity tests: device copies of seeded cases and the
tolerances of the parity contract.

Tolerances (checked against the NumPy oracle on the
same BF16 bits):
  * output: max |gpu - ref| <= 2^-7.
  * LSE:    |gpu - ref| <= 1e-5 * |ref|, with an absolute floor of
    1e-5 * 1e-3 where |ref| < 1e-3; -inf exactly where the oracle has -inf
    (empty partitions).  Where the caller passes the partition's score
    magnitude S (oracle.score_magnitudes: the largest sum_i |q_i k_i| * scale
    over its tokens), the bound is at least SCORE_ULPS * 2^-24 * (S + 1).
    Why: a partition's LSE is 1-Lipschitz in its scores, and an FP32 score
    (any FP32 dot product: the GPU's, the NumPy reference's) is rounded on
    the scale of S, not of its value; ln l adds the rounding of ex2/log2 on
    the scale of 1.  A partition of one or two tokens whose score is near 0
    therefore cannot be reproduced to 1e-5 *relative* by any FP32
    implementation; everywhere else the relative bound is what binds.
  * page addressing and partition bounds: bit-exact (checked through
    bit-identical outputs under page relocation and split re-layout).

The worst observed ratios (error / bound) of a session are kept in WORST and
printed at the end of the run (tests/conftest.py).
"""
import numpy as np
import pytest
import torch

OUT_ATOL = 2.0 ** -7
LSE_RTOL = 1e-5
LSE_FLOOR_BELOW = 1e-3
SCORE_ULPS = 8
U32 = 2.0 ** -24

# Worst (error / bound) ratios seen in this session, plus the largest
# relative LSE error where |ref| >= 1e-3 and no score allowance was needed.
WORST = {"output_abs_err": 0.0, "output_ratio": 0.0, "lse_ratio": 0.0,
         "lse_rel_err_strict": 0.0, "lse_checked": 0, "lse_needing_score_allowance": 0}

requires_cuda = pytest.mark.skipif(not torch.cuda.is_available(), reason="needs a CUDA device")


def bf16_tensor(bits, device="cuda"):
    """uint16 BF16 patterns -> torch.bfloat16 tensor with the same bits."""
    arr = np.ascontiguousarray(bits).view(np.int16)
    return torch.from_numpy(arr).to(device).view(torch.bfloat16)


def device_case(case, device="cuda"):
    return (bf16_tensor(case.q_bits, device), bf16_tensor(case.k_bits, device),
            bf16_tensor(case.v_bits, device),
            torch.from_numpy(np.ascontiguousarray(case.table)).to(device),
            torch.from_numpy(np.ascontiguousarray(case.lengths)).to(device))


def _np(x):
    return x.float().cpu().numpy() if torch.is_tensor(x) else np.asarray(x, dtype=np.float32)


def assert_out_close(actual, expected, what="output"):
    a, e = _np(actual), _np(expected)
    assert a.shape == e.shape, (a.shape, e.shape)
    assert np.isfinite(a).all(), f"{what}: non-finite values"
    err = np.abs(a - e)
    worst = float(err.max(initial=0.0))
    WORST["output_abs_err"] = max(WORST["output_abs_err"], worst)
    WORST["output_ratio"] = max(WORST["output_ratio"], worst / OUT_ATOL)
    at = np.unravel_index(np.argmax(err), err.shape) if err.size else ()
    assert worst <= OUT_ATOL, (f"{what}: max abs err {worst:.3e} > 2^-7 at {at}: "
                               f"got {a[at]}, want {e[at]}")
    return worst


def lse_bound(expected, score_mag=None):
    e = np.abs(np.asarray(expected, dtype=np.float64))
    bound = LSE_RTOL * np.maximum(e, LSE_FLOOR_BELOW)
    if score_mag is not None:
        bound = np.maximum(bound, SCORE_ULPS * U32 * (np.asarray(score_mag, np.float64) + 1.0))
    return bound


def assert_lse_close(actual, expected, what="lse", score_mag=None):
    a = _np(actual).astype(np.float64)
    e = np.asarray(_np(expected), dtype=np.float64)
    assert a.shape == e.shape, (a.shape, e.shape)
    np.testing.assert_array_equal(np.isneginf(a), np.isneginf(e), err_msg=f"{what}: -inf layout")
    fin = np.isfinite(e)
    assert np.isfinite(a[fin]).all()
    err = np.abs(a[fin] - e[fin])
    mag = None if score_mag is None else np.asarray(score_mag)[fin]
    bound = lse_bound(e[fin], mag)
    strict = LSE_RTOL * np.maximum(np.abs(e[fin]), LSE_FLOOR_BELOW)
    if err.size:
        WORST["lse_checked"] += int(err.size)
        WORST["lse_ratio"] = max(WORST["lse_ratio"], float((err / bound).max()))
        WORST["lse_needing_score_allowance"] += int((err > strict).sum())
        big = np.abs(e[fin]) >= LSE_FLOOR_BELOW
        if big.any():
            WORST["lse_rel_err_strict"] = max(WORST["lse_rel_err_strict"],
                                              float((err[big] / np.abs(e[fin][big])).max()))
    bad = err > bound
    assert not bad.any(), (f"{what}: {int(bad.sum())} LSE values outside the bound; worst "
                           f"|err| {err.max():.3e} at |ref| {np.abs(e[fin])[np.argmax(err / bound)]:.3e}")
