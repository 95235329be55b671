"""Helpers for the GPU parity tests: device copies of seeded cases and the
tolerances of the parity contract.

Tolerances (checked against the NumPy oracle on the
same BF16 bits):
  * output: |gpu - ref| <= 2^-7 + 2^-8 * |ref|  -- max-abs 2^-7, plus the
    half-ulp rounding of the BF16 output itself for |ref| > 1;
  * LSE:    |gpu - ref| <= 1e-5 * max(1, |ref|), and -inf exactly where the
    oracle has -inf (empty partitions);
  * page addressing and partition bounds: bit-exact (checked through
    bit-identical outputs under page relocation and split re-layout).
"""
import numpy as np
import pytest
import torch

OUT_ATOL = 2.0 ** -7
OUT_RTOL = 2.0 ** -8
LSE_RTOL = 1e-5

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


def assert_out_close(actual, expected, what="output"):
    a = actual.float().cpu().numpy() if torch.is_tensor(actual) else np.asarray(actual)
    e = expected.float().cpu().numpy() if torch.is_tensor(expected) else np.asarray(expected)
    assert a.shape == e.shape, (a.shape, e.shape)
    assert np.isfinite(a).all(), f"{what}: non-finite values"
    err = np.abs(a - e)
    bound = OUT_ATOL + OUT_RTOL * np.abs(e)
    worst = np.unravel_index(np.argmax(err - bound), err.shape)
    assert (err <= bound).all(), (f"{what}: max abs err {err.max():.3e}; worst at {worst}: "
                                  f"got {a[worst]}, want {e[worst]}")
    return float(err.max())


def assert_lse_close(actual, expected, what="lse"):
    a = actual.float().cpu().numpy() if torch.is_tensor(actual) else np.asarray(actual)
    e = np.asarray(expected, dtype=np.float32)
    assert a.shape == e.shape, (a.shape, e.shape)
    np.testing.assert_array_equal(np.isneginf(a), np.isneginf(e), err_msg=f"{what}: -inf layout")
    fin = np.isfinite(e)
    assert np.isfinite(a[fin]).all()
    err = np.abs(a[fin] - e[fin])
    bound = LSE_RTOL * np.maximum(1.0, np.abs(e[fin]))
    assert (err <= bound).all(), f"{what}: max rel err {(err / np.maximum(1, np.abs(e[fin]))).max():.3e}"
