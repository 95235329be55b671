"""GPU test of ``pdl_paged_decode_static_scratch``, the allocation-free entry point.

Callers such as an engine that has handed nearly all free HBM to its KV page
pool, or a host that must not call cudaMalloc/cudaFree on its decode path
(they can synchronise the device), cannot provide a split workspace.  This
entry point keeps the workspace in a 4 MiB device array inside the library.
The test calls it through the C ABI twice in a row -- with different lengths,
so stale contents of the shared array would show -- and compares each result
with ``pdl_paged_decode`` given a caller-allocated workspace, within the
output tolerance of the parity tests.  It also checks that a request larger
than the array is rejected with a clear error before anything is launched.

This file is named to be collected last, so a run that stops at the first
failure has already run every other test.
"""
import ctypes

import pytest
import torch

import cases
from gpu_util import assert_out_close, device_case, requires_cuda
from paged_decode import _lib, ops

pytestmark = [pytest.mark.gpu, requires_cuda]


def _call(entry, args, device):
    lib = _lib.load()
    with torch.cuda.device(device):
        stream = torch.cuda.current_stream(device).cuda_stream
        return getattr(lib, entry)(ctypes.byref(args), stream)


def _with_workspace(q, k, v, table, lens, splits, tokens):
    b, hq, d = q.shape
    out = torch.empty(b, hq, d, dtype=torch.bfloat16, device=q.device)
    partial = torch.empty(b, hq, splits, d, device=q.device)
    lse = torch.empty(b, hq, splits, device=q.device)
    args = ops.decode_args(q, k, v, table, lens, scale=d ** -0.5, tokens_per_split=tokens,
                           splits=splits, protocol=ops.PROTOCOL_LSE, out=out, partial=partial,
                           lse=lse)
    assert _call("pdl_paged_decode", args, q.device) == 0
    return out


def test_static_scratch_matches_workspace_entry_point_on_two_calls():
    case = cases.make_case([1500, 0, 257, 2048], 8, 2, 128, seed=21, capacity=2048)
    q, k, v, table, lens = device_case(case)
    splits, tokens = 4, 512
    for lengths in ([1500, 0, 257, 2048], [3, 2048, 0, 1025]):
        lens.copy_(torch.tensor(lengths, dtype=torch.int32, device="cuda"))
        expected = _with_workspace(q, k, v, table, lens, splits, tokens)
        out = torch.full_like(expected, float("nan"))
        args = ops.decode_args(q, k, v, table, lens, scale=128 ** -0.5, tokens_per_split=tokens,
                               splits=splits, protocol=ops.PROTOCOL_LSE, out=out)
        status = _call("pdl_paged_decode_static_scratch", args, q.device)
        assert status == 0, _lib.status_text(status)
        torch.cuda.synchronize()
        assert_out_close(out, expected, "static-scratch output")


def test_static_scratch_rejects_requests_beyond_its_size():
    # 16 rows * 32 heads * 16 splits * (128 + 1) floats = 4,227,072 bytes > 4 MiB.
    case = cases.make_case([4096] * 16, 32, 4, 128, seed=2, capacity=4096)
    q, k, v, table, lens = device_case(case)
    out = torch.zeros(16, 32, 128, dtype=torch.bfloat16, device="cuda")
    args = ops.decode_args(q, k, v, table, lens, scale=128 ** -0.5, tokens_per_split=256,
                           splits=16, protocol=ops.PROTOCOL_LSE, out=out)
    status = _call("pdl_paged_decode_static_scratch", args, q.device)
    assert status == 4  # PDL_ERR_WORKSPACE
    message = _lib.load().pdl_last_error().decode()
    assert "static scratch" in message and str(_lib.STATIC_SCRATCH_BYTES) in message
    torch.cuda.synchronize()
    assert not out.any()  # nothing was launched
