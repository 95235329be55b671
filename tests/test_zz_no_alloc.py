"""GPU test of ``pdl_paged_decode_static_scratch``, the allocation-free entry point.

Callers such as an engine that has handed nearly all free HBM to its KV page
pool, or a host that must not call cudaMalloc/cudaFree on its decode path
(they can synchronise the device), cannot provide a split workspace.  This
entry point keeps the workspace in a 4 MiB device array inside the library.
The test calls it through the C ABI twice in a row -- with different lengths,
so stale contents of the shared array would show -- and requires each result
to be bit-identical to ``pdl_paged_decode`` given a caller-allocated
workspace (same kernels, same plan), and the last one to match the oracle.  It also checks that a request larger
than the array is rejected with a clear error before anything is launched.

This file is named to be collected last, so a run that stops at the first
failure has already run every other test.
"""
import ctypes

import pytest
import torch

import cases
import oracle
from gpu_util import assert_out_close, device_case, requires_cuda
from paged_decode import _lib, ops

pytestmark = [pytest.mark.gpu, requires_cuda]


def _call(entry, args, device):
    lib = _lib.load()
    with torch.cuda.device(device):
        stream = torch.cuda.current_stream(device).cuda_stream
        return getattr(lib, entry)(ctypes.byref(args), stream)


def _with_workspace(q, k, v, table, lens, splits, tokens, flags):
    b, hq, d = q.shape
    out = torch.empty(b, hq, d, dtype=torch.bfloat16, device=q.device)
    partial = torch.empty(b, hq, splits, d, device=q.device)
    lse = torch.empty(b, hq, splits, device=q.device)
    args = ops.decode_args(q, k, v, table, lens, scale=d ** -0.5, tokens_per_split=tokens,
                           splits=splits, protocol=ops.PROTOCOL_LSE, flags=flags, out=out,
                           partial=partial, lse=lse)
    assert _call("pdl_paged_decode", args, q.device) == 0
    return out


def _static_scratch(q, k, v, table, lens, splits, tokens, flags):
    out = torch.full(q.shape, float("nan"), dtype=torch.bfloat16, device=q.device)
    args = ops.decode_args(q, k, v, table, lens, scale=q.shape[-1] ** -0.5,
                           tokens_per_split=tokens, splits=splits, protocol=ops.PROTOCOL_LSE,
                           flags=flags, out=out)
    status = _call("pdl_paged_decode_static_scratch", args, q.device)
    assert status == 0, _lib.status_text(status)
    return out


# (lengths of two calls in a row, splits, tokens per split, flags).  The same
# kernels run with the same plan on both paths, so outputs must be identical
# bits.  The second call of each pair reads a shared array that still holds the
# first call's partitions: PDL_FLAG_SKIP_EMPTY after a longer call leaves them
# there, and only the live partitions may be merged.
CALLS = [
    (([1500, 0, 257, 2048], [3, 2048, 0, 1025]), 4, 512, 0),
    (([2048, 2048, 2048, 2048], [1, 700, 0, 513]), 4, 512, ops.FLAG_SKIP_EMPTY),
    (([2048, 17, 0, 999], [5, 2048, 1024, 0]), 1, 0, 0),
    (([2048, 17, 0, 999], [5, 2048, 1024, 0]), 1, 2048, ops.FLAG_DIRECT_SINGLE),
]


@pytest.mark.parametrize("lengths,splits,tokens,flags", CALLS)
def test_static_scratch_matches_workspace_entry_point_on_two_calls(lengths, splits, tokens,
                                                                   flags):
    case = cases.make_case(list(lengths[0]), 8, 2, 128, seed=21, capacity=2048)
    q, k, v, table, lens = device_case(case)
    for values in lengths:
        lens.copy_(torch.tensor(values, dtype=torch.int32, device="cuda"))
        expected = _with_workspace(q, k, v, table, lens, splits, tokens, flags)
        out = _static_scratch(q, k, v, table, lens, splits, tokens, flags)
        torch.cuda.synchronize()
        assert torch.equal(out, expected), "static-scratch output differs from the workspace path"
    assert_out_close(out, oracle.dense_reference(case.q, case.k, case.v, case.table,
                                                 lens.cpu().numpy()), "static-scratch output")


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
