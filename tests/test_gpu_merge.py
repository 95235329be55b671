"""The stable LSE merge (``pdl_lse_merge``) around its shared-memory staging
boundary: the rows of up to 48 partitions arrive in one round trip, more in
chunks of 48.  Partition counts on both sides of every chunk edge must give
the float64 merge of the same inputs: outputs within the library's 2^-7, the
FP32 merged partial within 1e-5 of the largest value, the merged LSE within
1e-5 relative."""
import numpy as np
import pytest
import torch

from gpu_util import assert_out_close, requires_cuda
from paged_decode import ops

pytestmark = [pytest.mark.gpu, requires_cuda]

DEV = torch.device("cuda", 0)


def reference(partial, lse):
    p, l = partial.double().cpu().numpy(), lse.double().cpu().numpy()
    m = l.max(axis=1, keepdims=True)
    m[~np.isfinite(m)] = 0.0
    w = np.exp(l - m)
    tot = w.sum(axis=1)
    out = (w[:, :, None] * p).sum(axis=1) / np.where(tot > 0, tot, 1.0)[:, None]
    merged = np.where(tot > 0, np.log(np.where(tot > 0, tot, 1.0)) + m[:, 0], -np.inf)
    return out, merged


@pytest.mark.parametrize("d", [64, 128, 256])
@pytest.mark.parametrize("parts", [1, 31, 32, 47, 48, 49, 96, 97, 130])
def test_merge_across_staging_chunks(parts, d):
    rows = 24
    g = torch.Generator(device="cpu").manual_seed(parts * 1000 + d)
    partial = torch.randn(rows, parts, d, generator=g)
    lse = torch.randn(rows, parts, generator=g) * 3.0
    empty = torch.rand(rows, parts, generator=g) < 0.2
    lse[empty] = -float("inf")
    partial[empty] = 0.0
    lse[0] = -float("inf")  # an empty row
    partial[0] = 0.0
    lse[1, -1] = 30.0       # one dominant partition, the last one
    want_out, want_lse = reference(partial, lse)
    partial, lse = partial.to(DEV), lse.to(DEV)
    out = torch.empty(rows, d, dtype=torch.bfloat16, device=DEV)
    out_partial = torch.full((rows, d), float("nan"), device=DEV)
    out_lse = torch.full((rows,), float("nan"), device=DEV)
    ops.lse_merge(ops.merge_args(partial, lse, rows=rows, parts=parts, head_dim=d,
                                 row_stride=parts * d, part_stride=d, lse_row_stride=parts,
                                 lse_part_stride=1, out=out, out_partial=out_partial,
                                 out_lse=out_lse), DEV)
    torch.cuda.synchronize()
    assert ops.read_fault() == 0
    assert_out_close(out, want_out)
    got = out_partial.double().cpu().numpy()
    assert np.abs(got - want_out).max() <= 1e-5 * max(1.0, np.abs(want_out).max())
    got_lse = out_lse.double().cpu().numpy()
    assert np.isneginf(got_lse[0]) and np.isneginf(want_lse[0])
    fin = np.isfinite(want_lse)
    assert (np.abs(got_lse[fin] - want_lse[fin]) <= 1e-5 * np.maximum(np.abs(want_lse[fin]), 1.0)).all()
