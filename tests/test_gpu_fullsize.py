"""Parity at the BASELINE configurations' full sizes.

The NumPy oracle cannot gather a 524,288-token row in reasonable time, so
at full size the checks are:
  * sampled rows of configs 2-5 (first/last rows, config 4's longest, median
    and zero-length rows, both 524k-token rows of config 5; config 3 over its
    batch and context grid) against an FP64 reference evaluated on the GPU in
    64k-token chunks (oracle test infrastructure), within the output
    tolerance of the parity tests, and every partition's LSE of those rows
    against an FP64 logsumexp within the LSE tolerance;
  * size-independent properties, bit for bit: relocating every physical page
    (and rewriting the block table to match) leaves every output bit
    unchanged, and dynamic scheduling gives the bits of static scheduling.
The split plan is the bench's: the reference plan's 2 partitions for config 2,
this library's B200 plan otherwise (launched as launch_partitioning says: config 3 at
B=8 and 32 with partitions that follow each row's length).
"""
import pytest
import torch

from gpu_util import assert_lse_close, assert_out_close, requires_cuda
from oracle.torch_reference import chunked_partition_lse, chunked_reference_rows
from paged_decode import ops
from paged_decode.matched_splitkv import allocate_matched_resources, matched_decode
from paged_decode.splitkv_plan import launch_partitioning, make_b200_plan, make_splitkv_plan
from paged_decode.workloads import make_workload

pytestmark = [pytest.mark.gpu, requires_cuda]

DEV = torch.device("cuda", 0)


def plan_for(name, spec):
    sms = ops.sm_count(DEV)
    if name == "cfg2":
        return make_splitkv_plan(spec, sms, num_splits=2)
    return make_b200_plan(spec, sms)


def sample_rows(w):
    lens = w.lengths.cpu()
    b = lens.numel()
    rows = {0, b - 1}
    if w.name == "cfg4":
        order = torch.argsort(lens)
        rows |= {int(order[-1]), int(order[b // 2]), int((lens == 0).nonzero()[0])}
    return sorted(rows)


@pytest.fixture(autouse=True)
def _free_memory():
    yield
    torch.cuda.empty_cache()


@pytest.mark.parametrize("name,batch,context", [
    ("cfg2", None, None), ("cfg4", None, None), ("cfg5", None, None),
    # Config 3's grid: B in {1, 8, 32, 128, 256}, contexts 528 and 2064.
    ("cfg3", 1, 528), ("cfg3", 1, 2064), ("cfg3", 8, 528), ("cfg3", 8, 2064),
    ("cfg3", 32, 528), ("cfg3", 32, 2064), ("cfg3", 128, 2064), ("cfg3", 256, 528),
    ("cfg3", 256, 2064)])
def test_full_size_rows_and_partition_lse_match_fp64_reference(name, batch, context):
    """Sampled rows' outputs (max-abs 2^-7) and every partition's LSE of those
    rows (1e-5 relative; see gpu_util) against FP64 references on the GPU."""
    w = make_workload(name, device=DEV, batch=batch, context=context)
    plan = plan_for(name, w.spec)
    res = allocate_matched_resources(w.spec, DEV, plan=plan)
    out = matched_decode(w.q, w.k, w.v, w.table, w.lengths, resources=res, scale=w.scale)
    rows = sample_rows(w)
    want = chunked_reference_rows(w.q, w.k, w.v, w.table, w.lengths, rows, scale=w.scale)
    assert_out_close(out[rows], want.float(), what=f"{name} rows {rows}")
    assert torch.isfinite(out.float()).all()
    tokens, bounds = launch_partitioning(plan)
    lse, mag = chunked_partition_lse(w.q, w.k, w.table, w.lengths, rows, tokens, plan.splits,
                                     scale=w.scale, balanced=bool(bounds))
    assert_lse_close(res.lse[rows], lse.cpu().numpy(), what=f"{name} lse rows {rows}",
                     score_mag=mag.cpu().numpy())


@pytest.mark.parametrize("name", ["cfg4", "cfg5"])
def test_full_size_page_relocation_and_scheduling_are_bit_exact(name):
    w = make_workload(name, device=DEV)
    plan = plan_for(name, w.spec)
    res = allocate_matched_resources(w.spec, DEV, plan=plan)
    base = matched_decode(w.q, w.k, w.v, w.table, w.lengths, resources=res,
                          scale=w.scale).clone()

    # Every physical page moves to a new index; the table follows it.
    pages = w.k.shape[0]
    perm = torch.randperm(pages, generator=torch.Generator(device=DEV).manual_seed(3),
                          device=DEV)
    k2 = torch.empty_like(w.k)
    k2[perm] = w.k
    v2 = torch.empty_like(w.v)
    v2[perm] = w.v
    t2 = torch.where(w.table >= 0, perm[w.table.clamp(min=0).long()].to(torch.int32), w.table)
    res2 = allocate_matched_resources(w.spec, DEV, plan=plan)
    moved = matched_decode(w.q, k2, v2, t2, w.lengths, resources=res2, scale=w.scale)
    assert torch.equal(moved, base)
    del k2, v2

    # Static round-robin scheduling (no counters) against the dynamic default.
    out = torch.empty_like(res.out)
    partial, lse = torch.empty_like(res.partials), torch.empty_like(res.lse)
    tokens, bounds = launch_partitioning(plan)
    args = ops.decode_args(w.q, w.k, w.v, w.table, w.lengths, scale=w.scale,
                           tokens_per_split=tokens, splits=plan.splits, flags=bounds,
                           protocol=ops.PROTOCOL_LSE, out=out, partial=partial, lse=lse)
    ops.paged_decode(args, DEV)
    assert torch.equal(out, base)
    assert ops.read_fault() == 0
