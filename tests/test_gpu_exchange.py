"""Single-GPU tests of ``pdl_exchange_merge``, the peer-memory context-parallel combine.

The real exchange runs one process per GPU.  On one GPU, ranks are emulated
by ONE cooperative launch over every rank's slices and exchange buffers (the
same kernel code: local merge, sequence-tagged stores into every rank's
buffer, bounded wait for the peers' words, merge), so no kernel waits on
another launch.
Checks:
  * bit-identical to the two-kernel path (local ``pdl_lse_merge`` to a
    (partial, LSE) block per rank, the blocks concatenated as an all-gather
    leaves them, ``pdl_lse_merge`` over the ranks), for 1/2/4/8 ranks and
    D = 64/128/256, over consecutive calls (both buffer halves, sequence
    advance), and within the output tolerance of a float64 merge of all
    ranks' partitions at once;
  * partitions past a row's live count (``lengths``) are never read;
  * the non-emulated launch (world 1, rank 0) inside a CUDA graph, replayed
    with new inputs;
  * a wait that nothing satisfies (a peer buffer no process writes) gives up
    after its timeout, sets the fault bit, leaves the output rows unwritten,
    and the context stays usable.
"""
import numpy as np
import pytest
import torch

from gpu_util import assert_out_close, requires_cuda
from paged_decode import _lib, ops, parallel

pytestmark = [pytest.mark.gpu, requires_cuda]

DEV = torch.device("cuda", 0)


def make_inputs(world, rows, parts, d, seed, empty_frac=0.2):
    g = torch.Generator(device="cpu").manual_seed(seed)
    partial = torch.randn(world, rows, parts, d, generator=g)
    lse = torch.randn(world, rows, parts, generator=g) * 3.0
    empty = torch.rand(world, rows, parts, generator=g) < empty_frac
    lse[empty] = -float("inf")
    partial[empty] = 0.0
    lse[:, 0] = -float("inf")  # one row empty on every rank
    partial[:, 0] = 0.0
    return partial.to(DEV), lse.to(DEV)


def two_kernel(partial, lse, world, rows, parts, d):
    """Local merge per rank, an all-gather's layout, merge over the ranks."""
    layout = parallel.ExchangeLayout(rows, d, world)
    gathered = torch.zeros(world * layout.block, device=DEV)
    for r in range(world):
        send_p, send_l = layout.send_views(gathered[r * layout.block:(r + 1) * layout.block])
        ops.lse_merge(ops.merge_args(partial[r], lse[r], rows=rows, parts=parts, head_dim=d,
                                     row_stride=parts * d, part_stride=d, lse_row_stride=parts,
                                     lse_part_stride=1, out_partial=send_p, out_lse=send_l), DEV)
    out = torch.empty(rows, d, dtype=torch.bfloat16, device=DEV)
    rs, ps, lrs, lps = layout.merge_strides()
    ops.lse_merge(ops.merge_args(gathered, gathered[layout.lse_offset:], rows=rows, parts=world,
                                 head_dim=d, row_stride=rs, part_stride=ps, lse_row_stride=lrs,
                                 lse_part_stride=lps, out=out), DEV)
    return out


def flat_reference(partial, lse):
    """float64 merge of all ranks' partitions of each row at once."""
    p = partial.double().cpu().numpy().transpose(1, 0, 2, 3)  # rows, world, parts, d
    l = lse.double().cpu().numpy().transpose(1, 0, 2)
    rows, d = p.shape[0], p.shape[3]
    p, l = p.reshape(rows, -1, d), l.reshape(rows, -1)
    m = l.max(axis=1, keepdims=True)
    m[~np.isfinite(m)] = 0.0
    w = np.exp(l - m)
    tot = w.sum(axis=1, keepdims=True)
    out = (w[:, :, None] * p).sum(axis=1) / np.where(tot > 0, tot, 1.0)
    return out


class Emulated:
    """Exchange buffers of `world` emulated ranks on this GPU."""

    def __init__(self, world, rows, d):
        self.world, self.rows, self.d = world, rows, d
        self.plan = ops.exchange_plan(rows, d, world, ops.sm_count(DEV), emulate=True)
        self.buffers = [torch.zeros(self.plan.buffer_bytes, dtype=torch.uint8, device=DEV)
                        for _ in range(world)]
        self.out = torch.empty(world, rows, d, dtype=torch.bfloat16, device=DEV)

    def __call__(self, partial, lse, parts, lengths=None, num_heads=0, tokens_per_split=0):
        a = ops.exchange_args(partial, lse, rows=self.rows, parts=parts, head_dim=self.d,
                              world=self.world, buffers=[b.data_ptr() for b in self.buffers],
                              out=self.out, emulate=True, lengths=lengths, num_heads=num_heads,
                              tokens_per_split=tokens_per_split)
        ops.exchange_merge(a, DEV)
        return self.out


@pytest.mark.parametrize("d", [64, 128, 256])
@pytest.mark.parametrize("world", [1, 2, 4, 8])
def test_emulated_exchange_equals_two_kernel_path(world, d):
    rows, parts = 24, 5
    ex = Emulated(world, rows, d)
    ops.read_fault(clear=True)
    for call in range(3):  # halves 1, 0, 1 of the double buffer
        partial, lse = make_inputs(world, rows, parts, d, seed=100 * world + d + call)
        got = ex(partial, lse, parts).clone()
        want = two_kernel(partial, lse, world, rows, parts, d)
        for r in range(world):
            assert torch.equal(got[r], want), f"rank {r}, call {call}"
        assert_out_close(want, flat_reference(partial, lse))
        assert got[:, 0].abs().max().item() == 0.0  # all-empty row -> 0
    assert ops.read_fault() == 0
    seq = ex.buffers[0][:ex.plan.data_offset].view(torch.int32)[:ex.plan.ctas * 4]
    assert (seq == 3).all()  # every warp advanced its sequence once per call


def test_emulated_exchange_large_rows_loop_over_units():
    """More units than resident CTAs: every warp handles several (row, slice) units."""
    world, rows, parts, d = 2, 4096, 3, 256
    ex = Emulated(world, rows, d)
    assert ex.plan.ctas * 4 < rows * 2
    partial, lse = make_inputs(world, rows, parts, d, seed=7)
    got = ex(partial, lse, parts)
    want = two_kernel(partial, lse, world, rows, parts, d)
    assert torch.equal(got[0], want) and torch.equal(got[1], want)


def test_emulated_exchange_reads_only_live_partitions():
    world, batch, heads, parts, d, tps = 4, 5, 8, 6, 128, 512
    rows = batch * heads
    g = torch.Generator(device="cpu").manual_seed(3)
    lengths = torch.randint(0, parts * tps + 1, (world, batch), generator=g, dtype=torch.int32)
    lengths[:, 1] = 0
    partial, lse = make_inputs(world, rows, parts, d, seed=11, empty_frac=0.0)
    live = (lengths + tps - 1) // tps  # [world, batch]
    dead = torch.arange(parts)[None, None, :] >= live.repeat_interleave(heads, dim=1)[:, :, None]
    clean_p, clean_l = partial.clone(), lse.clone()
    clean_l[dead.to(DEV)] = -float("inf")
    clean_p[dead.to(DEV)] = 0.0
    dirty_p, dirty_l = partial.clone(), lse.clone()
    dirty_l[dead.to(DEV)] = 50.0          # would dominate the merge if read
    dirty_p[dead.to(DEV)] = float("nan")  # would poison it if read
    ex = Emulated(world, rows, d)
    got = ex(dirty_p, dirty_l, parts, lengths=lengths.to(DEV), num_heads=heads,
             tokens_per_split=tps).clone()
    want = two_kernel(clean_p, clean_l, world, rows, parts, d)
    for r in range(world):
        assert torch.equal(got[r], want)


def test_single_rank_exchange_in_a_cuda_graph():
    """The non-emulated launch (programmatic dependent launch, rank 0 of 1),
    captured once and replayed with new inputs: the sequence advances on the
    device."""
    rows, parts, d = 64, 4, 128
    plan = ops.exchange_plan(rows, d, 1, ops.sm_count(DEV))
    buf = ops.PeerBuffer(plan.buffer_bytes, DEV)
    try:
        partial, lse = make_inputs(1, rows, parts, d, seed=21)
        out = torch.empty(rows, d, dtype=torch.bfloat16, device=DEV)
        a = ops.exchange_args(partial[0], lse[0], rows=rows, parts=parts, head_dim=d, world=1,
                              rank=0, buffers=[buf.ptr], out=out)
        stream = torch.cuda.Stream(DEV)
        stream.wait_stream(torch.cuda.current_stream(DEV))
        with torch.cuda.stream(stream):
            for _ in range(3):
                ops.exchange_merge(a, DEV)
        torch.cuda.current_stream(DEV).wait_stream(stream)
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph):
            ops.exchange_merge(a, DEV)
        for call in range(3):
            p2, l2 = make_inputs(1, rows, parts, d, seed=30 + call)
            partial.copy_(p2)
            lse.copy_(l2)
            graph.replay()
            torch.cuda.synchronize(DEV)
            assert torch.equal(out, two_kernel(partial, lse, 1, rows, parts, d)), call
        del graph
        assert ops.read_fault() == 0
    finally:
        torch.cuda.synchronize(DEV)
        buf.free()


def test_exchange_wait_gives_up_when_no_peer_publishes():
    """Rank 0 of 2 whose peer buffer no process ever writes: the bounded wait
    runs out, the fault bit is set, the rows stay unwritten, and later work on
    the same context still runs."""
    rows, parts, d = 32, 2, 64
    plan = ops.exchange_plan(rows, d, 2, ops.sm_count(DEV))
    bufs = [ops.PeerBuffer(plan.buffer_bytes, DEV) for _ in range(2)]
    try:
        partial, lse = make_inputs(1, rows, parts, d, seed=5)
        sentinel = torch.full((rows, d), 7.0, dtype=torch.bfloat16, device=DEV)
        out = sentinel.clone()
        ops.read_fault(clear=True)
        a = ops.exchange_args(partial[0], lse[0], rows=rows, parts=parts, head_dim=d, world=2,
                              rank=0, buffers=[b.ptr for b in bufs], out=out, timeout_us=20_000)
        ops.exchange_merge(a, DEV)
        torch.cuda.synchronize(DEV)
        fault = ops.read_fault(clear=True)
        assert fault & _lib.FAULT_EXCHANGE_WAIT
        assert torch.equal(out, sentinel)
    finally:
        torch.cuda.synchronize(DEV)
        for b in bufs:
            b.free()
    ex = Emulated(2, rows, d)  # the context is still usable
    partial, lse = make_inputs(2, rows, parts, d, seed=6)
    assert torch.equal(ex(partial, lse, parts)[1], two_kernel(partial, lse, 2, rows, parts, d))
    assert ops.read_fault() == 0


def test_exchange_rejects_bad_arguments():
    rows, parts, d = 8, 2, 64
    partial, lse = make_inputs(1, rows, parts, d, seed=1)
    out = torch.empty(rows, d, dtype=torch.bfloat16, device=DEV)
    buf = torch.zeros(1 << 16, dtype=torch.uint8, device=DEV)
    base = dict(rows=rows, parts=parts, head_dim=d, world=1, buffers=[buf.data_ptr()], out=out)
    with pytest.raises(RuntimeError, match="rank"):
        ops.exchange_merge(ops.exchange_args(partial, lse, rank=1, **base), DEV)
    with pytest.raises(RuntimeError, match="aligned"):
        ops.exchange_merge(ops.exchange_args(partial, lse, **{**base, "buffers": [buf.data_ptr() + 16]}), DEV)
    with pytest.raises(RuntimeError, match="timeout"):
        ops.exchange_merge(ops.exchange_args(partial, lse, timeout_us=20_000_000, **base), DEV)
    with pytest.raises(RuntimeError, match="lengths"):
        lens = torch.zeros(rows, dtype=torch.int32, device=DEV)
        ops.exchange_merge(ops.exchange_args(partial, lse, lengths=lens, num_heads=3, tokens_per_split=1,
                                             **base), DEV)
