"""CPU tests of the multi-GPU host logic, with world-size-2 gloo process groups.

The GPU kernels are replaced by the oracle on each rank; what is under test is
the product's sharding plans, the device-side local-length rule, the exchange
buffer layout and the collective itself (``parallel.exchange``), and that
merging the exchanged (partial, LSE) pairs reproduces the unsharded result.
"""
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

import cases
import oracle
from paged_decode import parallel
from paged_decode.workloads import cfg4_lengths


def free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


# ---------------------------------------------------------------- planning
@pytest.mark.parametrize("world", [1, 2, 4, 8])
def test_batch_shards_cover_every_row_once_and_balance_tokens(world):
    lengths = cfg4_lengths()
    shards = parallel.batch_shards(lengths, world)
    rows = sorted(r for s in shards for r in s)
    assert rows == list(range(len(lengths)))
    loads = [int(sum(lengths[s])) for s in shards]
    assert max(loads) - min(loads) <= int(lengths.max())
    assert parallel.batch_shards(lengths, world) == shards  # deterministic
    contiguous = parallel.batch_shards(lengths, world, balanced=False)
    assert sorted(r for s in contiguous for r in s) == list(range(len(lengths)))


def test_head_and_context_shards():
    assert parallel.head_shard(64, 8, 4, 1) == (2, 4, 16, 32)
    with pytest.raises(ValueError):
        parallel.head_shard(32, 8, 3, 0)
    spans = [parallel.context_shard(2048, 8, r) for r in range(8)]
    assert spans[0] == (0, 256) and spans[-1] == (1792, 2048)
    spans = [parallel.context_shard(10, 4, r) for r in range(4)]
    assert spans == [(0, 3), (3, 6), (6, 9), (9, 10)]
    assert parallel.tokens_per_rank(10, 4) == 768


def test_local_lengths_rule():
    lengths = torch.tensor([0, 1, 767, 768, 769, 2000, 2560], dtype=torch.int32)
    per = parallel.tokens_per_rank(10, 4)
    got = [parallel.local_lengths(lengths, r, per).tolist() for r in range(4)]
    for i, n in enumerate(lengths.tolist()):
        assert sum(g[i] for g in got) == n
        for r in range(4):
            assert got[r][i] == min(max(n - r * per, 0), per)


def test_exchange_layout_alignment():
    for rows in (1, 3, 4, 128):
        lay = parallel.ExchangeLayout(rows, 128, 4)
        assert lay.block % 4 == 0 and lay.lse_offset % 4 == 0
        gathered = torch.arange(4 * lay.block, dtype=torch.float32)
        p, l = lay.gathered_views(gathered)
        assert p.shape == (4, rows, 128) and l.shape == (4, rows)
        assert float(p[2, 0, 0]) == 2 * lay.block
        assert float(l[1, 0]) == lay.block + lay.lse_offset


# ---------------------------------------------------------------- collectives
def merged_partial(partials, lse):
    """(partial, LSE) of a set of partitions -- the local merge, on the oracle's data."""
    lse = lse.astype(np.float64)
    top = lse.max(axis=-1, keepdims=True)
    top = np.where(np.isneginf(top), 0.0, top)
    total = np.exp(lse - top).sum(axis=-1)
    with np.errstate(divide="ignore"):
        merged = np.where(total > 0, np.log(np.where(total > 0, total, 1)) + top[..., 0], -np.inf)
    weights = np.exp(lse - merged[..., None])
    weights = np.where(np.isfinite(weights), weights, 0.0)
    return (weights[..., None] * partials).sum(axis=-2).astype(np.float32), merged.astype(np.float32)


def _context_rank(rank, world, port, result):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        case = cases.make_case([1700, 0, 513, 2048], 8, 2, 64, seed=31, capacity=2048)
        q, k, v, table, lengths = case.arrays()
        per = parallel.tokens_per_rank(table.shape[1], world)
        lo, hi = parallel.context_shard(table.shape[1], world, rank)
        local_table = np.full((table.shape[0], per // 256), -1, np.int32)
        local_table[:, :hi - lo] = table[:, lo:hi]
        local_len = parallel.local_lengths(torch.from_numpy(lengths), rank, per).numpy()
        # The oracle plays the GPU: local partitions, then the local merge.
        partials, lse = oracle.normalized_partitions(q, k, v, local_table, local_len, 256, per // 256)
        part, part_lse = merged_partial(partials, lse)
        rows = q.shape[0] * q.shape[1]
        layout = parallel.ExchangeLayout(rows, q.shape[2], world)
        send = torch.zeros(layout.block)
        send_p, send_l = layout.send_views(send)
        send_p.copy_(torch.from_numpy(part.reshape(rows, -1)))
        send_l.copy_(torch.from_numpy(part_lse.reshape(rows)))
        gathered = torch.empty(world * layout.block)
        parallel.exchange(send, gathered)
        gp, gl = layout.gathered_views(gathered)
        out = oracle.lse_merge(gp.permute(1, 0, 2).numpy(), gl.t().numpy())
        expected = oracle.dense_reference(*case.arrays()).reshape(rows, -1)
        result[rank] = float(np.abs(out - expected).max())
    finally:
        dist.destroy_process_group()


def test_context_parallel_exchange_reproduces_unsharded_result():
    world = 2
    manager = mp.get_context("spawn").Manager()
    result = manager.dict()
    mp.start_processes(_context_rank, args=(world, free_port(), result), nprocs=world,
                       start_method="spawn")
    assert sorted(result.keys()) == [0, 1]
    assert max(result.values()) < 1e-5


def _batch_rank(rank, world, port, result):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        case = cases.make_case([900, 10, 0, 2048, 300, 1500], 4, 2, 64, seed=4, capacity=2048)
        q, k, v, table, lengths = case.arrays()
        rows = parallel.batch_shards(lengths, world)[rank]
        mine = oracle.dense_reference(q[rows], k, v, table[rows], lengths[rows])
        gathered = [None] * world
        dist.all_gather_object(gathered, (rows, mine))
        full = np.zeros_like(q)
        for r_rows, r_out in gathered:
            full[r_rows] = r_out
        result[rank] = float(np.abs(full - oracle.dense_reference(*case.arrays())).max())
    finally:
        dist.destroy_process_group()


def test_batch_sharding_reassembles_unsharded_result():
    world = 2
    manager = mp.get_context("spawn").Manager()
    result = manager.dict()
    mp.start_processes(_batch_rank, args=(world, free_port(), result), nprocs=world,
                       start_method="spawn")
    assert sorted(result.keys()) == [0, 1] and max(result.values()) == 0.0


def _failing_rank(rank, world, port, result):
    """Rank 1 raises before the collective; rank 0 must see an error, not hang."""
    import datetime
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=5))
    try:
        if rank == 1:
            result[rank] = "raised"
            raise RuntimeError("injected host-side failure before the exchange")
        send = torch.zeros(8)
        gathered = torch.empty(16)
        try:
            parallel.exchange(send, gathered)
            result[rank] = "completed"
        except Exception as exc:  # gloo reports the lost peer or the timeout
            result[rank] = f"error: {type(exc).__name__}"
    finally:
        try:
            dist.destroy_process_group()
        except Exception:
            pass


def test_exchange_fails_instead_of_hanging_when_a_rank_dies():
    world = 2
    manager = mp.get_context("spawn").Manager()
    result = manager.dict()
    with pytest.raises(Exception):
        mp.start_processes(_failing_rank, args=(world, free_port(), result), nprocs=world,
                           start_method="spawn")
    assert result.get(1) == "raised"
    assert str(result.get(0, "")).startswith("error")


def _handles_rank(rank, world, port, result):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        result[rank] = parallel.share_handles(bytes([rank + 1]) * 64, 32)
    finally:
        dist.destroy_process_group()


def test_peer_exchange_handles_reach_every_rank():
    """The set-up collective of the p2p exchange: every rank learns every
    rank's IPC handle and planned grid, in rank order."""
    world = 2
    manager = mp.get_context("spawn").Manager()
    result = manager.dict()
    mp.start_processes(_handles_rank, args=(world, free_port(), result), nprocs=world,
                       start_method="spawn")
    expect = [(bytes([r + 1]) * 64, 32) for r in range(world)]
    assert result[0] == expect and result[1] == expect
    with pytest.raises(ValueError):
        parallel.share_handles(b"short", 1)


def test_shard_batch_pool_keeps_each_rows_pages():
    """A rank's compact pool holds exactly its rows' live pages, in order, and
    its table addresses them; padding stays -1."""
    gen = torch.Generator().manual_seed(5)
    lengths = torch.tensor([0, 700, 256, 1, 1024, 300], dtype=torch.int32)
    width, pages = 4, 6 * 4
    table = torch.randperm(pages, generator=gen).view(6, width).to(torch.int32)
    k = torch.randn(pages, 256, 2, 8, generator=gen)
    v = torch.randn(pages, 256, 2, 8, generator=gen)
    for rows in ([1, 4], [0, 2, 5], [3]):
        kl, vl, tl, ll = parallel.shard_batch_pool(k, v, table, lengths, rows)
        assert torch.equal(ll, lengths[rows]) and tl.shape == (len(rows), width)
        for i, row in enumerate(rows):
            live = -(-int(lengths[row]) // 256)
            for j in range(width):
                if j < live:
                    assert torch.equal(kl[tl[i, j]], k[table[row, j]])
                    assert torch.equal(vl[tl[i, j]], v[table[row, j]])
                else:
                    assert int(tl[i, j]) == -1
