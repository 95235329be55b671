"""Multi-GPU paged decode: one process per GPU, NCCL through torch.distributed.

Three ways to spread one decode step over N GPUs of a node:

* batch sharding -- rows are independent; each rank owns a subset of rows
  (token-balanced, decided on the host before capture) together with their
  pages.  No collective on the data path.
* KV-head sharding -- each rank owns KV heads [r*Hkv/N, (r+1)*Hkv/N) and the
  query heads that read them, with a head-sliced page pool
  [P, 256, Hkv/N, D].  No collective; the output stays head-sharded, as a
  tensor-parallel output projection expects.
* context parallel -- for very long rows, rank r owns the pages
  [r*W/N, (r+1)*W/N) of every row (page aligned).  Each rank decodes its token
  range to a normalised FP32 partial + LSE per (row, head); those
  (rows*(D+1) floats per rank) are exchanged and every rank runs the stable
  LSE merge over the N ranks.  The exchange is either one NCCL all-gather
  between a local and a global merge kernel, or (``exchange="p2p"``) one
  kernel that stores the local merge into every peer's buffer over NVLink
  and merges after a bounded flag wait (``PeerExchange``).

The reference has no multi-GPU attention path; the planning functions are
pure (no CUDA) so CPU process groups (gloo) can test them.
"""
import math

import torch
import torch.distributed as dist

from .spec import DecodeSpec, PAGE_SIZE


# ---------------------------------------------------------------- planning
def batch_shards(lengths, world, balanced=True):
    """Rows of each rank.

    balanced: longest-first greedy on live tokens (ties to the lowest rank), so
    variable-length batches give every GPU about the same KV bytes; otherwise
    contiguous, equally sized row ranges.  Each rank's rows are sorted.
    """
    lengths = [int(x) for x in lengths]
    if not balanced:
        bounds = [round(r * len(lengths) / world) for r in range(world + 1)]
        return [list(range(bounds[r], bounds[r + 1])) for r in range(world)]
    load = [0] * world
    shards = [[] for _ in range(world)]
    for row in sorted(range(len(lengths)), key=lambda i: (-lengths[i], i)):
        rank = min(range(world), key=lambda r: (load[r], r))
        shards[rank].append(row)
        load[rank] += lengths[row]
    return [sorted(s) for s in shards]


def head_shard(num_heads, num_kv_heads, world, rank):
    """(kv_lo, kv_hi, q_lo, q_hi) owned by `rank`; KV heads must split evenly."""
    if num_kv_heads % world:
        raise ValueError("KV-head sharding needs num_kv_heads divisible by the world size")
    per = num_kv_heads // world
    group = num_heads // num_kv_heads
    return rank * per, (rank + 1) * per, rank * per * group, (rank + 1) * per * group


def context_shard(table_width, world, rank):
    """Page columns [lo, hi) of the block table owned by `rank` (page aligned)."""
    per = -(-table_width // world)
    lo = min(rank * per, table_width)
    return lo, min(lo + per, table_width)


def tokens_per_rank(table_width, world):
    return -(-table_width // world) * PAGE_SIZE


def local_lengths(lengths, rank, per_rank_tokens, out=None):
    """Tokens of each row that fall in `rank`'s context range (device op, graph-safe)."""
    if out is None:
        out = torch.empty_like(lengths)
    torch.sub(lengths, rank * per_rank_tokens, out=out)
    return out.clamp_(0, per_rank_tokens)


class ExchangeLayout:
    """Per-rank block of the context-parallel exchange: partial [rows, D], then
    LSE [rows] padded to 4 floats, so every partial row of every rank starts on
    a 16-byte boundary in the gathered buffer [world, block]."""

    def __init__(self, rows, head_dim, world):
        self.rows, self.head_dim, self.world = rows, head_dim, world
        self.lse_offset = rows * head_dim
        self.block = self.lse_offset + 4 * (-(-rows // 4))

    def send_views(self, send):
        return (send[:self.lse_offset].view(self.rows, self.head_dim),
                send[self.lse_offset:self.lse_offset + self.rows])

    def gathered_views(self, gathered):
        g = gathered.view(self.world, self.block)
        return (g[:, :self.lse_offset].reshape(self.world, self.rows, self.head_dim),
                g[:, self.lse_offset:self.lse_offset + self.rows])

    def merge_strides(self):
        """(row_stride, part_stride, lse_row_stride, lse_part_stride) of the gathered buffer."""
        return self.head_dim, self.block, 1, self.block


def exchange(send, gathered, group=None):
    """The one collective of context parallelism: all-gather every rank's block."""
    dist.all_gather_into_tensor(gathered, send, group=group)


def share_handles(handle, ctas, group=None, device=None):
    """All-gather every rank's (64-byte IPC handle, planned CTA count).

    Travels as one uint8 tensor per rank: on ``device`` for NCCL groups, on
    the CPU otherwise.  Returns ``[(handle bytes, ctas)]`` indexed by rank.
    """
    if len(handle) != 64:
        raise ValueError("CUDA IPC handles are 64 bytes")
    world = dist.get_world_size(group)
    on = torch.device(device) if dist.get_backend(group) == "nccl" else torch.device("cpu")
    mine = torch.tensor(list(handle) + list(int(ctas).to_bytes(4, "little")),
                        dtype=torch.uint8, device=on)
    every = torch.empty(world * mine.numel(), dtype=torch.uint8, device=on)
    dist.all_gather_into_tensor(every, mine, group=group)
    rows = every.view(world, -1).cpu().tolist()
    return [(bytes(r[:64]), int.from_bytes(bytes(r[64:]), "little")) for r in rows]


# ---------------------------------------------------------------- GPU decoders
class PeerExchange:
    """Exchange buffers of a process group for ``pdl_exchange_merge``.

    Every rank creates one zeroed buffer (``PeerBuffer``) sized by
    ``pdl_exchange_plan``; the 64-byte CUDA IPC handles and the planned CTA
    count are all-gathered over ``group`` (on the GPU for NCCL groups), every
    rank maps the others' buffers, and a barrier makes sure all mappings
    exist before the first exchange.  ``ptrs[q]`` is rank q's buffer as seen
    from this process.  Call ``close`` on every rank (it synchronises).
    """

    def __init__(self, rows, head_dim, device, group=None):
        from . import ops
        self.ops = ops
        self.group = group
        self.device = torch.device(device)
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        self.plan = ops.exchange_plan(rows, head_dim, self.world, ops.sm_count(self.device))
        self.own = ops.PeerBuffer(self.plan.buffer_bytes, self.device)
        try:
            shared = share_handles(self.own.handle, self.plan.ctas, group, self.device)
        except Exception:
            self.own.free()
            raise
        ctas = [c for _, c in shared]
        if len(set(ctas)) != 1:
            self.own.free()
            raise RuntimeError(f"ranks planned different exchange grids {ctas}; "
                               "context parallelism needs identical GPUs")
        self.ptrs = []
        try:
            for q in range(self.world):
                self.ptrs.append(self.own.ptr if q == self.rank else
                                 ops.open_peer_buffer(shared[q][0], self.device))
        except Exception:
            self._release()
            raise
        dist.barrier(group)

    def _release(self):
        for q, ptr in enumerate(self.ptrs):
            if q != self.rank:
                self.ops.close_peer_buffer(ptr, self.device)
        self.ptrs = []
        self.own.free()

    def close(self):
        """Unmap the peers' buffers and free this rank's (after every rank is done)."""
        if self.own.ptr is None:
            return
        torch.cuda.synchronize(self.device)
        dist.barrier(self.group)
        for q, ptr in enumerate(self.ptrs):
            if q != self.rank:
                self.ops.close_peer_buffer(ptr, self.device)
        self.ptrs = []
        dist.barrier(self.group)
        self.own.free()


class ContextParallelDecode:
    """Context-parallel decode of a long-row batch across the ranks of `group`.

    Each rank holds only its page range: ``k_local``/``v_local`` pools and a
    local block table of ``tokens_per_rank / 256`` columns whose column j is
    the row's page ``context_shard(...)[0] + j``.  Global lengths come in;
    local lengths are derived on the device.  All buffers are allocated here,
    so the call itself (partition, local merge, all-gather, merge) can be
    captured in a CUDA graph.

    ``exchange="nccl"``: partition, local merge, NCCL all-gather, merge (four
    launches).  ``exchange="p2p"``: partition, then ``pdl_exchange_merge``
    (two launches; needs every rank on its own GPU of one node with peer
    access, and ``close()`` on every rank when done).  Both give the same bits.
    """

    def __init__(self, spec, device, group=None, local_splits=0, kernel="auto",
                 exchange="nccl"):
        """``local_splits`` 0 uses the B200 plan for the rank-local capacity."""
        if exchange not in ("nccl", "p2p"):
            raise ValueError("exchange must be 'nccl' or 'p2p'")
        from . import ops
        from .splitkv_plan import make_b200_plan, make_splitkv_plan
        self.ops = ops
        self.group = group
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        self.device = torch.device(device)
        self.spec = spec
        self.kernel = kernel
        self.per_rank = tokens_per_rank(spec.table_width, self.world)
        self.local_spec = DecodeSpec(spec.max_batch, spec.num_heads, spec.num_kv_heads,
                                     spec.head_dim, self.per_rank)
        sms = ops.sm_count(self.device)
        self.plan = (make_b200_plan(self.local_spec, sms) if not local_splits else
                     make_splitkv_plan(self.local_spec, sms, num_splits=local_splits))
        b, hq, d, s = spec.max_batch, spec.num_heads, spec.head_dim, self.plan.splits
        f32 = dict(device=self.device, dtype=torch.float32)
        self.partials = torch.empty(b, hq, s, d, **f32)
        self.lse = torch.empty(b, hq, s, **f32)
        self.layout = ExchangeLayout(b * hq, d, self.world)
        self.send = torch.zeros(self.layout.block, **f32)
        self.gathered = torch.zeros(self.world * self.layout.block, **f32)
        self.out = torch.empty(b, hq, d, device=self.device, dtype=torch.bfloat16)
        self.local_len = torch.zeros(b, device=self.device, dtype=torch.int32)
        # Dynamic-scheduler words of the local partition launch (left zeroed).
        self.counters = torch.zeros(2, device=self.device, dtype=torch.int32)
        self.exchange_mode = exchange
        self.peer = PeerExchange(b * hq, d, self.device, group) if exchange == "p2p" else None
        self._args = {}

    def close(self):
        """Release the peer-exchange buffers (p2p mode; call on every rank)."""
        if self.peer is not None:
            self.peer.close()
            self.peer = None

    def _launch_args(self, q, k_local, v_local, table_local, scale):
        ops = self.ops
        key = ops.tensor_key(q, k_local, v_local, table_local) + (scale,)
        if key not in self._args:
            rows, d = self.layout.rows, self.spec.head_dim
            s = self.plan.splits
            part = ops.decode_args(q, k_local, v_local, table_local, self.local_len, scale=scale,
                                   tokens_per_split=self.plan.tokens_per_split, splits=s,
                                   protocol=ops.PROTOCOL_LSE, kernel=self.kernel,
                                   partial=self.partials, lse=self.lse, counters=self.counters,
                                   flags=ops.FLAG_DYNAMIC)
            if self.peer is not None:
                ex = ops.exchange_args(self.partials, self.lse, rows=rows, parts=s, head_dim=d,
                                       rank=self.rank, world=self.world, buffers=self.peer.ptrs,
                                       out=self.out, lengths=self.local_len,
                                       num_heads=self.spec.num_heads,
                                       tokens_per_split=self.plan.tokens_per_split)
                self._args[key] = (part, ex, None)
                return self._args[key]
            send_p, send_l = self.layout.send_views(self.send)
            local = ops.merge_args(self.partials, self.lse, rows=rows, parts=s, head_dim=d,
                                   row_stride=s * d, part_stride=d, lse_row_stride=s,
                                   lse_part_stride=1, out_partial=send_p, out_lse=send_l)
            rs, ps, lrs, lps = self.layout.merge_strides()
            glob = ops.merge_args(self.gathered, self.gathered[self.layout.lse_offset:],
                                  rows=rows, parts=self.world, head_dim=d, row_stride=rs,
                                  part_stride=ps, lse_row_stride=lrs, lse_part_stride=lps,
                                  out=self.out)
            self._args[key] = (part, local, glob)
        return self._args[key]

    def __call__(self, q, k_local, v_local, table_local, lengths, scale=None):
        scale = q.shape[-1] ** -0.5 if scale is None else float(scale)
        if table_local.shape[1] * PAGE_SIZE != self.per_rank:
            raise ValueError("local block table must have tokens_per_rank / 256 columns")
        part, local, glob = self._launch_args(q, k_local, v_local, table_local, scale)
        local_lengths(lengths, self.rank, self.per_rank, out=self.local_len)
        self.ops.partition(part, self.device)
        if glob is None:
            self.ops.exchange_merge(local, self.device)
            return self.out
        self.ops.lse_merge(local, self.device)
        exchange(self.send, self.gathered, self.group)
        self.ops.lse_merge(glob, self.device)
        return self.out


def shard_context_pool(k, v, table, rank, world):
    """Build rank `rank`'s local pools and table from global ones (setup helper).

    Pages of columns [lo, hi) of every row are copied into a compact local pool;
    the local table has ``tokens_per_rank / 256`` columns (padding -1).
    """
    width = table.shape[1]
    lo, hi = context_shard(width, world, rank)
    per = -(-width // world)
    cols = table[:, lo:hi]
    flat = cols.reshape(-1).long()
    live = flat >= 0
    idx = torch.nonzero(live).flatten()
    local_k = k[flat[idx]].contiguous() if idx.numel() else k[:1].clone()
    local_v = v[flat[idx]].contiguous() if idx.numel() else v[:1].clone()
    local_table = torch.full((table.shape[0], per), -1, dtype=torch.int32, device=table.device)
    mapping = torch.full_like(flat, -1)
    mapping[idx] = torch.arange(idx.numel(), device=table.device)
    local_table[:, :hi - lo] = mapping.view(table.shape[0], hi - lo).to(torch.int32)
    return local_k, local_v, local_table


def shard_head_pool(k, v, q, rank, world, num_heads, num_kv_heads):
    """Rank `rank`'s head slice: (q_local, k_local, v_local) for KV-head sharding."""
    kv_lo, kv_hi, q_lo, q_hi = head_shard(num_heads, num_kv_heads, world, rank)
    return (q[:, q_lo:q_hi].contiguous(), k[:, :, kv_lo:kv_hi].contiguous(),
            v[:, :, kv_lo:kv_hi].contiguous())


def shard_batch_pool(k, v, table, lengths, rows):
    """Rank-local pools and table for the batch rows `rows` (setup helper).

    Only the live pages of those rows are copied, in row order, into a compact
    local pool; the local table keeps the global width (padding -1) so the
    geometry contract is unchanged.  Returns (k_local, v_local, table_local,
    lengths_local).
    """
    idx = torch.as_tensor(rows, device=table.device, dtype=torch.long)
    sub = table[idx]
    lens = lengths[idx]
    live = -(-lens.to(torch.int64) // PAGE_SIZE)
    cols = torch.arange(table.shape[1], device=table.device)
    mask = cols[None, :] < live[:, None]
    pages = sub[mask].long()
    local_table = torch.full_like(sub, -1)
    local_table[mask] = torch.arange(pages.numel(), device=table.device, dtype=sub.dtype)
    if pages.numel() == 0:
        return k[:1].clone(), v[:1].clone(), local_table, lens.clone()
    return k[pages].contiguous(), v[pages].contiguous(), local_table, lens.clone()
