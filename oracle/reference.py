"""NumPy restatement of the reference decode-attention algorithm (oracle only).

TEST INFRASTRUCTURE: see ``oracle/__init__.py`` for who may import this.

Layouts follow the reference exactly:
  q       [B, Hq, D]            float32 (values of BF16 inputs)
  k, v    [P, 256, Hkv, D]      NHD pages, float32 (values of BF16 inputs)
  table   [B, W]  int32         logical page j of row b -> physical page
  lengths [B]     int32         live tokens per row
Logical token t of row b lives at page ``table[b, t // 256]``, slot ``t % 256``
(reference ``src/paged_decode/kernels.py:26-28``); query head h reads KV head
``h // (Hq // Hkv)``.
"""
import numpy as np

PAGE = 256          # reference src/paged_decode/spec.py:6
PARTITION = 1024    # reference src/paged_decode/spec.py:7
TILE = 64           # reference src/paged_decode/spec.py:8


# --------------------------------------------------------------------------
# BF16 helpers: NumPy has no bfloat16, so inputs are generated as float32,
# rounded to BF16 with round-to-nearest-even on the raw bits, and the same
# 16-bit patterns are fed to the GPU (as bfloat16) and to this oracle (as the
# float32 values they denote).
# --------------------------------------------------------------------------
def bf16_bits(x):
    """float32 array -> uint16 BF16 bit patterns, round-to-nearest-even."""
    u = np.ascontiguousarray(x, dtype=np.float32).view(np.uint32).astype(np.uint64)
    rounded = (u + 0x7FFF + ((u >> 16) & 1)) >> 16
    nan = np.isnan(np.asarray(x, dtype=np.float32))
    out = rounded.astype(np.uint16)
    out[nan] = 0x7FC0
    return out


def bits_to_f32(bits):
    """uint16 BF16 bit patterns -> the float32 values they denote."""
    return (np.asarray(bits, dtype=np.uint16).astype(np.uint32) << 16).view(np.float32)


def round_bf16(x):
    """Round float32 values to the nearest BF16 value (returned as float32)."""
    return bits_to_f32(bf16_bits(x))


# --------------------------------------------------------------------------
# reference src/paged_decode/reference.py
# --------------------------------------------------------------------------
def validate_metadata(table, lengths, num_pages, max_context_len, page_size=PAGE):
    """Metadata contract of reference.py:10-21.

    Lengths must lie in [0, max_context_len]; the first ceil(len/page) table
    entries of each row must be valid physical pages.  Entries past that are
    padding (may be -1) and are never read.
    """
    table, lengths = np.asarray(table), np.asarray(lengths)
    if table.ndim != 2 or lengths.ndim != 1 or table.shape[0] != lengths.shape[0]:
        raise ValueError("metadata batch dimensions differ")
    if not (np.issubdtype(table.dtype, np.integer) and np.issubdtype(lengths.dtype, np.integer)):
        raise ValueError("metadata must be integral")
    if lengths.size and (lengths.min() < 0 or lengths.max() > max_context_len):
        raise ValueError("context length outside configured capacity")
    for b in range(table.shape[0]):
        live = -(-int(lengths[b]) // page_size)
        if live > table.shape[1]:
            raise ValueError("invalid live page mapping")
        pages = table[b, :live]
        if live and (pages.min() < 0 or pages.max() >= num_pages):
            raise ValueError("invalid live page mapping")


def gather_kv(cache, table_row, length):
    """Rows of one sequence in logical order, as float32 (reference.py:24-28)."""
    page_size = cache.shape[1]
    if length == 0:
        return np.empty((0,) + cache.shape[2:], dtype=np.float32)
    t = np.arange(length)
    return np.asarray(cache[table_row[t // page_size], t % page_size], dtype=np.float32)


def _default_scale(q, scale):
    return q.shape[-1] ** -0.5 if scale is None else scale


def dense_reference(q, k, v, table, lengths, scale=None):
    """Independent dense softmax oracle (reference.py:31-46); zero rows for len 0."""
    q = np.asarray(q, dtype=np.float32)
    scale = _default_scale(q, scale)
    validate_metadata(table, lengths, k.shape[0], table.shape[1] * k.shape[1], k.shape[1])
    out = np.zeros_like(q)
    group = q.shape[1] // k.shape[2]
    for b in range(q.shape[0]):
        n = int(lengths[b])
        if n == 0:
            continue
        keys, vals = gather_kv(k, table[b], n), gather_kv(v, table[b], n)
        for h in range(q.shape[1]):
            kv = h // group
            s = (keys[:, kv] @ q[b, h]) * scale
            w = np.exp(s - s.max())
            out[b, h] = (w @ vals[:, kv]) / w.sum()
    return out


def partial(q, keys, vals, scale, tile=TILE):
    """Tile-wise online softmax over one token range (reference.py:49-60).

    Returns (m, l, acc): m is the running maximum of the *scaled* scores,
    l the sum of exp(score - m), acc the unnormalised weighted sum of rows.
    An empty range gives (-inf, 0, zeros).
    """
    m = np.float32(-np.inf)
    l = np.float32(0.0)
    acc = np.zeros(q.shape, dtype=np.float32)
    for lo in range(0, keys.shape[0], tile):
        s = (keys[lo:lo + tile] @ q) * scale
        m_new = np.maximum(m, s.max())
        alpha = np.exp(m - m_new)
        p = np.exp(s - m_new)
        acc = acc * alpha + p @ vals[lo:lo + tile]
        l = l * alpha + p.sum()
        m = m_new
    return m, l, acc


def merge_partials(parts, dim):
    """Combine (m, l, acc) triples of disjoint ranges (reference.py:63-71)."""
    live = [part for part in parts if part[1] > 0]
    if not live:
        return np.zeros(dim, dtype=np.float32)
    top = max(part[0] for part in live)
    weights = [np.exp(part[0] - top) for part in live]
    num = sum(w * part[2] for w, part in zip(weights, live))
    den = sum(w * part[1] for w, part in zip(weights, live))
    return num / den


def streaming_reference(q, k, v, table, lengths, split=False, scale=None,
                        partition=PARTITION):
    """Streaming model of the kernels (reference.py:74-88).

    ``split=True`` cuts every row into ``partition``-token ranges (the
    reference fixes 1024, spec.py:7) and merges them; ``split=False`` runs one
    range per row.  ``partition`` is exposed so 512-token splits can be
    modelled with the same arithmetic.
    """
    scale = _default_scale(q, scale)
    validate_metadata(table, lengths, k.shape[0], table.shape[1] * k.shape[1], k.shape[1])
    out = np.zeros(q.shape, dtype=np.float32)
    group = q.shape[1] // k.shape[2]
    for b in range(q.shape[0]):
        n = int(lengths[b])
        keys, vals = gather_kv(k, table[b], n), gather_kv(v, table[b], n)
        step = partition if split else max(1, n)
        for h in range(q.shape[1]):
            kv = h // group
            qh = np.asarray(q[b, h], dtype=np.float32)
            parts = [partial(qh, keys[s:s + step, kv], vals[s:s + step, kv], scale)
                     for s in range(0, n, step)]
            out[b, h] = merge_partials(parts, q.shape[-1])
    return out


# --------------------------------------------------------------------------
# Split-KV protocols of the GPU kernels
# --------------------------------------------------------------------------
def balanced_span(length, splits, granule):
    """Tokens per partition of a row split into ``splits`` partitions that
    follow its length, in whole granules: G * ceil(ceil(L / S) / G).  This
    library's PDL_FLAG_BALANCED; no counterpart in the reference."""
    per = -(-int(length) // splits)
    return -(-per // granule) * granule


def partition_bounds(length, tokens_per_split, splits, balanced=False):
    """[start, end) of each partition (matched_splitkv.py:75-76, kernels.py:58-60).

    Partition p covers [p*T, min((p+1)*T, length)); it is empty when
    p*T >= length.  With ``balanced`` (no reference counterpart), T is
    balanced_span(length, splits, tokens_per_split) instead.  Integer
    arithmetic -- the GPU must match it bit-exactly.
    """
    span = balanced_span(length, splits, tokens_per_split) if balanced else tokens_per_split
    bounds = []
    for p in range(splits):
        start = p * span
        end = min(start + span, int(length))
        bounds.append((start, max(start, end)))
    return bounds


def normalized_partitions(q, k, v, table, lengths, tokens_per_split, splits, scale=None,
                          balanced=False):
    """Normalised partial + LSE per partition (matched_splitkv.py:52-98).

    partial = acc / l and lse = m + ln(l) with m in scaled-score units
    (matched_splitkv.py:92-95); an empty partition gives partial 0 and
    lse -inf.  Shapes: partials [B,Hq,S,D], lse [B,Hq,S].
    """
    q = np.asarray(q, dtype=np.float32)
    scale = _default_scale(q, scale)
    batch, heads, dim = q.shape
    group = heads // k.shape[2]
    partials = np.zeros((batch, heads, splits, dim), dtype=np.float32)
    lse = np.full((batch, heads, splits), -np.inf, dtype=np.float32)
    for b in range(batch):
        n = int(lengths[b])
        keys, vals = gather_kv(k, table[b], n), gather_kv(v, table[b], n)
        for p, (start, end) in enumerate(partition_bounds(n, tokens_per_split, splits, balanced)):
            if end <= start:
                continue
            for h in range(heads):
                kv = h // group
                m, l, acc = partial(q[b, h], keys[start:end, kv], vals[start:end, kv], scale)
                if l > 0:
                    partials[b, h, p] = acc / l
                    lse[b, h, p] = m + np.log(l)
    return partials, lse


def score_magnitudes(q, k, table, lengths, tokens_per_split, splits, scale=None,
                     balanced=False):
    """Per partition, the largest sum_i |q_i * k_ti| * |scale| over its tokens.

    This is the magnitude an FP32 dot product's rounding error scales with
    (a score near 0 can come from terms of size ~1), so it bounds how
    closely any FP32 implementation -- the reference's NumPy one included --
    can reproduce an LSE whose value is near 0.  0 for empty partitions.
    Shape [B, Hq, S].  (Test-side tolerance helper; no reference counterpart.)
    """
    q = np.asarray(q, dtype=np.float32)
    scale = abs(_default_scale(q, scale))
    batch, heads, dim = q.shape
    group = heads // k.shape[2]
    mags = np.zeros((batch, heads, splits), dtype=np.float64)
    for b in range(batch):
        n = int(lengths[b])
        keys = np.abs(gather_kv(k, table[b], n).astype(np.float64))
        for p, (start, end) in enumerate(partition_bounds(n, tokens_per_split, splits, balanced)):
            if end <= start:
                continue
            for h in range(heads):
                kv = h // group
                mags[b, h, p] = (keys[start:end, kv] @ np.abs(q[b, h].astype(np.float64))).max() * scale
    return mags


def lse_merge(partials, lse):
    """Stable LSE merge of normalised partials (matched_splitkv.py:101-127).

    M = max lse (an all -inf row uses 0), total = sum exp(lse - M),
    logsum = ln(total) + M (+inf when total is 0), and
    out = sum_p exp(lse_p - logsum) * partial_p.  All-empty rows give 0.
    """
    lse = np.asarray(lse, dtype=np.float32)
    top = lse.max(axis=-1, keepdims=True)
    top = np.where(np.isneginf(top), np.float32(0), top)
    total = np.exp(lse - top).sum(axis=-1, keepdims=True)
    with np.errstate(divide="ignore"):
        logsum = np.where(total > 0, np.log(np.where(total > 0, total, 1)) + top, np.inf)
    weights = np.exp(lse - logsum)
    return (weights[..., None] * partials).sum(axis=-2).astype(np.float32)


def unnormalized_partitions(q, k, v, table, lengths, tokens_per_split, splits, scale=None,
                            balanced=False):
    """(m, l, acc) per partition as stored by the split kernel (kernels.py:44-80).

    m is in scaled-score units, -inf with l = 0 and acc = 0 for empty
    partitions.  Shapes: maxima/denoms [B,Hq,S], accums [B,Hq,S,D].
    """
    q = np.asarray(q, dtype=np.float32)
    scale = _default_scale(q, scale)
    batch, heads, dim = q.shape
    group = heads // k.shape[2]
    maxima = np.full((batch, heads, splits), -np.inf, dtype=np.float32)
    denoms = np.zeros((batch, heads, splits), dtype=np.float32)
    accums = np.zeros((batch, heads, splits, dim), dtype=np.float32)
    for b in range(batch):
        n = int(lengths[b])
        keys, vals = gather_kv(k, table[b], n), gather_kv(v, table[b], n)
        for p, (start, end) in enumerate(partition_bounds(n, tokens_per_split, splits, balanced)):
            if end <= start:
                continue
            for h in range(heads):
                kv = h // group
                m, l, acc = partial(q[b, h], keys[start:end, kv], vals[start:end, kv], scale)
                maxima[b, h, p], denoms[b, h, p], accums[b, h, p] = m, l, acc
    return maxima, denoms, accums


def merge_unnormalized(maxima, denoms, accums):
    """Merge (m, l, acc) partitions (kernels.py:83-100).

    The maximum of an all-empty row is replaced by 0 before subtracting, and
    the total is guarded so such rows give exactly 0.
    """
    top = maxima.max(axis=-1, keepdims=True)
    top = np.where(np.isneginf(top), np.float32(0), top)
    factors = np.exp(maxima - top)
    total = (denoms * factors).sum(axis=-1)
    num = (accums * factors[..., None]).sum(axis=-2)
    return (num / np.where(total > 0, total, 1)[..., None]).astype(np.float32)


def matched_reference(q, k, v, table, lengths, tokens_per_split, splits, scale=None,
                      balanced=False):
    """Partition + LSE merge, the two-kernel path of matched_splitkv.py:130-150.

    Returns (out [B,Hq,D], partials [B,Hq,S,D], lse [B,Hq,S]).
    """
    partials, lse = normalized_partitions(q, k, v, table, lengths, tokens_per_split,
                                          splits, scale, balanced)
    return lse_merge(partials, lse), partials, lse
