"""FP32 gather + dense softmax on the GPU (oracle only; TEST INFRASTRUCTURE).

Restates the reference's Torch oracle (src/paged_decode/torch_reference.py:5-17)
for inputs too large for the NumPy oracle: every live row is gathered by its
block table, upcast to FP32 and attended densely -- an algorithm independent
of the split-K kernels it checks.  Rows of length 0 give zeros.
"""
import torch

from .reference import balanced_span


def dense_reference(q, k, v, tables, lengths, scale=None):
    scale = q.shape[-1] ** -0.5 if scale is None else scale
    out = torch.zeros_like(q, dtype=torch.float32)
    group = q.shape[1] // k.shape[2]
    for b, n in enumerate(lengths.cpu().tolist()):
        if n == 0:
            continue
        t = torch.arange(n, device=q.device)
        pages = tables[b, t // 256].long()
        keys = k[pages, t % 256].float().repeat_interleave(group, dim=1)
        vals = v[pages, t % 256].float().repeat_interleave(group, dim=1)
        scores = torch.einsum("hd,nhd->hn", q[b].float(), keys) * scale
        out[b] = torch.einsum("hn,nhd->hd", scores.softmax(-1), vals)
    return out


def dense_lse(q, k, v, tables, lengths, start, stop, scale=None):
    """Natural-log LSE of the scaled scores over tokens [start, stop) of each row."""
    scale = q.shape[-1] ** -0.5 if scale is None else scale
    lse = torch.full(q.shape[:2], float("-inf"), dtype=torch.float32, device=q.device)
    group = q.shape[1] // k.shape[2]
    for b, n in enumerate(lengths.cpu().tolist()):
        hi = min(stop, n)
        if hi <= start:
            continue
        t = torch.arange(start, hi, device=q.device)
        pages = tables[b, t // 256].long()
        keys = k[pages, t % 256].float().repeat_interleave(group, dim=1)
        scores = torch.einsum("hd,nhd->hn", q[b].float(), keys) * scale
        lse[b] = torch.logsumexp(scores, dim=-1)
    return lse


def chunked_reference_rows(q, k, v, tables, lengths, rows, scale=None, chunk=65536):
    """FP64 decode output [len(rows), Hq, D] of the selected rows, for rows too long
    to gather whole (a 524,288-token row): per KV head, tokens in chunks, with a
    running max / sum / weighted sum in FP64 -- the same dense softmax, only
    evaluated piecewise.  Rows of length 0 give zeros."""
    scale = q.shape[-1] ** -0.5 if scale is None else scale
    hkv = k.shape[2]
    group = q.shape[1] // hkv
    out = torch.zeros((len(rows), q.shape[1], q.shape[2]), dtype=torch.float64, device=q.device)
    lens = lengths.cpu().tolist()
    for i, b in enumerate(rows):
        n = lens[b]
        for h in range(hkv):
            qh = q[b, h * group:(h + 1) * group].double()             # [G, D]
            m = torch.full((group, 1), float("-inf"), dtype=torch.float64, device=q.device)
            s = torch.zeros((group, 1), dtype=torch.float64, device=q.device)
            acc = torch.zeros((group, q.shape[2]), dtype=torch.float64, device=q.device)
            for t0 in range(0, n, chunk):
                t = torch.arange(t0, min(n, t0 + chunk), device=q.device)
                pages = tables[b, t // 256].long()
                keys = k[pages, t % 256, h].double()                   # [n, D]
                vals = v[pages, t % 256, h].double()
                sc = (qh @ keys.T) * scale                              # [G, n]
                m_new = torch.maximum(m, sc.max(dim=1, keepdim=True).values)
                alpha = torch.exp(m - m_new)
                p = torch.exp(sc - m_new)
                s = s * alpha + p.sum(dim=1, keepdim=True)
                acc = acc * alpha + p @ vals
                m = m_new
            if n:
                out[i, h * group:(h + 1) * group] = acc / s
    return out


def chunked_partition_lse(q, k, tables, lengths, rows, tokens_per_split, splits, scale=None,
                          balanced=False):
    """FP64 natural-log LSE of the scaled scores of every partition
    [p * T, min((p + 1) * T, len)) of the selected rows, [len(rows), Hq, S],
    -inf for empty partitions (``balanced``: the partitions of
    reference.balanced_span instead); and each partition's score magnitude (the
    largest sum_i |q_i k_i| * |scale| over its tokens, 0 when empty), the
    scale an FP32 score's rounding error grows with.  Evaluated on the GPU,
    one partition of one KV head at a time."""
    scale = q.shape[-1] ** -0.5 if scale is None else scale
    hkv = k.shape[2]
    group = q.shape[1] // hkv
    lse = torch.full((len(rows), q.shape[1], splits), float("-inf"), dtype=torch.float64,
                     device=q.device)
    mag = torch.zeros((len(rows), q.shape[1], splits), dtype=torch.float64, device=q.device)
    lens = lengths.cpu().tolist()
    for i, b in enumerate(rows):
        n = lens[b]
        span = balanced_span(n, splits, tokens_per_split) if balanced else tokens_per_split
        for p in range(splits):
            lo, hi = p * span, min(n, (p + 1) * span)
            if hi <= lo:
                continue
            t = torch.arange(lo, hi, device=q.device)
            pages = tables[b, t // 256].long()
            for h in range(hkv):
                qh = q[b, h * group:(h + 1) * group].double()          # [G, D]
                keys = k[pages, t % 256, h].double()                    # [n, D]
                sc = (qh @ keys.T) * scale
                lse[i, h * group:(h + 1) * group, p] = torch.logsumexp(sc, dim=1)
                mag[i, h * group:(h + 1) * group, p] = (qh.abs() @ keys.abs().T).max(dim=1).values \
                    * abs(scale)
    return lse, mag
