"""Seeded synthetic workloads with the shapes of the five BASELINE configs.

No dataset exists for this operator; every config is synthetic and seeded:
q/K/V ~ N(0,1) rounded to BF16, NHD pages of 256 tokens, block tables that
scatter each row over a shuffled pool.  Tensors are generated on the device
(torch RNG), so multi-GB pools take milliseconds.

  cfg1  B=4,   Hq=8,  Hkv=2,  D=128, pool 64 pages, len ~ U[0,1024] (one 0, one 1024)
  cfg2  B=64,  Hq=Hkv=32,     D=64,  ctx 2048, pool 1.25x the pages needed
  cfg3  Hq=16, Hkv=4,         D=256, ctx 528 | 2064, B in {1,8,32,128,256},
        capacity 2320 (room for 256 decode steps), 2% of K channels x8
  cfg4  B=128, Hq=32, Hkv=8,  D=128, len ~ lognormal(median 4096, sigma 1)
        clipped to [1, 32768], every 32nd row 0 (seed 20261201: sum 750,637);
        a smaller batch takes the first rows of the same draw
  cfg5  B=2,   Hq=64, Hkv=8,  D=128, ctx 524288 (2048 pages per row)
"""
from dataclasses import dataclass, field
import math

import numpy as np
import torch

from .spec import DecodeSpec

PAGE = 256


@dataclass
class Workload:
    name: str
    q: torch.Tensor
    k: torch.Tensor
    v: torch.Tensor
    table: torch.Tensor
    lengths: torch.Tensor
    spec: DecodeSpec
    scale: float
    meta: dict = field(default_factory=dict)

    @property
    def kv_bytes(self):
        """Algorithmic KV bytes of one decode step: sum_b len_b * Hkv * D * 2 (K,V) * 2 B."""
        total = int(self.lengths.to(torch.int64).sum().item())
        return total * self.spec.num_kv_heads * self.spec.head_dim * 2 * 2

    def args(self):
        return self.q, self.k, self.v, self.table, self.lengths


def _randn_bf16(shape, gen, device):
    return torch.randn(shape, generator=gen, device=device, dtype=torch.float32).to(torch.bfloat16)


def _pool(batch, width, pages, hkv, dim, gen, device):
    perm = torch.randperm(pages, generator=gen, device=device)
    table = perm[:batch * width].view(batch, width).to(torch.int32).contiguous()
    k = _randn_bf16((pages, PAGE, hkv, dim), gen, device)
    v = _randn_bf16((pages, PAGE, hkv, dim), gen, device)
    return table, k, v


def cfg4_lengths(seed=20261201, batch=128):
    """Lognormal lengths (median 4096, sigma 1.0), clipped to [1, 32768], every 32nd zeroed."""
    rng = np.random.default_rng(seed)
    x = rng.lognormal(mean=math.log(4096), sigma=1.0, size=batch)
    lengths = np.clip(np.round(x), 1, 32768).astype(np.int32)
    lengths[::32] = 0
    return lengths


def make_workload(name, device="cuda", seed=0, batch=None, context=None, rank=0):
    """Build config `name` on `device`; `rank` decorrelates per-GPU shards."""
    gen = torch.Generator(device=device).manual_seed(1_000_003 * rank + 7919 * seed + 17)
    if name == "cfg1":
        b, hq, hkv, d, cap, pool = 4, 8, 2, 128, 1024, 64
        table, k, v = _pool(b, cap // PAGE, pool, hkv, d, gen, device)
        lengths = torch.randint(0, cap + 1, (b,), generator=gen, device=device, dtype=torch.int32)
        lengths[0], lengths[1] = 0, cap
        meta = dict(tokens_per_split=1024)
    elif name == "cfg2":
        b, hq, hkv, d = batch or 64, 32, 32, 64
        cap = context or 2048
        width = -(-cap // PAGE)
        pool = int(math.ceil(1.25 * b * width))
        table, k, v = _pool(b, width, pool, hkv, d, gen, device)
        lengths = torch.full((b,), cap, dtype=torch.int32, device=device)
        meta = dict(tokens_per_split=1024)
    elif name == "cfg3":
        b, hq, hkv, d = batch or 32, 16, 4, 256
        ctx = context or 2064
        cap = 2320
        width = -(-cap // PAGE)
        table, k, v = _pool(b, width, b * width, hkv, d, gen, device)
        channels = torch.randperm(hkv * d, generator=gen, device=device)[:round(0.02 * hkv * d)]
        scale_ch = torch.ones(hkv * d, device=device)
        scale_ch[channels] = 8.0
        k = (k.float() * scale_ch.view(1, 1, hkv, d)).to(torch.bfloat16)
        lengths = torch.full((b,), ctx, dtype=torch.int32, device=device)
        meta = dict(outlier_channels=int(channels.numel()))
    elif name == "cfg4":
        # `batch` (default 128) takes the first rows of the same draw, e.g. a
        # smaller case of the same lengths for profiling.
        b, hq, hkv, d, cap = batch or 128, 32, 8, 128, 32768
        lens_np = cfg4_lengths(batch=b)
        lengths = torch.from_numpy(lens_np).to(device)
        need = [-(-int(n) // PAGE) for n in lens_np]
        pool = max(1, sum(need))
        width = cap // PAGE
        perm = torch.randperm(pool, generator=gen, device=device).to(torch.int32)
        table = torch.full((b, width), -1, dtype=torch.int32, device=device)
        offset = 0
        for row, n in enumerate(need):
            table[row, :n] = perm[offset:offset + n]
            offset += n
        k = _randn_bf16((pool, PAGE, hkv, d), gen, device)
        v = _randn_bf16((pool, PAGE, hkv, d), gen, device)
        meta = dict(sum_len=int(lens_np.sum()))
    elif name == "cfg5":
        b, hq, hkv, d = batch or 2, 64, 8, 128
        cap = context or 524288
        width = cap // PAGE
        table, k, v = _pool(b, width, b * width, hkv, d, gen, device)
        lengths = torch.full((b,), cap, dtype=torch.int32, device=device)
        meta = dict()
    else:
        raise ValueError(f"unknown workload {name!r}")
    q = _randn_bf16((b, hq, d), gen, device)
    spec = DecodeSpec(b, hq, hkv, d, cap)
    return Workload(name, q, k, v, table, lengths, spec, d ** -0.5, meta)
