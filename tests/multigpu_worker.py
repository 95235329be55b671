"""torchrun worker for tests/test_gpu_multi.py (one process per GPU, NCCL).

Every rank builds the same seeded global workload on its own GPU, computes
the unsharded single-GPU result locally, then checks:
  * context parallel (local partial + LSE, one all-gather, LSE merge) against
    the single-GPU output, eager and replayed from a CUDA graph;
  * the same with the peer-memory exchange (``exchange="p2p"``: one kernel
    stores into every rank's IPC-mapped buffer and merges after a bounded
    flag wait): bit-identical to the all-gather path, eager and in a graph;
  * batch sharding: its rows, decoded alone, equal the unsharded rows bit for bit;
  * KV-head sharding: its head slice equals the unsharded heads bit for bit.
Rank 0 prints one JSON line with the results; any failure raises.
"""
import datetime
import json
import os
import sys
from pathlib import Path

ROOT = Path(__file__).resolve().parents[1]
sys.path.insert(0, str(ROOT / "paged-decode-lab_b200"))

import torch  # noqa: E402
import torch.distributed as dist  # noqa: E402

from paged_decode import ops, parallel  # noqa: E402
from paged_decode.spec import DecodeSpec  # noqa: E402

TOL = 2.0 ** -7


def decode(q, k, v, table, lens, tokens, splits):
    """Unsharded reference decode with an explicit split layout."""
    out = torch.empty(q.shape, dtype=torch.bfloat16, device=q.device)
    partial = torch.empty(q.shape[0], q.shape[1], splits, q.shape[2], device=q.device)
    lse = torch.empty(q.shape[0], q.shape[1], splits, device=q.device)
    ops.paged_decode(ops.decode_args(q, k, v, table, lens, scale=q.shape[-1] ** -0.5,
                                     tokens_per_split=tokens, splits=splits,
                                     protocol=ops.PROTOCOL_LSE, out=out, partial=partial,
                                     lse=lse), q.device)
    return out


def main():
    local = int(os.environ["LOCAL_RANK"])
    torch.cuda.set_device(local)
    device = torch.device("cuda", local)
    dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=60), device_id=device)
    rank, world = dist.get_rank(), dist.get_world_size()
    gen = torch.Generator(device=device).manual_seed(1234)
    report = {}

    # ---- context parallel: B=2, Hq=64, Hkv=8, D=128, 65536-token capacity
    b, hq, hkv, d, width = 2, 64, 8, 128, 256
    pages = b * width
    table = torch.randperm(pages, generator=gen, device=device).view(b, width).to(torch.int32)
    k = torch.randn(pages, 256, hkv, d, generator=gen, device=device).to(torch.bfloat16)
    v = torch.randn(pages, 256, hkv, d, generator=gen, device=device).to(torch.bfloat16)
    q = torch.randn(b, hq, d, generator=gen, device=device).to(torch.bfloat16)
    lens = torch.tensor([width * 256, 40_000], dtype=torch.int32, device=device)
    spec = DecodeSpec(b, hq, hkv, d, width * 256)
    full = decode(q, k, v, table, lens, 4096, width * 256 // 4096)
    k_loc, v_loc, t_loc = parallel.shard_context_pool(k, v, table, rank, world)
    cp = parallel.ContextParallelDecode(spec, device, local_splits=0)
    out = cp(q, k_loc, v_loc, t_loc, lens).clone()
    report["context_eager_err"] = (out.float() - full.float()).abs().max().item()
    stream = torch.cuda.Stream(device)
    stream.wait_stream(torch.cuda.current_stream(device))
    with torch.cuda.stream(stream):
        for _ in range(3):
            cp(q, k_loc, v_loc, t_loc, lens)
    torch.cuda.current_stream(device).wait_stream(stream)
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        cp(q, k_loc, v_loc, t_loc, lens)
    lens.copy_(torch.tensor([12_345, width * 256 - 7], dtype=torch.int32, device=device))
    graph.replay()
    torch.cuda.synchronize(device)
    replayed = cp.out.clone()
    full2 = decode(q, k, v, table, lens, 4096, width * 256 // 4096)
    report["context_graph_err"] = (replayed.float() - full2.float()).abs().max().item()
    eager = cp(q, k_loc, v_loc, t_loc, lens)
    report["context_graph_equals_eager"] = bool(torch.equal(eager, replayed))
    del graph

    # ---- context parallel over peer memory (one exchange kernel)
    p2p = parallel.ContextParallelDecode(spec, device, local_splits=0, exchange="p2p")
    lens.copy_(torch.tensor([width * 256, 40_000], dtype=torch.int32, device=device))
    nccl_out = cp(q, k_loc, v_loc, t_loc, lens).clone()
    p2p_out = p2p(q, k_loc, v_loc, t_loc, lens).clone()
    report["p2p_equals_nccl"] = bool(torch.equal(p2p_out, nccl_out))
    with torch.cuda.stream(stream):
        stream.wait_stream(torch.cuda.current_stream(device))
        for _ in range(3):
            p2p(q, k_loc, v_loc, t_loc, lens)
    torch.cuda.current_stream(device).wait_stream(stream)
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        p2p(q, k_loc, v_loc, t_loc, lens)
    ok = True
    for new_lens in ([12_345, width * 256 - 7], [0, 1], [width * 256, 256]):
        lens.copy_(torch.tensor(new_lens, dtype=torch.int32, device=device))
        graph.replay()
        torch.cuda.synchronize(device)
        ok &= bool(torch.equal(p2p.out, cp(q, k_loc, v_loc, t_loc, lens)))
    report["p2p_graph_equals_nccl"] = ok
    del graph
    torch.cuda.synchronize(device)
    report["p2p_fault_word"] = ops.read_fault()
    p2p.close()

    # ---- batch sharding (variable lengths): rows decode independently
    b, hq, hkv, d, width = 16, 32, 8, 128, 32
    pages = b * width
    table = torch.randperm(pages, generator=gen, device=device).view(b, width).to(torch.int32)
    k = torch.randn(pages, 256, hkv, d, generator=gen, device=device).to(torch.bfloat16)
    v = torch.randn(pages, 256, hkv, d, generator=gen, device=device).to(torch.bfloat16)
    q = torch.randn(b, hq, d, generator=gen, device=device).to(torch.bfloat16)
    lens = torch.randint(0, width * 256 + 1, (b,), generator=gen, device=device,
                         dtype=torch.int32)
    full = decode(q, k, v, table, lens, 1024, width // 4)
    rows = parallel.batch_shards(lens.tolist(), world)[rank]
    idx = torch.tensor(rows, device=device)
    mine = decode(q[idx].contiguous(), k, v, table[idx].contiguous(), lens[idx].contiguous(),
                  1024, width // 4)
    report["batch_bit_exact"] = bool(torch.equal(mine, full[idx]))

    # ---- KV-head sharding
    q_l, k_l, v_l = parallel.shard_head_pool(k, v, q, rank, world, hq, hkv)
    mine = decode(q_l, k_l, v_l, table, lens, 1024, width // 4)
    _, _, q_lo, q_hi = parallel.head_shard(hq, hkv, world, rank)
    report["head_bit_exact"] = bool(torch.equal(mine, full[:, q_lo:q_hi]))

    flags = torch.tensor([report["context_eager_err"] <= TOL, report["context_graph_err"] <= TOL,
                          report["context_graph_equals_eager"], report["p2p_equals_nccl"],
                          report["p2p_graph_equals_nccl"], report["p2p_fault_word"] == 0,
                          report["batch_bit_exact"],
                          report["head_bit_exact"]], device=device, dtype=torch.int32)
    dist.all_reduce(flags, op=dist.ReduceOp.MIN)
    report["all_ranks_ok"] = bool(flags.min().item())
    if rank == 0:
        print(json.dumps(report), flush=True)
    dist.barrier()
    dist.destroy_process_group()
    return 0 if report["all_ranks_ok"] else 1


if __name__ == "__main__":
    sys.exit(main())
