"""Benchmark of the paged decode-attention operator (one JSON line on rank 0).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--config cfg4] [--impl ours|reference]

A step is one decode call (partition + LSE merge) over one batch of the chosen
BASELINE config with inputs resident in HBM.  Default workload: config 4, the
largest config stated for one GPU -- variable-length serving batch, B=128,
Hq=32, Hkv=8, D=128, lognormal lengths (median 4096, clipped to [1, 32768],
every 32nd row 0; 3.07 GB of KV per step) -- split with this library's B200
plan (8 partitions of 4096 tokens, dynamic scheduling).

* ``value``: KV GB/s = algorithmic KV bytes / device time.  K steps are
  captured in one CUDA graph; that K-step window is replayed R times back to
  back (R sized to about half a second so the clock sampler sees it) between
  CUDA events, max over ranks.  When a config's KV pool is smaller than 2x L2,
  steps rotate over independent input copies so every step reads HBM.
* ``convergence``: the same step captured as 32- and 128-step graphs;
  |t32 - t128| / t128 (required <= 0.05).
* ``e2e``: the same metric through the public API (``matched_decode``, or
  ``ContextParallelDecode``) with host buffers: each step copies q / block
  table / lengths from pinned host memory and the output back, inside the
  timed region.  The KV cache is resident device state, as in serving.  The
  API call is captured once in a CUDA graph and replayed per step, as the
  engines replay their decode step (their inputs are copied in outside the
  graph); the copies are ordinary stream copies each step.
* ``roofline``: the partition kernel alone (K launches per graph window) vs
  the measured HBM copy bandwidth in MEASURED_PEAKS.json; ``traffic`` is the
  per-launch DRAM bytes of the ncu summary committed under profiles/.
* ``cpu_baseline``: the NumPy oracle (the reference's CPU algorithm) over a
  bounded sample of the same workload on the host cores (rank 0, N = 1).
* ``--impl reference``: that CPU implementation alone, on all host cores.

Multi-GPU (torchrun), ``--mode``:
  batch    (default) one global batch, rows split token-balanced over the
           ranks, no collective on the data path ("scaling": "strong");
  head     one global batch, KV heads split over the ranks ("strong");
  context  one global batch, each row's pages split over the ranks, one
           exchange of (partial, LSE) per step (default for cfg5; "strong");
  replica  every rank decodes its own batch ("weak").
``value`` = the global batch's KV bytes (every rank's for replica) / the
slowest rank's time.  Before timing, the ranks' outputs are gathered and
compared with a one-GPU decode of the global batch on rank 0: bit-exact for
head and batch sharding (same partition bounds), within 2^-7 for context
parallelism (other partition bounds); the line carries ``parity``.
"""
import argparse
import copy
import datetime
import json
import math
import os
import re
import subprocess
import sys
import threading
import time
from pathlib import Path

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT / "paged-decode-lab_b200"))
sys.path.insert(0, str(ROOT))

METRIC = "decode-attn achieved KV HBM GB/s"
UNIT = "GB/s"
L2_BYTES = 126e6
CONVERGENCE_LIMIT = 0.05


def parse_args(argv=None):
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=("ours", "reference"), default="ours")
    ap.add_argument("--config", default="cfg4", choices=("cfg1", "cfg2", "cfg3", "cfg4", "cfg5"))
    ap.add_argument("--batch", type=int, default=None)
    ap.add_argument("--context", type=int, default=None)
    ap.add_argument("--splits", type=int, default=None, help="matched plan split count")
    ap.add_argument("--kernel", default="auto", choices=("auto", "simt", "mma"))
    ap.add_argument("--mode", default="auto", choices=("auto", "head", "batch", "context", "replica"),
                    help="N>1: split one batch by rows, by KV head or by context (strong "
                         "scaling), or run an independent batch per rank (weak); auto = context "
                         "for cfg5, else batch")
    ap.add_argument("--exchange", default="p2p", choices=("nccl", "p2p"),
                    help="context mode: NCCL all-gather between two merge kernels, or one "
                         "kernel storing into peers' buffers over NVLink (pdl_exchange_merge)")
    ap.add_argument("--append", action="store_true",
                    help="each step first appends the new token's K/V through the block table "
                         "(pdl_append_kv, lengths += 1 on the device) and then decodes, as a "
                         "decode loop does; lengths restart at each replayed window")
    ap.add_argument("--hot", action="store_true",
                    help="reuse one input copy every step (L2-resident when it fits), as the "
                         "reference measured its A100 numbers; default rotates copies past L2")
    ap.add_argument("--window-seconds", type=float, default=0.5)
    ap.add_argument("--cpu-seconds", type=float, default=10.0)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-parity", action="store_true", help="skip the N>1 parity check")
    ap.add_argument("--sweep", action="store_true",
                    help="partition-kernel GB/s for every (head_dim, group, kernel) at ~1 GB of "
                         "KV (one JSON line per point; not the contract line)")
    ap.add_argument("--exchange-micro", action="store_true",
                    help="under torchrun (N>1): time the context-parallel combine alone, NCCL "
                         "path (local merge, all-gather, merge) vs the peer-memory exchange "
                         "kernel (one JSON line per shape; not the contract line)")
    return ap.parse_args(argv)


def resolve_mode(args, world):
    """The multi-GPU mode of this run ("single" on one GPU)."""
    if world == 1:
        return "single"
    if args.mode != "auto":
        return args.mode
    return "context" if args.config == "cfg5" else "batch"


def sweep(reps=20):
    """Partition kernel alone, graph-timed, ctx 4096, Hkv 8, ~1 GB of KV per launch."""
    import torch
    from paged_decode import ops
    for dim in (64, 128, 256):
        for group in (1, 2, 4, 8, 16):
            for kernel in ("simt", "mma"):
                ctx, hkv = 4096, 8
                batch = max(1, int(1.0e9 // (ctx * hkv * dim * 4)))
                width, hq = ctx // 256, hkv * group
                gen = torch.Generator(device="cuda").manual_seed(0)
                table = torch.randperm(batch * width, generator=gen, device="cuda")
                table = table.view(batch, width).to(torch.int32)
                k = torch.randn(batch * width, 256, hkv, dim, generator=gen,
                                device="cuda").to(torch.bfloat16)
                v = torch.randn_like(k)
                q = torch.randn(batch, hq, dim, generator=gen, device="cuda").to(torch.bfloat16)
                lens = torch.full((batch,), ctx, dtype=torch.int32, device="cuda")
                splits = 4 if batch * hkv < 600 else 1
                partial = torch.empty(batch, hq, splits, dim, device="cuda")
                lse = torch.empty(batch, hq, splits, device="cuda")
                a = ops.decode_args(q, k, v, table, lens, scale=dim ** -0.5,
                                    tokens_per_split=ctx // splits, splits=splits,
                                    protocol=ops.PROTOCOL_LSE, kernel=kernel, partial=partial,
                                    lse=lse)
                for _ in range(3):
                    ops.partition(a, q.device)
                side = torch.cuda.Stream()
                side.wait_stream(torch.cuda.current_stream())
                with torch.cuda.stream(side):
                    ops.partition(a, q.device)
                torch.cuda.current_stream().wait_stream(side)
                graph = torch.cuda.CUDAGraph()
                with torch.cuda.graph(graph):
                    for _ in range(reps):
                        ops.partition(a, q.device)
                graph.replay()
                torch.cuda.synchronize()
                e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                e0.record()
                graph.replay()
                graph.replay()
                e1.record()
                torch.cuda.synchronize()
                us = e0.elapsed_time(e1) * 1e3 / (2 * reps)
                kv = batch * ctx * hkv * dim * 4
                print(json.dumps(dict(head_dim=dim, group=group, kernel=kernel, batch=batch,
                                      splits=splits, us=round(us, 2),
                                      gbs=round(kv / us / 1e3, 1))), flush=True)
                del graph, k, v
                torch.cuda.empty_cache()


def config_plan(name, args, spec, sm_count):
    """Split plan per config: cfg2 keeps its specified 1024-token partitions, --splits
    asks the reference heuristic for an explicit count, otherwise this library's
    B200 plan (``make_b200_plan``)."""
    from paged_decode.splitkv_plan import make_b200_plan, make_splitkv_plan
    if args.splits is not None:
        return make_splitkv_plan(spec, sm_count, num_splits=args.splits)
    if name == "cfg2":
        return make_splitkv_plan(spec, sm_count, num_splits=2)
    return make_b200_plan(spec, sm_count)


# ---------------------------------------------------------------- CPU legs
def cpu_sample_rows(name):
    return {"cfg1": 4, "cfg2": 16, "cfg3": 8, "cfg4": 16, "cfg5": 2}[name]


def cpu_sample_cap(name):
    return 65536 if name == "cfg5" else None


def blas_info():
    """The BLAS library NumPy uses (the CPU baseline's matrix products)."""
    try:
        import numpy as np
        deps = np.show_config(mode="dicts").get("Build Dependencies", {})
        blas = deps.get("blas", {})
        return f"{blas.get('name', 'unknown')} {blas.get('version', '')}".strip()
    except Exception as exc:  # depends on how NumPy was built
        return f"unknown ({type(exc).__name__})"


def run_cpu(name, steps, warmup, seconds=None):
    """Time the oracle port on host cores; returns (GB/s, cores, sample, s/pass, passes)."""
    from oracle import cpu_runner
    sample = cpu_runner.build_sample(name, cpu_sample_rows(name), max_tokens=cpu_sample_cap(name))
    runner = cpu_runner.Runner(sample)
    try:
        for _ in range(warmup):
            runner.run_once()
        times = []
        t_end = None if seconds is None else time.perf_counter() + seconds
        while True:
            times.append(runner.run_once())
            if seconds is None and len(times) >= steps:
                break
            if seconds is not None and time.perf_counter() >= t_end:
                break
        per_pass = sum(times) / len(times)
        return (sample.kv_bytes / per_pass / 1e9, runner.workers, sample.description,
                per_pass, len(times))
    finally:
        runner.close()
        cpu_runner.release()


def cpu_line(gbs, cores, desc):
    """The cpu_baseline object: the oracle port on `cores` single-threaded BLAS workers."""
    return {"value": round(gbs, 4), "unit": UNIT, "cores": cores, "kind": "port",
            "sample": desc, "blas": blas_info(), "blas_threads_per_worker": 1,
            "workers": cores}


# ---------------------------------------------------------------- clocks
class ClockSampler:
    """nvidia-smi every 100 ms on a reader thread; samples carry arrival times."""

    QUERY = ("clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.hw_slowdown,"
             "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,"
             "clocks_event_reasons.sw_power_cap")
    REASONS = ("hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap")

    def __init__(self, index):
        self.index = index
        self.samples = []
        self.proc = None

    def start(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.index}", f"--query-gpu={self.QUERY}",
                 "--format=csv,noheader,nounits", "-lms", "100"],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except (OSError, FileNotFoundError):
            self.proc = None
            return self
        self.thread = threading.Thread(target=self._read, daemon=True)
        self.thread.start()
        return self

    def _read(self):
        for line in self.proc.stdout:
            self.samples.append((time.monotonic(), line.strip()))

    def stop(self):
        if self.proc is not None:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()

    def summary(self, windows):
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        sm, mx, reasons = [], None, set()
        for t, line in self.samples:
            if not any(t0 - 0.05 <= t <= t1 + 0.15 for t0, t1 in windows):
                continue
            f = [x.strip() for x in line.split(",")]
            try:
                sm.append(float(f[0]))
                mx = float(f[1])
            except (ValueError, IndexError):
                continue
            for name, val in zip(self.REASONS, f[3:7]):
                if val.lower() == "active":
                    reasons.add(name)
        sm.sort()
        return {"sm_mhz": sm[len(sm) // 2] if sm else None, "sm_max_mhz": mx,
                "samples": len(sm), "reasons": sorted(reasons)}


def gpu_sharing(index):
    """Read-only check for other processes computing on this GPU (nvidia-smi).

    Returns {"gpu_shared": bool or None, "foreign_compute_apps": n or None};
    None when the query is unavailable (no nvidia-smi, or a PID namespace
    hides the processes).
    """
    try:
        uuid = subprocess.run(["nvidia-smi", f"--id={index}", "--query-gpu=uuid",
                               "--format=csv,noheader"], capture_output=True, text=True,
                              timeout=20).stdout.strip()
        apps = subprocess.run(["nvidia-smi", "--query-compute-apps=pid,gpu_uuid",
                               "--format=csv,noheader"], capture_output=True, text=True,
                              timeout=20)
    except (OSError, subprocess.SubprocessError):
        return {"gpu_shared": None, "foreign_compute_apps": None}
    if apps.returncode != 0 or not uuid:
        return {"gpu_shared": None, "foreign_compute_apps": None}
    mine, foreign = os.getpid(), 0
    for line in apps.stdout.splitlines():
        parts = [p.strip() for p in line.split(",")]
        if len(parts) >= 2 and parts[1] == uuid and parts[0].isdigit() and int(parts[0]) != mine:
            foreign += 1
    return {"gpu_shared": foreign > 0, "foreign_compute_apps": foreign}


# ---------------------------------------------------------------- helpers
def measured_peak():
    path = ROOT / "MEASURED_PEAKS.json"
    if path.exists():
        data = json.loads(path.read_text())
        return float(data["hbm_gbs"]), "measured (MEASURED_PEAKS.json hbm_gbs)"
    return 6650.0, "fallback 6.65 TB/s"


def committed_traffic(workload, kernel, kv_bytes):
    """Per-launch DRAM bytes from the ncu summary committed under profiles/
    (line ``traffic[workload][kernel]: BYTES of KV_BYTES``), scaled by the KV
    bytes when this launch reads a different amount than the captured one."""
    for path in sorted((ROOT / "profiles").glob("*.md")):
        m = re.search(rf"^traffic\[{re.escape(workload)}\]\[{re.escape(kernel)}\]:\s*(\d+)"
                      rf"(?:\s+of\s+(\d+))?", path.read_text(), re.M)
        if m:
            src = f"committed ncu summary profiles/{path.name}"
            traffic, captured = int(m.group(1)), int(m.group(2) or 0)
            if captured and captured != kv_bytes:
                traffic = int(traffic * kv_bytes / captured)
                src += f" (scaled from {captured} KV bytes)"
            return traffic, src
    return None, None


def reference_line(args):
    gbs, cores, desc, per_pass, n = run_cpu(args.config, args.steps, args.warmup)
    return {"metric": METRIC, "value": round(gbs, 4), "unit": UNIT, "impl": "reference",
            "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": round(per_pass * 1e3, 3), "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "f32 (bf16-valued inputs)",
            "data": "synthetic (seeded, NumPy)",
            "config": {"workload": args.config, "sample": desc},
            "cpu_baseline": cpu_line(gbs, cores, desc),
            "e2e": {"value": round(gbs, 4), "unit": UNIT, "h2d_bytes_per_step": 0,
                    "d2h_bytes_per_step": 0}}


def exchange_micro(reps=20, steps=20):
    """Context-parallel combine alone on every rank, graph-timed, max over ranks:
    rows = B*Hq merged over `splits` local partitions, then across the ranks."""
    import torch
    import torch.distributed as dist
    from paged_decode import ops, parallel
    local = int(os.environ["LOCAL_RANK"])
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=60), device_id=dev)
    rank, world = dist.get_rank(), dist.get_world_size()

    def timed(fn):
        side = torch.cuda.Stream(dev)
        side.wait_stream(torch.cuda.current_stream(dev))
        with torch.cuda.stream(side):
            for _ in range(3):
                fn()
        torch.cuda.current_stream(dev).wait_stream(side)
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph):
            for _ in range(steps):
                fn()
        graph.replay()
        torch.cuda.synchronize(dev)
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        dist.barrier()
        torch.cuda.synchronize(dev)
        e0.record()
        for _ in range(reps):
            graph.replay()
        e1.record()
        torch.cuda.synchronize(dev)
        t = torch.tensor([e0.elapsed_time(e1) * 1e3 / (reps * steps)], device=dev,
                         dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        del graph
        return round(t.item(), 2)

    # (rows, local splits, head_dim): config 5 at 64k / 524k tokens per row,
    # a wide batch, and the config-3 geometry.
    for rows, splits, d in [(128, 19, 128), (128, 64, 128), (1024, 8, 128), (32, 40, 256)]:
        gen = torch.Generator(device=dev).manual_seed(rank + 1)
        partial = torch.randn(rows, splits, d, device=dev, generator=gen)
        lse = torch.randn(rows, splits, device=dev, generator=gen)
        out = torch.empty(rows, d, dtype=torch.bfloat16, device=dev)
        layout = parallel.ExchangeLayout(rows, d, world)
        send = torch.zeros(layout.block, device=dev)
        gathered = torch.zeros(world * layout.block, device=dev)
        sp, sl = layout.send_views(send)
        lm = ops.merge_args(partial, lse, rows=rows, parts=splits, head_dim=d,
                            row_stride=splits * d, part_stride=d, lse_row_stride=splits,
                            lse_part_stride=1, out_partial=sp, out_lse=sl)
        rs, ps, lrs, lps = layout.merge_strides()
        gm = ops.merge_args(gathered, gathered[layout.lse_offset:], rows=rows, parts=world,
                            head_dim=d, row_stride=rs, part_stride=ps, lse_row_stride=lrs,
                            lse_part_stride=lps, out=out)

        def nccl_path():
            ops.lse_merge(lm, dev)
            dist.all_gather_into_tensor(gathered, send)
            ops.lse_merge(gm, dev)

        peers = parallel.PeerExchange(rows, d, dev)
        ea = ops.exchange_args(partial, lse, rows=rows, parts=splits, head_dim=d, rank=rank,
                               world=world, buffers=peers.ptrs, out=out)
        line = {"rows": rows, "splits": splits, "head_dim": d, "world": world,
                "local_merge_us": timed(lambda: ops.lse_merge(lm, dev)),
                "all_gather_us": timed(lambda: dist.all_gather_into_tensor(gathered, send)),
                "global_merge_us": timed(lambda: ops.lse_merge(gm, dev)),
                "nccl_path_us": timed(nccl_path),
                "p2p_exchange_us": timed(lambda: ops.exchange_merge(ea, dev))}
        torch.cuda.synchronize(dev)
        line["fault_word"] = ops.read_fault()
        peers.close()
        if rank == 0:
            print(json.dumps(line), flush=True)
    dist.barrier()
    dist.destroy_process_group()


# ---------------------------------------------------------------- multi-GPU parity
def full_decode(w, tokens_per_split, splits, kernel, device, flags=0):
    """One-GPU decode of a whole batch with the given partitioning: the
    parity reference of the sharded modes (same kernels and bounds per row)."""
    import torch
    from paged_decode import ops
    b, hq, d = w.q.shape
    out = torch.empty(b, hq, d, dtype=torch.bfloat16, device=device)
    partial = torch.empty(b, hq, splits, d, device=device)
    lse = torch.empty(b, hq, splits, device=device)
    ops.paged_decode(ops.decode_args(w.q, w.k, w.v, w.table, w.lengths, scale=w.scale,
                                     tokens_per_split=tokens_per_split, splits=splits,
                                     protocol=ops.PROTOCOL_LSE, kernel=kernel, out=out,
                                     partial=partial, lse=lse, flags=flags), device)
    torch.cuda.synchronize(device)
    return out


def check_parity(mode, out, full, plan, shards, kernel, world, rank, device):
    """Gather every rank's output and compare it on rank 0 with a one-GPU
    decode of the global batch; every rank takes the same collective steps."""
    import torch
    import torch.distributed as dist
    ok, err = True, 0.0
    if mode == "context":
        if rank == 0:
            from paged_decode import ops
            from paged_decode.splitkv_plan import make_b200_plan
            g = make_b200_plan(full.spec, ops.sm_count(device))
            want = full_decode(full, g.tokens_per_split, g.splits, kernel, device)  # fixed bounds
            err = float((out.float() - want.float()).abs().max().item())
            ok = err <= 2.0 ** -7 and bool(torch.isfinite(out.float()).all().item())
        reference = "one-GPU decode of the global batch (B200 plan), max-abs 2^-7"
    elif mode == "head":
        gathered = torch.empty((world,) + tuple(out.shape), dtype=out.dtype, device=device)
        dist.all_gather_into_tensor(gathered, out.contiguous())
        if rank == 0:
            got = torch.cat(list(gathered), dim=1)
            from paged_decode.splitkv_plan import launch_partitioning
            tokens, bounds = launch_partitioning(plan)
            want = full_decode(full, tokens, plan.splits, kernel, device, flags=bounds)
            ok = torch.equal(got, want)
            err = float((got.float() - want.float()).abs().max().item())
        reference = "one-GPU decode of the global batch, same partitions: bit-exact"
    elif mode == "batch":
        most = max(len(s) for s in shards)
        pad = torch.zeros((most,) + tuple(out.shape[1:]), dtype=out.dtype, device=device)
        pad[:out.shape[0]] = out
        gathered = torch.empty((world, most) + tuple(out.shape[1:]), dtype=out.dtype,
                               device=device)
        dist.all_gather_into_tensor(gathered, pad)
        if rank == 0:
            got = torch.empty_like(full.q)
            for r, rows in enumerate(shards):
                got[torch.as_tensor(rows, device=device)] = gathered[r, :len(rows)]
            from paged_decode.splitkv_plan import launch_partitioning
            tokens, bounds = launch_partitioning(plan)
            want = full_decode(full, tokens, plan.splits, kernel, device, flags=bounds)
            ok = torch.equal(got, want)
            err = float((got.float() - want.float()).abs().max().item())
        reference = "one-GPU decode of the global batch, same partitions: bit-exact"
    else:  # replica: independent batches, nothing to gather
        return {"mode": mode, "ok": True, "reference": "none (independent batches)"}
    flag = torch.tensor([1 if ok else 0], device=device)
    dist.broadcast(flag, 0)
    return {"mode": mode, "ok": bool(flag.item()), "max_abs_err": err, "reference": reference}


# ---------------------------------------------------------------- main
def main(argv=None):
    args = parse_args(argv)
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))

    if args.impl == "reference":
        if rank == 0:
            print(json.dumps(reference_line(args)), flush=True)
        return 0
    if args.sweep:
        sweep()
        return 0
    if args.exchange_micro:
        if world < 2:
            print(json.dumps({"exchange_micro": "needs torchrun with 2 or more ranks"}))
            return 0
        exchange_micro()
        return 0

    mode = resolve_mode(args, world)
    if args.append and mode == "context":
        raise SystemExit("--append is not supported with --mode context")

    # CPU baseline first (rank 0, N = 1): its spawn pool starts before any CUDA work.
    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        gbs, cores, desc, per_pass, n = run_cpu(args.config, 1, 1, seconds=args.cpu_seconds)
        cpu = cpu_line(gbs, cores, f"{desc}; {n} passes, {per_pass * 1e3:.1f} ms each")

    import torch
    import torch.distributed as dist
    from paged_decode import ops, parallel
    from paged_decode.matched_splitkv import allocate_matched_resources, matched_decode
    from paged_decode.spec import DecodeSpec
    from paged_decode.workloads import make_workload

    if world > 1:
        torch.cuda.set_device(local)
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                device_id=torch.device("cuda", local))
    device = torch.device("cuda", local if world > 1 else 0)
    torch.cuda.set_device(device)
    sharing = gpu_sharing(device.index)
    clocks = ClockSampler(device.index).start()
    windows = []
    sms = ops.sm_count(device)

    def max_over_ranks(x):
        if world == 1:
            return x
        t = torch.tensor([x], device=device, dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    strong = mode in ("head", "batch", "context")
    stream = torch.cuda.current_stream(device)
    K = args.steps
    seed_rank = rank if mode == "replica" else 0

    # ---- this rank's work --------------------------------------------------
    glob = make_workload(args.config, device=device, batch=args.batch, context=args.context,
                         rank=seed_rank)
    gspec = glob.spec
    launch_kv_bytes = glob.kv_bytes  # one decode of the global workload
    job_bytes = launch_kv_bytes * (world if mode == "replica" else 1)
    shards = None
    if mode == "batch":
        shards = parallel.batch_shards(glob.lengths.cpu().tolist(), world)
        if not all(shards):
            raise SystemExit("batch mode needs at least one row per rank")
    # Rank 0 keeps the global batch for the parity check (a shallow copy: the
    # tensors survive when the workload below is cut to this rank's share).
    full = copy.copy(glob) if world > 1 and rank == 0 and not args.no_parity else None

    def local_workload(seed):
        """This rank's tensors for input copy `seed` (copy 0 is the global batch)."""
        w = glob if seed == 0 else make_workload(args.config, device=device, batch=args.batch,
                                                 context=args.context, rank=seed_rank, seed=seed)
        if mode == "head":
            w.q, w.k, w.v = parallel.shard_head_pool(w.k, w.v, w.q, rank, world,
                                                     gspec.num_heads, gspec.num_kv_heads)
            w.spec = DecodeSpec(gspec.max_batch, gspec.num_heads // world,
                                gspec.num_kv_heads // world, gspec.head_dim,
                                gspec.max_context_len)
        elif mode == "batch":
            rows = shards[rank]
            w.k, w.v, w.table, w.lengths = parallel.shard_batch_pool(w.k, w.v, w.table,
                                                                     w.lengths, rows)
            w.q = w.q[torch.as_tensor(rows, device=device)].contiguous()
            w.spec = DecodeSpec(len(rows), gspec.num_heads, gspec.num_kv_heads, gspec.head_dim,
                                gspec.max_context_len)
        return w

    cp = None
    if mode == "context":
        w0 = copy.copy(glob)
        w0.k, w0.v, w0.table = parallel.shard_context_pool(glob.k, glob.v, glob.table, rank,
                                                           world)
        glob = None
        torch.cuda.empty_cache()
        cp = parallel.ContextParallelDecode(gspec, device, kernel=args.kernel,
                                            local_splits=args.splits or 0,
                                            exchange=args.exchange)
        cp(w0.q, w0.k, w0.v, w0.table, w0.lengths)
        plan = cp.plan
        local_bytes = int(cp.local_len.to(torch.int64).sum().item()) * gspec.num_kv_heads * \
            gspec.head_dim * 4
        copies, wls, out_slots = 1, [w0], None

        def decode_call(w, slot=0):
            return cp(w.q, w.k, w.v, w.table, w.lengths, scale=w.scale)

        part_args = [cp._launch_args(w0.q, w0.k, w0.v, w0.table, w0.scale)[0]]
        out_buf = cp.out
    else:
        w0 = local_workload(0)
        pool_bytes = w0.k.numel() * 2 * 2
        copies = 1 if (pool_bytes >= 2 * L2_BYTES or args.hot) else \
            min(64, math.ceil(2 * L2_BYTES / pool_bytes))
        wls = [w0] + [local_workload(c) for c in range(1, copies)]
        if mode == "batch":
            # One partition size on every rank (the plan of the largest shard),
            # so each row's bounds equal the one-GPU decode's.
            most = max(len(s) for s in shards)
            plan = config_plan(args.config, args, DecodeSpec(most, gspec.num_heads,
                                                             gspec.num_kv_heads, gspec.head_dim,
                                                             gspec.max_context_len), sms)
        else:
            plan = config_plan(args.config, args, w0.spec, sms)
        res = allocate_matched_resources(w0.spec, device, plan=plan)
        local_bytes = w0.kv_bytes
        # A second resource set lets step i+1 compute while step i's output
        # is still being copied to the host.
        out_slots = [res, allocate_matched_resources(w0.spec, device, plan=plan)]
        if args.append:
            from paged_decode.kvcache import append_decode_kv
            for w in wls:
                gen = torch.Generator(device=device).manual_seed(99)
                shape = (w.spec.max_batch, w.spec.num_kv_heads, w.spec.head_dim)
                w.k_new = torch.randn(shape, generator=gen, device=device).to(torch.bfloat16)
                w.v_new = torch.randn(shape, generator=gen, device=device).to(torch.bfloat16)
                w.len0 = w.lengths.clone()

        def decode_call(w, slot=0):
            if args.append:
                append_decode_kv(w.k_new, w.v_new, w.k, w.v, w.table, w.lengths)
            return matched_decode(w.q, w.k, w.v, w.table, w.lengths,
                                  resources=out_slots[slot], scale=w.scale, kernel=args.kernel)

        from paged_decode.splitkv_plan import launch_partitioning
        tokens, bounds = launch_partitioning(plan)
        part_args = [ops.decode_args(w.q, w.k, w.v, w.table, w.lengths, scale=w.scale,
                                     tokens_per_split=tokens, splits=plan.splits,
                                     protocol=ops.PROTOCOL_LSE, kernel=args.kernel, out=res.out,
                                     partial=res.partials, lse=res.lse, counters=res.counters,
                                     flags=ops.FLAG_DYNAMIC | bounds) for w in wls]
        out_buf = res.out

    def step(i):
        if args.append and i < copies:  # each window starts from the same lengths
            wls[i].lengths.copy_(wls[i].len0)
        decode_call(wls[i % copies])

    def partition_only(i):
        ops.partition(part_args[i % copies], device)

    for i in range(max(3, args.warmup)):
        step(i)
        partition_only(i)
    torch.cuda.synchronize(device)

    # ---- multi-GPU parity: every rank's output against one GPU --------------
    parity = None
    if world > 1 and not args.no_parity and not args.append:
        out = decode_call(wls[0]).clone()
        torch.cuda.synchronize(device)
        parity = check_parity(mode, out, full, plan, shards, args.kernel, world, rank, device)
        del out
    full = None
    torch.cuda.empty_cache()

    def capture(fn, n):
        side = torch.cuda.Stream(device)
        side.wait_stream(stream)
        with torch.cuda.stream(side):
            fn(0)
        stream.wait_stream(side)
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph):
            for i in range(n):
                fn(i)
        graph.replay()
        torch.cuda.synchronize(device)
        return graph

    def timed(graph, seconds, record=True):
        """Replay a graph in back-to-back windows; returns (ms, max over ranks; replays)."""
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        graph.replay()
        e1.record(stream)
        torch.cuda.synchronize(device)
        reps = max(1, min(500, math.ceil(seconds * 1e3 / max(e0.elapsed_time(e1), 1e-3))))
        reps = int(max_over_ranks(reps))
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize(device)
        t0 = time.monotonic()
        e0.record(stream)
        for _ in range(reps):
            graph.replay()
        e1.record(stream)
        torch.cuda.synchronize(device)
        if record:
            windows.append((t0, time.monotonic()))
        return max_over_ranks(e0.elapsed_time(e1)), reps

    step_graph = capture(step, K)
    total_ms, reps = timed(step_graph, args.window_seconds)
    del step_graph
    ms_per_step = total_ms / (reps * K)
    value = job_bytes / (ms_per_step / 1e3) / 1e9

    part_graph = capture(partition_only, K)
    part_total, part_reps = timed(part_graph, args.window_seconds / 2)
    del part_graph
    part_ms = part_total / (part_reps * K)
    peak, peak_src = measured_peak()
    achieved = local_bytes / (part_ms / 1e3) / 1e9
    group = gspec.num_heads // gspec.num_kv_heads
    kernel_name = "mma" if (args.kernel == "mma" or (args.kernel == "auto" and group >= 3)) \
        else "simt"
    traffic, traffic_src = committed_traffic(args.config, kernel_name, launch_kv_bytes)
    if traffic is not None and strong:
        global_bytes = job_bytes
        traffic = int(traffic * local_bytes / max(global_bytes, 1))  # this rank's share
        traffic_src += " (scaled to this rank's share of the batch)"

    # Unroll convergence: per-step time of 32- and 128-step graphs.
    conv = {}
    for n in (32, 128):
        g = capture(step, n)
        tot, r = timed(g, 0.15, record=False)
        conv[n] = tot * 1e3 / (r * n)
        del g
    convergence = abs(conv[32] - conv[128]) / conv[128]

    # e2e: public API with host buffers.  Each step's inputs (q, block table,
    # lengths) sit in one pinned staging buffer, copied to the device with one
    # H2D copy (the workload tensors are views into its device twin, as a
    # serving engine stages them); the output is copied back to pinned memory.
    # As in a serving loop, copies run on their own streams, double-buffered:
    # step i+1's inputs are copied in and step i's output is copied out while
    # the next step computes.  Every copy of every step is inside the timed
    # region (the end event waits for the last copy out).
    def staged(w):
        parts = [w.q, w.table, w.lengths]
        sizes = [t.numel() * t.element_size() for t in parts]
        offs, total = [], 0
        for n in sizes:
            offs.append(total)
            total += -(-n // 16) * 16
        dev = torch.empty(total, dtype=torch.uint8, device=device)
        views = [dev[o:o + n].view(t.dtype).view(t.shape) for o, n, t in zip(offs, sizes, parts)]
        for view, t in zip(views, parts):
            view.copy_(t)
        w.q, w.table, w.lengths = views
        host = torch.empty(total, dtype=torch.uint8).pin_memory()
        host.copy_(dev)
        return dev, host

    e2e_wls = list(wls)
    if len(e2e_wls) < 2:  # a second staging set for the same workload
        twin = copy.copy(wls[0])
        twin.q, twin.table, twin.lengths = (wls[0].q.clone(), wls[0].table.clone(),
                                            wls[0].lengths.clone())
        e2e_wls.append(twin)
    stages = [staged(w) for w in e2e_wls]
    n_stage = len(stages)
    hout = [torch.empty(out_buf.shape, dtype=out_buf.dtype).pin_memory() for _ in range(2)]
    dout = None if out_slots is not None else [torch.empty_like(out_buf) for _ in range(2)]
    h2d = stages[0][0].numel()
    d2h = hout[0].numel() * hout[0].element_size()
    copy_in, copy_out = torch.cuda.Stream(device), torch.cuda.Stream(device)
    ev = lambda: torch.cuda.Event()  # noqa: E731
    in_ready, stage_free = [ev() for _ in range(n_stage)], [ev() for _ in range(n_stage)]
    computed, out_free = [ev(), ev()], [ev(), ev()]

    # The API call of every (staging set, output slot) pair the loop uses,
    # warmed up eagerly and captured once (the graph contract of the API).
    pairs = sorted({(i % n_stage, i % 2) for i in range(K + 3)})
    side = torch.cuda.Stream(device)
    side.wait_stream(stream)
    with torch.cuda.stream(side):
        for s, j in pairs:
            decode_call(e2e_wls[s], j)
    stream.wait_stream(side)
    torch.cuda.synchronize(device)
    def capture_call(s, j):
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph):
            decode_call(e2e_wls[s], j)
        return graph

    e2e_graphs = {pair: capture_call(*pair) for pair in pairs}
    torch.cuda.synchronize(device)

    def e2e_step(i):
        s, j = i % n_stage, i % 2
        dev, host = stages[s]
        copy_in.wait_event(stage_free[s])           # step i - n_stage has read it
        with torch.cuda.stream(copy_in):
            dev.copy_(host, non_blocking=True)
        in_ready[s].record(copy_in)
        stream.wait_event(in_ready[s])
        stream.wait_event(out_free[j])               # step i - 2's output is on the host
        e2e_graphs[(s, j)].replay()
        out = out_slots[j].out if out_slots is not None else out_buf
        if dout is not None:
            dout[j].copy_(out, non_blocking=True)
            out = dout[j]
        stage_free[s].record(stream)
        computed[j].record(stream)
        copy_out.wait_event(computed[j])
        with torch.cuda.stream(copy_out):
            hout[j].copy_(out, non_blocking=True)
        out_free[j].record(copy_out)

    for i in range(3):
        e2e_step(i)
    torch.cuda.synchronize(device)
    if world > 1:
        dist.barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    copy_in.wait_stream(stream)  # the first copy in starts after the start event
    for i in range(K):
        e2e_step(i)
    stream.wait_stream(copy_out)
    e1.record(stream)
    torch.cuda.synchronize(device)
    e2e_ms = max_over_ranks(e0.elapsed_time(e1))
    e2e_value = job_bytes * K / (e2e_ms / 1e3) / 1e9
    e2e_graphs.clear()  # graphs that hold NCCL calls must go before the process group
    fault = ops.read_fault()
    clocks.stop()

    if world > 1:  # shared if any rank's GPU is
        flag = torch.tensor([1 if sharing["gpu_shared"] else 0], device=device)
        dist.all_reduce(flag, op=dist.ReduceOp.MAX)
        if sharing["gpu_shared"] is not None:
            sharing["gpu_shared"] = bool(flag.item())

    if rank == 0:
        parallelism = {
            "single": "single GPU",
            "head": f"KV-head-sharded x{world} (no collective on the data path)",
            "batch": f"batch-sharded x{world}: token-balanced rows of one batch (no collective)",
            "replica": f"independent batch per GPU x{world}",
            "context": f"context-parallel x{world} (" + (
                "one peer-memory exchange kernel over NVLink" if args.exchange == "p2p"
                else "NCCL all-gather + LSE merge") + ")",
        }[mode]
        line = {
            "metric": METRIC, "value": round(value, 2), "unit": UNIT, "n_gpus": world,
            "steps": K, "warmup": args.warmup, "ms_per_step": round(ms_per_step, 5),
            "us_per_call": round(ms_per_step * 1e3, 3), "higher_is_better": True,
            "scaling": "strong" if strong else "weak", "vs_baseline": None,
            "dtype": "bf16 in, fp32 softmax/accumulate",
            "data": "synthetic (seeded N(0,1) BF16 q/K/V, shuffled page pool)",
            "config": {"workload": args.config, "batch": gspec.max_batch,
                       "num_heads": gspec.num_heads, "num_kv_heads": gspec.num_kv_heads,
                       "head_dim": gspec.head_dim, "context": gspec.max_context_len,
                       "splits": plan.splits, "tokens_per_split": plan.tokens_per_split,
                       "balanced_partitions": bool(plan.balanced),
                       "kv_bytes_per_step": job_bytes, "kernel": kernel_name,
                       "mode": mode, "parallelism": parallelism,
                       "timing": f"{K}-step CUDA graph replayed {reps}x back to back",
                       "step": ("KV append (lengths += 1 on the device) + decode; KV bytes "
                                "counted at the starting lengths" if args.append else "decode"),
                       "l2": ("inputs larger than L2 (KV pool >> 126 MB)"
                              if copies == 1 and not args.hot else
                              "hot: one input copy reused every step (L2-resident)" if args.hot
                              else f"{copies} independent input copies rotated (> 2x L2)")},
            "roofline": {"bound": "hbm", "achieved": round(achieved, 2), "peak": peak,
                         "unit": "GB/s", "frac": round(achieved / peak, 4),
                         "traffic": traffic, "kernel_us": round(part_ms * 1e3, 3),
                         "bytes_per_launch": local_bytes, "peak_source": peak_src,
                         "traffic_source": traffic_src},
            "cpu_baseline": cpu,
            "e2e": {"value": round(e2e_value, 2), "unit": UNIT, "h2d_bytes_per_step": h2d,
                    "d2h_bytes_per_step": d2h, "us_per_call": round(e2e_ms / K * 1e3, 3),
                    "api": ("paged_decode.parallel.ContextParallelDecode" if mode == "context"
                            else "paged_decode.matched_splitkv.matched_decode")
                           + " (captured once, replayed per step)"},
            "convergence": {"us_per_step_unroll32": round(conv[32], 3),
                            "us_per_step_unroll128": round(conv[128], 3),
                            "delta": round(convergence, 4),
                            "ok": convergence <= CONVERGENCE_LIMIT},
            "parity": parity,
            "gpu_shared": sharing["gpu_shared"],
            "foreign_compute_apps": sharing["foreign_compute_apps"],
            # Own kernels per step: partition + merge; context mode adds the
            # local merge (nccl) or replaces both merges by the exchange (p2p).
            "gpu_launches": (((3 if args.exchange == "nccl" else 2) if mode == "context" else 2)
                             + (1 if args.append else 0)) * K * reps,
            "clocks": clocks.summary(windows),
            "fault_word": fault,
        }
        print(json.dumps(line), flush=True)
    if cp is not None:
        cp.close()
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()
    return 0


if __name__ == "__main__":
    sys.exit(main())
