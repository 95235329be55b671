"""Benchmark of the paged decode-attention operator (one JSON line on rank 0).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--config cfg2] [--impl ours|reference]

A step is one decode call over one batch of the chosen BASELINE config (inputs
resident in HBM, larger than L2).  Default workload: config 2 (MHA D=64,
B=64, Hq=Hkv=32, 2048 tokens per row, 1024-token split-K partitions + LSE
merge), the single-GPU config the metric is quoted on.

* ``value``: KV GB/s = algorithmic KV bytes / device time, for K steps replayed
  from a CUDA graph between CUDA events (max over ranks); ``us_per_call`` beside it.
* ``e2e``: the same metric through the public API (``matched_decode``) with
  host buffers: each step copies q / block table / lengths from pinned host
  memory, decodes, and reads the output back.  The KV cache is resident
  device state, as in serving.
* ``roofline``: the partition kernel alone (CUDA events on its stream) against
  the measured HBM copy bandwidth in MEASURED_PEAKS.json; ``traffic`` is the
  per-launch DRAM bytes of the ncu summary committed under profiles/.
* ``cpu_baseline``: the NumPy oracle (the reference's CPU algorithm) over a
  bounded sample of the same workload on the host cores (rank 0, N = 1).
* ``--impl reference``: that CPU implementation alone, on all host cores.

Multi-GPU (torchrun): every rank decodes its own independent batch (batch
sharding, no collective on the data path); ``value`` = all ranks' bytes / the
slowest rank's time ("scaling": "weak").
"""
import argparse
import datetime
import json
import os
import re
import subprocess
import sys
import time
from pathlib import Path

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT / "paged-decode-lab_b200"))
sys.path.insert(0, str(ROOT))

METRIC = "decode-attn achieved KV HBM GB/s"
UNIT = "GB/s"


def parse_args():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=("ours", "reference"), default="ours")
    ap.add_argument("--config", default="cfg2", choices=("cfg1", "cfg2", "cfg3", "cfg4", "cfg5"))
    ap.add_argument("--batch", type=int, default=None)
    ap.add_argument("--context", type=int, default=None)
    ap.add_argument("--splits", type=int, default=None, help="matched plan split count")
    ap.add_argument("--kernel", default="auto", choices=("auto", "simt", "mma"))
    ap.add_argument("--cpu-seconds", type=float, default=10.0)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    return ap.parse_args()


def config_splits(name, args):
    """Split count of the matched plan per config (None = the plan's own heuristic)."""
    if args.splits is not None:
        return args.splits
    return {"cfg1": 1, "cfg2": 2, "cfg3": 0, "cfg4": 0, "cfg5": 16}[name]


# ---------------------------------------------------------------- CPU legs
def cpu_sample_rows(name):
    return {"cfg1": 4, "cfg2": 16, "cfg3": 8, "cfg4": 16, "cfg5": 2}[name]


def cpu_sample_cap(name):
    return 65536 if name == "cfg5" else None


def run_cpu(name, steps, warmup, seconds=None):
    """Time the oracle port on host cores; returns (GB/s, cores, sample text, s/step)."""
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
            if seconds is not None and time.perf_counter() >= t_end and len(times) >= 1:
                break
        per_step = sum(times) / len(times)
        return (sample.kv_bytes / per_step / 1e9, runner.workers, sample.description,
                per_step, len(times))
    finally:
        runner.close()
        cpu_runner.release()


# ---------------------------------------------------------------- clocks
class ClockSampler:
    QUERY = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
             "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
             "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, index):
        self.index = index
        self.proc = None
        self.path = Path(os.environ.get("TMPDIR", "/tmp")) / f"pdl_clocks_{os.getpid()}.csv"

    def __enter__(self):
        try:
            self.fh = open(self.path, "w")
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.index}", f"--query-gpu={self.QUERY}",
                 "--format=csv,noheader,nounits", "-lms", "100"],
                stdout=self.fh, stderr=subprocess.DEVNULL)
            time.sleep(0.3)
        except (OSError, FileNotFoundError):
            self.proc = None
        return self

    def __exit__(self, *exc):
        if self.proc is not None:
            time.sleep(0.2)
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()
            self.fh.close()

    def summary(self):
        if self.proc is None or not self.path.exists():
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        rows = [r.split(",") for r in self.path.read_text().strip().splitlines() if r.strip()]
        self.path.unlink(missing_ok=True)
        sm, mx, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for r in rows:
            try:
                sm.append(float(r[1]))
                mx = float(r[2])
                for name, val in zip(names, r[5:9]):
                    if val.strip().lower() == "active":
                        reasons.add(name)
            except (ValueError, IndexError):
                continue
        sm.sort()
        return {"sm_mhz": sm[len(sm) // 2] if sm else None, "sm_max_mhz": mx,
                "samples": len(sm), "reasons": sorted(reasons)}


# ---------------------------------------------------------------- helpers
def measured_peak():
    path = ROOT / "MEASURED_PEAKS.json"
    if path.exists():
        data = json.loads(path.read_text())
        return float(data["hbm_gbs"]), "measured (MEASURED_PEAKS.json hbm_gbs)"
    return 6650.0, "fallback 6.65 TB/s"


def committed_traffic(workload, kernel):
    """Per-launch DRAM bytes from the ncu summary committed under profiles/."""
    for path in sorted((ROOT / "profiles").glob("*.md")):
        text = path.read_text()
        m = re.search(rf"^traffic\[{re.escape(workload)}\]\[{re.escape(kernel)}\]:\s*(\d+)",
                      text, re.M)
        if m:
            return int(m.group(1)), path.name
    return None, None


def main():
    args = parse_args()
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))

    if args.impl == "reference":
        if rank != 0:
            return 0
        gbs, cores, desc, per_step, n = run_cpu(args.config, args.steps, args.warmup)
        line = {"metric": METRIC, "value": round(gbs, 4), "unit": UNIT, "impl": "reference",
                "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
                "ms_per_step": round(per_step * 1e3, 3), "higher_is_better": True,
                "scaling": "weak", "vs_baseline": None, "dtype": "f32 (bf16-valued inputs)",
                "data": "synthetic (seeded, NumPy)",
                "config": {"workload": args.config, "sample": desc},
                "cpu_baseline": {"value": round(gbs, 4), "unit": UNIT, "cores": cores,
                                 "kind": "port", "sample": desc},
                "e2e": {"value": round(gbs, 4), "unit": UNIT, "h2d_bytes_per_step": 0,
                        "d2h_bytes_per_step": 0}}
        print(json.dumps(line), flush=True)
        return 0

    import torch
    import torch.distributed as dist
    from paged_decode import ops
    from paged_decode.matched_splitkv import allocate_matched_resources, matched_decode
    from paged_decode.workloads import make_workload

    if world > 1:
        torch.cuda.set_device(local)
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                device_id=torch.device("cuda", local))
    device = torch.device("cuda", local if world > 1 else 0)
    torch.cuda.set_device(device)

    # CPU baseline first (rank 0, N = 1): its spawn pool starts before heavy GPU work.
    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        gbs, cores, desc, per_step, n = run_cpu(args.config, 1, 1, seconds=args.cpu_seconds)
        cpu = {"value": round(gbs, 4), "unit": UNIT, "cores": cores, "kind": "port",
               "sample": f"{desc}; {n} passes, {per_step * 1e3:.1f} ms each"}

    wl = make_workload(args.config, device=device, batch=args.batch, context=args.context,
                       rank=rank)
    q, k, v, table, lens = wl.args()
    res = allocate_matched_resources(wl.spec, device, num_splits=config_splits(args.config, args))
    kv_bytes = wl.kv_bytes
    stream = torch.cuda.current_stream(device)

    def step():
        matched_decode(q, k, v, table, lens, resources=res, scale=wl.scale, kernel=args.kernel)

    for _ in range(max(3, args.warmup)):
        step()
    torch.cuda.synchronize(device)

    # value: K steps replayed from one captured graph.
    side = torch.cuda.Stream(device)
    side.wait_stream(stream)
    with torch.cuda.stream(side):
        step()
    stream.wait_stream(side)
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        step()
    graph.replay()
    torch.cuda.synchronize(device)
    if world > 1:
        dist.barrier()
    start, stop = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(device.index) as clocks:
        torch.cuda.synchronize(device)
        start.record(stream)
        for _ in range(args.steps):
            graph.replay()
        stop.record(stream)
        torch.cuda.synchronize(device)
    elapsed = start.elapsed_time(stop)
    if world > 1:
        t = torch.tensor([elapsed], device=device)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        elapsed = float(t.item())
    ms_per_step = elapsed / args.steps
    value = world * kv_bytes * args.steps / (elapsed / 1e3) / 1e9

    # roofline: the partition kernel alone.
    plan = res.plan
    part_args = ops.decode_args(q, k, v, table, lens, scale=wl.scale,
                                tokens_per_split=plan.tokens_per_split, splits=plan.splits,
                                protocol=ops.PROTOCOL_LSE, kernel=args.kernel, out=res.out,
                                partial=res.partials, lse=res.lse)
    for _ in range(3):
        ops.partition(part_args, device)
    reps = max(5, args.steps)
    torch.cuda.synchronize(device)
    start.record(stream)
    for _ in range(reps):
        ops.partition(part_args, device)
    stop.record(stream)
    torch.cuda.synchronize(device)
    part_ms = start.elapsed_time(stop) / reps
    peak, peak_src = measured_peak()
    achieved = kv_bytes / (part_ms / 1e3) / 1e9
    group = wl.spec.num_heads // wl.spec.num_kv_heads
    kernel_name = "mma" if (args.kernel == "mma" or (args.kernel == "auto" and group >= 8)) \
        else "simt"
    traffic, traffic_src = committed_traffic(args.config, kernel_name)

    # e2e: public API with host buffers (pinned), copies inside the timed region.
    hq = torch.empty_like(q, device="cpu").pin_memory()
    hq.copy_(q)
    htable = table.cpu().pin_memory()
    hlens = lens.cpu().pin_memory()
    hout = torch.empty(res.out.shape, dtype=res.out.dtype).pin_memory()
    h2d = hq.numel() * hq.element_size() + htable.numel() * 4 + hlens.numel() * 4
    d2h = hout.numel() * hout.element_size()

    def e2e_step():
        q.copy_(hq, non_blocking=True)
        table.copy_(htable, non_blocking=True)
        lens.copy_(hlens, non_blocking=True)
        out = matched_decode(q, k, v, table, lens, resources=res, scale=wl.scale,
                             kernel=args.kernel)
        hout.copy_(out, non_blocking=True)

    for _ in range(3):
        e2e_step()
    torch.cuda.synchronize(device)
    if world > 1:
        dist.barrier()
    start.record(stream)
    for _ in range(args.steps):
        e2e_step()
    stop.record(stream)
    torch.cuda.synchronize(device)
    e2e_ms = start.elapsed_time(stop)
    if world > 1:
        t = torch.tensor([e2e_ms], device=device)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        e2e_ms = float(t.item())
    e2e_value = world * kv_bytes * args.steps / (e2e_ms / 1e3) / 1e9
    fault = ops.read_fault()

    if rank == 0:
        line = {
            "metric": METRIC, "value": round(value, 2), "unit": UNIT, "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms_per_step, 5),
            "us_per_call": round(ms_per_step * 1e3, 3), "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "bf16 in, fp32 softmax/accumulate",
            "data": "synthetic (seeded N(0,1) BF16 q/K/V, shuffled page pool)",
            "config": {"workload": args.config, "batch": wl.spec.max_batch,
                       "num_heads": wl.spec.num_heads, "num_kv_heads": wl.spec.num_kv_heads,
                       "head_dim": wl.spec.head_dim, "context": wl.spec.max_context_len,
                       "splits": plan.splits, "tokens_per_split": plan.tokens_per_split,
                       "kv_bytes_per_step": kv_bytes, "kernel": kernel_name,
                       "parallelism": f"batch-sharded x{world}" if world > 1 else "single GPU",
                       "l2": "inputs larger than L2 (KV pool >> 126 MB); no flush needed"
                       if kv_bytes > 126e6 else "working set below L2 size"},
            "roofline": {"bound": "hbm", "achieved": round(achieved, 2), "peak": peak,
                         "unit": "GB/s", "frac": round(achieved / peak, 4),
                         "traffic": traffic, "kernel_us": round(part_ms * 1e3, 3),
                         "peak_source": peak_src, "traffic_source": traffic_src},
            "cpu_baseline": cpu,
            "e2e": {"value": round(e2e_value, 2), "unit": UNIT, "h2d_bytes_per_step": h2d,
                    "d2h_bytes_per_step": d2h, "us_per_call": round(e2e_ms / args.steps * 1e3, 3),
                    "api": "paged_decode.matched_splitkv.matched_decode"},
            "gpu_launches": 2 * args.steps,
            "clocks": clocks.summary(),
            "fault_word": fault,
        }
        print(json.dumps(line), flush=True)
    del graph
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()
    return 0


if __name__ == "__main__":
    sys.exit(main())
