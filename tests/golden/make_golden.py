"""Generate the golden fixtures by running the REFERENCE's own CPU code.

Run once, in a checkout that has the reference project available:

    python tests/golden/make_golden.py --reference-src <reference>/src

It imports the reference package ``paged_decode`` from that directory
(``reference.py``, ``spec.py``, ``splitkv_plan.py``; NumPy only), rebuilds the
seeded cases of ``cases.py`` and records the reference's outputs:

* ``golden_cases.npz`` -- dense / streaming / split outputs and per-partition
  (m, l, acc) -> (normalised partial, LSE) for every case;
* ``golden_plans.json`` -- ``make_splitkv_plan`` and ``DecodeSpec`` geometry
  for a grid of specs at 108 and 148 SMs.

The fixtures store outputs and input checksums only; inputs are rebuilt from
their seeds by ``cases.py``.  Nothing at test time reads the reference.
"""
import argparse
import os
import importlib
import json
import sys
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
sys.path.insert(0, str(HERE))
import cases  # noqa: E402


def load_reference(src):
    sys.path.insert(0, str(src))
    ref = importlib.import_module("paged_decode.reference")
    spec = importlib.import_module("paged_decode.spec")
    plan = importlib.import_module("paged_decode.splitkv_plan")
    return ref, spec, plan


def partitions_from_reference(ref, arrays, tokens, scale=None):
    """Per-partition (m, l, acc) from the reference's ``partial``; LSE = m + ln l."""
    q, k, v, table, lengths = arrays
    batch, heads, dim = q.shape
    group = heads // k.shape[2]
    scale = dim ** -0.5 if scale is None else scale
    splits = max(1, -(-int(table.shape[1] * 256) // tokens))
    partial = np.zeros((batch, heads, splits, dim), np.float32)
    lse = np.full((batch, heads, splits), -np.inf, np.float32)
    m_out = np.full((batch, heads, splits), -np.inf, np.float32)
    l_out = np.zeros((batch, heads, splits), np.float32)
    acc_out = np.zeros((batch, heads, splits, dim), np.float32)
    for b in range(batch):
        n = int(lengths[b])
        keys = ref.gather_kv(k, table[b], n)
        vals = ref.gather_kv(v, table[b], n)
        for p in range(splits):
            start, end = p * tokens, min((p + 1) * tokens, n)
            if start >= end:
                continue
            for h in range(heads):
                m, l, acc = ref.partial(q[b, h], keys[start:end, h // group],
                                        vals[start:end, h // group], scale)
                m_out[b, h, p], l_out[b, h, p], acc_out[b, h, p] = m, l, acc
                if l > 0:
                    partial[b, h, p] = acc / l
                    lse[b, h, p] = m + np.log(l)
    return dict(partial=partial, lse=lse, m=m_out, l=l_out, acc=acc_out)


def record_case(out, meta, name, case, ref, parts=(512, 1024), scale_mul=None):
    arrays = list(case.arrays())
    if scale_mul is not None:               # reference tests/test_reference.py:46-51
        arrays[0] = arrays[0] * scale_mul
        arrays[1] = arrays[1] * scale_mul
    out[f"{name}/dense"] = ref.dense_reference(*arrays)
    out[f"{name}/stream"] = ref.streaming_reference(*arrays, split=False)
    out[f"{name}/split"] = ref.streaming_reference(*arrays, split=True)
    for tokens in parts:
        for key, value in partitions_from_reference(ref, arrays, tokens).items():
            out[f"{name}/p{tokens}/{key}"] = value
    meta[name] = dict(checksum=case.checksum(), parts=list(parts), scale_mul=scale_mul)


def main():
    parser = argparse.ArgumentParser()
    parser.add_argument("--reference-src", default=os.environ.get("PAGED_DECODE_REFERENCE_SRC"),
                        help="the reference project's src/ directory (or set "
                             "PAGED_DECODE_REFERENCE_SRC)")
    args = parser.parse_args()
    if not args.reference_src:
        parser.error("--reference-src is required")
    ref, spec_mod, plan_mod = load_reference(args.reference_src)

    out, meta = {}, {}
    for length in cases.SWEEP_LENGTHS:
        for dim, hq, hkv in cases.SWEEP_GEOMETRIES:
            record_case(out, meta, f"sweep_{length}_{dim}_{hq}_{hkv}",
                        cases.sweep_case(length, dim, hq, hkv), ref)
    poisoned = cases.poison_tails(cases.make_case([257, 0], capacity=1025))
    record_case(out, meta, "poison", poisoned, ref)
    record_case(out, meta, "large_logits", cases.make_case([1025], seed=23), ref,
                scale_mul=80.0)
    cfg1 = cases.config1()
    plan148 = plan_mod.make_splitkv_plan(spec_mod.DecodeSpec(4, 8, 2, 128, 1024), 148)
    record_case(out, meta, "cfg1", cfg1, ref, parts=(512, 1024, plan148.tokens_per_split))
    np.savez_compressed(HERE / "golden_cases.npz", **out)

    plans = []
    grid = [(b, hq, hkv, d, cap) for b in (1, 2, 3, 8, 32, 128, 256)
            for hq, hkv in ((8, 2), (16, 4), (32, 8), (32, 32), (64, 8), (16, 1))
            for d in (64, 128, 256) for cap in (1, 255, 528, 1024, 2064, 2176, 2320, 8192)]
    grid += [(4, 8, 2, 128, 1024), (64, 32, 32, 64, 2048), (128, 32, 8, 128, 32768),
             (2, 64, 8, 128, 524288)]
    for b, hq, hkv, d, cap in grid:
        spec = spec_mod.DecodeSpec(b, hq, hkv, d, cap)
        for sms in (108, 148):
            for n in (0, 3):
                p = plan_mod.make_splitkv_plan(spec, sms, num_splits=n)
                plans.append([b, hq, hkv, d, cap, sms, n, p.splits, p.tile_tokens,
                              p.tokens_per_split, p.table_capacity_tokens, p.lse_lanes,
                              p.policy])
    geometry = [dict(spec=[b, hq, hkv, d, cap],
                     partitions=spec_mod.DecodeSpec(b, hq, hkv, d, cap).partitions,
                     table_width=spec_mod.DecodeSpec(b, hq, hkv, d, cap).table_width,
                     split_workspace_bytes=spec_mod.DecodeSpec(b, hq, hkv, d, cap).split_workspace_bytes)
                for b, hq, hkv, d, cap in grid[::7]]
    fields = ["max_batch", "num_heads", "num_kv_heads", "head_dim", "max_context_len",
              "sm_count", "num_splits", "splits", "tile_tokens", "tokens_per_split",
              "table_capacity_tokens", "lse_lanes", "policy"]
    (HERE / "golden_plans.json").write_text(json.dumps(
        dict(plan_fields=fields, plans=plans, geometry=geometry, cases=meta),
        separators=(",", ":"), sort_keys=True))
    print(f"wrote {len(out)} arrays, {len(plans)} plans")


if __name__ == "__main__":
    main()
