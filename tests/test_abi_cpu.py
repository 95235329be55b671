"""CPU tests of the C ABI and the host-side logic (no GPU calls).

* the shared library loads and exports every symbol ``include/pdl_b200.h`` declares;
* the native plan / geometry equal the reference's golden values exactly;
* ``DecodeSpec`` and the engine-option checks keep the reference's contract
  (reference tests/test_reference.py:60-81, tests/test_splitkv_plan.py).
"""
import ctypes
import json
import re
from pathlib import Path

import pytest

import oracle
from paged_decode import _lib
from paged_decode.spec import DecodeSpec, validate_engine_options
from paged_decode.splitkv_plan import make_splitkv_plan

ROOT = Path(__file__).resolve().parents[1]
HEADER = ROOT / "include" / "pdl_b200.h"
PLANS = json.loads((ROOT / "tests" / "golden" / "golden_plans.json").read_text())


def declared_symbols():
    text = HEADER.read_text()
    return sorted(set(re.findall(r"^\s*(?:int|const char \*)\s*(pdl_\w+)\s*\(", text, re.M)))


def test_library_exports_every_declared_symbol():
    lib = _lib.load()
    names = declared_symbols()
    assert names == sorted(_lib.SYMBOLS)
    for name in names:
        assert hasattr(lib, name), name
    assert lib.pdl_abi_version() == _lib.ABI_VERSION


def test_status_strings():
    lib = _lib.load()
    assert lib.pdl_status_string(0) == b"ok"
    assert b"workspace" in lib.pdl_status_string(4)
    assert lib.pdl_status_string(999) == b"unknown status"


def test_native_plan_matches_reference_golden():
    lib = _lib.load()
    fields = PLANS["plan_fields"]
    for row in PLANS["plans"]:
        rec = dict(zip(fields, row))
        spec = _lib.PdlSpec(rec["max_batch"], rec["num_heads"], rec["num_kv_heads"],
                            rec["head_dim"], rec["max_context_len"], 256)
        plan = _lib.PdlPlan()
        assert lib.pdl_splitkv_plan(ctypes.byref(spec), rec["sm_count"], rec["num_splits"],
                                    ctypes.byref(plan)) == 0
        got = [plan.splits, plan.tile_tokens, plan.tokens_per_split, plan.table_capacity_tokens,
               plan.lse_lanes, "explicit" if plan.explicit_splits else "pinned_geometry"]
        assert got == row[7:], rec


def test_native_plan_matches_oracle_on_unseen_specs():
    for batch in (1, 5, 17, 64, 100, 300):
        for hq, hkv in ((12, 4), (16, 2), (40, 8), (64, 4)):
            for dim in (64, 128, 256):
                for cap in (100, 777, 4096, 40000):
                    for sms in (132, 148, 160):
                        spec = DecodeSpec(batch, hq, hkv, dim, cap)
                        got = make_splitkv_plan(spec, sms)
                        want = oracle.make_splitkv_plan(batch, hq, hkv, dim, cap, sms)
                        assert (got.splits, got.tokens_per_split, got.lse_lanes) == \
                            (want.splits, want.tokens_per_split, want.lse_lanes)


def test_native_geometry_matches_reference_golden():
    lib = _lib.load()
    for rec in PLANS["geometry"]:
        b, hq, hkv, d, cap = rec["spec"]
        parts, width, ws = ctypes.c_int32(), ctypes.c_int32(), ctypes.c_int64()
        spec = _lib.PdlSpec(b, hq, hkv, d, cap, 256)
        assert lib.pdl_spec_geometry(ctypes.byref(spec), ctypes.byref(parts), ctypes.byref(width),
                                     ctypes.byref(ws)) == 0
        assert (parts.value, width.value, ws.value) == \
            (rec["partitions"], rec["table_width"], rec["split_workspace_bytes"])
        py = DecodeSpec(b, hq, hkv, d, cap)
        assert (py.partitions, py.table_width, py.split_workspace_bytes) == \
            (rec["partitions"], rec["table_width"], rec["split_workspace_bytes"])


def test_native_geometry_rejects_bad_specs():
    lib = _lib.load()
    for bad in ((0, 8, 2, 128, 10), (1, 8, 3, 128, 10), (1, 8, 2, 80, 10)):
        spec = _lib.PdlSpec(*bad, 256)
        assert lib.pdl_spec_geometry(ctypes.byref(spec), None, None, None) != 0
    spec = _lib.PdlSpec(1, 8, 2, 128, 10, 16)
    assert lib.pdl_spec_geometry(ctypes.byref(spec), None, None, None) == 2


def test_launch_entry_points_reject_null_args_without_a_gpu():
    lib = _lib.load()
    for name in ("pdl_partition", "pdl_merge", "pdl_paged_decode",
                 "pdl_paged_decode_static_scratch", "pdl_lse_merge", "pdl_append_kv"):
        assert getattr(lib, name)(None, 0) == 1


def test_spec_and_memory():
    spec = DecodeSpec(32, 32, 8, 128, 8192)
    assert spec.partitions == 8
    assert spec.table_width == 32
    assert spec.split_workspace_bytes == 32 * 32 * 8 * 130 * 4


@pytest.mark.parametrize("kwargs", [{"head_dim": 80}, {"page_size": 16}, {"num_kv_heads": 3},
                                    {"max_batch": 0}, {"max_context_len": -1}])
def test_unsupported_geometry(kwargs):
    values = dict(max_batch=8, num_heads=4, num_kv_heads=2, head_dim=64, max_context_len=2048)
    values.update(kwargs)
    with pytest.raises(ValueError):
        DecodeSpec(**values)


@pytest.mark.parametrize("backend,tp,page", [("typo", 1, 256), ("triton_base", 2, 256),
                                            ("triton_splitk", 1, 512)])
def test_engine_rejects_unsupported_options(backend, tp, page):
    with pytest.raises(ValueError):
        validate_engine_options(backend, tp, page, 32, 8192)


def test_explicit_count_partitions_capacity_in_tiles():
    plan = make_splitkv_plan(DecodeSpec(1, 16, 4, 256, 2176), 108, num_splits=3)
    assert plan.splits == 3 and plan.tokens_per_split == 768
    assert plan.policy == "explicit"


@pytest.mark.parametrize("count", [-1, 129, 1.5])
def test_unsupported_explicit_counts(count):
    with pytest.raises(ValueError, match="num_splits"):
        make_splitkv_plan(DecodeSpec(1, 8, 2, 256, 1024), 108, num_splits=count)


def test_unsupported_group():
    with pytest.raises(ValueError, match="16"):
        make_splitkv_plan(DecodeSpec(1, 32, 1, 256, 1024), 108)


def test_b200_plan_invariants():
    from paged_decode.splitkv_plan import make_b200_plan
    for b, hq, hkv, d, cap in [(4, 8, 2, 128, 1024), (64, 32, 32, 64, 2048), (1, 16, 4, 256, 2320),
                               (32, 16, 4, 256, 2320), (128, 32, 8, 128, 32768),
                               (2, 64, 8, 128, 524288), (1, 1, 1, 64, 1)]:
        plan = make_b200_plan(DecodeSpec(b, hq, hkv, d, cap), 148)
        capacity = -(-cap // 256) * 256
        assert plan.tokens_per_split % plan.tile_tokens == 0
        assert plan.splits * plan.tokens_per_split >= capacity
        assert (plan.splits - 1) * plan.tokens_per_split < capacity  # no always-empty partition
        assert plan.tokens_per_split <= max(4096, plan.tile_tokens)
    assert make_b200_plan(DecodeSpec(128, 32, 8, 128, 32768), 148).splits == 8


def test_b200_plan_recommends_balanced_partitions_for_one_wave_of_long_d256_items():
    from paged_decode.splitkv_plan import launch_partitioning, make_b200_plan
    plan = make_b200_plan(DecodeSpec(32, 16, 4, 256, 2320), 148)
    assert (plan.splits, plan.tokens_per_split, plan.balanced) == (2, 1280, True)
    assert launch_partitioning(plan) == (64, _lib.FLAG_BALANCED)
    # Between one and two waves of whole rows: two balanced partitions per row.
    plan = make_b200_plan(DecodeSpec(128, 16, 4, 256, 2320), 148)
    assert (plan.splits, plan.tokens_per_split, plan.balanced) == (2, 1280, True)
    # B=1 (40 items of 64 tokens), one wave of whole rows, three waves, D = 128: fixed bounds.
    for spec in (DecodeSpec(1, 16, 4, 256, 2320), DecodeSpec(64, 16, 4, 256, 2320),
                 DecodeSpec(256, 16, 4, 256, 2320), DecodeSpec(128, 32, 8, 128, 32768)):
        plan = make_b200_plan(spec, 148)
        assert not plan.balanced and launch_partitioning(plan) == (plan.tokens_per_split, 0)


def test_exchange_plan_arithmetic():
    lib = _lib.load()

    def plan(rows, d, world, sms=148, emulate=0):
        p = _lib.PdlExchangePlan()
        status = lib.pdl_exchange_plan(rows, d, world, sms, emulate, ctypes.byref(p))
        return status, p

    status, p = plan(128, 128, 2)  # config 5: B=2 x Hq=64 rows
    assert status == 0 and p.ctas == 32
    assert p.block_words == 128 * 128 + 128 and p.data_offset == 4096 * 4
    assert p.buffer_bytes == p.data_offset + 2 * 2 * p.block_words * 8
    status, p = plan(3, 64, 1)
    assert status == 0 and p.ctas == 1 and p.block_words == 3 * 64 + 4
    status, p = plan(16384, 256, 8)  # two column slices per row; 4 CTAs per SM at most
    assert status == 0 and p.ctas == 4 * 148
    status, p = plan(16384, 256, 8, emulate=1)  # every emulated rank co-resident
    assert status == 0 and p.ctas == 4 * 148 // 8
    status, p = plan(1 << 20, 64, 2, sms=1000)
    assert status == 0 and p.ctas == 1024  # flag arrays hold 1024 CTAs
    for bad in [(128, 96, 2), (0, 128, 2), (128, 128, 0), (128, 128, 9)]:
        assert plan(*bad)[0] != 0
    assert lib.pdl_exchange_plan(1, 64, 1, 148, 0, None) == 1


def test_exchange_entry_points_reject_null_without_a_gpu():
    lib = _lib.load()
    assert lib.pdl_exchange_merge(None, 0) == 1
    assert lib.pdl_peer_buffer_create(0, None, None) == 1
    assert lib.pdl_peer_buffer_open(None, None) == 1
    assert lib.pdl_peer_buffer_close(None) == 1
    assert lib.pdl_peer_buffer_free(None) == 1


def test_exchange_args_need_one_buffer_per_rank():
    import torch
    from paged_decode import ops
    t = torch.zeros(8)
    with pytest.raises(ValueError):
        ops.exchange_args(t, t, rows=1, parts=1, head_dim=64, world=2, buffers=[0], out=t)
    a = ops.exchange_args(t, t, rows=1, parts=1, head_dim=64, world=2, buffers=[256, 512],
                          out=t, rank=1, timeout_us=5)
    assert a.world == 2 and a.rank == 1 and list(a.buffers)[:2] == [256, 512]
