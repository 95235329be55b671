"""Pin the CPU oracle against the reference's own outputs (golden fixtures).

The fixtures were produced by ``tests/golden/make_golden.py`` from the
reference's NumPy code; these tests rebuild each seeded case, check its input
checksum, and require the oracle restatement to reproduce every recorded
output.  Plans and geometry must match exactly (integer work).
"""
import json
from pathlib import Path

import numpy as np
import pytest

import cases
import oracle

GOLDEN = Path(__file__).resolve().parent / "golden"
ARRAYS = np.load(GOLDEN / "golden_cases.npz")
META = json.loads((GOLDEN / "golden_plans.json").read_text())

# The oracle repeats the reference's arithmetic in the same order, so the
# residual is BLAS summation order only.
ATOL, RTOL = 2e-6, 2e-6


def _case(name):
    if name.startswith("sweep_"):
        _, length, dim, hq, hkv = name.split("_")
        case = cases.sweep_case(int(length), int(dim), int(hq), int(hkv))
    elif name == "poison":
        case = cases.poison_tails(cases.make_case([257, 0], capacity=1025))
    elif name == "large_logits":
        case = cases.make_case([1025], seed=23)
    elif name == "cfg1":
        case = cases.config1()
    else:
        raise KeyError(name)
    assert case.checksum() == META["cases"][name]["checksum"], "case generator drifted"
    arrays = list(case.arrays())
    mul = META["cases"][name]["scale_mul"]
    if mul is not None:
        arrays[0], arrays[1] = arrays[0] * mul, arrays[1] * mul
    return case, arrays


def _close(actual, expected, atol=ATOL, rtol=RTOL):
    np.testing.assert_allclose(actual, expected, atol=atol, rtol=rtol)


@pytest.mark.parametrize("name", sorted(META["cases"]))
def test_outputs_match_reference(name):
    _, arrays = _case(name)
    tol = dict(atol=1e-4, rtol=1e-5) if name == "large_logits" else {}
    _close(oracle.dense_reference(*arrays), ARRAYS[f"{name}/dense"], **tol)
    _close(oracle.streaming_reference(*arrays), ARRAYS[f"{name}/stream"], **tol)
    _close(oracle.streaming_reference(*arrays, split=True), ARRAYS[f"{name}/split"], **tol)


@pytest.mark.parametrize("name", sorted(META["cases"]))
def test_partitions_match_reference(name):
    case, arrays = _case(name)
    q, k, v, table, lengths = arrays
    for tokens in META["cases"][name]["parts"]:
        splits = max(1, -(-table.shape[1] * 256 // tokens))
        partial, lse = oracle.normalized_partitions(q, k, v, table, lengths, tokens, splits)
        m, l, acc = oracle.unnormalized_partitions(q, k, v, table, lengths, tokens, splits)
        key = f"{name}/p{tokens}"
        _close(partial, ARRAYS[f"{key}/partial"], atol=1e-5)
        # LSE is compared relative to its magnitude, +-inf positions exactly.
        np.testing.assert_array_equal(np.isinf(lse), np.isinf(ARRAYS[f"{key}/lse"]))
        finite = np.isfinite(lse)
        _close(lse[finite], ARRAYS[f"{key}/lse"][finite], atol=1e-5, rtol=1e-6)
        _close(m, ARRAYS[f"{key}/m"])
        _close(l, ARRAYS[f"{key}/l"], rtol=1e-5)
        _close(acc, ARRAYS[f"{key}/acc"], atol=1e-4, rtol=1e-5)
        # Both merges rebuild the reference's split output for 1024 partitions.
        merged = oracle.lse_merge(partial, lse)
        unnorm = oracle.merge_unnormalized(m, l, acc)
        _close(merged, ARRAYS[f"{name}/dense"], atol=5e-6, rtol=5e-5)
        _close(unnorm, ARRAYS[f"{name}/dense"], atol=5e-6, rtol=5e-5)


def test_zero_length_rows_are_exact_zero():
    _, arrays = _case("poison")
    assert not oracle.dense_reference(*arrays)[1].any()
    assert not ARRAYS["poison/split"][1].any()


def test_plans_match_reference_exactly():
    fields = META["plan_fields"]
    for row in META["plans"]:
        rec = dict(zip(fields, row))
        plan = oracle.make_splitkv_plan(rec["max_batch"], rec["num_heads"], rec["num_kv_heads"],
                                        rec["head_dim"], rec["max_context_len"],
                                        rec["sm_count"], rec["num_splits"])
        got = [plan.splits, plan.tile_tokens, plan.tokens_per_split,
               plan.table_capacity_tokens, plan.lse_lanes, plan.policy]
        assert got == row[7:], rec


def test_geometry_matches_reference():
    for rec in META["geometry"]:
        parts, width, ws = oracle.spec_geometry(*rec["spec"])
        assert (parts, width, ws) == (rec["partitions"], rec["table_width"],
                                      rec["split_workspace_bytes"])


# Known answers copied as numbers from the reference's own plan tests
# (tests/test_splitkv_plan.py:7-30, sm_count 108).
@pytest.mark.parametrize("batch,heads,kv,capacity,splits,tokens", [
    (8, 8, 2, 1024, 8, 128), (8, 16, 4, 1024, 6, 192),
    (1, 16, 4, 2176, 36, 64), (1, 8, 2, 2176, 36, 64), (32, 32, 8, 8192, 1, 8192)])
def test_reference_plan_known_answers(batch, heads, kv, capacity, splits, tokens):
    plan = oracle.make_splitkv_plan(batch, heads, kv, 256, capacity, 108)
    assert (plan.splits, plan.tokens_per_split) == (splits, tokens)
    assert plan.table_capacity_tokens == (capacity + 255) // 256 * 256


def test_partition_bounds_integer_contract():
    assert oracle.partition_bounds(2051, 1024, 3) == [(0, 1024), (1024, 2048), (2048, 2051)]
    assert oracle.partition_bounds(0, 512, 2) == [(0, 0), (512, 512)]
    assert oracle.partition_bounds(1024, 1024, 2) == [(0, 1024), (1024, 1024)]


def test_balanced_partition_bounds_cover_each_row_in_equal_granule_multiples():
    assert oracle.partition_bounds(2064, 64, 2, balanced=True) == [(0, 1088), (1088, 2064)]
    assert oracle.partition_bounds(0, 64, 3, balanced=True) == [(0, 0)] * 3
    for n in range(0, 3000, 37):
        for splits in (1, 2, 3, 7, 40):
            for granule in (32, 64, 128):
                b = oracle.partition_bounds(n, granule, splits, balanced=True)
                span = oracle.balanced_span(n, splits, granule)
                assert span % granule == 0 and span * splits >= n
                live = [(s, e) for s, e in b if e > s]
                assert [s for s, _ in live] == [p * span for p in range(len(live))]
                assert sum(e - s for s, e in live) == n
                assert all(e - s == span for s, e in live[:-1])


def test_all_empty_lse_merge_gives_zero():
    partials = np.zeros((1, 2, 3, 8), np.float32)
    lse = np.full((1, 2, 3), -np.inf, np.float32)
    assert not oracle.lse_merge(partials, lse).any()


def test_bf16_rounding_is_nearest_even():
    x = np.array([1.0, 1.0 + 2 ** -8, 1.0 + 3 * 2 ** -8, -2.5, 3.0e38], np.float32)
    got = oracle.round_bf16(x)
    np.testing.assert_array_equal(got[:4], [1.0, 1.0, 1.0 + 2 ** -6, -2.5])
    assert np.isfinite(got[4]) or np.isinf(got[4])
