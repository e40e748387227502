"""Pin the CPU oracle to the reference's own oracles and known answers (no GPU)."""

import numpy as np
import pytest

from golden_io import known_answers, load, rel_l2
from oracle import cpu_reference as ref


def _row_case(slices):
    d = load(f"row_case_s{slices}.npz")
    meta = {
        k: d[k]
        for k in (
            "b_offsets", "b_strides", "ranks", "scales", "segment_indptr", "segment_slots",
            "token_indices", "slice_offsets",
        )
    }
    meta["segment_count"] = int(d["segment_count"][0])
    lo, hi = d["output_columns"]
    return d, meta, d["storage"][:, lo:hi]


@pytest.mark.parametrize("slices", [1, 2, 3])
def test_row_shrink_oracle_matches_reference(slices):
    d, meta, _ = _row_case(slices)
    x = ref.bf16_value(d["x"])
    a = ref.bf16_value(d["a"])
    z = ref.row_shrink(x, a, d["z"], d["routes"], meta["ranks"], slices, 64)
    np.testing.assert_array_equal(z, d["expected_z"])


@pytest.mark.parametrize("slices", [1, 2, 3])
def test_row_expand_fp64_oracle_matches_reference(slices):
    d, meta, output = _row_case(slices)
    y = ref.row_expand_fp64(d["expected_z"], d["b"], output, meta)
    np.testing.assert_array_equal(y, d["expected_y"])


@pytest.mark.parametrize("slices", [1, 2, 3])
def test_exact_row_expand_within_reference_gate(slices):
    # The FP32 kernel arithmetic against the reference's FP64 oracle: the reference's
    # own relative-L2 gate (tests/test_row_operators_gpu.py:137-141).
    d, meta, output = _row_case(slices)
    y = ref.row_expand(
        d["expected_z"], d["b"], output, meta["b_offsets"], meta["b_strides"], meta["ranks"],
        meta["scales"], meta["segment_indptr"], meta["segment_slots"], meta["token_indices"],
        meta["slice_offsets"], meta["segment_count"],
    )
    assert rel_l2(ref.bf16_value(y), ref.bf16_value(d["expected_y"])) < 0.005
    routes = d["routes"]
    skipped = (routes == -1) | (routes == 8)
    np.testing.assert_array_equal(y[skipped], output[skipped])


def test_rounding_known_answer():
    kat = known_answers()["rounding"]
    bits = lambda v: ref.bf16_bits(np.array(v, dtype=np.float32))  # noqa: E731
    y = ref.row_expand(
        bits([[kat["z"]]]), bits([kat["b"]]), bits([[kat["y"]]]), [0], [1], [1],
        [kat["scale"]], [0, 1], [0], [0], [0, 1], 1,
    )
    assert ref.bf16_value(y)[0, 0] == kat["expected"]
    assert ref.round_bf16(np.float32(kat["scale"] + kat["y"])) == kat["single_rounding"]


def test_example_known_answer():
    kat = known_answers()["example"]
    f = lambda v: np.array(v, dtype=np.float32)  # noqa: E731
    x, a = f(kat["x"]), f(kat["a"])
    z = ref.row_shrink(x, a, np.zeros((3, 2), np.uint16), kat["routes"], kat["ranks"], 1, kat["max_rank"])
    y = ref.row_expand(
        z, ref.bf16_bits(f(kat["b"])), ref.bf16_bits(f(kat["y"])), [0], [2], kat["ranks"],
        kat["scales"], kat["segment_indptr"], kat["segment_slots"], kat["token_indices"],
        kat["slice_offsets"], 1,
    )
    np.testing.assert_array_equal(ref.bf16_value(y), f(kat["expected"]))


def _gemv_cases():
    from golden_io import GOLDEN

    return sorted(p.name for p in GOLDEN.glob("gemv_case_*.npz"))


def _values(array, dtype):
    if dtype == "bfloat16":
        return ref.bf16_value(array)
    return np.asarray(array, dtype=np.float32)


@pytest.mark.parametrize("name", _gemv_cases())
def test_bgmv_oracle_matches_reference(name):
    d = load(name)
    dtype = name.split("_")[2]
    x, a, b, base = (_values(d[k], dtype) for k in ("x", "a", "b", "base"))
    got = ref.bgmv_reference(x, a, b, d["ranks"], d["routes"], d["scales"], d["offsets"], base, dtype)
    expected = _values(d["expected"], dtype)
    tol = {"float32": 2e-5, "float16": 3e-3, "bfloat16": 2e-2}[dtype]
    np.testing.assert_allclose(got, expected, rtol=tol, atol=tol)


def _vllm_cases():
    from golden_io import GOLDEN

    return sorted(p.name for p in GOLDEN.glob("vllm_case_*.npz"))


@pytest.mark.parametrize("name", _vllm_cases())
def test_vllm_oracle_matches_reference(name):
    d = load(name)
    dtype = name.split("_")[2]
    x = _values(d["x"], dtype)
    a = [_values(d[f"a{i}"], dtype) for i in range(3)]
    b = [_values(d[f"b{i}"], dtype) for i in range(3)]
    y = _values(d["y"], dtype)
    got = ref.vllm_reference(x, a, b, d["routes"], y, scale=0.7, offset=3, add=False, dtype=dtype)
    np.testing.assert_array_equal(got, _values(d["expected"], dtype))
    got = ref.vllm_reference(x, a, b, d["routes"], y, scale=0.7, offset=0, add=True, dtype=dtype)
    np.testing.assert_array_equal(got, _values(d["expected_add"], dtype))


def _naive_grouping(slots, num_slots, chunk):
    buckets = {}
    for t, s in enumerate(slots):
        buckets.setdefault(s if 0 <= s < num_slots else None, []).append(t)
    perm, indptr, seg_slots = [], [], []
    for s in range(num_slots):
        tokens = buckets.get(s, [])
        step = chunk if chunk > 0 else max(1, len(tokens))
        for j in range(0, len(tokens), step):
            indptr.append(len(perm) + j)
            seg_slots.append(s)
        perm.extend(tokens)
    n_active = len(perm)
    perm.extend(buckets.get(None, []))
    return indptr + [n_active], seg_slots, perm


@pytest.mark.parametrize("seed", range(6))
@pytest.mark.parametrize("chunk", [0, 1, 5, 16])
def test_grouping_oracle_against_naive(seed, chunk):
    rng = np.random.default_rng(seed)
    num_slots = int(rng.integers(1, 40))
    T = int(rng.integers(0, 300))
    slots = rng.integers(-3, num_slots + 3, size=T)
    indptr, seg_slots, perm, count = ref.group_tokens(slots, num_slots, chunk)
    e_indptr, e_slots, e_perm = _naive_grouping(slots.tolist(), num_slots, chunk)
    assert indptr.tolist() == e_indptr
    assert seg_slots.tolist() == e_slots
    assert perm.tolist() == e_perm
    assert count == len(e_slots)


def test_grouping_oracle_reproduces_reference_fixture_segments():
    # The reference fixture's segments (tests/test_row_operators_gpu.py:55-65) are
    # contiguous runs of one slot each, sizes [1,2,3,4,8,16,15,16,3,2]; grouping its
    # routes with chunk 16 gives the same per-slot token sets.
    d = load("row_case_s1.npz")
    routes = d["routes"]
    indptr, seg_slots, perm, count = ref.group_tokens(routes, 9, 16)
    for seg in range(count):
        tokens = set(perm[indptr[seg] : indptr[seg + 1]].tolist())
        assert all(routes[t] == seg_slots[seg] for t in tokens)
    ref_slots = d["segment_slots"][: int(d["segment_count"][0])]
    ref_indptr = d["segment_indptr"]
    for g in range(9):
        ours = {t for s in range(count) if seg_slots[s] == g for t in perm[indptr[s] : indptr[s + 1]]}
        theirs = {
            t for s in range(len(ref_slots)) if ref_slots[s] == g
            for t in d["token_indices"][ref_indptr[s] : ref_indptr[s + 1]]
        }
        assert ours == theirs
