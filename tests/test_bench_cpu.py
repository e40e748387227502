"""bench.py's host-side logic on the CPU: the seeded batches, the shard layout, and the
reference arm, which must run without this repository's package or library."""

import json
import subprocess
import sys

import numpy as np
import pytest

import bench

ROOT = bench.ROOT


def test_every_rank_routes_the_same_batch():
    a = bench.config_routing(4, np.random.default_rng(7))
    b = bench.config_routing(4, np.random.default_rng(7))
    for u, v in zip(a, b):
        assert np.array_equal(u, v)


@pytest.mark.parametrize("world", [1, 2, 4, 8])
def test_shards_partition_inputs_and_outputs(world):
    c = bench.CONFIGS[4]
    for index, (name, k, widths, role) in enumerate(c["projections"]):
        hp = type("HP", (), dict(K=k, N=sum(widths), widths=widths, role=role))()
        k_cover, rows_cover = np.zeros(k, int), np.zeros(sum(widths), int)
        for rank in range(world):
            (k0, k1), rows, shard_widths = bench.shard_spec(hp, rank, world)
            k_cover[k0:k1] += 1
            rows_cover[rows] += 1
            assert sum(shard_widths) == len(rows)
        # column-parallel: every rank reads all of x; row-parallel: the inputs partition.
        assert np.all(k_cover == (world if role == "column" else 1))
        assert np.all(rows_cover == 1)


def test_host_weights_are_reproducible_per_slot():
    p1 = bench.HostProjection(0, "p", 64, (32,), None, np.array([4, 8]), 8, [1], seed=3)
    p2 = bench.HostProjection(0, "p", 64, (32,), None, np.array([4, 8]), 8, [0, 1], seed=3)
    assert p1.a[1].equal(p2.a[1]) and p1.b[1].equal(p2.b[1])
    assert float(p2.b[1][:, 8:].abs().sum()) == 0.0 if p2.b[1].shape[1] > 8 else True


def test_reference_arm_never_loads_the_package():
    code = (
        "import sys, bench; bench.main(['--impl', 'reference', '--config', '2', '--steps', '1', "
        "'--warmup', '1']); assert not any(m.startswith('loraforge_b200') for m in sys.modules), "
        "'package imported'"
    )
    out = subprocess.run([sys.executable, "-c", code], cwd=ROOT, capture_output=True, text=True,
                         timeout=600)
    assert out.returncode == 0, out.stderr[-2000:]
    line = json.loads(out.stdout.strip().splitlines()[-1])
    assert line["impl"] == "reference" and line["value"] > 0
    assert line["config"] == bench.config_record(2, 1)
    assert line["e2e"]["h2d_bytes_per_step"] == 0


def test_sub_records_run_in_a_seeded_random_order():
    first, again, other = (bench.sub_record_order(seed) for seed in (1234, 1234, 7))
    assert sorted(first) == list(range(len(bench.SUB_RECORDS)))
    assert first == again
    assert first != other or len(first) < 3
    names = [bench.sub_record_name(c, p) for c, p in bench.SUB_RECORDS]
    assert len(set(names)) == len(names) and "config1" in names and "config1_bgmv" in names
