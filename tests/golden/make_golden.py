"""Generate the golden fixtures in this directory from the reference's own oracles.

Run in a checkout that has the reference source tree (lishenghui/loraforge):

    python tests/golden/make_golden.py /path/to/loraforge

It imports the reference's test modules on CPU and records, for the reference's
own fixture recipes, the inputs and the outputs of the reference oracles:

* row_case_s{1,2,3}.npz — ``case()`` of tests/test_row_operators_gpu.py:40-96
  (seed 31) with ``shrink_reference`` / ``expand_reference`` (:99-134) outputs;
* gemv_case_*.npz — the ``fixture()`` recipe of tests/test_gemv_gpu.py:16-49 on a
  CPU generator (seed 23) with the output of its ``reference()`` (:52-67);
* vllm_case_*.npz — ``tensors()`` of tests/test_vllm_gpu.py:11-25 on CPU
  (seed 123) with the output of its ``reference()`` (:26-39);
* retained_layout.npz — ``RetainedLayout`` (src/loraforge/runtime/retained.py:119-205)
  driven through the load sequence of tests/test_retained_layout.py:24-61;
* known_answers.json — the rounding known answer (tests/test_row_operators_gpu.py:233-259)
  and examples/row_operators.py.

BF16 tensors are stored as uint16 bit patterns, FP16 as float16.  A rows that the
operators never read (rows at or beyond slices*rank of each slot) are zeroed after
the reference outputs are computed, to keep the files small.
"""

from __future__ import annotations

import importlib.util
import json
import sys
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent


def _module(root: Path, relative: str, name: str):
    spec = importlib.util.spec_from_file_location(name, root / relative)
    module = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(module)
    return module


def bits(t):
    import torch

    if t.dtype == torch.bfloat16:
        return t.contiguous().view(torch.int16).numpy().view(np.uint16)
    return t.contiguous().numpy()


def row_cases(root: Path):
    import torch

    m = _module(root, "tests/test_row_operators_gpu.py", "ref_row_tests")
    for slices in (1, 2, 3):
        x, a, z, b, storage, output, routes, meta = m.case(slices, device="cpu")
        expected_z = m.shrink_reference(x, a, z, routes, meta["ranks"], slices)
        expected_y = m.expand_reference(expected_z, b, output, meta)
        ranks = meta["ranks"].tolist()
        a_live = a.clone()
        for g, r in enumerate(ranks):
            a_live[g, slices * r :] = 0
        np.savez_compressed(
            HERE / f"row_case_s{slices}.npz",
            x=bits(x.contiguous()),
            a=bits(a_live),
            z=bits(z),
            b=bits(b),
            storage=bits(storage),
            output_columns=np.array([3, 3 + output.shape[1]]),
            routes=routes.numpy(),
            expected_z=bits(expected_z),
            expected_y=bits(expected_y),
            **{k: v.numpy() for k, v in meta.items()},
        )


def gemv_cases(root: Path):
    import torch

    m = _module(root, "tests/test_gemv_gpu.py", "ref_gemv_tests")
    cases = [(d, s, 8) for d in (torch.float32, torch.float16, torch.bfloat16) for s in (1, 3)]
    cases.append((torch.bfloat16, 2, 33))
    for dtype, slices, capacity in cases:
        g = torch.Generator().manual_seed(23)
        sizes = [5, 3, 7][:slices]
        x = (torch.randn(14, 777, generator=g, dtype=torch.float32) / 10).to(dtype)[::2]
        a = (torch.randn(4, slices * capacity, 777, generator=g) / 10).to(dtype)
        b = (torch.randn(4, sum(sizes), capacity, generator=g) / 10).to(dtype)
        ranks = torch.tensor([0, 1, min(3, capacity), capacity], dtype=torch.int64)
        routes = torch.tensor([0, 3, 2, 1, 3, 0, 2], dtype=torch.int64)
        scales = torch.tensor([0, 0.25, 1.5, 0.75])
        offsets = torch.tensor(
            [0] + [sum(sizes[: i + 1]) for i in range(slices)], dtype=torch.int64
        )
        base = (torch.randn(7, sum(sizes) + 4, generator=g) / 10).to(dtype)
        expected = m.reference(x, a, b, ranks, routes, scales, offsets, base)
        for slot, r in enumerate(ranks.tolist()):
            a[slot, slices * r :] = 0  # rows the operator never reads
        name = str(dtype).split(".")[-1]
        np.savez_compressed(
            HERE / f"gemv_case_{name}_s{slices}_c{capacity}.npz",
            x=bits(x.contiguous()),
            a=bits(a),
            b=bits(b),
            ranks=ranks.numpy(),
            routes=routes.numpy(),
            scales=scales.numpy(),
            offsets=offsets.numpy(),
            base=bits(base),
            expected=bits(expected),
            max_slice=np.array(max(sizes)),
        )


def vllm_cases(root: Path):
    import torch

    m = _module(root, "tests/test_vllm_gpu.py", "ref_vllm_tests")
    cases = [(d, r) for d in (torch.float32, torch.float16, torch.bfloat16) for r in (1, 7)]
    cases.append((torch.bfloat16, 33))
    for dtype, rank in cases:
        torch.manual_seed(123)
        x = torch.randn(7, 514, dtype=dtype)[:, :513]
        a = [torch.randn(4, rank, 513, dtype=dtype) * 0.1 for _ in range(3)]
        b = [torch.randn(4, n, rank, dtype=dtype) * 0.1 for n in (17, 13, 21)]
        routes = (torch.arange(7, dtype=torch.int32) % 5) - 1
        y = torch.randn(7, 57, dtype=dtype) * 0.1
        expected = m.reference(x, a, b, routes, y, offset=3, add=False)
        expected_add = m.reference(x, a, b, routes, y, offset=0, add=True)
        name = str(dtype).split(".")[-1]
        np.savez_compressed(
            HERE / f"vllm_case_{name}_r{rank}.npz",
            x=bits(x.contiguous()),
            **{f"a{i}": bits(t) for i, t in enumerate(a)},
            **{f"b{i}": bits(t) for i, t in enumerate(b)},
            routes=routes.numpy(),
            y=bits(y),
            expected=bits(expected),
            expected_add=bits(expected_add),
        )


def retained_layout(root: Path):
    import torch

    sys.path.insert(0, str(root / "src"))
    from loraforge.runtime.retained import RetainedLayout, effective_rank

    def ranks(k, other=None):
        return {
            f"base_model.model.model.layers.0.mlp.{name}.lora_A.weight": value
            for name, value in (("gate_proj", k), ("up_proj", k if other is None else other))
        }

    a = torch.arange(2 * 2 * 128 * 8).reshape(2, 256, 8).to(torch.bfloat16)
    b = torch.arange(2 * 32 * 128).reshape(2, 32, 128).to(torch.bfloat16)
    original_a = a.clone()
    catalog = {"low": ranks(3, 2), "high": ranks(32), "fallback": ranks(128)}
    e = RetainedLayout(a, b, "gate_up_proj", 0, catalog)
    record = {
        "a0": bits(a.clone()),
        "b": bits(b),
        "regions": np.array([e.regions[k] for k in ("low", "high", "fallback")]),
        "max_rank": np.array(e.max_rank),
        "store_numel": np.array(e.store.numel()),
    }
    steps = [("low", 1, 128), ("fallback", 1, 128), ("high", 1, 128), (None, 1, 0)]
    for i, (path, slot, rank) in enumerate(steps):
        a[1].copy_(original_a[1])  # native reload before every repack
        e.load(path, slot, rank)
        record[f"step{i}_a"] = bits(a.clone())
        record[f"step{i}_store"] = bits(e.store.clone())
        for field in ("rank", "supported", "unsupported", "low", "high", "bucket", "boff"):
            record[f"step{i}_{field}"] = getattr(e, field).numpy().copy()
    record["effective_rank"] = np.array(
        [
            effective_rank(ranks(3, 7), "gate_up_proj", 0),
            effective_rank(ranks(3), "gate_up_proj", 1),
            effective_rank(ranks(3), "qkv_proj", 0),
        ]
    )
    np.savez_compressed(HERE / "retained_layout.npz", **record)


def known_answers():
    data = {
        "rounding": {
            "z": 1.0,
            "b": 1.0,
            "scale": 1.00390625,
            "y": 0.0078125,
            "expected": 1.0078125,
            "single_rounding": 1.015625,
            "source": "tests/test_row_operators_gpu.py:233-259",
        },
        "example": {
            "x": [[1.0] * 8] * 3,
            "a": [[[1.0] * 8] * 2],
            "b": [1.0] * 6,
            "y": [[1.0] * 3] * 3,
            "routes": [0, -1, 0],
            "ranks": [2],
            "max_rank": 2,
            "scales": [0.5],
            "segment_indptr": [0, 2],
            "segment_slots": [0],
            "token_indices": [2, 0],
            "slice_offsets": [0, 3],
            "expected": [[9, 9, 9], [1, 1, 1], [9, 9, 9]],
            "source": "examples/row_operators.py:15-38",
        },
    }
    (HERE / "known_answers.json").write_text(json.dumps(data, indent=1) + "\n")


def main(argv):
    if len(argv) != 2:
        raise SystemExit("usage: python tests/golden/make_golden.py <reference source tree>")
    root = Path(argv[1]).resolve()
    sys.path.insert(0, str(root / "src"))
    row_cases(root)
    gemv_cases(root)
    vllm_cases(root)
    retained_layout(root)
    known_answers()


if __name__ == "__main__":
    main(sys.argv)
