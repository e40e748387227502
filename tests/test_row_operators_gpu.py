"""row_shrink / row_expand on the B200 against the reference's outputs and the oracle.

Mirrors tests/test_row_operators_gpu.py of lishenghui/loraforge: mixed ranks,
slices and segments, projection-sized widths, graph replay after metadata
mutation, the two-stage rounding known answer, rejections and empty batches.
Expand results are additionally required to be bit-identical to the oracle's
restatement of the reference kernel arithmetic.
"""

import numpy as np
import pytest

torch = pytest.importorskip("torch")
pytestmark = [
    pytest.mark.gpu,
    pytest.mark.skipif(not torch.cuda.is_available(), reason="CUDA device required"),
]

from cases import golden_row_case, oracle_expand, oracle_shrink, row_case, values  # noqa: E402
from golden_io import bf16_bits, known_answers, rel_l2  # noqa: E402

from loraforge_b200.ops import row_expand, row_shrink  # noqa: E402


def close(actual, expected):
    # The reference's gate: relative L2 < 0.005 (tests/test_row_operators_gpu.py:137-141).
    assert rel_l2(values(actual), values(expected)) < 0.005


def live_mask(routes, ranks, slices, width):
    r = np.where(routes >= 0, ranks[np.clip(routes, 0, None)], 0)
    return np.arange(width)[None, :] < (slices * r)[:, None]


@pytest.mark.parametrize("slices", [1, 2, 3])
@pytest.mark.parametrize("threads", [128, 256])
def test_mixed_ranks_slices_segments_and_base(slices, threads):
    (x, a, z, b, storage, output, routes, meta), gold = golden_row_case(slices)
    before, all_before = output.clone(), storage.clone()
    row_shrink(x, a, z, routes, meta["ranks"], num_slices=slices)
    torch.cuda.synchronize()
    got_z = bf16_bits(z)
    live = live_mask(gold["routes"], gold["ranks"], slices, got_z.shape[1])
    for row in range(got_z.shape[0]):
        if live[row].any():
            close(got_z[row][live[row]], gold["expected_z"][row][live[row]])
    np.testing.assert_array_equal(got_z[~live], gold["expected_z"][~live])  # untouched 3.0
    # Expand the reference's own z so the comparison isolates the expand kernel.
    z_ref = torch.from_numpy(gold["expected_z"].view(np.int16)).view(torch.bfloat16).cuda()
    row_expand(z_ref, b, output, **meta, threads=threads, blocks=1)
    torch.cuda.synchronize()
    np.testing.assert_array_equal(bf16_bits(output), oracle_expand(z_ref, b, before, meta))
    close(bf16_bits(output), gold["expected_y"])
    delta = torch.zeros_like(output)
    row_expand(z_ref, b, delta, **meta, threads=threads, blocks=2)
    np.testing.assert_array_equal(
        bf16_bits(delta), oracle_expand(z_ref, b, torch.zeros_like(output), meta)
    )
    torch.testing.assert_close(storage[:, :3], all_before[:, :3], rtol=0, atol=0)
    torch.testing.assert_close(storage[:, -3:], all_before[:, -3:], rtol=0, atol=0)
    skipped = (routes == -1) | (routes == 8)
    torch.testing.assert_close(output[skipped], before[skipped], rtol=0, atol=0)


@pytest.mark.parametrize("width,columns", [(4096, 14336), (14336, 4096)])
def test_model_projection_sizes(width, columns):
    x, a, z, b, _, output, routes, meta = row_case(width=width, columns=columns)
    expected_z = oracle_shrink(x, a, z, routes, meta["ranks"], 1)
    row_shrink(x, a, z, routes, meta["ranks"])
    got = bf16_bits(z)
    live = live_mask(routes.cpu().numpy(), meta["ranks"].cpu().numpy(), 1, got.shape[1])
    close(got[live], expected_z[live])
    np.testing.assert_array_equal(got[~live], expected_z[~live])
    expected = oracle_expand(z, b, output, meta)
    row_expand(z, b, output, **meta)
    np.testing.assert_array_equal(bf16_bits(output), expected)


def test_graph_replay_changed_routes_ranks_offsets_and_weights():
    x, a, z, b, _, output, routes, meta = row_case(slices=3)
    base = output.clone()

    def run():
        row_shrink(x, a, z, routes, meta["ranks"], num_slices=3)
        row_expand(z, b, output, **meta)

    stream = torch.cuda.Stream()
    stream.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(stream):
        run()
    torch.cuda.current_stream().wait_stream(stream)
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        run()
    # Slot 2 is reloaded with rank 7 and points at slot 3's compact region; both
    # kernels must see the new metadata at the same addresses on replay.
    meta["ranks"][2] = 7
    meta["b_strides"][2] = 8
    meta["b_offsets"][2] = meta["b_offsets"][3]
    a[2].mul_(0.5)
    b.mul_(0.75)
    x.mul_(0.75)
    meta["scales"].mul_(0.5)
    meta["token_indices"].copy_(meta["token_indices"].flip(0))
    for seg, slot in enumerate(meta["segment_slots"].tolist()):
        start, end = meta["segment_indptr"][seg : seg + 2].tolist()
        routes[meta["token_indices"][start:end].long()] = slot
    meta["segment_count"].sub_(2)  # drop the base and empty trailing segments
    output.copy_(base)
    z.fill_(3)
    expected_z = oracle_shrink(x, a, z, routes, meta["ranks"], 3)
    graph.replay()
    torch.cuda.synchronize()
    live = live_mask(routes.cpu().numpy(), meta["ranks"].cpu().numpy(), 3, z.shape[1])
    got_z = bf16_bits(z)
    close(got_z[live], expected_z[live])
    np.testing.assert_array_equal(bf16_bits(output), oracle_expand(z, b, base, meta))
    replay = output.clone()
    output.copy_(base)
    run()
    torch.testing.assert_close(output, replay, rtol=0, atol=0)


def test_scaled_delta_rounding_contract():
    kat = known_answers()["rounding"]
    device = "cuda:0"
    z = torch.tensor([[kat["z"]]], device=device, dtype=torch.bfloat16)
    b = torch.tensor([kat["b"]], device=device, dtype=torch.bfloat16)
    y = torch.tensor([[kat["y"]]], device=device, dtype=torch.bfloat16)

    def i(values, dtype=torch.int32):
        return torch.tensor(values, device=device, dtype=dtype)

    row_expand(
        z, b, y, b_offsets=i([0], torch.int64), b_strides=i([1]), ranks=i([1]),
        scales=i([kat["scale"]], torch.float32), segment_indptr=i([0, 1]),
        segment_slots=i([0]), token_indices=i([0]), slice_offsets=i([0, 1]),
        segment_count=i([1]),
    )
    assert y.item() == kat["expected"]
    assert torch.tensor(kat["scale"] + kat["y"]).bfloat16().item() == kat["single_rounding"]


def test_example_known_answer():
    kat = known_answers()["example"]
    device = "cuda:0"
    x = torch.tensor(kat["x"], device=device, dtype=torch.bfloat16)
    a = torch.tensor(kat["a"], device=device, dtype=torch.bfloat16)
    z = torch.zeros(3, 2, device=device, dtype=torch.bfloat16)
    b = torch.tensor(kat["b"], device=device, dtype=torch.bfloat16)
    y = torch.tensor(kat["y"], device=device, dtype=torch.bfloat16)

    def md(values, dtype=torch.int32):
        return torch.tensor(values, device=device, dtype=dtype)

    ranks = md(kat["ranks"])
    row_shrink(x, a, z, md(kat["routes"]), ranks, max_rank=kat["max_rank"])
    row_expand(
        z, b, y, b_offsets=md([0], torch.int64), b_strides=md([2]), ranks=ranks,
        scales=md(kat["scales"], torch.float32), segment_indptr=md(kat["segment_indptr"]),
        segment_slots=md(kat["segment_slots"]), token_indices=md(kat["token_indices"]),
        slice_offsets=md(kat["slice_offsets"]), segment_count=md([1]),
    )
    torch.testing.assert_close(y.cpu(), torch.tensor(kat["expected"], dtype=torch.bfloat16))


def test_reject_invalid_structures_and_aliases():
    x, a, z, b, _, output, routes, meta = row_case()
    with pytest.raises(ValueError, match="same CUDA"):
        row_shrink(x, a.cpu(), z, routes, meta["ranks"])
    with pytest.raises(ValueError, match="aligned"):
        row_shrink(x[:, 1:513], a[:, :, :512].contiguous(), z, routes, meta["ranks"])
    with pytest.raises(ValueError, match="inference"):
        row_expand(z.requires_grad_(), b, output, **meta)
    z.requires_grad_(False)
    with pytest.raises(ValueError, match="length"):
        row_expand(z, b, output, **(meta | {"b_offsets": meta["b_offsets"][:2]}))
    with pytest.raises(ValueError, match="threads"):
        row_expand(z, b, output, **meta, threads=64)
    with pytest.raises(ValueError, match="share storage"):
        row_expand(z, b, z[:, : output.shape[1]], **meta)


def test_empty_batch_and_zero_active_segments():
    x, a, z, b, _, output, routes, meta = row_case()
    before = output.clone()
    meta["segment_count"].zero_()
    row_expand(z, b, output, **meta)
    torch.testing.assert_close(output, before, rtol=0, atol=0)
    row_shrink(x[:0], a, z[:0], routes[:0], meta["ranks"])
    row_expand(z[:0], b, output[:0], **meta)


def test_repeated_calls_are_deterministic():
    x, a, z, b, _, output, routes, meta = row_case(slices=3, width=4096)
    row_shrink(x, a, z, routes, meta["ranks"], num_slices=3)
    first = z.clone()
    for _ in range(3):
        z.fill_(3)
        row_shrink(x, a, z, routes, meta["ranks"], num_slices=3)
        torch.testing.assert_close(z, first, rtol=0, atol=0)


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="two visible GPUs required")
def test_device_guard():
    x, a, z, b, _, output, routes, meta = row_case(device="cuda:1")
    with torch.cuda.device(0):
        row_shrink(x, a, z, routes, meta["ranks"])
        row_expand(z, b, output, **meta)
        assert torch.cuda.current_device() == 0
