"""Padded-slot decode BGMV (lora_shrink / lora_expand) on the B200.

Mirrors tests/test_gemv_gpu.py of lishenghui/loraforge: golden cases produced by
the reference's own oracle (FP32/FP16/BF16, 1-3 slices, capacities 8 and 33),
CUDA-graph replay with slot reload at fixed addresses, and large capacities.
"""

import numpy as np
import pytest

torch = pytest.importorskip("torch")
pytestmark = [
    pytest.mark.gpu,
    pytest.mark.skipif(not torch.cuda.is_available(), reason="CUDA device required"),
]

from golden_io import GOLDEN, load, to_torch  # noqa: E402
from oracle import cpu_reference as ref  # noqa: E402

from loraforge_b200.ops import lora_expand, lora_shrink  # noqa: E402

DTYPES = {"float32": torch.float32, "float16": torch.float16, "bfloat16": torch.bfloat16}
TOL = {torch.float32: 2e-5, torch.float16: 3e-3, torch.bfloat16: 2e-2}


def golden(name):
    d = load(name)
    dtype = DTYPES[name.split("_")[2]]
    dev = "cuda:0"
    xs = to_torch(d["x"], device=dev).to(dtype)
    # The reference's x is a stride-2 row view of a [14, 777] tensor.
    full = torch.zeros(2 * xs.shape[0], xs.shape[1], dtype=dtype, device=dev)
    full[::2] = xs
    x = full[::2]
    t = lambda k: to_torch(d[k], device=dev)  # noqa: E731
    return (
        x, t("a").to(dtype), t("b").to(dtype), t("ranks"), t("routes"), t("scales"),
        t("offsets"), int(d["max_slice"]), t("base").to(dtype), t("expected").to(dtype),
    )


@pytest.mark.parametrize("name", sorted(p.name for p in GOLDEN.glob("gemv_case_*.npz")))
def test_dense_decode(name):
    x, a, b, ranks, routes, scales, offsets, max_slice, base, expected = golden(name)
    slices = offsets.numel() - 1
    z = lora_shrink(x, a, ranks, routes, slices)
    result = lora_expand(z, b, ranks, scales, routes, offsets, max_slice, base)
    assert result.data_ptr() == base.data_ptr()
    tol = TOL[x.dtype]
    torch.testing.assert_close(result, expected, rtol=tol, atol=tol)
    assert z.dtype == x.dtype


def fixture(dtype, slices, capacity, seed=23):
    g = torch.Generator().manual_seed(seed)
    sizes = [5, 3, 7][:slices]
    x = (torch.randn(14, 777, generator=g) / 10).to(dtype).cuda()[::2]
    a = (torch.randn(4, slices * capacity, 777, generator=g) / 10).to(dtype).cuda()
    b = (torch.randn(4, sum(sizes), capacity, generator=g) / 10).to(dtype).cuda()
    ranks = torch.tensor([0, 1, min(3, capacity), capacity], device="cuda", dtype=torch.int64)
    routes = torch.tensor([0, 3, 2, 1, 3, 0, 2], device="cuda", dtype=torch.int64)
    scales = torch.tensor([0, 0.25, 1.5, 0.75], device="cuda")
    offsets = torch.tensor([0] + [sum(sizes[: i + 1]) for i in range(slices)], device="cuda")
    base = (torch.randn(7, sum(sizes) + 4, generator=g) / 10).to(dtype).cuda()
    return x, a, b, ranks, routes, scales, offsets, sizes, base


def expected_of(x, a, b, ranks, routes, scales, offsets, base):
    name = str(x.dtype).split(".")[-1]
    f = lambda t: t.float().cpu().numpy()  # noqa: E731
    out = ref.bgmv_reference(
        f(x), f(a), f(b), ranks.cpu().numpy(), routes.cpu().numpy(), scales.cpu().numpy(),
        offsets.cpu().numpy(), f(base), name,
    )
    return torch.from_numpy(out).to(x.dtype).cuda()


@pytest.mark.parametrize("dtype", [torch.float32, torch.float16, torch.bfloat16])
@pytest.mark.parametrize("slices", [1, 3])
def test_graph_routing_and_slot_reload(dtype, slices):
    x, a, b, ranks, routes, scales, offsets, sizes, _ = fixture(dtype, slices, 8)
    pointers = tuple(t.data_ptr() for t in (a, b, ranks, routes, scales))
    stream = torch.cuda.Stream()
    stream.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(stream):
        for _ in range(3):
            z = lora_shrink(x, a, ranks, routes, slices)
            lora_expand(z, b, ranks, scales, routes, offsets, max(sizes))
    stream.synchronize()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph, stream=stream):
        z = lora_shrink(x, a, ranks, routes, slices)
        result = lora_expand(z, b, ranks, scales, routes, offsets, max(sizes))
    for rank in (2, 0, 5):
        a[3].fill_(0.125)
        b[3].fill_(0.25)
        ranks[3] = rank
        scales[3] = 0.5 + rank
        routes.copy_(torch.tensor([3, 0, 1, 2, 3, 3, 0], device="cuda"))
        zeros = torch.zeros(7, sum(sizes), dtype=dtype, device="cuda")
        expected = expected_of(x, a, b, ranks, routes, scales, offsets, zeros)
        graph.replay()
        torch.cuda.synchronize()
        tol = TOL[dtype]
        torch.testing.assert_close(result, expected, rtol=tol, atol=tol)
    assert pointers == tuple(t.data_ptr() for t in (a, b, ranks, routes, scales))


@pytest.mark.parametrize("capacity", [128, 256])
def test_large_rank_capacity(capacity):
    x, a, b, ranks, routes, scales, offsets, sizes, base = fixture(torch.bfloat16, 1, capacity)
    expected = expected_of(x, a, b, ranks, routes, scales, offsets, base)
    z = lora_shrink(x, a, ranks, routes)
    actual = lora_expand(z, b, ranks, scales, routes, offsets, max(sizes), base)
    torch.testing.assert_close(actual, expected, rtol=0.02, atol=0.02)


def test_int32_metadata_and_aligned_vector_path():
    g = torch.Generator().manual_seed(5)
    x = (torch.randn(33, 4096, generator=g) / 10).bfloat16().cuda()
    a = (torch.randn(6, 3 * 16, 4096, generator=g) / 10).bfloat16().cuda()
    b = (torch.randn(6, 6144, 16, generator=g) / 10).bfloat16().cuda()
    ranks = torch.tensor([16, 8, 0, 16, 4, 16], dtype=torch.int32, device="cuda")
    routes = torch.randint(0, 6, (33,), generator=g, dtype=torch.int32).cuda()
    scales = torch.full((6,), 2.0, device="cuda")
    offsets = torch.tensor([0, 4096, 5120, 6144], dtype=torch.int32, device="cuda")
    base = torch.zeros(33, 6144, dtype=torch.bfloat16, device="cuda")
    expected = expected_of(x, a, b, ranks, routes, scales, offsets.long(), base)
    z = lora_shrink(x, a, ranks, routes, 3)
    out = lora_expand(z, b, ranks, scales, routes, offsets, 4096, base)
    torch.testing.assert_close(out, expected, rtol=2e-2, atol=2e-2)
    assert np.isfinite(out.float().cpu().numpy()).all()


@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16])
@pytest.mark.parametrize("capacity", [8, 16, 32, 64, 128])
@pytest.mark.parametrize("tokens", [3, 300])
def test_vector_expand_matches_scalar_form(dtype, capacity, tokens):
    # Unit-stride output rows take the 16-byte-vector walker kernel, a column-major output the
    # element-wise one; both do the same arithmetic, so the outputs agree bit for bit.
    g = torch.Generator().manual_seed(capacity * 7 + tokens)
    sizes = [1000, 2500, 777]
    width = sum(sizes)
    z = (torch.randn(tokens, 3 * capacity, generator=g) / 4).to(dtype).cuda()
    b = (torch.randn(5, width, capacity, generator=g) / 4).to(dtype).cuda()
    ranks = torch.tensor([capacity, 0, max(1, capacity // 2), 3, capacity], device="cuda")
    routes = torch.randint(-1, 5, (tokens,), generator=g).cuda()
    scales = torch.tensor([0.5, 1.0, 2.0, 0.25, 1.5], device="cuda")
    offsets = torch.tensor([0, 1000, 3500, width], device="cuda")
    base = (torch.randn(tokens, width, generator=g) / 4).to(dtype).cuda()
    vec = lora_expand(z, b, ranks, scales, routes, offsets, max(sizes), base.clone())
    column_major = base.t().contiguous().t()
    assert column_major.stride(1) != 1
    scalar = lora_expand(z, b, ranks, scales, routes, offsets, max(sizes), column_major)
    assert torch.equal(vec, scalar)
    assert torch.equal(vec[routes < 0], base[routes < 0])
    if (routes == 0).any():
        assert not torch.equal(vec[routes == 0], base[routes == 0])
