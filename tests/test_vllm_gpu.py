"""vLLM padded-slot BGMV (vllm_gemv.shrink / expand) on the B200.

Mirrors test_raw_gemv of tests/test_vllm_gpu.py in lishenghui/loraforge against
golden outputs of the reference's FP64 oracle, plus determinism (the reference's
split-K atomics are replaced by sums in a fixed order) and bit identity of the walker
and element-wise expand kernels.
"""

import pytest

torch = pytest.importorskip("torch")
pytestmark = [
    pytest.mark.gpu,
    pytest.mark.skipif(not torch.cuda.is_available(), reason="CUDA device required"),
]

from golden_io import GOLDEN, load, to_torch  # noqa: E402

from loraforge_b200.ops.vllm_gemv import expand, shrink  # noqa: E402

DTYPES = {"float32": torch.float32, "float16": torch.float16, "bfloat16": torch.bfloat16}


def close(actual, expected):
    error = (actual.double() - expected.double()).norm()
    limit = 2e-5 if actual.dtype == torch.float32 else 0.01
    assert (error / expected.double().norm().clamp_min(1e-20)).item() < limit


def golden(name):
    d = load(name)
    dtype = DTYPES[name.split("_")[2]]
    dev = "cuda:0"
    t = lambda k: to_torch(d[k], device=dev).to(dtype)  # noqa: E731
    xs = t("x")
    full = torch.zeros(xs.shape[0], xs.shape[1] + 1, dtype=dtype, device=dev)
    full[:, : xs.shape[1]] = xs
    x = full[:, : xs.shape[1]]  # the reference's x is a [:, :513] view of [7, 514]
    rank = int(name.split("_r")[-1].split(".")[0])
    a = [t(f"a{i}") for i in range(3)]
    b = [t(f"b{i}") for i in range(3)]
    if rank != 7:  # padded 4D layouts, as the reference test uses for rank != 7
        a, b = [w.unsqueeze(1) for w in a], [w.unsqueeze(1) for w in b]
    routes = to_torch(d["routes"], device=dev)
    return x, a, b, routes, t("y"), t("expected"), t("expected_add"), rank


@pytest.mark.parametrize("name", sorted(p.name for p in GOLDEN.glob("vllm_case_*.npz")))
def test_raw_gemv(name):
    x, a, b, routes, y, expected, expected_add, rank = golden(name)
    before = y.clone()
    buf = torch.empty(3, x.shape[0], rank, device=x.device, dtype=torch.float32)
    shrink(x, a, buf, routes, scale=0.7)
    expand(buf, b, y, routes, offset=3, add=False)
    close(y, expected)
    torch.testing.assert_close(y[routes < 0], before[routes < 0], rtol=0, atol=0)
    torch.testing.assert_close(y[:, :3], before[:, :3], rtol=0, atol=0)
    torch.testing.assert_close(y[:, 54:], before[:, 54:], rtol=0, atol=0)
    y2 = before.clone()
    expand(buf, b, y2, routes, offset=0, add=True)
    close(y2, expected_add)


def test_deterministic_shrink_and_base_routes_zero():
    torch.manual_seed(1)
    x = torch.randn(64, 4096, device="cuda", dtype=torch.bfloat16)
    a = [torch.randn(8, 1, 32, 4096, device="cuda", dtype=torch.bfloat16) * 0.1 for _ in range(2)]
    routes = (torch.arange(64, device="cuda", dtype=torch.int32) % 9) - 1
    first = torch.empty(2, 64, 32, device="cuda")
    shrink(x, a, first, routes, scale=0.5)
    again = torch.empty_like(first)
    for _ in range(3):
        shrink(x, a, again, routes, scale=0.5)
        torch.testing.assert_close(again, first, rtol=0, atol=0)
    assert not first[:, routes < 0].any()


@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16])
@pytest.mark.parametrize("rank", [8, 16, 32, 64, 128])
@pytest.mark.parametrize("add", [False, True])
@pytest.mark.parametrize("tokens", [3, 300])
def test_vector_expand_matches_scalar_form(dtype, rank, add, tokens):
    # Slices with row strides of a multiple of 8 elements take the 16-byte-vector walker
    # kernel; the same values in rows padded by one element take the element-wise one.  Same
    # arithmetic, so the outputs agree bit for bit.
    g = torch.Generator().manual_seed(rank + (1 if add else 0) + tokens)
    sizes = [1000, 2500, 777]
    b = [(torch.randn(6, 1, n, rank, generator=g) / 4).to(dtype).cuda() for n in sizes]
    padded = []
    for w in b:
        p = torch.zeros(6, 1, w.shape[2], rank + 1, dtype=dtype, device="cuda")[..., :rank]
        p.copy_(w)
        assert p.stride(-2) % 8 != 0
        padded.append(p)
    v = (torch.randn(3, tokens, rank, generator=g) / 4).cuda()
    routes = torch.randint(-1, 6, (tokens,), generator=g, dtype=torch.int32).cuda()
    y = (torch.randn(tokens, sum(sizes) + 9, generator=g) / 4).to(dtype).cuda()
    vec, scalar = y.clone(), y.clone()
    expand(v, b, vec, routes, offset=5, add=add)
    expand(v, padded, scalar, routes, offset=5, add=add)
    assert torch.equal(vec, scalar)
    assert torch.equal(vec[routes < 0], y[routes < 0])
    end = 5 + sum(sizes)
    assert torch.equal(vec[:, :5], y[:, :5]) and torch.equal(vec[:, end:], y[:, end:])
