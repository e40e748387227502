"""Device grouping must be bit-exact against the oracle's stable grouping."""

import numpy as np
import pytest

torch = pytest.importorskip("torch")
pytestmark = [
    pytest.mark.gpu,
    pytest.mark.skipif(not torch.cuda.is_available(), reason="CUDA device required"),
]

from oracle import cpu_reference as ref  # noqa: E402

from loraforge_b200.ops.grouping import empty_routing, group_tokens  # noqa: E402


def check(slots_np, num_slots, chunk):
    slots = torch.tensor(slots_np, dtype=torch.int32, device="cuda")
    routing = group_tokens(slots, num_slots, chunk=chunk)
    torch.cuda.synchronize()
    indptr, seg_slots, perm, count = ref.group_tokens(slots_np, num_slots, chunk)
    got_count = int(routing.segment_count.item())
    assert got_count == count
    assert routing.segment_indptr[: count + 1].tolist() == indptr.tolist()
    assert routing.segment_slots[:count].tolist() == seg_slots.tolist()
    assert routing.token_indices[: len(slots_np)].tolist() == perm.tolist()


@pytest.mark.parametrize("seed", range(4))
@pytest.mark.parametrize("chunk", [0, 1, 16])
def test_random_routing(seed, chunk):
    rng = np.random.default_rng(seed)
    num_slots = int(rng.integers(1, 300))
    T = int(rng.integers(1, 3000))
    check(rng.integers(-2, num_slots + 2, size=T), num_slots, chunk)


@pytest.mark.parametrize(
    "T,num_slots,chunk",
    [(0, 4, 16), (1, 1, 16), (256, 128, 16), (512, 1024, 0), (8192, 64, 16), (40000, 16384, 16)],
)
def test_edge_sizes(T, num_slots, chunk):
    rng = np.random.default_rng(T)
    check(rng.integers(-1, num_slots, size=T), num_slots, chunk)


def test_all_inactive_and_single_slot():
    check(np.full(100, -1), 8, 16)
    check(np.full(100, 3), 8, 16)
    check(np.arange(100) % 2 - 1, 1, 0)


def test_zipf_decode_batch_and_reuse_of_buffers():
    rng = np.random.default_rng(7)
    ranks = np.arange(1, 129)
    p = 1.0 / ranks**1.1
    slots = rng.choice(128, size=256, p=p / p.sum()).astype(np.int32)
    out = empty_routing(256, "cuda")
    for _ in range(2):
        routing = group_tokens(torch.from_numpy(slots).cuda(), 128, chunk=16, out=out)
        assert routing.segment_indptr.data_ptr() == out.segment_indptr.data_ptr()
    indptr, seg_slots, perm, count = ref.group_tokens(slots, 128, 16)
    assert out.segment_indptr[: count + 1].tolist() == indptr.tolist()
    assert out.token_indices.tolist() == perm.tolist()


def test_graph_capture_replays_with_new_routes():
    slots = torch.zeros(300, dtype=torch.int32, device="cuda")
    out = empty_routing(300, "cuda")
    group_tokens(slots, 32, out=out)
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        group_tokens(slots, 32, out=out)
    rng = np.random.default_rng(3)
    for _ in range(3):
        new = rng.integers(-1, 32, size=300).astype(np.int32)
        slots.copy_(torch.from_numpy(new))
        graph.replay()
        torch.cuda.synchronize()
        indptr, seg_slots, perm, count = ref.group_tokens(new, 32, 16)
        assert out.segment_count.item() == count
        assert out.token_indices.tolist() == perm.tolist()
        assert out.segment_slots[:count].tolist() == seg_slots.tolist()


@pytest.mark.parametrize("chunk", [1, 16, 128])
def test_segment_routes_inverts_grouping(chunk):
    from loraforge_b200.ops.grouping import segment_routes

    rng = np.random.default_rng(chunk)
    slots_np = rng.integers(-1, 40, size=3000).astype(np.int32)
    slots = torch.from_numpy(slots_np).cuda()
    routing = group_tokens(slots, 40, chunk=chunk)
    routes = segment_routes(*routing, len(slots_np))
    torch.cuda.synchronize()
    # Grouping skips inactive tokens and slots outside [0, num_slots); they come back as -1.
    assert routes.cpu().numpy().tolist() == np.where(slots_np >= 0, slots_np, -1).tolist()


def test_segment_routes_ignores_padded_segments():
    from loraforge_b200.ops.grouping import segment_routes

    # Two live segments, then padding whose ranges point past the token table.
    indptr = torch.tensor([0, 2, 3, 9, 9], dtype=torch.int32, device="cuda")
    seg_slots = torch.tensor([5, 7, 9, 9], dtype=torch.int32, device="cuda")
    perm = torch.tensor([3, 0, 1], dtype=torch.int32, device="cuda")
    count = torch.tensor([2], dtype=torch.int32, device="cuda")
    routes = segment_routes(indptr, seg_slots, perm, count, 5)
    torch.cuda.synchronize()
    assert routes.tolist() == [5, 7, -1, 5, -1]
    count.fill_(4)  # padded segments now counted: their index range is clipped to the table
    routes = segment_routes(indptr, seg_slots, perm, count, 5)
    torch.cuda.synchronize()
    assert routes.tolist() == [5, 7, -1, 5, -1]


def split_runs_reference(indptr, seg_slots, perm, chunk):
    """Segments of the same grouping cut at every gap in token order, each run into pieces
    of at most `chunk` tokens from its own start (chunk <= 0: one piece per run)."""
    out_indptr, out_slots = [], []
    for s in range(len(seg_slots)):
        if s > 0 and seg_slots[s - 1] == seg_slots[s]:
            continue  # the slot's range was handled from its first segment
        e = s
        while e + 1 < len(seg_slots) and seg_slots[e + 1] == seg_slots[s]:
            e += 1
        lo, hi = int(indptr[s]), int(indptr[e + 1])
        p = lo
        while p < hi:
            q = p + 1
            while q < hi and perm[q] == perm[q - 1] + 1:
                q += 1
            step = chunk if chunk > 0 else q - p
            for a in range(p, q, step):
                out_indptr.append(a)
                out_slots.append(int(seg_slots[s]))
            p = q
    out_indptr.append(int(indptr[len(seg_slots)]))
    return out_indptr, out_slots


def runs_reference(slots_np, num_slots, chunk):
    """Runs of consecutive tokens with one slot, in token order, cut every `chunk` tokens
    from each run's start; active tokens in token order, then the others."""
    active = [0 <= int(s) < num_slots for s in slots_np]
    perm = [t for t, a in enumerate(active) if a] + [t for t, a in enumerate(active) if not a]
    indptr, seg_slots, pos, prev, start = [], [], 0, -1, 0
    for t, s in enumerate(slots_np):
        s = int(s) if active[t] else -1
        if s >= 0:
            if s != prev:
                start = t
            if s != prev or (chunk > 0 and (t - start) % chunk == 0):
                indptr.append(pos)
                seg_slots.append(s)
            pos += 1
        prev = s
    indptr.append(pos)
    return indptr, seg_slots, perm


def check_runs(slots_np, num_slots, chunk):
    slots = torch.tensor(slots_np, dtype=torch.int32, device="cuda")
    routing = group_tokens(slots, num_slots, chunk=chunk, runs=True)
    torch.cuda.synchronize()
    want_indptr, want_slots, want_perm = runs_reference(slots_np, num_slots, chunk)
    count = int(routing.segment_count.item())
    assert count == len(want_slots)
    assert routing.segment_indptr[: count + 1].tolist() == want_indptr
    assert routing.segment_slots[:count].tolist() == want_slots
    assert routing.token_indices[: len(slots_np)].tolist() == want_perm
    # Every segment is one run of one slot, at most `chunk` tokens.
    ind = routing.segment_indptr[: count + 1].cpu().numpy()
    tok = routing.token_indices.cpu().numpy()
    for s in range(count):
        run = tok[ind[s] : ind[s + 1]]
        assert len(run) >= 1 and (chunk <= 0 or len(run) <= chunk)
        assert np.all(np.diff(run) == 1)
        assert np.all(slots_np[run] == routing.segment_slots[s].item())


def check_split(slots_np, num_slots, chunk):
    # lf_split_runs on the slot-ordered grouping: the same token_indices, segments cut at
    # every gap in token order.
    from loraforge_b200 import _native

    T = len(slots_np)
    slots = torch.tensor(slots_np, dtype=torch.int32, device="cuda")
    first = group_tokens(slots, num_slots, chunk=chunk)
    out = empty_routing(T, "cuda")
    _native.call("lf_split_runs", first.segment_indptr.data_ptr(), first.segment_slots.data_ptr(),
                 first.token_indices.data_ptr(), first.segment_count.data_ptr(), T, chunk,
                 out.segment_indptr.data_ptr(), out.segment_slots.data_ptr(), out.segment_count.data_ptr(),
                 _native.stream_of(slots.device))
    torch.cuda.synchronize()
    indptr, seg_slots, perm, _ = ref.group_tokens(slots_np, num_slots, chunk)
    want_indptr, want_slots = split_runs_reference(indptr, seg_slots, perm, chunk)
    count = int(out.segment_count.item())
    assert count == len(want_slots)
    assert out.segment_indptr[: count + 1].tolist() == want_indptr
    assert out.segment_slots[:count].tolist() == want_slots


@pytest.mark.parametrize("chunk", [0, 5, 16, 128])
@pytest.mark.parametrize("seed", range(3))
def test_split_runs_prefill_batches(seed, chunk):
    # Requests of geometric lengths, adapters drawn with repeats, some without adapter.
    rng = np.random.default_rng(100 + seed)
    num_slots = int(rng.integers(2, 40))
    lengths = np.maximum(1, rng.geometric(1 / 200, size=int(rng.integers(1, 60))))
    owners = rng.integers(-1, num_slots, size=len(lengths))
    check_runs(np.repeat(owners, lengths), num_slots, chunk)
    check_split(np.repeat(owners, lengths), num_slots, chunk)


@pytest.mark.parametrize("chunk", [0, 3, 16])
def test_split_runs_scattered_and_edge_cases(chunk):
    rng = np.random.default_rng(7)
    for check in (check_runs, check_split):
        check(rng.integers(-2, 9, size=5000), 8, chunk)  # decode-like: many one-token runs
        check(np.full(1, 3), 4, chunk)
        check(np.full(300, -1), 4, chunk)  # no active token: no segment
        check(np.arange(70) % 2, 2, chunk)  # every run one token long
    # A batch past the split kernel's shared-memory codes (global-memory walks there).
    lengths = np.maximum(1, rng.geometric(1 / 900, size=90))
    big = np.repeat(rng.integers(-1, 12, size=len(lengths)), lengths)[:70000]
    check_runs(big, 12, chunk)
    check_split(big, 12, chunk)
