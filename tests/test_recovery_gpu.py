"""Recovery after a bounded device wait runs out, and after a workspace is overwritten.

No test here faults, traps or hangs a GPU:

* the peer z sum is run on one device as rank 0 of a two-rank group whose second buffer
  belongs to no process, so the flag it waits for is never set; with a spin limit of a few
  thousand polls the kernel gives up within milliseconds, keeps this rank's partial z, sets
  the status word the host reads, and the context stays usable;
* the completion counters of a decode workspace are overwritten from the host (as a
  workspace shared with foreign code might be); ``reset_workspace`` restores them and the
  next call is bit-identical to one on a fresh workspace; the library's built-in scratch
  gets the same check through ``reset_builtin_workspace``.
"""

import ctypes
import time

import pytest

torch = pytest.importorskip("torch")
pytestmark = [
    pytest.mark.gpu,
    pytest.mark.skipif(not torch.cuda.is_available(), reason="CUDA device required"),
]

from test_fused_gpu import decode_case  # noqa: E402

from loraforge_b200 import _native  # noqa: E402
from loraforge_b200.ops.fused import (  # noqa: E402
    lora_shrink_expand,
    sgmv_expand,
    sgmv_shrink,
    reset_builtin_workspace,
    reset_workspace,
    workspace_floats,
    z_rows,
)


def _peer_buffer(capacity):
    lib = _native.library()
    handle = (ctypes.c_char * lib.lf_peer_handle_bytes())()
    ptr = ctypes.c_void_p()
    _native.call("lf_peer_alloc", capacity, ctypes.byref(ptr), handle)
    return ptr.value


def _status(buffer, reset=False):
    v = ctypes.c_int32(-1)
    _native.call("lf_peer_status", buffer, ctypes.byref(v), 1 if reset else 0)
    return v.value


def test_peer_sum_wait_for_absent_rank_expires_with_status():
    torch.cuda.set_device(0)
    capacity = 4096
    own, absent = _peer_buffer(capacity), _peer_buffer(capacity)
    try:
        bases = torch.tensor([own, absent], dtype=torch.int64, device="cuda")
        z = torch.randn(capacity, device="cuda")
        before = z.clone()
        torch.cuda.synchronize()
        t0 = time.perf_counter()
        _native.call("lf_peer_sum", bases.data_ptr(), 0, 2, z.data_ptr(), z.numel(), capacity, 4000,
                     _native.stream_of(z.device))
        torch.cuda.synchronize()
        elapsed = time.perf_counter() - t0
        assert elapsed < 1.5, elapsed  # bounded: well under the default limit
        assert _status(own) == 1
        assert torch.equal(z, before)  # z keeps this rank's partial
        assert _status(own, reset=True) == 1 and _status(own) == 0
        # The context is still usable: a one-rank sum over the own buffer returns z itself.
        one = torch.tensor([own], dtype=torch.int64, device="cuda")
        _native.call("lf_peer_sum", one.data_ptr(), 0, 1, z.data_ptr(), z.numel(), capacity, 0,
                     _native.stream_of(z.device))
        torch.cuda.synchronize()
        assert torch.equal(z, before) and _status(own) == 0
    finally:
        torch.cuda.synchronize()
        _native.call("lf_peer_free", own)
        _native.call("lf_peer_free", absent)


def test_peer_all_reduce_raises_on_expiry(monkeypatch):
    from loraforge_b200.ops.sharded import PeerAllReduce

    peer = PeerAllReduce(1024)
    try:
        z = torch.ones(1024, device="cuda")
        peer(z)
        peer.raise_on_expiry()  # one rank: nothing to wait for, status 0
        # The status word as a rank whose wait ran out leaves it (the kernel path is
        # covered by the test above): the operator reports it and clears it.
        calls = []
        monkeypatch.setattr(peer, "status", lambda reset=False: calls.append(reset) or 1)
        with pytest.raises(RuntimeError, match="expired"):
            peer.raise_on_expiry()
        assert calls == [True]
    finally:
        monkeypatch.undo()
        peer.close()


def _two_launches(x, a, b, y, meta, S, ws):
    # The split-K shrink and the expand as two launches on one workspace: the path whose
    # per-segment completion counters live in the workspace (row-parallel calls take it; a
    # whole lora_shrink_expand call of rank <= 64 runs as one launch without a workspace).
    sgmv_shrink(x, a, b, y, workspace=ws, **meta, num_slices=S)
    sgmv_expand(x, a, b, y, workspace=ws, **meta, num_slices=S)


def test_overwritten_workspace_counters_are_restored_by_reset():
    x, a, b, base, slots_t, meta, S, cap = decode_case(seed=21, widths=(14336, 14336))
    T, K = x.shape
    fresh = torch.zeros(workspace_floats(T, K, S, cap), dtype=torch.float32, device="cuda")
    want = base.clone()
    _two_launches(x, a, b, want, meta, S, fresh)
    ws = torch.zeros_like(fresh)
    offset = z_rows(ws, T, K, S, cap).data_ptr() // 4 - ws.data_ptr() // 4
    row = z_rows(ws, T, K, S, cap).shape[1]
    counters = ws[offset + T * row : offset + T * row + T].view(torch.int32)
    counters.fill_(3)  # foreign values where the per-segment counters live
    reset_workspace(ws, T, K, S, cap)
    got = base.clone()
    _two_launches(x, a, b, got, meta, S, ws)
    torch.cuda.synchronize()
    assert torch.equal(got, want)
    assert int(counters.abs().sum()) == 0
    # And again on the same workspace: every call leaves the counters at zero.
    again = base.clone()
    _two_launches(x, a, b, again, meta, S, ws)
    torch.cuda.synchronize()
    assert torch.equal(again, want)


def test_builtin_scratch_reset_then_call_matches_workspace():
    x, a, b, base, slots_t, meta, S, cap = decode_case(seed=22)
    want = base.clone()
    lora_shrink_expand(x, a, b, want, **meta, num_slices=S)
    reset_builtin_workspace()
    got = base.clone()
    lora_shrink_expand(x, a, b, got, **meta, num_slices=S, workspace="builtin")
    torch.cuda.synchronize()
    assert torch.equal(got, want)
    assert _native.device_wait_timeouts(reset=True) == 0
