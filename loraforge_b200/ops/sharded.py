"""Megatron-style tensor-parallel LoRA over B200 ranks (one process per GPU).

The reference runs this path only at tensor parallelism 1 (the fleet backend rejects
TP != 1, src/loraforge/integrations/_sglang_fleet.py:177-178); these helpers add the two
natural shardings of a LoRA-augmented projection:

* column-parallel (QKV, gate/up): rank g owns a 1/G slice of every output slice's
  columns.  A is replicated, so each rank runs the full shrink and expands only its
  columns; there is no communication.
* row-parallel (down): rank g owns a 1/G slice of the input columns of x and A.  Each
  rank's shrink gives a partial z; one all-reduce (sum) of the FP32 z rows
  ([tokens, S*r]) over the group makes it whole, and each rank expands its 1/G slice of
  the output columns (its B rows), so no B row is read twice.

The weight helpers run at load time on either device; the two operators are
asynchronous on the current stream.  The row-parallel z sum is the group's all-reduce,
or ``PeerAllReduce``: one kernel over NVLink peer memory (CUDA IPC buffers, release /
acquire flags between the GPUs), which at decode sizes (tens of KiB) is bound by latency
rather than bandwidth.
"""

from __future__ import annotations

from loraforge_b200 import _native
from loraforge_b200.ops.fused import lora_shrink_expand, sgmv_expand, sgmv_shrink, z_rows


def shard_bounds(width: int, rank: int, world: int) -> tuple[int, int]:
    """[begin, end) of rank's equal share of `width` columns (width % world == 0)."""
    if world < 1 or not 0 <= rank < world:
        raise ValueError("rank must be in [0, world)")
    if width % world:
        raise ValueError(f"width {width} is not divisible by {world} ranks")
    share = width // world
    return rank * share, (rank + 1) * share


def shard_a_columns(a, rank: int, world: int):
    """A [slots, S*cap, K] -> rank's input-column shard [slots, S*cap, K/world] (contiguous)."""
    lo, hi = shard_bounds(a.shape[2], rank, world)
    return a[:, :, lo:hi].contiguous()


def shard_b_columns(b, b_offsets, b_strides, slice_widths, rank: int, world: int):
    """Compact B store of rank's output-column shard of every slice.

    b: flat BF16 store; slot g's [N, bucket_g] rows at b_offsets[g] (N = sum of the slice
    widths).  Returns (b_shard, offsets_shard, slice_widths_shard): the slot blocks keep
    their buckets, hold rank's rows of each slice in slice order, and start at 8-element
    boundaries.
    """
    import torch

    offsets = [int(v) for v in b_offsets.tolist()]
    strides = [int(v) for v in b_strides.tolist()]
    n = sum(slice_widths)
    bounds, start = [], 0
    for w in slice_widths:
        lo, hi = shard_bounds(w, rank, world)
        bounds.append((start + lo, start + hi))
        start += w
    pieces, new_offsets, cursor = [], [], 0
    for off, bucket in zip(offsets, strides):
        pad = (-cursor) % 8
        if pad:
            pieces.append(torch.zeros(pad, dtype=b.dtype, device=b.device))
            cursor += pad
        rows = b[off : off + n * bucket].view(n, bucket)
        block = torch.cat([rows[lo:hi] for lo, hi in bounds]).reshape(-1)
        new_offsets.append(cursor)
        pieces.append(block)
        cursor += block.numel()
    shard = torch.cat(pieces) if pieces else b[:0]
    offsets_t = torch.tensor(new_offsets, dtype=torch.int64, device=b_offsets.device)
    return shard, offsets_t, tuple(w // world for w in slice_widths)


def column_parallel(x, a, b_shard, y_shard, **meta) -> None:
    """Column-parallel LoRA: full shrink, expand of this rank's output columns only.

    ``b_shard`` / ``y_shard`` and the routing/metadata keywords as for
    ``lora_shrink_expand`` (``slice_offsets`` of the shard's slice widths).
    """
    lora_shrink_expand(x, a, b_shard, y_shard, **meta)


def row_parallel(x_shard, a_shard, b_shard, y_shard, *, workspace, group=None, peer=None,
                 check_peer: bool = True, **meta) -> None:
    """Row-parallel LoRA: partial shrink, all-reduce of the FP32 z rows, sharded expand.

    ``x_shard`` / ``a_shard`` hold this rank's input columns, ``b_shard`` / ``y_shard``
    its output columns; ``workspace`` (zero-filled before first use) must not be shared
    with another call in flight.  ``peer`` (a ``PeerAllReduce`` of the group) sums the z
    rows over NVLink peer memory in one kernel; without it the group's all-reduce is used.
    With ``group`` None and no initialised process group this is the single-rank
    computation.

    A peer sum whose wait for another rank ran out leaves this rank's partial z, so the
    output is invalid.  With ``check_peer`` (default) the call reads the peer status after
    launching the expand (a synchronising read, skipped while the stream is being
    captured) and raises ``RuntimeError`` on expiry; pass ``check_peer=False`` in a hot
    loop and call ``peer.raise_on_expiry()`` at step boundaries instead.
    """
    import torch
    import torch.distributed as dist

    sgmv_shrink(x_shard, a_shard, b_shard, y_shard, workspace=workspace, **meta)
    num_slices = meta.get("num_slices", 1)
    z = z_rows(workspace, x_shard.shape[0], x_shard.shape[1], num_slices, a_shard.shape[1] // num_slices)
    if peer is not None:
        peer(z)
    elif dist.is_available() and dist.is_initialized() and dist.get_world_size(group) > 1:
        dist.all_reduce(z, op=dist.ReduceOp.SUM, group=group)
    sgmv_expand(x_shard, a_shard, b_shard, y_shard, workspace=workspace, **meta)
    if peer is not None and check_peer and not torch.cuda.is_current_stream_capturing():
        peer.raise_on_expiry()


class PeerAllReduce:
    """Sum of FP32 tensors over a process group through NVLink peer memory, one kernel.

    The row-parallel z rows are tens of KiB, so a library all-reduce costs its launch and
    protocol latency, not bandwidth.  Every rank owns one buffer mapped by all the others
    (CUDA IPC); ``__call__`` runs ``lf_peer_sum``: copy the local values into the own
    buffer, flag every peer, wait for every peer's flag (bounded), add the ranks' buffers
    in rank order into the tensor.  Every rank gets the same bits.

    Construction and ``close`` are collective (every rank, same order; construction
    allocates and maps, calls do not).  ``capacity`` is the largest tensor (in floats) it
    will sum.  Calls are asynchronous on the tensor device's current stream and may be
    captured in a CUDA graph.  ``status()`` is 1 after a wait for a peer ran out;
    ``spin_limit`` bounds that wait in polls of the flag (None: the library default, well
    under 2 s).
    """

    def __init__(self, capacity: int, *, group=None, device=None, spin_limit: int | None = None):
        import ctypes

        import torch
        import torch.distributed as dist

        if type(capacity) is not int or capacity < 1:
            raise ValueError("capacity must be a positive integer")
        distributed = dist.is_available() and dist.is_initialized()
        self.world = dist.get_world_size(group) if distributed else 1
        self.rank = dist.get_rank(group) if distributed else 0
        if self.world > 16:
            raise ValueError("peer sums support up to 16 ranks")
        if spin_limit is not None and (type(spin_limit) is not int or spin_limit < 1):
            raise ValueError("spin_limit must be a positive integer")
        self.capacity, self.group, self.spin_limit = capacity, group, spin_limit or 0
        self.device = torch.device("cuda", torch.cuda.current_device()) if device is None else torch.device(device)
        lib = _native.library()
        handle = (ctypes.c_char * lib.lf_peer_handle_bytes())()
        own = ctypes.c_void_p()
        with torch.cuda.device(self.device):
            _native.call("lf_peer_alloc", capacity, ctypes.byref(own), handle)
        self._own = own.value
        handles = [bytes(handle)] * self.world
        if self.world > 1:
            dist.all_gather_object(handles, bytes(handle), group=group)
        self._opened, bases = [], []
        with torch.cuda.device(self.device):
            for r, h in enumerate(handles):
                if r == self.rank:
                    bases.append(self._own)
                    continue
                mapped = ctypes.c_void_p()
                _native.call("lf_peer_open", (ctypes.c_char * len(h)).from_buffer_copy(h), ctypes.byref(mapped))
                self._opened.append(mapped.value)
                bases.append(mapped.value)
        self.bases = torch.tensor(bases, dtype=torch.int64, device=self.device)

    def __call__(self, z) -> None:
        import torch

        if not isinstance(z, torch.Tensor):
            raise TypeError("z must be a torch.Tensor")
        if z.dtype != torch.float32 or z.device != self.device or not z.is_contiguous():
            raise ValueError("z must be a contiguous FP32 tensor on the buffers' device")
        if z.numel() > self.capacity or z.data_ptr() % 16:
            raise ValueError(f"z must be 16-byte aligned with at most {self.capacity} elements")
        with torch.cuda.device(self.device):
            _native.call("lf_peer_sum", self.bases.data_ptr(), self.rank, self.world, z.data_ptr(), z.numel(),
                         self.capacity, self.spin_limit, _native.stream_of(self.device))

    def status(self, reset: bool = False) -> int:
        """1 if a wait for a peer expired since the last reset (synchronous)."""
        import ctypes

        import torch

        value = ctypes.c_int32(0)
        with torch.cuda.device(self.device):
            _native.call("lf_peer_status", self._own, ctypes.byref(value), 1 if reset else 0)
        return value.value

    def raise_on_expiry(self) -> None:
        """Raise RuntimeError (and clear the status) if a wait for a peer ran out."""
        if self.status(reset=True):
            raise RuntimeError(
                "peer z sum: a wait for another rank expired; this rank's z kept its partial "
                "sum and the step's outputs are invalid"
            )

    def close(self) -> None:
        """Collective: wait for every rank's last sum, then unmap and free the buffers."""
        import torch
        import torch.distributed as dist

        if self._own is None:
            return
        with torch.cuda.device(self.device):
            torch.cuda.synchronize()
            if self.world > 1:
                dist.barrier(group=self.group)
            for ptr in self._opened:
                _native.call("lf_peer_close", ptr)
            _native.call("lf_peer_free", self._own)
        self._own, self._opened = None, []
