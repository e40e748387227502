"""CPU restatement of the reference's multi-LoRA shrink/expand semantics.

TEST INFRASTRUCTURE ONLY (see ``oracle/__init__.py``).  Arrays are numpy; BF16
tensors are carried as ``uint16`` bit patterns so every rounding is explicit.

Functions and the reference code they restate (paths inside lishenghui/loraforge):

* ``bf16_bits`` — ``round_bf16``, src/loraforge/ops/csrc/lora_rows.cu:27-33.
* ``row_shrink`` — the FP64 ``shrink_reference`` of
  tests/test_row_operators_gpu.py:99-106, with the kernel's rank/max_rank packing
  of src/loraforge/ops/csrc/lora_rows.cu:39-51.
* ``row_expand`` — the kernel arithmetic of src/loraforge/ops/csrc/lora_rows.cu:67-162
  (FP32 fused multiply-add over k = 0..bucket-1, BF16 scaled delta, BF16 sum),
  bit-exact: every product of two BF16 values is exact in FP32, so
  ``float32(acc + z*b)`` equals ``fmaf(z, b, acc)``.
* ``row_expand_fp64`` — ``expand_reference``, tests/test_row_operators_gpu.py:109-134.
* ``group_tokens`` — stable grouping by slot (SGLang 0.5.22 ``prepare_lora_batch``
  is not vendored; its order is restated as a stable sort, chunked like
  ``max_len`` 16 segments, cf. src/loraforge/integrations/_sglang_fleet.py:228-229).
* ``bgmv_reference`` — tests/test_gemv_gpu.py:52-67 (delta rounded to the dtype).
* ``vllm_reference`` — tests/test_vllm_gpu.py:30-44 (FP64, single final cast).
* ``lora_delta_fp32`` — the FP32 einsum over per-adapter gathers that BASELINE's
  tolerance gate and CPU baseline are defined on (torch CPU, all host threads).
"""

from __future__ import annotations

import numpy as np

F32 = np.float32


# ----------------------------------------------------------------------------- BF16
def bf16_bits(values) -> np.ndarray:
    """Round FP32 values to BF16 bit patterns (RNE; Inf/NaN exponents truncate)."""
    u = np.ascontiguousarray(values, dtype=F32).view(np.uint32).astype(np.uint64)
    finite = (u & 0x7F800000) != 0x7F800000
    u = np.where(finite, u + 0x7FFF + ((u >> 16) & 1), u)
    return ((u >> 16) & 0xFFFF).astype(np.uint16)


def bf16_value(bits) -> np.ndarray:
    """BF16 bit patterns -> FP32 values."""
    return (np.asarray(bits, dtype=np.uint16).astype(np.uint32) << 16).view(F32)


def round_bf16(values) -> np.ndarray:
    return bf16_value(bf16_bits(values))


def round_to(dtype: str, values) -> np.ndarray:
    """Round FP32/FP64 values through ``dtype`` ('float32', 'float16', 'bfloat16')."""
    v = np.asarray(values, dtype=np.float64).astype(F32)
    if dtype == "float32":
        return v
    if dtype == "float16":
        return v.astype(np.float16).astype(F32)
    if dtype == "bfloat16":
        return round_bf16(v)
    raise ValueError(dtype)


# ----------------------------------------------------------------------------- grouping
def group_tokens(slots, num_slots: int, chunk: int):
    """Stable grouping of tokens by slot.

    Returns (segment_indptr, segment_slots, token_indices, segment_count): active
    tokens sorted by slot with ties in token order, then tokens whose slot is
    outside [0, num_slots) in token order; per active slot ceil(count/chunk)
    segments (one per slot when chunk <= 0).
    """
    slots = np.asarray(slots, dtype=np.int64)
    active = (slots >= 0) & (slots < num_slots)
    key = np.where(active, slots, num_slots)
    perm = np.argsort(key, kind="stable").astype(np.int32)
    counts = np.bincount(slots[active], minlength=num_slots)
    indptr, seg_slots, pos = [], [], 0
    for s in range(num_slots):
        c = int(counts[s])
        if c == 0:
            continue
        pieces = -(-c // chunk) if chunk > 0 else 1
        for j in range(pieces):
            indptr.append(pos + (j * chunk if chunk > 0 else 0))
            seg_slots.append(s)
        pos += c
    indptr.append(pos)
    return (
        np.asarray(indptr, dtype=np.int32),
        np.asarray(seg_slots, dtype=np.int32),
        perm,
        len(seg_slots),
    )


# ----------------------------------------------------------------------------- row ops
def row_shrink(x, a, z_bits, slots, ranks, num_slices: int, max_rank: int) -> np.ndarray:
    """Retained-rank shrink in FP64, rounded (via FP32, as torch does) to BF16 bits.

    x: FP32 [T, K] (BF16 values); a: FP32 [slots, S*cap, K]; z_bits: uint16
    [T, S*cap].  Returns a new z bit array; untouched entries keep their bits.
    """
    out = np.array(z_bits, dtype=np.uint16, copy=True)
    S = num_slices
    cap = a.shape[1] // S
    nslots = len(ranks)
    for t, g in enumerate(np.asarray(slots)[: x.shape[0]]):
        if g < 0 or g >= nslots:
            continue
        r = int(ranks[g])
        if r <= 0:
            continue
        kk = min(r, max_rank)
        cols = np.array([s * r + k for s in range(S) for k in range(kk)], dtype=np.int64)
        cols = cols[cols < S * cap]
        vals = a[g, cols].astype(np.float64) @ x[t].astype(np.float64)
        out[t, cols] = bf16_bits(vals.astype(F32))
    return out


def _slice_of_columns(slice_offsets, n_cols):
    n = np.arange(n_cols)
    sl = np.zeros(n_cols, dtype=np.int64)
    for i in range(1, len(slice_offsets) - 1):
        sl[n >= slice_offsets[i]] = i
    return sl


def row_expand(
    z_bits, b_bits, y_bits, b_offsets, b_strides, ranks, scales, segment_indptr,
    segment_slots, token_indices, slice_offsets, segment_count,
) -> np.ndarray:
    """Bit-exact restatement of the reference RowExpand kernel; returns new y bits."""
    y = np.array(y_bits, dtype=np.uint16, copy=True)
    zf = bf16_value(z_bits)
    bf = bf16_value(b_bits)
    S = len(slice_offsets) - 1
    N = y.shape[1]
    cap = z_bits.shape[1] // S
    nslots = len(ranks)
    nseg = min(int(segment_count), len(segment_slots))
    slice_of = _slice_of_columns(slice_offsets, N)
    for seg in range(nseg):
        start, end = int(segment_indptr[seg]), int(segment_indptr[seg + 1])
        T = end - start
        g = int(segment_slots[seg])
        if T <= 0 or T > 16 or g < 0 or g >= nslots:
            continue
        rank, bucket = int(ranks[g]), int(b_strides[g])
        if rank <= 0 or rank > 64 or rank > cap:
            continue
        if bucket < 1 or bucket > 64 or bucket & (bucket - 1):
            continue
        off = int(b_offsets[g])
        B = bf[off : off + N * bucket].reshape(N, bucket)
        scale = F32(scales[g])
        for t in token_indices[start:end]:
            zs = np.zeros((S, bucket), dtype=F32)
            for s in range(S):
                live = min(bucket, rank)
                zs[s, :live] = zf[t, s * rank : s * rank + live]
            acc = np.zeros(N, dtype=F32)
            for k in range(bucket):
                acc = (acc + zs[slice_of, k] * B[:, k]).astype(F32)
            delta = round_bf16((acc * scale).astype(F32))
            y[t] = bf16_bits((bf16_value(y[t]) + delta).astype(F32))
    return y


def row_expand_fp64(z_bits, b_bits, y_bits, meta) -> np.ndarray:
    """FP64 dot, BF16 delta, BF16 sum: tests/test_row_operators_gpu.py:109-134."""
    y = np.array(y_bits, dtype=np.uint16, copy=True)
    zf = bf16_value(z_bits).astype(np.float64)
    bf = bf16_value(b_bits).astype(np.float64)
    ranks, bounds = meta["ranks"], meta["slice_offsets"]
    indptr, slots, indices = meta["segment_indptr"], meta["segment_slots"], meta["token_indices"]
    N = y.shape[1]
    base = bf16_value(y_bits)
    for seg in range(int(meta["segment_count"])):
        g = int(slots[seg])
        if g < 0 or not ranks[g]:
            continue
        r = int(ranks[g])
        off, bucket = int(meta["b_offsets"][g]), int(meta["b_strides"][g])
        w = bf[off : off + N * bucket].reshape(N, bucket)
        for row in indices[indptr[seg] : indptr[seg + 1]]:
            for s in range(len(bounds) - 1):
                lo, hi = int(bounds[s]), int(bounds[s + 1])
                value = w[lo:hi, :r] @ zf[row, s * r : (s + 1) * r]
                delta = round_bf16((value * float(meta["scales"][g])).astype(F32))
                y[row, lo:hi] = bf16_bits(base[row, lo:hi] + delta)
    return y


# ----------------------------------------------------------------------------- padded BGMV
def bgmv_reference(x, a, b, ranks, routes, scales, offsets, base, dtype: str):
    """tests/test_gemv_gpu.py:52-67 — z and delta rounded to ``dtype``; returns FP32."""
    expected = np.array(base, dtype=F32, copy=True)
    for row, slot in enumerate(routes):
        rank = int(ranks[slot])
        if not rank:
            continue
        for i in range(len(offsets) - 1):
            lo, hi = int(offsets[i]), int(offsets[i + 1])
            zz = round_to(dtype, x[row].astype(F32) @ a[slot, i * rank : (i + 1) * rank].astype(F32).T)
            delta = round_to(
                dtype, (zz @ b[slot, lo:hi, :rank].astype(F32).T) * F32(scales[slot])
            )
            expected[row, lo:hi] = round_to(dtype, expected[row, lo:hi] + delta)
    return expected


# ----------------------------------------------------------------------------- vLLM BGMV
def vllm_reference(x, a_slices, b_slices, routes, base, *, scale, offset=0, add=True, dtype="float32"):
    """tests/test_vllm_gpu.py:30-44 — FP64 shrink/expand, one final cast."""
    result = np.array(base, dtype=np.float64, copy=True)
    for aa, bb in zip(a_slices, b_slices):
        aa = aa.reshape(aa.shape[0], -1, x.shape[-1]).astype(np.float64)
        bb = bb.reshape(bb.shape[0], bb.shape[-2], -1).astype(np.float64)
        for t, g in enumerate(routes):
            if g >= 0:
                delta = (bb[g] @ (aa[g] @ x[t].astype(np.float64))) * scale
                cols = slice(offset, offset + bb.shape[-2])
                result[t, cols] = delta + (np.asarray(base, np.float64)[t, cols] if add else 0)
        offset += bb.shape[-2]
    return round_to(dtype, result)


# ----------------------------------------------------------------------------- FP32 einsum
def lora_delta_fp32(x, a, b_rows, slots, ranks, scales, slice_offsets, threads=None):
    """FP32 LoRA delta by einsum over per-adapter gathers (torch CPU).

    x: [T, K]; a: [slots, S*cap, K]; b_rows(g) -> [N, >=r] B rows of slot g;
    ranks/scales per slot.  Returns FP32 delta [T, N]; tokens with slot -1 (or
    rank 0) get zeros.  This is the computation BASELINE's tolerance gate and
    the CPU baseline are defined on.
    """
    import torch

    if threads is not None:
        torch.set_num_threads(threads)
    x = torch.as_tensor(x, dtype=torch.float32)
    slots_t = torch.as_tensor(np.asarray(slots), dtype=torch.int64)
    T = x.shape[0]
    S = len(slice_offsets) - 1
    N = int(slice_offsets[-1])
    out = torch.zeros(T, N, dtype=torch.float32)
    for g in torch.unique(slots_t).tolist():
        if g < 0:
            continue
        r = int(ranks[g])
        if r <= 0:
            continue
        idx = torch.nonzero(slots_t == g).flatten()
        A = torch.as_tensor(a[g][: S * r], dtype=torch.float32)
        zz = torch.einsum("tk,rk->tr", x[idx], A)
        B = torch.as_tensor(b_rows(g), dtype=torch.float32)[:, :r]
        for s in range(S):
            lo, hi = int(slice_offsets[s]), int(slice_offsets[s + 1])
            out[idx, lo:hi] += float(scales[g]) * torch.einsum(
                "tr,nr->tn", zz[:, s * r : (s + 1) * r], B[lo:hi]
            )
    return out.numpy()


# ----------------------------------------------------------------------------- gates
def half_ulp_bf16(values) -> np.ndarray:
    """Half a BF16 unit in the last place of each value (the rounding of an exact value)."""
    v = np.abs(np.asarray(values, dtype=np.float64))
    _, e = np.frexp(v)  # v = m * 2**e, m in [0.5, 1)
    return np.where(v > 0, np.ldexp(1.0, e - 9), 0.0)


def fp32_gate(out_values, ref32) -> dict:
    """BASELINE's max-abs gate for a BF16 output against the FP32 einsum.

    ``raw``: max|out - ref| / RMS(ref) (>= the output rounding itself, ~0.015 for
    Gaussian outputs); ``excess``: the same after discounting the half-ulp rounding
    that any BF16 output must incur — this is the number compared with 1e-2;
    ``exact``: the fraction of outputs equal to bf16(ref).
    """
    out = np.asarray(out_values, dtype=np.float64)
    ref = np.asarray(ref32, dtype=np.float64)
    rms = float(np.sqrt(np.mean(ref * ref))) or 1.0
    err = np.abs(out - ref)
    excess = np.maximum(err - half_ulp_bf16(ref), 0.0)
    exact = float(np.mean(round_bf16(ref.astype(F32)) == out.astype(F32)))
    return {"raw": float(err.max()) / rms, "excess": float(excess.max()) / rms, "exact": exact}
