// LoRA expand kernels: out[t, n] += scale * B_g[n, :] · z[t, slice(n) packed rank].
//
// row_expand_kernel keeps the reference's per-element arithmetic exactly
// (src/loraforge/ops/csrc/lora_rows.cu:67-117: FP32 products accumulated over
// k = 0..bucket-1 in order with fused multiply-adds, the scaled delta rounded to
// BF16, added to the BF16 base and rounded again), so it is bit-identical to the
// reference kernel on identical inputs.  Its work item is a (segment or row-tile
// sub-segment, block of 2 x blockDim.x columns) pair of a persistent grid.  The
// reference walks an item's tokens with one read-modify-write of y after another,
// each a full memory round trip; here a thread keeps the B rows of its two columns
// in registers as packed BF16 and loads the old y values of every token of the item
// before the first product, so an item costs one round trip for all its tokens.
// The sub-tile's z values are staged in shared memory as FP32.
//
// bgmv_expand_kernel and vllm_expand_kernel serve the padded SGLang and vLLM
// layouts for FP32/FP16/BF16 activations, one CTA per (token, 256-column block).
// Where the element type is 16-bit and the B rows are aligned for 16-byte loads, the
// same arithmetic runs in *_vec_kernel forms: a CTA walks column blocks for one token
// with several 16-byte B loads per thread in flight.
#include <algorithm>

#include "launch.cuh"

namespace lfb {
namespace {

constexpr int kMaxSlices = 4;
constexpr int kSegRows = 16;
constexpr int kColsPerThread = 2;  // output columns per thread and item

// B row n of an item's slot held as packed BF16 pairs; the FP32 value of element k is
// recovered at the multiply (bits << 16 is exact).
template <int BR>
struct BRow {
  static constexpr int kWords = BR >= 2 ? BR / 2 : 1;
  uint32_t w[kWords];

  __device__ __forceinline__ void load(const uint16_t* bp) {
    if constexpr (BR >= 8) {
#pragma unroll
      for (int q = 0; q < BR / 8; ++q) {
        const uint4 v = reinterpret_cast<const uint4*>(bp)[q];
        w[4 * q] = v.x;
        w[4 * q + 1] = v.y;
        w[4 * q + 2] = v.z;
        w[4 * q + 3] = v.w;
      }
    } else if constexpr (BR == 4) {
      const uint2 v = *reinterpret_cast<const uint2*>(bp);
      w[0] = v.x;
      w[1] = v.y;
    } else if constexpr (BR == 2) {
      w[0] = *reinterpret_cast<const uint32_t*>(bp);
    } else {
      w[0] = bp[0];
    }
  }
  __device__ __forceinline__ float at(int k) const {
    if constexpr (BR == 1) return __uint_as_float(w[0] << 16);
    return (k & 1) ? __uint_as_float(w[k >> 1] & 0xffff0000u) : __uint_as_float(w[k >> 1] << 16);
  }
};

// The reference's per-element arithmetic for one (token, column): FP32 fused
// multiply-adds over k = 0..BR-1 in order from zero, the scaled sum rounded to BF16,
// added to the old BF16 value and rounded again.  Rows of up to 16 elements are held
// in registers (`head`); longer rows continue the same chain with 16-element chunks
// read again from L1 for every token, which keeps the register count of the kernel
// at the 16-element case.
constexpr int kHeld = 16;

template <int BR>
__device__ __forceinline__ uint16_t expand_value(const float* zt, const uint16_t* brow,
                                                 const BRow<(BR < kHeld ? BR : kHeld)>& head,
                                                 float scale, uint32_t old) {
  constexpr int H = BR < kHeld ? BR : kHeld;
  float acc = 0.f;
#pragma unroll
  for (int k = 0; k < H; ++k) acc = fmaf(zt[k], head.at(k), acc);
#pragma unroll 1
  for (int q = 1; q < BR / H; ++q) {
    BRow<H> b;
    b.load(brow + q * H);
#pragma unroll
    for (int k = 0; k < H; ++k) acc = fmaf(zt[q * H + k], b.at(k), acc);
  }
  const float delta = round_through_bf16(acc * scale);
  return uint16_t(float_to_bf16_bits(bf16_bits_to_float(old) + delta));
}

__device__ __forceinline__ void cp_async4(void* smem, const void* gmem) {
  asm volatile("cp.async.ca.shared.global [%0], [%1], 4;" ::"r"(
                   static_cast<uint32_t>(__cvta_generic_to_shared(smem))),
               "l"(gmem)
               : "memory");
}

// One item (sub-tile of T <= 16 rows, 2 * blockDim.x columns) for one thread, which
// owns two columns c0, c1.  PAIRED (even row stride, 4-byte aligned output): the
// columns are adjacent and one 4-byte value holds both.  Otherwise they are
// blockDim.x apart and move as 2-byte values.
//
// Before the barrier that publishes the z values, the thread issues its B rows (into
// registers) and, PAIRED, one asynchronous 4-byte copy per row of the old y values
// into its own shared-memory column `ys` (token t at ys[t * pitch]), so the HBM round
// trips of B, old y and z overlap.  A row listed twice in one item (malformed
// routing) voids the snapshot: the item is then updated in token order with one
// read-modify-write after another, as the reference's loop does.
template <int BR, bool PAIRED>
__device__ __noinline__ void expand_item(const uint16_t* __restrict__ z, const uint16_t* __restrict__ bslot,
                                            uint16_t* y, int64_t y_stride, int base, int N,
                                            const int* offs, int S, int cap, int rank, int T,
                                            const int* rows, float* zs, float scale, uint32_t* ys) {
  constexpr int H = BR < kHeld ? BR : kHeld;
  const int tid = threadIdx.x, pitch = blockDim.x;
  const int c0 = PAIRED ? base + 2 * tid : base + tid;
  const int c1 = PAIRED ? c0 + 1 : c0 + pitch;
  const bool one = c0 < N, two = c1 < N;
  const uint16_t* brow0 = bslot + int64_t(c0) * BR;
  const uint16_t* brow1 = bslot + int64_t(c1) * BR;
  BRow<H> b0, b1;
  if (one) b0.load(brow0);
  if (two) b1.load(brow1);
  if (PAIRED && two) {
#pragma unroll
    for (int t = 0; t < kSegRows; ++t)
      if (t < T) cp_async4(ys + t * pitch, y + int64_t(rows[t]) * y_stride + c0);
    asm volatile("cp.async.commit_group;" ::: "memory");
  }
  bool dup = false;
  if (tid < T)
    for (int u = 0; u < tid; ++u) dup |= rows[u] == rows[tid];
  for (int i = tid; i < T * S * BR; i += pitch) {
    const int t = i / (S * BR);
    const int rem = i - t * S * BR;
    const int s = rem / BR;
    const int k = rem - s * BR;
    zs[(t * kMaxSlices + s) * 64 + k] =
        k < rank ? bf16_bits_to_float(z[int64_t(rows[t]) * S * cap + s * rank + k]) : 0.f;
  }
  const bool distinct = !__syncthreads_or(dup);
  if (PAIRED && two) asm volatile("cp.async.wait_group 0;" ::: "memory");
  if (!one) return;
  int s0 = 0, s1 = 0;
  for (int i = 1; i < S; ++i) {
    if (c0 >= offs[i]) s0 = i;
    if (c1 >= offs[i]) s1 = i;
  }
  if (!distinct) {
    for (int t = 0; t < T; ++t) {
      uint16_t* yp = y + int64_t(rows[t]) * y_stride;
      const float* zt = zs + t * kMaxSlices * 64;
      yp[c0] = expand_value<BR>(zt + s0 * 64, brow0, b0, scale, yp[c0]);
      if (two) yp[c1] = expand_value<BR>(zt + s1 * 64, brow1, b1, scale, yp[c1]);
    }
    return;
  }
  if (!(PAIRED && two)) {  // 2-byte columns: both columns' old values, 8 rows at a time
    uint16_t* ys16 = reinterpret_cast<uint16_t*>(ys);
#pragma unroll 1
    for (int t0 = 0; t0 < T; t0 += 8) {
      uint16_t o0[8], o1[8];
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        const uint16_t* yp = y + int64_t(rows[min(t0 + j, T - 1)]) * y_stride;
        o0[j] = yp[c0];
        o1[j] = two ? yp[c1] : 0;
      }
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        ys16[2 * (t0 + j) * pitch] = o0[j];
        ys16[2 * (t0 + j) * pitch + 1] = o1[j];
      }
    }
  }
#pragma unroll 1
  for (int t = 0; t < T; ++t) {
    const uint32_t w = ys[t * pitch];
    const float* zt = zs + t * kMaxSlices * 64;
    uint16_t* yp = y + int64_t(rows[t]) * y_stride;
    const uint16_t v0 = expand_value<BR>(zt + s0 * 64, brow0, b0, scale, w & 0xffffu);
    if (!two) {
      yp[c0] = v0;
      continue;
    }
    const uint16_t v1 = expand_value<BR>(zt + s1 * 64, brow1, b1, scale, w >> 16);
    if (PAIRED) {
      *reinterpret_cast<uint32_t*>(yp + c0) = uint32_t(v0) | (uint32_t(v1) << 16);
    } else {
      yp[c0] = v0;
      yp[c1] = v1;
    }
  }
}

// Persistent grid over items = (segment sub-tile of row_tile tokens, block of
// blockDim.x * kColsPerThread output columns).  Per item: the sub-tile's rows and
// their z values (FP32, zero past the rank) are staged in shared memory, then each
// thread updates its columns for every row of the sub-tile.
template <bool PAIRED>
__global__ void __launch_bounds__(256, 4) row_expand_kernel(
    const uint16_t* __restrict__ z, const uint16_t* __restrict__ B,
    const int64_t* __restrict__ b_offsets, const int32_t* __restrict__ b_strides, uint16_t* y,
    int64_t y_stride, const int32_t* __restrict__ indptr, const int32_t* __restrict__ seg_slots,
    const int32_t* __restrict__ perm, const int32_t* __restrict__ ranks,
    const float* __restrict__ scales, const int32_t* __restrict__ slice_offsets,
    const int32_t* __restrict__ seg_count, int T_tokens, int N, int S, int cap, int num_slots,
    int max_segments, int row_tile) {
  __shared__ int rows[kSegRows];
  __shared__ int offs[kMaxSlices + 1];
  __shared__ __align__(16) float zs[kSegRows * kMaxSlices * 64];
  __shared__ uint32_t ys_all[kSegRows * 256];  // old y: both columns of a token, per thread
  const int tid = threadIdx.x;
  if (tid <= S) offs[tid] = slice_offsets[tid];
  const int parts = kSegRows / row_tile;
  const int span = blockDim.x * kColsPerThread;
  const int column_blocks = (N + span - 1) / span;
  const int nseg = min(*seg_count, max_segments);
  const int items = nseg * parts * column_blocks;
  for (int item = blockIdx.x; item < items; item += gridDim.x) {
    const int part = item / column_blocks;
    const int cb = item - part * column_blocks;
    const int seg = part / parts;
    const int seg_start = indptr[seg], seg_end = indptr[seg + 1];
    if (seg_end - seg_start > kSegRows) continue;  // segment contract: <= 16 tokens
    const int start = seg_start + (part - seg * parts) * row_tile;
    const int T = min(seg_end, start + row_tile) - start;
    const int g = seg_slots[seg];
    if (T <= 0 || g < 0 || g >= num_slots) continue;
    const int rank = ranks[g];
    const int bucket = b_strides[g];
    if (rank <= 0 || rank > 64 || rank > cap) continue;
    if (bucket < 1 || bucket > 64 || (bucket & (bucket - 1))) continue;
    __syncthreads();  // the previous item is done with rows and zs
    int row = -1;
    if (tid < T) {
      row = perm[start + tid];
      if (row < 0 || row >= T_tokens) row = -1;
      rows[tid] = row;
    }
    if (__syncthreads_or(tid < T && row < 0)) continue;  // uniform: one bad row skips the item
    const int base = cb * span;
    const uint16_t* bslot = B + b_offsets[g];
    const float scale = scales[g];
    uint32_t* ys = ys_all + tid;
    switch (bucket) {  // uniform across the CTA: expand_item's barrier is reached by all
      case 1: expand_item<1, PAIRED>(z, bslot, y, y_stride, base, N, offs, S, cap, rank, T, rows, zs, scale, ys); break;
      case 2: expand_item<2, PAIRED>(z, bslot, y, y_stride, base, N, offs, S, cap, rank, T, rows, zs, scale, ys); break;
      case 4: expand_item<4, PAIRED>(z, bslot, y, y_stride, base, N, offs, S, cap, rank, T, rows, zs, scale, ys); break;
      case 8: expand_item<8, PAIRED>(z, bslot, y, y_stride, base, N, offs, S, cap, rank, T, rows, zs, scale, ys); break;
      case 16: expand_item<16, PAIRED>(z, bslot, y, y_stride, base, N, offs, S, cap, rank, T, rows, zs, scale, ys); break;
      case 32: expand_item<32, PAIRED>(z, bslot, y, y_stride, base, N, offs, S, cap, rank, T, rows, zs, scale, ys); break;
      default: expand_item<64, PAIRED>(z, bslot, y, y_stride, base, N, offs, S, cap, rank, T, rows, zs, scale, ys); break;
    }
  }
}

// ------------------------------------------------------------------ padded BGMV expand
// One CTA per (token, 256-column block); the token's packed z row is staged as FP32.
template <typename T, typename I, typename OI, typename SC>
__global__ void bgmv_expand_kernel(const typename T::storage* __restrict__ z,
                                   const typename T::storage* __restrict__ B,
                                   const void* ranks, const typename SC::storage* scales,
                                   const void* map, const void* offsets,
                                   typename T::storage* y, int64_t ys0, int64_t ys1, int N,
                                   int num_slots, int S, int rmax) {
  extern __shared__ float zt[];  // S * rmax
  __shared__ int offs[17];
  const int t = blockIdx.x;
  const int g = load_index<I>(map, t);
  if (g < 0 || g >= num_slots) return;
  const int r = min(load_index<I>(ranks, g), rmax);
  if (r <= 0) return;
  for (int i = threadIdx.x; i < S * r; i += blockDim.x)
    zt[i] = T::to_float(z[int64_t(t) * S * rmax + i]);
  for (int i = threadIdx.x; i <= S && i < 17; i += blockDim.x) offs[i] = load_index<OI>(offsets, i);
  __syncthreads();
  const int n = blockIdx.y * blockDim.x + threadIdx.x;
  if (n >= N || n < offs[0] || n >= offs[S]) return;
  int s = 0;
  while (s + 1 < S && n >= offs[s + 1]) ++s;
  const typename T::storage* bp = B + (int64_t(g) * N + n) * rmax;
  const float* zs = zt + s * r;
  float acc = 0.f;
  for (int k = 0; k < r; ++k) acc = fmaf(zs[k], T::to_float(bp[k]), acc);
  const float delta = round_through<T>(acc * SC::to_float(scales[g]));
  typename T::storage* yp = y + int64_t(t) * ys0 + int64_t(n) * ys1;
  *yp = T::from_float(T::to_float(*yp) + delta);
}

// ------------------------------------------------------------------ column walkers
// The first RQ 16-byte pieces (8 * RQ elements) of one B row and the old output value of one
// (token, column), loaded ahead of their use.
template <int RQ>
struct RowPiece {
  uint4 w[RQ];
  float old;
};

template <typename T, int RQ>
__device__ __forceinline__ void load_piece(RowPiece<RQ>& p, const typename T::storage* row,
                                           int count, const typename T::storage* yp, bool live,
                                           bool read_old = true) {
  const uint4* v = reinterpret_cast<const uint4*>(row);
#pragma unroll
  for (int q = 0; q < RQ; ++q) p.w[q] = live && q * 8 < count ? __ldg(v + q) : make_uint4(0, 0, 0, 0);
  p.old = live && read_old ? T::to_float(*yp) : 0.f;
}

// acc = fma(lhs[k], row[k], acc) for k = 0 .. r - 1 in order: the piece's elements first, then
// the rest of the row (ranks above 8 * RQ) read 8 elements at a time.  An FMA's product is
// exact before its one rounding, so the operand order does not change the result.
template <typename T, int RQ>
__device__ __forceinline__ float row_products(const RowPiece<RQ>& p, const typename T::storage* row,
                                              const float* lhs, int r) {
  float acc = 0.f;
#pragma unroll
  for (int q = 0; q < RQ; ++q) {
    float b[8];
    unpack8<T>(p.w[q], b);
#pragma unroll
    for (int j = 0; j < 8; ++j)
      if (8 * q + j < r) acc = fmaf(lhs[8 * q + j], b[j], acc);
  }
  const uint4* v = reinterpret_cast<const uint4*>(row);
  for (int k0 = 8 * RQ; k0 < r; k0 += 8) {
    float b[8];
    unpack8<T>(__ldg(v + k0 / 8), b);
#pragma unroll
    for (int j = 0; j < 8; ++j)
      if (k0 + j < r) acc = fmaf(lhs[k0 + j], b[j], acc);
  }
  return acc;
}

// The staged z (or v) values of one slice, held in registers by a walker thread and reloaded
// from shared memory only when its column moves into another slice, so the products read no
// shared memory.  Used for rows of up to 32 elements (RQ <= 4).
template <int RQ>
struct HeldSlice {
  float v[8 * RQ];
  int slice = -1;

  __device__ __forceinline__ void select(int s, const float* values, int r) {
    if (s == slice) return;
    slice = s;
#pragma unroll
    for (int k = 0; k < 8 * RQ; ++k) v[k] = k < r ? values[k] : 0.f;
  }
};

// row_products with the left-hand values held in registers and the whole row in the piece
// (r <= 8 * RQ); full-length rows skip the per-element rank test.
template <typename T, int RQ>
__device__ __forceinline__ float held_products(const RowPiece<RQ>& p, const HeldSlice<RQ>& h,
                                               int r) {
  float acc = 0.f;
  if (r == 8 * RQ) {
#pragma unroll
    for (int q = 0; q < RQ; ++q) {
      float b[8];
      unpack8<T>(p.w[q], b);
#pragma unroll
      for (int j = 0; j < 8; ++j) acc = fmaf(h.v[8 * q + j], b[j], acc);
    }
  } else {
#pragma unroll
    for (int q = 0; q < RQ; ++q) {
      float b[8];
      unpack8<T>(p.w[q], b);
#pragma unroll
      for (int j = 0; j < 8; ++j)
        if (8 * q + j < r) acc = fmaf(h.v[8 * q + j], b[j], acc);
    }
  }
  return acc;
}

// RQ for a row capacity that is a multiple of 8: the whole row when it has at most 64 elements.
inline int row_pieces(int64_t elems) { return elems <= 8 ? 1 : elems <= 16 ? 2 : elems <= 32 ? 4 : 8; }

// Pieces in flight per thread: the next column's.  Rings of 2 and 4 pieces (more registers,
// fewer resident CTAs) measured slower on the decode shapes.
template <int RQ>
constexpr int ring_depth() { return 1; }

// Column walkers: about kWalkersPerSm CTAs per SM over all tokens (16 measured 2 % ahead of 8
// on the decode shapes over repeated runs, 4 level with 8, 32 slower).
constexpr int kWalkersPerSm = 16;

// bgmv_expand_kernel's arithmetic for 16-bit elements whose B rows are 16-byte aligned and a
// multiple of 8 elements long, with unit column stride.  A CTA stages its token's z once and
// walks the column blocks blockIdx.y, blockIdx.y + gridDim.y, ...; each thread keeps the B
// rows and old output values of its next D columns in flight (a ring of D pieces in
// registers, each refilled as soon as it is used), read as 16-byte vectors, and holds the z
// values of its column's slice in registers.  The chain of dependent loads (route, rank, z)
// is paid once per CTA instead of once per 256 columns.
template <typename T, typename I, typename OI, typename SC, int RQ>
__global__ void __launch_bounds__(256)
bgmv_expand_vec_kernel(const typename T::storage* __restrict__ z,
                       const typename T::storage* __restrict__ B, const void* ranks,
                       const typename SC::storage* scales, const void* map, const void* offsets,
                       typename T::storage* y, int64_t ys0, int N, int num_slots, int S, int rmax) {
  using St = typename T::storage;
  constexpr int D = ring_depth<RQ>();
  extern __shared__ float zt[];  // S * rmax
  __shared__ int offs[17];
  const int t = blockIdx.x;
  const int g = load_index<I>(map, t);
  if (g < 0 || g >= num_slots) return;
  const int r = min(load_index<I>(ranks, g), rmax);
  if (r <= 0) return;
  const St* bslot = B + int64_t(g) * N * rmax;
  St* yrow = y + int64_t(t) * ys0;
  const int step = gridDim.y * blockDim.x;
  const int first = blockIdx.y * blockDim.x + threadIdx.x;
  RowPiece<RQ> ring[D];
  const auto fetch = [&](RowPiece<RQ>& p, int col, bool live) {
    const int c = min(col, N - 1);
    load_piece<T, RQ>(p, bslot + int64_t(c) * rmax, r, yrow + c, live && col < N);
  };
#pragma unroll
  for (int d = 0; d < D; ++d) fetch(ring[d], first + d * step, true);
  for (int i = threadIdx.x; i < S * r; i += blockDim.x)
    zt[i] = T::to_float(z[int64_t(t) * S * rmax + i]);
  for (int i = threadIdx.x; i <= S && i < 17; i += blockDim.x) offs[i] = load_index<OI>(offsets, i);
  __syncthreads();
  const int lo = max(offs[0], 0), hi = min(offs[S], N);
  const float scale = SC::to_float(scales[g]);
  int s = 0;  // slice of the thread's column: its columns only increase
  HeldSlice<(RQ <= 4 ? RQ : 1)> held;
  for (int n = first; n < hi; n += D * step) {  // no barrier below: threads leave independently
#pragma unroll
    for (int d = 0; d < D; ++d) {
      const int col = n + d * step;
      if (col >= lo && col < hi) {
        while (s + 1 < S && col >= offs[s + 1]) ++s;
        float acc;
        if constexpr (RQ <= 4) {
          held.select(s, zt + s * r, r);
          acc = held_products<T, RQ>(ring[d], held, r);
        } else {
          acc = row_products<T, RQ>(ring[d], bslot + int64_t(col) * rmax, zt + s * r, r);
        }
        yrow[col] = T::from_float(ring[d].old + round_through<T>(acc * scale));
      }
      const int ahead = col + D * step;
      fetch(ring[d], ahead, ahead >= lo && ahead < hi);
    }
  }
}

// ------------------------------------------------------------------ vLLM expand
struct VllmSlices {
  lf_slice_desc d[8];
  int64_t begin[9];  // cumulative output columns of the slices
};

template <typename T>
__global__ void vllm_expand_kernel(const float* __restrict__ v, const __grid_constant__ VllmSlices sl,
                                   int S, int R, typename T::storage* y, int64_t y_stride,
                                   const int32_t* __restrict__ routes, int T_tokens,
                                   int num_slots, int64_t offset, int add) {
  extern __shared__ float vt[];  // S * R
  const int t = blockIdx.x;
  const int g = routes[t];
  if (g < 0 || g >= num_slots) return;
  for (int i = threadIdx.x; i < S * R; i += blockDim.x) {
    const int s = i / R, k = i - s * R;
    vt[i] = v[(int64_t(s) * T_tokens + t) * R + k];
  }
  __syncthreads();
  const int64_t n = int64_t(blockIdx.y) * blockDim.x + threadIdx.x;
  if (n >= sl.begin[S]) return;
  int s = 0;
  while (s + 1 < S && n >= sl.begin[s + 1]) ++s;
  const lf_slice_desc& d = sl.d[s];
  const typename T::storage* bp = reinterpret_cast<const typename T::storage*>(d.ptr) +
                                  int64_t(g) * d.slot_stride + (n - sl.begin[s]) * d.row_stride;
  const float* vs = vt + s * R;
  float acc = 0.f;
  for (int k = 0; k < R; ++k) acc = fmaf(T::to_float(bp[k]), vs[k], acc);
  typename T::storage* yp = y + int64_t(t) * y_stride + offset + n;
  if (add) acc += T::to_float(*yp);
  *yp = T::from_float(acc);
}

// vllm_expand_kernel's arithmetic for 16-bit elements whose slices all have 16-byte aligned
// bases and slot / row strides of a multiple of 8 elements, as a column walker with a ring of
// D pieces in flight per thread and the slice's v values held in registers (see
// bgmv_expand_vec_kernel).
template <typename T, int RQ>
__global__ void __launch_bounds__(256)
vllm_expand_vec_kernel(const float* __restrict__ v, const __grid_constant__ VllmSlices sl, int S,
                       int R, typename T::storage* y, int64_t y_stride,
                       const int32_t* __restrict__ routes, int T_tokens, int num_slots,
                       int64_t offset, int add) {
  using St = typename T::storage;
  constexpr int D = ring_depth<RQ>();
  extern __shared__ float vt[];  // S * R
  const int t = blockIdx.x;
  const int g = routes[t];
  if (g < 0 || g >= num_slots) return;
  const int64_t total = sl.begin[S];
  St* yrow = y + int64_t(t) * y_stride + offset;
  const auto row_of = [&](int64_t col, int& s) {
    s = 0;
    while (s + 1 < S && col >= sl.begin[s + 1]) ++s;
    return reinterpret_cast<const St*>(sl.d[s].ptr) + int64_t(g) * sl.d[s].slot_stride +
           (col - sl.begin[s]) * sl.d[s].row_stride;
  };
  const auto fetch = [&](RowPiece<RQ>& p, int64_t col) {
    const int64_t c = min(col, total - 1);
    int s;
    load_piece<T, RQ>(p, row_of(c, s), R, yrow + c, col < total, add != 0);
  };
  const int64_t step = int64_t(gridDim.y) * blockDim.x;
  const int64_t first = int64_t(blockIdx.y) * blockDim.x + threadIdx.x;
  RowPiece<RQ> ring[D];
#pragma unroll
  for (int d = 0; d < D; ++d) fetch(ring[d], first + d * step);
  for (int i = threadIdx.x; i < S * R; i += blockDim.x) {
    const int si = i / R, k = i - si * R;
    vt[i] = v[(int64_t(si) * T_tokens + t) * R + k];
  }
  __syncthreads();
  HeldSlice<(RQ <= 4 ? RQ : 1)> held;
  for (int64_t n = first; n < total; n += D * step) {  // no barrier below
#pragma unroll
    for (int d = 0; d < D; ++d) {
      const int64_t col = n + d * step;
      if (col < total) {
        int s;
        const St* row = row_of(col, s);
        float acc;
        if constexpr (RQ <= 4) {
          held.select(s, vt + s * R, R);
          acc = held_products<T, RQ>(ring[d], held, R);
        } else {
          acc = row_products<T, RQ>(ring[d], row, vt + s * R, R);
        }
        if (add) acc += ring[d].old;
        yrow[col] = T::from_float(acc);
      }
      fetch(ring[d], col + D * step);
    }
  }
}

// Column-block walkers per token for the *_vec_kernel forms: about kWalkersPerSm CTAs per SM
// over all tokens, at most one per column block.
inline unsigned column_walkers(int64_t tokens, unsigned column_blocks) {
  static int sms[64] = {};
  int device = 0;
  cudaGetDevice(&device);
  int& count = sms[device & 63];
  if (count == 0) cudaDeviceGetAttribute(&count, cudaDevAttrMultiProcessorCount, device);
  const int64_t want = (int64_t(std::max(count, 1)) * kWalkersPerSm + tokens - 1) /
                       std::max<int64_t>(tokens, 1);
  return unsigned(std::max<int64_t>(1, std::min<int64_t>(want, column_blocks)));
}

template <typename T, typename I, typename OI, typename SC>
int launch_bgmv_expand(const void* z, const void* b, const void* ranks, const void* scales,
                       const void* map, const void* offsets, void* y, int64_t ys0, int64_t ys1,
                       int64_t T_tokens, int N, int num_slots, int S, int rmax,
                       cudaStream_t stream) {
  using St = typename T::storage;
  const dim3 grid(unsigned(T_tokens), unsigned((N + 255) / 256));
  const size_t smem = sizeof(float) * size_t(S) * rmax;
  // S * rmax <= 16 * 256 FP32 values: always within the default 48 KiB of shared memory.
  if constexpr (sizeof(St) == 2) {
    if (rmax % 8 == 0 && ys1 == 1 && aligned16(b)) {
      auto kernel = bgmv_expand_vec_kernel<T, I, OI, SC, 8>;
      switch (row_pieces(rmax)) {
        case 1: kernel = bgmv_expand_vec_kernel<T, I, OI, SC, 1>; break;
        case 2: kernel = bgmv_expand_vec_kernel<T, I, OI, SC, 2>; break;
        case 4: kernel = bgmv_expand_vec_kernel<T, I, OI, SC, 4>; break;
      }
      const dim3 vgrid(unsigned(T_tokens), column_walkers(T_tokens, grid.y));
      kernel<<<vgrid, 256, smem, stream>>>(
          static_cast<const St*>(z), static_cast<const St*>(b), ranks,
          static_cast<const typename SC::storage*>(scales), map, offsets, static_cast<St*>(y),
          ys0, N, num_slots, S, rmax);
      return check_launch("bgmv_expand");
    }
  }
  bgmv_expand_kernel<T, I, OI, SC><<<grid, 256, smem, stream>>>(
      static_cast<const St*>(z), static_cast<const St*>(b), ranks,
      static_cast<const typename SC::storage*>(scales), map, offsets, static_cast<St*>(y), ys0,
      ys1, N, num_slots, S, rmax);
  return check_launch("bgmv_expand");
}

template <typename T, typename I, typename OI>
int bgmv_expand_sc(int32_t scale_dtype, const void* z, const void* b, const void* ranks,
                   const void* scales, const void* map, const void* offsets, void* y,
                   int64_t ys0, int64_t ys1, int64_t T_tokens, int N, int num_slots, int S,
                   int rmax, cudaStream_t stream) {
  switch (scale_dtype) {
    case LF_F32:
      return launch_bgmv_expand<T, I, OI, f32_t>(z, b, ranks, scales, map, offsets, y, ys0, ys1,
                                                 T_tokens, N, num_slots, S, rmax, stream);
    case LF_F16:
      return launch_bgmv_expand<T, I, OI, f16_t>(z, b, ranks, scales, map, offsets, y, ys0, ys1,
                                                 T_tokens, N, num_slots, S, rmax, stream);
    case LF_BF16:
      return launch_bgmv_expand<T, I, OI, bf16_t>(z, b, ranks, scales, map, offsets, y, ys0, ys1,
                                                  T_tokens, N, num_slots, S, rmax, stream);
  }
  return fail(LF_E_INVALID, "bgmv_expand: unsupported scale dtype");
}

template <typename T>
int bgmv_expand_t(int32_t scale_dtype, const void* z, const void* b, const void* ranks,
                  const void* scales, const void* map, int index_bits, const void* offsets,
                  int offset_bits, void* y, int64_t ys0, int64_t ys1, int64_t T_tokens, int N,
                  int num_slots, int S, int rmax, cudaStream_t stream) {
  if (index_bits == 32 && offset_bits == 32)
    return bgmv_expand_sc<T, int32_t, int32_t>(scale_dtype, z, b, ranks, scales, map, offsets, y,
                                               ys0, ys1, T_tokens, N, num_slots, S, rmax, stream);
  if (index_bits == 32)
    return bgmv_expand_sc<T, int32_t, int64_t>(scale_dtype, z, b, ranks, scales, map, offsets, y,
                                               ys0, ys1, T_tokens, N, num_slots, S, rmax, stream);
  if (offset_bits == 32)
    return bgmv_expand_sc<T, int64_t, int32_t>(scale_dtype, z, b, ranks, scales, map, offsets, y,
                                               ys0, ys1, T_tokens, N, num_slots, S, rmax, stream);
  return bgmv_expand_sc<T, int64_t, int64_t>(scale_dtype, z, b, ranks, scales, map, offsets, y,
                                             ys0, ys1, T_tokens, N, num_slots, S, rmax, stream);
}

template <typename T>
int launch_vllm_vec(dim3 grid, size_t smem, cudaStream_t s, const float* v, const VllmSlices& sl,
                    int num_slices, int rank, void* y, int64_t y_stride, const int32_t* routes,
                    int64_t num_tokens, int num_slots, int64_t offset, int add) {
  auto kernel = vllm_expand_vec_kernel<T, 8>;
  switch (row_pieces(rank)) {
    case 1: kernel = vllm_expand_vec_kernel<T, 1>; break;
    case 2: kernel = vllm_expand_vec_kernel<T, 2>; break;
    case 4: kernel = vllm_expand_vec_kernel<T, 4>; break;
  }
  const dim3 vgrid(grid.x, column_walkers(num_tokens, grid.y));
  kernel<<<vgrid, 256, smem, s>>>(v, sl, num_slices, rank, static_cast<typename T::storage*>(y),
                                  y_stride, routes, int(num_tokens), num_slots, offset, add);
  return check_launch("vllm_expand");
}

}  // namespace
}  // namespace lfb

using namespace lfb;

extern "C" int lf_row_expand(const void* z, const void* b, const int64_t* b_offsets,
                             const int32_t* b_strides, void* y, int64_t y_stride,
                             const int32_t* segment_indptr, const int32_t* segment_slots,
                             const int32_t* token_indices, const int32_t* ranks,
                             const float* scales, const int32_t* slice_offsets,
                             const int32_t* segment_count, int64_t num_tokens, int32_t out_width,
                             int32_t num_slices, int32_t capacity, int32_t num_slots,
                             int32_t max_segments, int32_t blocks, int32_t threads,
                             int32_t row_tile, void* stream) {
  if (num_tokens < 0 || num_tokens >= (int64_t(1) << 31) || out_width < 1)
    return fail(LF_E_INVALID, "row_expand: invalid token count or output width");
  if (num_slices < 1 || num_slices > kMaxSlices || capacity < 1 || num_slots < 1)
    return fail(LF_E_INVALID, "row_expand: invalid slice count, capacity or slot count");
  if (threads != 128 && threads != 256) return fail(LF_E_INVALID, "row_expand: threads must be 128 or 256");
  if (blocks < 0 || blocks > 65535) return fail(LF_E_INVALID, "row_expand: blocks must be in 0..65535");
  if (row_tile != 2 && row_tile != 4 && row_tile != 8 && row_tile != 16)
    return fail(LF_E_INVALID, "row_tile must be 2, 4, 8, or 16");
  if (y_stride < out_width || !aligned16(b))
    return fail(LF_E_INVALID, "row_expand: expected aligned B and nonoverlapping output rows");
  if (max_segments < 0) return fail(LF_E_INVALID, "row_expand: negative segment capacity");
  if (num_tokens == 0 || max_segments == 0) return LF_OK;
  const int span = threads * kColsPerThread;
  const int column_blocks = (out_width + span - 1) / span;
  if (int64_t(max_segments) * (kSegRows / row_tile) * column_blocks >= (int64_t(1) << 31))
    return fail(LF_E_INVALID, "row_expand: segment work count must fit signed int32 indexing");
  // Adjacent column pairs move as one 4-byte value when every row start is 4-byte aligned.
  const bool paired = y_stride % 2 == 0 && (reinterpret_cast<uintptr_t>(y) & 3u) == 0;
  auto kernel = paired ? row_expand_kernel<true> : row_expand_kernel<false>;
  if (blocks == 0) {  // automatic: every CTA the SMs hold at once
    int device = 0, sms = 0, per_sm = 0;
    cudaGetDevice(&device);
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, device);
    cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kernel, threads, 0);
    blocks = max(1, min(65535, sms * max(1, per_sm)));
  }
  kernel<<<blocks, threads, 0, static_cast<cudaStream_t>(stream)>>>(
      static_cast<const uint16_t*>(z), static_cast<const uint16_t*>(b), b_offsets, b_strides,
      static_cast<uint16_t*>(y), y_stride, segment_indptr, segment_slots, token_indices, ranks,
      scales, slice_offsets, segment_count, int(num_tokens), out_width, num_slices, capacity,
      num_slots, max_segments, row_tile);
  return check_launch("row_expand");
}

extern "C" int lf_bgmv_expand(int32_t dtype, const void* z, const void* b, const void* ranks,
                              const void* scales, int32_t scale_dtype, const void* token_map,
                              int32_t index_bits, const void* offsets, int32_t offset_bits,
                              void* y, int64_t y_stride0, int64_t y_stride1, int64_t num_tokens,
                              int32_t out_width, int32_t num_slots, int32_t num_slices,
                              int32_t rmax, void* stream) {
  if (num_tokens < 0 || num_tokens >= (int64_t(1) << 31) || out_width < 1 || num_slots < 1)
    return fail(LF_E_INVALID, "bgmv_expand: invalid sizes");
  if (num_slices < 1 || num_slices > 16 || rmax < 1 || rmax > 256)
    return fail(LF_E_INVALID, "bgmv_expand: 1..16 slices and rank capacity 1..256 required");
  if ((index_bits != 32 && index_bits != 64) || (offset_bits != 32 && offset_bits != 64))
    return fail(LF_E_INVALID, "bgmv_expand: index widths must be 32 or 64 bits");
  if (num_tokens == 0) return LF_OK;
  const cudaStream_t s = static_cast<cudaStream_t>(stream);
  switch (dtype) {
    case LF_F32:
      return bgmv_expand_t<f32_t>(scale_dtype, z, b, ranks, scales, token_map, index_bits,
                                  offsets, offset_bits, y, y_stride0, y_stride1, num_tokens,
                                  out_width, num_slots, num_slices, rmax, s);
    case LF_F16:
      return bgmv_expand_t<f16_t>(scale_dtype, z, b, ranks, scales, token_map, index_bits,
                                  offsets, offset_bits, y, y_stride0, y_stride1, num_tokens,
                                  out_width, num_slots, num_slices, rmax, s);
    case LF_BF16:
      return bgmv_expand_t<bf16_t>(scale_dtype, z, b, ranks, scales, token_map, index_bits,
                                   offsets, offset_bits, y, y_stride0, y_stride1, num_tokens,
                                   out_width, num_slots, num_slices, rmax, s);
  }
  return fail(LF_E_INVALID, "bgmv_expand: unsupported dtype");
}

extern "C" int lf_vllm_expand(int32_t dtype, const float* v, const lf_slice_desc* slices,
                              int32_t num_slices, int32_t num_slots, void* y, int64_t y_stride,
                              const int32_t* routes, int64_t num_tokens, int32_t rank,
                              int64_t offset, int32_t add, void* stream) {
  if (num_tokens < 0 || num_tokens >= (int64_t(1) << 31) || num_slots < 1)
    return fail(LF_E_INVALID, "vllm_expand: invalid sizes");
  if (num_slices < 1 || num_slices > 8 || !slices)
    return fail(LF_E_INVALID, "vllm_expand: 1..8 slices required");
  if (rank < 1 || rank > 256) return fail(LF_E_INVALID, "vllm_expand: rank must be in 1..256");
  if (num_tokens == 0) return LF_OK;
  VllmSlices sl{};
  sl.begin[0] = 0;
  for (int s = 0; s < num_slices; ++s) {
    sl.d[s] = slices[s];
    sl.begin[s + 1] = sl.begin[s] + slices[s].rows;
  }
  const int64_t total = sl.begin[num_slices];
  if (total < 1 || (total + 255) / 256 > 65535) return fail(LF_E_INVALID, "vllm_expand: invalid output width");
  const dim3 grid(unsigned(num_tokens), unsigned((total + 255) / 256));
  const size_t smem = sizeof(float) * size_t(num_slices) * rank;
  const cudaStream_t s = static_cast<cudaStream_t>(stream);
  bool vec = rank % 8 == 0;  // 16-byte B pieces: aligned bases, strides of 8 elements
  for (int i = 0; i < num_slices; ++i)
    vec = vec && aligned16(sl.d[i].ptr) && sl.d[i].slot_stride % 8 == 0 &&
          sl.d[i].row_stride % 8 == 0;
  switch (dtype) {
    case LF_F32:
      vllm_expand_kernel<f32_t><<<grid, 256, smem, s>>>(v, sl, num_slices, rank,
                                                        static_cast<float*>(y), y_stride, routes,
                                                        int(num_tokens), num_slots, offset, add);
      break;
    case LF_F16:
      if (vec)
        return launch_vllm_vec<f16_t>(grid, smem, s, v, sl, num_slices, rank, y, y_stride, routes,
                                      num_tokens, num_slots, offset, add);
      vllm_expand_kernel<f16_t><<<grid, 256, smem, s>>>(v, sl, num_slices, rank,
                                                        static_cast<__half*>(y), y_stride, routes,
                                                        int(num_tokens), num_slots, offset, add);
      break;
    case LF_BF16:
      if (vec)
        return launch_vllm_vec<bf16_t>(grid, smem, s, v, sl, num_slices, rank, y, y_stride, routes,
                                       num_tokens, num_slots, offset, add);
      vllm_expand_kernel<bf16_t><<<grid, 256, smem, s>>>(
          v, sl, num_slices, rank, static_cast<__nv_bfloat16*>(y), y_stride, routes,
          int(num_tokens), num_slots, offset, add);
      break;
    default:
      return fail(LF_E_INVALID, "vllm_expand: unsupported dtype");
  }
  return check_launch("vllm_expand");
}
