// LoRA expand kernels: out[t, n] += scale * B_g[n, :] · z[t, slice(n) packed rank].
//
// row_expand_kernel keeps the reference's per-element arithmetic exactly
// (src/loraforge/ops/csrc/lora_rows.cu:67-117: FP32 products accumulated over
// k = 0..bucket-1 in order with fused multiply-adds, the scaled delta rounded to
// BF16, added to the BF16 base and rounded again), so it is bit-identical to the
// reference kernel on identical inputs.  Its work item is a (segment or row-tile
// sub-segment, column block) pair of a persistent grid; each thread keeps its B row
// in registers and walks the segment's <= 16 tokens, whose z values are staged in
// shared memory as FP32.
//
// bgmv_expand_kernel and vllm_expand_kernel serve the padded SGLang and vLLM
// layouts for FP32/FP16/BF16 activations.
#include "launch.cuh"

namespace lfb {
namespace {

constexpr int kMaxSlices = 4;
constexpr int kSegRows = 16;

template <int BR>
__device__ __forceinline__ void load_b_row(const uint16_t* bp, float* b) {
  if constexpr (BR >= 8) {
#pragma unroll
    for (int q = 0; q < BR; q += 8) unpack_bf16x8(*reinterpret_cast<const uint4*>(bp + q), b + q);
  } else if constexpr (BR == 4) {
    const uint2 v = *reinterpret_cast<const uint2*>(bp);
    b[0] = __uint_as_float(v.x << 16);
    b[1] = __uint_as_float(v.x & 0xffff0000u);
    b[2] = __uint_as_float(v.y << 16);
    b[3] = __uint_as_float(v.y & 0xffff0000u);
  } else if constexpr (BR == 2) {
    const uint32_t v = *reinterpret_cast<const uint32_t*>(bp);
    b[0] = __uint_as_float(v << 16);
    b[1] = __uint_as_float(v & 0xffff0000u);
  } else {
    b[0] = bf16_bits_to_float(bp[0]);
  }
}

// One output column n for the tokens of the current item.
template <int BR>
__device__ __forceinline__ void expand_column(const uint16_t* bp, uint16_t* y, int64_t y_stride,
                                              int n, int slice, int T, const int* rows,
                                              const float* zs, float scale) {
  float b[BR];
  load_b_row<BR>(bp + int64_t(n) * BR, b);
  for (int t = 0; t < T; ++t) {
    const float* zt = zs + (t * kMaxSlices + slice) * 64;
    float acc = 0.f;
#pragma unroll
    for (int k = 0; k < BR; ++k) acc = fmaf(zt[k], b[k], acc);
    uint16_t* yp = y + int64_t(rows[t]) * y_stride + n;
    const float delta = bf16_bits_to_float(float_to_bf16_bits(acc * scale));
    *yp = uint16_t(float_to_bf16_bits(bf16_bits_to_float(*yp) + delta));
  }
}

__global__ void row_expand_kernel(const uint16_t* __restrict__ z, const uint16_t* __restrict__ B,
                                  const int64_t* __restrict__ b_offsets,
                                  const int32_t* __restrict__ b_strides, uint16_t* y,
                                  int64_t y_stride, const int32_t* __restrict__ indptr,
                                  const int32_t* __restrict__ seg_slots,
                                  const int32_t* __restrict__ perm,
                                  const int32_t* __restrict__ ranks,
                                  const float* __restrict__ scales,
                                  const int32_t* __restrict__ slice_offsets,
                                  const int32_t* __restrict__ seg_count, int T_tokens, int N,
                                  int S, int cap, int num_slots, int max_segments,
                                  int row_tile) {
  __shared__ int rows[kSegRows];
  __shared__ int offs[kMaxSlices + 1];
  __shared__ float zs[kSegRows * kMaxSlices * 64];
  const int tid = threadIdx.x;
  if (tid <= S) offs[tid] = slice_offsets[tid];
  const int parts = kSegRows / row_tile;
  const int column_blocks = (N + blockDim.x - 1) / blockDim.x;
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
    __syncthreads();  // the previous item is done with rows/zs
    if (tid < T) {
      const int row = perm[start + tid];
      rows[tid] = (row >= 0 && row < T_tokens) ? row : -1;
    }
    __syncthreads();
    bool valid = true;
    for (int t = 0; t < T; ++t) valid &= rows[t] >= 0;
    if (!valid) continue;  // uniform: every thread read the same rows
    for (int i = tid; i < T * S * bucket; i += blockDim.x) {
      const int t = i / (S * bucket);
      const int rem = i - t * S * bucket;
      const int s = rem / bucket;
      const int k = rem - s * bucket;
      zs[(t * kMaxSlices + s) * 64 + k] =
          k < rank ? bf16_bits_to_float(z[int64_t(rows[t]) * S * cap + s * rank + k]) : 0.f;
    }
    __syncthreads();
    const int n = cb * blockDim.x + tid;
    if (n < N) {
      int slice = 0;
      for (int i = 1; i < S; ++i)
        if (n >= offs[i]) slice = i;
      const uint16_t* bp = B + b_offsets[g];
      const float scale = scales[g];
      switch (bucket) {
        case 1: expand_column<1>(bp, y, y_stride, n, slice, T, rows, zs, scale); break;
        case 2: expand_column<2>(bp, y, y_stride, n, slice, T, rows, zs, scale); break;
        case 4: expand_column<4>(bp, y, y_stride, n, slice, T, rows, zs, scale); break;
        case 8: expand_column<8>(bp, y, y_stride, n, slice, T, rows, zs, scale); break;
        case 16: expand_column<16>(bp, y, y_stride, n, slice, T, rows, zs, scale); break;
        case 32: expand_column<32>(bp, y, y_stride, n, slice, T, rows, zs, scale); break;
        default: expand_column<64>(bp, y, y_stride, n, slice, T, rows, zs, scale); break;
      }
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

template <typename T, typename I, typename OI, typename SC>
int launch_bgmv_expand(const void* z, const void* b, const void* ranks, const void* scales,
                       const void* map, const void* offsets, void* y, int64_t ys0, int64_t ys1,
                       int64_t T_tokens, int N, int num_slots, int S, int rmax,
                       cudaStream_t stream) {
  using St = typename T::storage;
  const dim3 grid(unsigned(T_tokens), unsigned((N + 255) / 256));
  const size_t smem = sizeof(float) * size_t(S) * rmax;
  static int flags[64] = {};
  auto kernel = bgmv_expand_kernel<T, I, OI, SC>;
  if (int rc = ensure_smem(kernel, int(smem), flags)) return rc;
  kernel<<<grid, 256, smem, stream>>>(static_cast<const St*>(z), static_cast<const St*>(b),
                                      ranks, static_cast<const typename SC::storage*>(scales),
                                      map, offsets, static_cast<St*>(y), ys0, ys1, N, num_slots,
                                      S, rmax);
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
  if (blocks < 1 || blocks > 65535) return fail(LF_E_INVALID, "row_expand: blocks must be in 1..65535");
  if (row_tile != 2 && row_tile != 4 && row_tile != 8 && row_tile != 16)
    return fail(LF_E_INVALID, "row_tile must be 2, 4, 8, or 16");
  if (y_stride < out_width || !aligned16(b))
    return fail(LF_E_INVALID, "row_expand: expected aligned B and nonoverlapping output rows");
  if (max_segments < 0) return fail(LF_E_INVALID, "row_expand: negative segment capacity");
  if (num_tokens == 0 || max_segments == 0) return LF_OK;
  const int column_blocks = (out_width + threads - 1) / threads;
  if (int64_t(max_segments) * (kSegRows / row_tile) * column_blocks >= (int64_t(1) << 31))
    return fail(LF_E_INVALID, "row_expand: segment work count must fit signed int32 indexing");
  row_expand_kernel<<<blocks, threads, 0, static_cast<cudaStream_t>(stream)>>>(
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
  switch (dtype) {
    case LF_F32:
      vllm_expand_kernel<f32_t><<<grid, 256, smem, s>>>(v, sl, num_slices, rank,
                                                        static_cast<float*>(y), y_stride, routes,
                                                        int(num_tokens), num_slots, offset, add);
      break;
    case LF_F16:
      vllm_expand_kernel<f16_t><<<grid, 256, smem, s>>>(v, sl, num_slices, rank,
                                                        static_cast<__half*>(y), y_stride, routes,
                                                        int(num_tokens), num_slots, offset, add);
      break;
    case LF_BF16:
      vllm_expand_kernel<bf16_t><<<grid, 256, smem, s>>>(
          v, sl, num_slices, rank, static_cast<__nv_bfloat16*>(y), y_stride, routes,
          int(num_tokens), num_slots, offset, add);
      break;
    default:
      return fail(LF_E_INVALID, "vllm_expand: unsupported dtype");
  }
  return check_launch("vllm_expand");
}
