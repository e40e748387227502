// LoRA shrink kernels: z = A_g · x_t for every token t routed to slot g.
//
//   token_shrink_kernel  BF16 / FP16 operands with 16-byte aligned rows (the row_shrink,
//                        fleet direct_shrink, padded BGMV and vLLM shrinks on their usual
//                        inputs): one CTA per (token, 8 A rows), one warp per row, each row
//                        summed in the reference's order, so BF16 z is bit-identical to the
//                        reference kernel's (src/loraforge/ops/csrc/lora_rows.cu:35-65).
//   slot_shrink_kernel   every other case (FP32 operands, unaligned rows): grid (slot, block
//                        of 16 A rows, K part); a CTA finds its slot's tokens with a ballot
//                        scan of the routing vector, stages tiles of up to 8 of their x rows
//                        in shared memory as FP32 and streams its A rows once per tile; K is
//                        split across a thread-block cluster of up to 8 CTAs whose partial
//                        sums are added in a fixed order through distributed shared memory.
//
// Both serve three operand layouts through a small policy struct:
//   RetainedShrink  — retained-rank BF16 (row_shrink / fleet direct_shrink);
//   PaddedShrink    — SGLang padded-A decode layout (lora_shrink), any float dtype;
//   VllmShrink      — vLLM per-slice padded layout with FP32 output (vllm_gemv.shrink).
// Results are deterministic (no atomics) and no scratch memory is used.
#include <cooperative_groups.h>

#include <type_traits>
#include <utility>

#include "launch.cuh"

namespace cg = cooperative_groups;

namespace lfb {
namespace {

constexpr int kThreads = 256;
constexpr int kWarps = kThreads / 32;
constexpr int kRowsPerWarp = 2;
constexpr int kRowsPerCta = kWarps * kRowsPerWarp;  // 16
constexpr int kTokTile = 8;
constexpr int kKChunk = 1024;     // x elements staged per token per pass
constexpr int kListWindow = 2048; // tokens scanned per routing window

// ------------------------------------------------------------------ vector loads
template <typename T, int VEC>
__device__ __forceinline__ void load_vec(const typename T::storage* p, float* out);

template <>
__device__ __forceinline__ void load_vec<bf16_t, 8>(const __nv_bfloat16* p, float* out) {
  unpack_bf16x8(*reinterpret_cast<const uint4*>(p), out);
}
template <>
__device__ __forceinline__ void load_vec<f16_t, 8>(const __half* p, float* out) {
  const uint4 v = *reinterpret_cast<const uint4*>(p);
  const __half2* h = reinterpret_cast<const __half2*>(&v);
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const float2 f = __half22float2(h[i]);
    out[2 * i] = f.x;
    out[2 * i + 1] = f.y;
  }
}
template <>
__device__ __forceinline__ void load_vec<f32_t, 4>(const float* p, float* out) {
  const float4 v = *reinterpret_cast<const float4*>(p);
  out[0] = v.x;
  out[1] = v.y;
  out[2] = v.z;
  out[3] = v.w;
}
template <>
__device__ __forceinline__ void load_vec<bf16_t, 1>(const __nv_bfloat16* p, float* out) {
  out[0] = __bfloat162float(*p);
}
template <>
__device__ __forceinline__ void load_vec<f16_t, 1>(const __half* p, float* out) {
  out[0] = __half2float(*p);
}
template <>
__device__ __forceinline__ void load_vec<f32_t, 1>(const float* p, float* out) {
  out[0] = *p;
}

// ------------------------------------------------------------------ layouts
// Retained-rank layout (src/loraforge/ops/csrc/lora_rows.cu:39-51): logical row
// j < S*min(r, max_rank) maps to slice s = j / kk, row k = j % kk and packed
// column s*r + k; z gets the reference's RNE BF16 rounding.
struct RetainedShrink {
  using Elem = bf16_t;
  struct State {
    int r, kk;
  };
  const __nv_bfloat16* a;
  uint16_t* z;
  const int32_t* slots;
  const int32_t* ranks;
  int num_slots, S, cap, max_rank;
  int64_t K;

  __device__ int slot_of(int t) const {
    const int s = slots[t];
    return (s >= 0 && s < num_slots) ? s : -1;
  }
  __device__ int prepare(int g, State& st) const {
    st.r = ranks[g];
    if (st.r <= 0) return 0;
    st.kk = min(st.r, max_rank);
    return S * st.kk;
  }
  __device__ static int column(int j, const State& st) {
    return (j / st.kk) * st.r + (j % st.kk);
  }
  __device__ const __nv_bfloat16* a_row(int g, int j, const State& st) const {
    const int col = column(j, st);
    return col < S * cap ? a + (int64_t(g) * S * cap + col) * K : nullptr;
  }
  __device__ void store(int t, int j, float v, const State& st) const {
    const int col = column(j, st);
    if (col < S * cap) z[int64_t(t) * S * cap + col] = uint16_t(float_to_bf16_bits(v));
  }
};

// SGLang padded layout (src/loraforge/ops/_gemv_kernels.py:136-176): rank is
// clamped to the capacity Rmax and slices are packed at s*rank.
template <typename T, typename I>
struct PaddedShrink {
  using Elem = T;
  struct State {
    int r;
  };
  const typename T::storage* a;
  typename T::storage* z;
  const void* ranks;
  const void* map;
  int num_slots, S, rmax;
  int64_t K;

  __device__ int slot_of(int t) const {
    const int g = load_index<I>(map, t);
    return (g >= 0 && g < num_slots) ? g : -1;
  }
  __device__ int prepare(int g, State& st) const {
    st.r = min(load_index<I>(ranks, g), rmax);
    return st.r > 0 ? S * st.r : 0;
  }
  __device__ const typename T::storage* a_row(int g, int j, const State&) const {
    return a + (int64_t(g) * S * rmax + j) * K;
  }
  __device__ void store(int t, int j, float v, const State&) const {
    z[int64_t(t) * S * rmax + j] = T::from_float(v);
  }
};

// vLLM per-slice layout (src/loraforge/ops/_vllm_gemv_kernels.py:12-53): every
// slice has the same rank R; out[s, t, k] = scale * dot, FP32.
template <typename T>
struct VllmShrink {
  using Elem = T;
  struct State {};
  lf_slice_desc slices[8];
  float* out;
  const int32_t* routes;
  int num_slots, S, R, T_tokens;
  float scale;

  __device__ int slot_of(int t) const {
    const int g = routes[t];
    return (g >= 0 && g < num_slots) ? g : -1;
  }
  __device__ int prepare(int, State&) const { return S * R; }
  __device__ const typename T::storage* a_row(int g, int j, const State&) const {
    const lf_slice_desc& d = slices[j / R];
    return reinterpret_cast<const typename T::storage*>(d.ptr) + int64_t(g) * d.slot_stride +
           int64_t(j % R) * d.row_stride;
  }
  __device__ void store(int t, int j, float v, const State&) const {
    out[(int64_t(j / R) * T_tokens + t) * R + (j % R)] = v * scale;
  }
};

// ------------------------------------------------------------------ kernel
template <typename T, int VEC, typename L>
__global__ void __launch_bounds__(kThreads)
slot_shrink_kernel(const __grid_constant__ L layout, const typename T::storage* __restrict__ x,
                   int64_t x_stride,
                   int T_tokens, int64_t K) {
  using S = typename T::storage;
  extern __shared__ float smem_f[];
  float* xs = smem_f;                                          // kTokTile * kKChunk
  float* part = xs + kTokTile * kKChunk;                       // kTokTile * kRowsPerCta
  int* list = reinterpret_cast<int*>(part + kTokTile * kRowsPerCta);  // kListWindow
  __shared__ int warp_count[kWarps];
  __shared__ int list_len;

  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int g = blockIdx.x;
  typename L::State st;
  const int nrows = layout.prepare(g, st);
  const int row0 = blockIdx.y * kRowsPerCta;
  if (row0 >= nrows) return;  // uniform across the cluster (same slot and row block)

  const int parts = gridDim.z;
  const int part_id = blockIdx.z;
  const int64_t kvec = (K + VEC - 1) / VEC;
  const int64_t per_part = (kvec + parts - 1) / parts * VEC;
  const int64_t kb = min(K, int64_t(part_id) * per_part);
  const int64_t ke = min(K, kb + per_part);

  // Each warp owns two consecutive logical rows of the block.
  const int j0 = row0 + warp * kRowsPerWarp;
  const S* arow[kRowsPerWarp];
#pragma unroll
  for (int rr = 0; rr < kRowsPerWarp; ++rr)
    arow[rr] = (j0 + rr < nrows) ? layout.a_row(g, j0 + rr, st) : nullptr;

  const unsigned lower = (1u << lane) - 1u;
  for (int w0 = 0; w0 < T_tokens; w0 += kListWindow) {
    const int wend = min(T_tokens, w0 + kListWindow);
    // Ballot scan of the routing window: the list keeps token order.
    if (tid == 0) list_len = 0;
    __syncthreads();
    for (int base = w0; base < wend; base += kThreads) {
      const int t = base + tid;
      const bool mine = t < wend && layout.slot_of(t) == g;
      const unsigned ballot = __ballot_sync(0xffffffffu, mine);
      if (lane == 0) warp_count[warp] = __popc(ballot);
      __syncthreads();
      int offset = list_len;
      for (int w = 0; w < warp; ++w) offset += warp_count[w];
      if (mine) list[offset + __popc(ballot & lower)] = t;
      __syncthreads();
      if (tid == 0) {
        int total = 0;
        for (int w = 0; w < kWarps; ++w) total += warp_count[w];
        list_len += total;
      }
      __syncthreads();
    }
    const int n = list_len;
    for (int tb = 0; tb < n; tb += kTokTile) {
      const int nt = min(kTokTile, n - tb);
      float acc[kTokTile][kRowsPerWarp];
#pragma unroll
      for (int i = 0; i < kTokTile; ++i)
#pragma unroll
        for (int rr = 0; rr < kRowsPerWarp; ++rr) acc[i][rr] = 0.f;

      for (int64_t k0 = kb; k0 < ke; k0 += kKChunk) {
        const int kc = ke - k0 < kKChunk ? int(ke - k0) : kKChunk;
        const int cvec = (kc + VEC - 1) / VEC;
        __syncthreads();  // previous chunk fully consumed
        for (int idx = tid; idx < nt * cvec; idx += kThreads) {
          const int i = idx / cvec, c = (idx - i * cvec) * VEC;
          const S* src = x + int64_t(list[tb + i]) * x_stride + k0 + c;
          float v[VEC];
          load_vec<T, VEC>(src, v);  // kc is a multiple of VEC on the vector path
#pragma unroll
          for (int e = 0; e < VEC; ++e) xs[i * kKChunk + c + e] = v[e];
        }
        __syncthreads();
        if (arow[0] != nullptr) {
          for (int c = lane * VEC; c < kc; c += 32 * VEC) {
            float a0[VEC], a1[VEC];
            load_vec<T, VEC>(arow[0] + k0 + c, a0);
            if (arow[1] != nullptr) {
              load_vec<T, VEC>(arow[1] + k0 + c, a1);
            } else {
#pragma unroll
              for (int e = 0; e < VEC; ++e) a1[e] = 0.f;
            }
#pragma unroll
            for (int i = 0; i < kTokTile; ++i) {
              if (i < nt) {
                const float* xv = xs + i * kKChunk + c;
#pragma unroll
                for (int e = 0; e < VEC; ++e) {
                  acc[i][0] = fmaf(a0[e], xv[e], acc[i][0]);
                  acc[i][1] = fmaf(a1[e], xv[e], acc[i][1]);
                }
              }
            }
          }
        }
      }
      // Reduce over the warp's lanes; lane 0 owns the CTA's partial sums.
#pragma unroll
      for (int i = 0; i < kTokTile; ++i)
#pragma unroll
        for (int rr = 0; rr < kRowsPerWarp; ++rr) acc[i][rr] = warp_sum(acc[i][rr]);
      if (parts == 1) {
        if (lane == 0) {
#pragma unroll
          for (int i = 0; i < kTokTile; ++i)
#pragma unroll
            for (int rr = 0; rr < kRowsPerWarp; ++rr)
              if (i < nt && arow[rr] != nullptr) layout.store(list[tb + i], j0 + rr, acc[i][rr], st);
        }
      } else {
        if (lane == 0) {
#pragma unroll
          for (int i = 0; i < kTokTile; ++i)
#pragma unroll
            for (int rr = 0; rr < kRowsPerWarp; ++rr)
              part[i * kRowsPerCta + warp * kRowsPerWarp + rr] = acc[i][rr];
        }
        cg::cluster_group cluster = cg::this_cluster();
        cluster.sync();
        if (cluster.block_rank() == 0 && tid < nt * kRowsPerCta) {
          const int i = tid / kRowsPerCta, rl = tid - i * kRowsPerCta;
          const int j = row0 + rl;
          if (j < nrows) {
            float sum = 0.f;
            for (int p = 0; p < parts; ++p) sum += cluster.map_shared_rank(part, p)[tid];
            layout.store(list[tb + i], j, sum, st);
          }
        }
        cluster.sync();
      }
    }
  }
}

constexpr size_t kShrinkSmem =
    sizeof(float) * (kTokTile * kKChunk + kTokTile * kRowsPerCta) + sizeof(int) * kListWindow;

// Cluster size along K: about one CTA per 1024 input columns, at most 8.
inline int k_parts(int64_t K) {
  const int64_t p = K / 1024;
  return int(p < 1 ? 1 : (p > 8 ? 8 : p));
}

// ------------------------------------------------------------------ token-major kernel
// 16-bit operands with 16-byte aligned rows.  One CTA of eight warps per (token, group of
// eight A rows), one warp per row, like the reference (src/loraforge/ops/csrc/lora_rows.cu:
// 35-65, grid at :178-180), and every row summed in the reference's order: lane l takes
// the 8-element chunks starting at 8l, 8l + 256, ... and accumulates their products with
// fused multiply-adds in element order, then the lanes' sums are added by the same
// shuffle-down tree (offsets 16, 8, 4, 2, 1).  The FP32 dot products, and the BF16 z after
// rounding, are therefore bit-identical to the reference kernel's on the same inputs.
//
// Each chunk's A load (the long-latency stream: HBM, or L2 for a popular slot's later
// tokens) is issued before its x load (L1 after the first warp of the CTA); that order
// measured 25-35 % faster than x first at the same arithmetic, and the unrolled loop keeps
// several chunks in flight.  A slot-major kernel on the tensor cores (one CTA per slot and
// K part, every token of the slot in one pass, K parts summed through distributed shared
// memory) read each A row once but measured slower on config 1 (qkv 36.8, gate_up 26.5,
// down 32.9 us against 20.4, 18.4, 26.5): its chain of scan, copy and reduction latencies
// left the SMs idle.
constexpr int kTokWarps = 8;
constexpr int kTokThreads = kTokWarps * 32;

template <typename T, typename L>
__global__ void __launch_bounds__(kTokThreads)
token_shrink_kernel(const __grid_constant__ L layout, const typename T::storage* __restrict__ x,
                    int64_t x_stride, int K) {
  using S = typename T::storage;
  const int t = blockIdx.x;
  const int g = layout.slot_of(t);
  if (g < 0) return;
  typename L::State st;
  const int nrows = layout.prepare(g, st);
  const int lane = threadIdx.x & 31;
  const int j = blockIdx.y * kTokWarps + (threadIdx.x >> 5);
  if (j >= nrows) return;  // no barrier in this kernel: warps leave independently
  const S* arow = layout.a_row(g, j, st);
  if (arow == nullptr) return;
  const S* xr = x + int64_t(t) * x_stride;
  float acc = 0.f;
#pragma unroll 8
  for (int k = lane * 8; k < K; k += 256) {
    const uint4 av = *reinterpret_cast<const uint4*>(arow + k);  // A first: the long-latency stream
    const uint4 xv = *reinterpret_cast<const uint4*>(xr + k);
    float a8[8], x8[8];
    unpack8<T>(av, a8);
    unpack8<T>(xv, x8);
#pragma unroll
    for (int e = 0; e < 8; ++e) acc = fmaf(a8[e], x8[e], acc);
  }
#pragma unroll
  for (int d = 16; d > 0; d >>= 1) acc += __shfl_down_sync(0xffffffffu, acc, d);
  if (lane == 0) layout.store(t, j, acc, st);
}

template <typename T, typename L>
int launch_token_shrink(const L& layout, const typename T::storage* x, int64_t x_stride,
                        int64_t T_tokens, int64_t K, int max_rows, cudaStream_t stream,
                        const char* what) {
  const int groups = (max_rows + kTokWarps - 1) / kTokWarps;
  if (groups < 1 || groups > 65535) return fail(LF_E_INVALID, "shrink: too many rank rows");
  if (K >= (int64_t(1) << 31) - 256) return fail(LF_E_INVALID, "shrink: width too large");
  token_shrink_kernel<T, L><<<dim3(unsigned(T_tokens), unsigned(groups)), kTokThreads, 0, stream>>>(
      layout, x, x_stride, int(K));
  const cudaError_t err = cudaGetLastError();
  if (err != cudaSuccess) {
    last_error() = std::string(what) + ": " + cudaGetErrorString(err);
    return LF_E_CUDA;
  }
  return LF_OK;
}

template <typename T, int VEC, typename L>
int launch_shrink(const L& layout, const typename T::storage* x, int64_t x_stride,
                  int64_t T_tokens, int64_t K, int num_slots, int max_rows,
                  cudaStream_t stream, const char* what) {
  static int flags[64] = {};
  auto kernel = slot_shrink_kernel<T, VEC, L>;
  if (int rc = ensure_smem(kernel, int(kShrinkSmem), flags)) return rc;
  const int row_blocks = (max_rows + kRowsPerCta - 1) / kRowsPerCta;
  if (row_blocks < 1 || row_blocks > 65535) return fail(LF_E_INVALID, "shrink: too many rank rows");
  const int parts = k_parts(K);
  const dim3 grid(num_slots, row_blocks, parts);
  cudaError_t err;
  if (parts == 1) {
    kernel<<<grid, kThreads, kShrinkSmem, stream>>>(layout, x, x_stride, int(T_tokens), K);
    err = cudaGetLastError();
  } else {
    err = launch_cluster_z(kernel, grid, dim3(kThreads), kShrinkSmem, stream, parts, layout, x,
                           x_stride, int(T_tokens), K);
  }
  if (err != cudaSuccess) {
    last_error() = std::string(what) + ": " + cudaGetErrorString(err);
    return LF_E_CUDA;
  }
  return LF_OK;
}

template <typename T, typename L>
int dispatch_vec(const L& layout, const void* x, int64_t x_stride, int64_t T_tokens, int64_t K,
                 int num_slots, int max_rows, bool vec_ok, cudaStream_t stream,
                 const char* what) {
  using S = typename T::storage;
  constexpr int V = 16 / sizeof(S);
  const S* xp = static_cast<const S*>(x);
  if constexpr (!std::is_same<T, f32_t>::value) {
    if (vec_ok)
      return launch_token_shrink<T>(layout, xp, x_stride, T_tokens, K, max_rows, stream, what);
  }
  if (vec_ok)
    return launch_shrink<T, V>(layout, xp, x_stride, T_tokens, K, num_slots, max_rows, stream,
                               what);
  return launch_shrink<T, 1>(layout, xp, x_stride, T_tokens, K, num_slots, max_rows, stream,
                             what);
}

}  // namespace
}  // namespace lfb

using namespace lfb;

extern "C" int lf_row_shrink(const void* x, int64_t x_stride, const void* a, void* z,
                             const int32_t* slots, const int32_t* ranks, int64_t num_tokens,
                             int64_t width, int32_t num_slots, int32_t num_slices,
                             int32_t capacity, int32_t max_rank, void* stream) {
  if (num_tokens < 0 || num_tokens >= (int64_t(1) << 31) || width < 1)
    return fail(LF_E_INVALID, "row_shrink: invalid token count or width");
  if (num_slices < 1 || num_slices > 4 || max_rank < 1 || max_rank > 64 || capacity < max_rank)
    return fail(LF_E_INVALID, "row_shrink: num_slices must be 1..4 and max_rank 1..64 <= capacity");
  if (num_slots < 1) return fail(LF_E_INVALID, "row_shrink: no slots");
  if (width % 8 || x_stride % 8 || x_stride < width || !aligned16(x) || !aligned16(a))
    return fail(LF_E_INVALID, "row_shrink: expected aligned A/x with width and stride multiples of 8");
  if (num_tokens == 0) return LF_OK;
  RetainedShrink L{static_cast<const __nv_bfloat16*>(a), static_cast<uint16_t*>(z), slots, ranks,
                   num_slots, num_slices, capacity, max_rank, width};
  return dispatch_vec<bf16_t>(L, x, x_stride, num_tokens, width, num_slots,
                              num_slices * max_rank, true, static_cast<cudaStream_t>(stream),
                              "row_shrink");
}

template <typename T>
static int bgmv_shrink_t(const void* x, int64_t x_stride, const void* a, void* z,
                         const void* ranks, const void* map, int index_bits, int64_t T_tokens,
                         int64_t width, int num_slots, int S, int rmax, cudaStream_t stream) {
  using St = typename T::storage;
  constexpr int V = 16 / sizeof(St);
  const bool vec_ok = width % V == 0 && x_stride % V == 0 && aligned16(x) && aligned16(a);
  if (index_bits == 32) {
    PaddedShrink<T, int32_t> L{static_cast<const St*>(a), static_cast<St*>(z), ranks, map,
                               num_slots, S, rmax, width};
    return dispatch_vec<T>(L, x, x_stride, T_tokens, width, num_slots, S * rmax, vec_ok, stream,
                           "bgmv_shrink");
  }
  PaddedShrink<T, int64_t> L{static_cast<const St*>(a), static_cast<St*>(z), ranks, map,
                             num_slots, S, rmax, width};
  return dispatch_vec<T>(L, x, x_stride, T_tokens, width, num_slots, S * rmax, vec_ok, stream,
                         "bgmv_shrink");
}

extern "C" int lf_bgmv_shrink(int32_t dtype, const void* x, int64_t x_stride, const void* a,
                              void* z, const void* ranks, const void* token_map,
                              int32_t index_bits, int64_t num_tokens, int64_t width,
                              int32_t num_slots, int32_t num_slices, int32_t rmax,
                              void* stream) {
  if (num_tokens < 0 || num_tokens >= (int64_t(1) << 31) || width < 1 || num_slots < 1)
    return fail(LF_E_INVALID, "bgmv_shrink: invalid sizes");
  if (num_slices < 1 || rmax < 1 || rmax > 256 || int64_t(num_slices) * rmax > 65535 * 16)
    return fail(LF_E_INVALID, "bgmv_shrink: rank capacity must be 1..256");
  if (index_bits != 32 && index_bits != 64)
    return fail(LF_E_INVALID, "bgmv_shrink: index_bits must be 32 or 64");
  if (num_tokens == 0) return LF_OK;
  const cudaStream_t s = static_cast<cudaStream_t>(stream);
  switch (dtype) {
    case LF_F32:
      return bgmv_shrink_t<f32_t>(x, x_stride, a, z, ranks, token_map, index_bits, num_tokens,
                                  width, num_slots, num_slices, rmax, s);
    case LF_F16:
      return bgmv_shrink_t<f16_t>(x, x_stride, a, z, ranks, token_map, index_bits, num_tokens,
                                  width, num_slots, num_slices, rmax, s);
    case LF_BF16:
      return bgmv_shrink_t<bf16_t>(x, x_stride, a, z, ranks, token_map, index_bits, num_tokens,
                                   width, num_slots, num_slices, rmax, s);
  }
  return fail(LF_E_INVALID, "bgmv_shrink: unsupported dtype");
}

template <typename T>
static int vllm_shrink_t(const void* x, int64_t x_stride, const lf_slice_desc* slices,
                         int S, float* out, const int32_t* routes, int64_t T_tokens,
                         int64_t width, int rank, int num_slots, float scale,
                         cudaStream_t stream) {
  using St = typename T::storage;
  constexpr int V = 16 / sizeof(St);
  VllmShrink<T> L{};
  bool vec_ok = width % V == 0 && x_stride % V == 0 && aligned16(x);
  for (int s = 0; s < S; ++s) {
    L.slices[s] = slices[s];
    vec_ok = vec_ok && aligned16(slices[s].ptr) && slices[s].slot_stride % V == 0 &&
             slices[s].row_stride % V == 0;
  }
  L.out = out;
  L.routes = routes;
  L.num_slots = num_slots;
  L.S = S;
  L.R = rank;
  L.T_tokens = int(T_tokens);
  L.scale = scale;
  return dispatch_vec<T>(L, x, x_stride, T_tokens, width, num_slots, S * rank, vec_ok, stream,
                         "vllm_shrink");
}

extern "C" int lf_vllm_shrink(int32_t dtype, const void* x, int64_t x_stride,
                              const lf_slice_desc* slices, int32_t num_slices,
                              int32_t num_slots, float* out, const int32_t* routes,
                              int64_t num_tokens, int64_t width, int32_t rank, float scale,
                              void* stream) {
  if (num_tokens < 0 || num_tokens >= (int64_t(1) << 31) || width < 1 || num_slots < 1)
    return fail(LF_E_INVALID, "vllm_shrink: invalid sizes");
  if (num_slices < 1 || num_slices > 8 || !slices)
    return fail(LF_E_INVALID, "vllm_shrink: 1..8 slices required");
  if (rank < 1 || rank > 256) return fail(LF_E_INVALID, "vllm_shrink: rank must be in 1..256");
  if (num_tokens == 0) return LF_OK;
  const cudaStream_t s = static_cast<cudaStream_t>(stream);
  switch (dtype) {
    case LF_F32:
      return vllm_shrink_t<f32_t>(x, x_stride, slices, num_slices, out, routes, num_tokens,
                                  width, rank, num_slots, scale, s);
    case LF_F16:
      return vllm_shrink_t<f16_t>(x, x_stride, slices, num_slices, out, routes, num_tokens,
                                  width, rank, num_slots, scale, s);
    case LF_BF16:
      return vllm_shrink_t<bf16_t>(x, x_stride, slices, num_slices, out, routes, num_tokens,
                                   width, rank, num_slots, scale, s);
  }
  return fail(LF_E_INVALID, "vllm_shrink: unsupported dtype");
}
