// Grouped (SGMV) LoRA shrink -> expand for decode segments of <= 16 tokens (one slot each).
//
// Two streaming kernels per call, chained with programmatic dependent launch:
//
//   sgmv_shrink_kernel   z[t, j] = sum_k x[t, k] * A_g[j, k]  (j < S*r), FP32, for every
//                        token t of a segment.  Grid = (K part, segment); the K parts of a
//                        segment form one thread-block cluster and their partial [16 x S*r]
//                        tiles are summed in a fixed rank order through distributed shared
//                        memory by rank 0, which writes z to the FP32 workspace.  Every A
//                        row is read from HBM once per segment; no atomics.
//   sgmv_expand_kernel   y[t, n] += scale_g * sum_k z[t, slice(n)*r + k] * B_g[n, k] for a
//                        (column chunk, segment) tile; z is read back from the workspace.
//
// Both run on the tensor cores (mma.sync m16n8k16 / m16n8k8, BF16 operands, FP32
// accumulate) with the segment's tokens as the M dimension.  Fragments are loaded
// straight from global memory with 16-byte vector loads: inside each 32-element K
// block the MMA fragment slots carry a permutation of k that is the same for both
// operands, so a lane's 16 contiguous bytes feed two MMAs with no shared-memory
// staging.  Output columns are permuted the same way so that each lane owns four
// consecutive outputs (8-byte read-modify-write of y).
//
// Numerics: kFp32 keeps z in FP32 (split into BF16 hi + lo for the expand MMAs, about
// 16 significant bits) and rounds the output once: y = bf16(y + scale*acc).
// kReference reproduces the retained-rank operators' contract: z rounded to BF16,
// delta = bf16(acc*scale), y = bf16(y + delta)
// (src/loraforge/ops/csrc/lora_rows.cu:64 and :113).
#include <cooperative_groups.h>

#include "launch.cuh"
#include "tma.cuh"

namespace cg = cooperative_groups;

namespace lfb {
namespace {

constexpr int kMaxCluster = 16;  // non-portable cluster size on sm_100
constexpr int kThreads = 256;
constexpr int kWarps = kThreads / 32;
constexpr int kSeg = 16;          // tokens per segment (one m16 tile)
constexpr int kMaxRows = 4 * 64;  // S*r <= 4 slices x rank 64
constexpr int kMaxKp = 64;
constexpr int kMaxSlices = 4;
constexpr int kMaxTilesPerWarp = kMaxRows / 8 / kWarps;  // 4
// 16-column units a warp keeps in flight: fewer for wide buckets (register budget).
template <int KP>
struct UnitBatch {
  static constexpr int value = KP >= 64 ? 1 : (KP >= 32 ? 2 : 4);
};

enum Numerics { kFp32 = 0, kReference = 1 };

struct FusedParams {
  const uint16_t* x;
  int64_t x_stride;
  const uint16_t* a;
  const uint16_t* b;
  const int64_t* b_offsets;
  const int32_t* b_strides;
  uint16_t* y;
  int64_t y_stride;
  const int32_t* indptr;
  const int32_t* seg_slots;
  const int32_t* perm;
  const int32_t* ranks;
  const float* scales;
  const int32_t* slice_offsets;
  const int32_t* seg_count;
  float* z;          // FP32 workspace, row t at z + t * z_stride
  int64_t z_stride;  // >= S * cap
  int T, K, N, S, cap, num_slots, max_segments;
  int units_per_chunk;  // expand: 16-column units per CTA
};

// ------------------------------------------------------------------ tensor-core helpers
__device__ __forceinline__ void mma16816(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2,
                                         uint32_t a3, uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, "
      "{%8,%9}, {%0,%1,%2,%3};\n"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

__device__ __forceinline__ void mma1688(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t b0) {
  asm volatile(
      "mma.sync.aligned.m16n8k8.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5}, {%6}, "
      "{%0,%1,%2,%3};\n"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a0), "r"(a1), "r"(b0));
}

__device__ __forceinline__ uint4 ldg16(const uint16_t* p) {
  return __ldg(reinterpret_cast<const uint4*>(p));
}

__device__ __forceinline__ uint32_t pack2(uint32_t lo_bits, uint32_t hi_bits) {
  return (lo_bits & 0xffffu) | (hi_bits << 16);
}

// z (FP32) -> BF16 "hi" pair and the BF16 residual "lo" pair.
__device__ __forceinline__ void split2(float v0, float v1, uint32_t& hi, uint32_t& lo) {
  const uint32_t h0 = float_to_bf16_bits(v0), h1 = float_to_bf16_bits(v1);
  hi = pack2(h0, h1);
  lo = pack2(float_to_bf16_bits(v0 - bf16_bits_to_float(h0)),
             float_to_bf16_bits(v1 - bf16_bits_to_float(h1)));
}

struct SegmentInfo {
  int g, n, r, bucket, kp;
  float scale;
  int64_t boff;
};

// ------------------------------------------------------------------ phase 2 (expand)
// One warp, a batch of 16-column units starting at unit u0 (stride ustride).
// zs: padded FP32 z tile [kSeg][kMaxSlices][kMaxKp] in shared memory.
template <int KP, int MODE>
__device__ __forceinline__ void expand_units(const FusedParams& p, const SegmentInfo& si,
                                             const int* tok, const float* zs, const int* offs,
                                             int u_begin, int u_end, int lane, int warp) {
  constexpr int KSTEPS = KP >= 16 ? KP / 16 : 1;  // k16 MMAs (or one k8 MMA when KP == 8)
  constexpr int kUnitBatch = UnitBatch<KP>::value;
  const int g = lane >> 2, t = lane & 3;
  const int tok_lo = g < si.n ? tok[g] : -1;
  const int tok_hi = g + 8 < si.n ? tok[g + 8] : -1;
  const uint16_t* bbase = p.b + si.boff;
  int cached_slice = -1;
  // z fragments of the current slice: [kstep][hi/lo][4 regs]
  uint32_t zf[KSTEPS][2][4];

  auto load_z = [&](int s) {
    const float* z0 = zs + (g * kMaxSlices + s) * kMaxKp;
    const float* z1 = zs + ((g + 8) * kMaxSlices + s) * kMaxKp;
#pragma unroll
    for (int ks = 0; ks < KSTEPS; ++ks) {
      if constexpr (KP == 8) {
        // m16n8k8: slots (2t, 2t+1) hold k = 2t, 2t+1.
        const float v0 = z0[2 * t], v1 = z0[2 * t + 1], w0 = z1[2 * t], w1 = z1[2 * t + 1];
        if (MODE == kFp32) {
          split2(v0, v1, zf[ks][0][0], zf[ks][1][0]);
          split2(w0, w1, zf[ks][0][1], zf[ks][1][1]);
        } else {
          zf[ks][0][0] = pack2(float_to_bf16_bits(v0), float_to_bf16_bits(v1));
          zf[ks][0][1] = pack2(float_to_bf16_bits(w0), float_to_bf16_bits(w1));
        }
      } else {
        // KP == 16: one k16 MMA over k = 4t..4t+3 per lane.
        // KP >= 32: k32 blocks; block kb = ks/2 covers 32 k, lane t owns 8t..8t+7 of it,
        // MMA (ks even) uses 8t..8t+3, (ks odd) uses 8t+4..8t+7.
        int k0;
        if constexpr (KP == 16) {
          k0 = 4 * t;
        } else {
          k0 = (ks >> 1) * 32 + 8 * t + (ks & 1) * 4;
        }
        const float4 va = *reinterpret_cast<const float4*>(z0 + k0);
        const float4 vb = *reinterpret_cast<const float4*>(z1 + k0);
        if (MODE == kFp32) {
          split2(va.x, va.y, zf[ks][0][0], zf[ks][1][0]);
          split2(vb.x, vb.y, zf[ks][0][1], zf[ks][1][1]);
          split2(va.z, va.w, zf[ks][0][2], zf[ks][1][2]);
          split2(vb.z, vb.w, zf[ks][0][3], zf[ks][1][3]);
        } else {
          zf[ks][0][0] = pack2(float_to_bf16_bits(va.x), float_to_bf16_bits(va.y));
          zf[ks][0][1] = pack2(float_to_bf16_bits(vb.x), float_to_bf16_bits(vb.y));
          zf[ks][0][2] = pack2(float_to_bf16_bits(va.z), float_to_bf16_bits(va.w));
          zf[ks][0][3] = pack2(float_to_bf16_bits(vb.z), float_to_bf16_bits(vb.w));
        }
      }
    }
  };

  // B fragment of one 8-column tile: output column `col`, this lane's k slots.
  auto load_b = [&](int col, uint32_t (&bf)[KSTEPS][2]) {
    const bool ok = col < p.N;
    const uint16_t* row = bbase + int64_t(ok ? col : 0) * si.bucket;
    if constexpr (KP == 8) {
      // k = 2t, 2t+1; buckets below 8 are zero-padded here.
      uint32_t v = 0;
      if (ok) {
        if (si.bucket >= 8 || 2 * t + 1 < si.bucket) {
          v = *reinterpret_cast<const uint32_t*>(row + 2 * t);
        } else if (2 * t < si.bucket) {
          v = row[2 * t];
        }
      }
      bf[0][0] = v;
      bf[0][1] = 0;
    } else if constexpr (KP == 16) {
      uint2 v = make_uint2(0, 0);
      if (ok) v = *reinterpret_cast<const uint2*>(row + 4 * t);
      bf[0][0] = v.x;
      bf[0][1] = v.y;
    } else {
#pragma unroll
      for (int kb = 0; kb < KP / 32; ++kb) {
        uint4 v = make_uint4(0, 0, 0, 0);
        if (ok) v = ldg16(row + kb * 32 + 8 * t);
        bf[2 * kb][0] = v.x;
        bf[2 * kb][1] = v.y;
        bf[2 * kb + 1][0] = v.z;
        bf[2 * kb + 1][1] = v.w;
      }
    }
  };

  auto slice_of = [&](int col) {
    int s = 0;
    for (int i = 1; i < p.S; ++i)
      if (col >= offs[i]) s = i;
    return s;
  };

  for (int u0 = u_begin + warp; u0 < u_end; u0 += kWarps * kUnitBatch) {
    uint32_t bfr[kUnitBatch][2][KSTEPS][2];
    uint2 yv[kUnitBatch][2];
    int n0s[kUnitBatch];
#pragma unroll
    for (int ub = 0; ub < kUnitBatch; ++ub) {
      const int u = u0 + ub * kWarps;
      const int n0 = u * 16;
      n0s[ub] = n0;
      const int c0 = n0 + 4 * (g >> 1) + (g & 1);
      if (u < u_end) {
        load_b(c0, bfr[ub][0]);
        load_b(c0 + 2, bfr[ub][1]);
      }
      // Output values this lane owns: columns n0+4t..n0+4t+3 of tokens g and g+8.
      const int col = n0 + 4 * t;
      const bool full = u < u_end && col + 3 < p.N;
      yv[ub][0] = make_uint2(0, 0);
      yv[ub][1] = make_uint2(0, 0);
      if (full && tok_lo >= 0)
        yv[ub][0] = *reinterpret_cast<const uint2*>(p.y + int64_t(tok_lo) * p.y_stride + col);
      if (full && tok_hi >= 0)
        yv[ub][1] = *reinterpret_cast<const uint2*>(p.y + int64_t(tok_hi) * p.y_stride + col);
    }
#pragma unroll
    for (int ub = 0; ub < kUnitBatch; ++ub) {
      const int u = u0 + ub * kWarps;
      if (u >= u_end) break;
      const int n0 = n0s[ub];
      const int s_first = slice_of(n0);
      const int s_last = slice_of(min(n0 + 15, p.N - 1));
      float out[2][4];  // [token row g / g+8][4 consecutive columns]
      for (int s = s_first; s <= s_last; ++s) {
        if (s != cached_slice) {
          load_z(s);
          cached_slice = s;
        }
        float acc[2][4];
#pragma unroll
        for (int tile = 0; tile < 2; ++tile) {
#pragma unroll
          for (int i = 0; i < 4; ++i) acc[tile][i] = 0.f;
#pragma unroll
          for (int ks = 0; ks < KSTEPS; ++ks) {
#pragma unroll
            for (int part = 0; part < (MODE == kFp32 ? 2 : 1); ++part) {
              if constexpr (KP == 8) {
                mma1688(acc[tile], zf[ks][part][0], zf[ks][part][1], bfr[ub][tile][ks][0]);
              } else {
                mma16816(acc[tile], zf[ks][part][0], zf[ks][part][1], zf[ks][part][2],
                         zf[ks][part][3], bfr[ub][tile][ks][0], bfr[ub][tile][ks][1]);
              }
            }
          }
        }
        // tile 0 holds columns n0+4t, +1; tile 1 holds n0+4t+2, +3.
        const float v[2][4] = {{acc[0][0], acc[0][1], acc[1][0], acc[1][1]},
                               {acc[0][2], acc[0][3], acc[1][2], acc[1][3]}};
#pragma unroll
        for (int c = 0; c < 4; ++c) {
          const int col = n0 + 4 * t + c;
          const bool mine = s_first == s_last || (col < p.N && slice_of(col) == s);
          if (mine) {
            out[0][c] = v[0][c];
            out[1][c] = v[1][c];
          }
        }
      }
      const int col = n0 + 4 * t;
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        const int token = h ? tok_hi : tok_lo;
        if (token < 0) continue;
        uint16_t* yp = p.y + int64_t(token) * p.y_stride + col;
        if (col + 3 < p.N) {
          const uint2 old = yv[ub][h];
          const uint32_t w[2] = {old.x, old.y};
          uint32_t res[2];
#pragma unroll
          for (int q = 0; q < 2; ++q) {
            uint32_t bits2[2];
#pragma unroll
            for (int e = 0; e < 2; ++e) {
              const float base = bf16_bits_to_float((w[q] >> (16 * e)) & 0xffffu);
              const float acc = out[h][2 * q + e];
              float sum;
              if (MODE == kFp32) {
                sum = base + si.scale * acc;
              } else {
                sum = base + bf16_bits_to_float(float_to_bf16_bits(acc * si.scale));
              }
              bits2[e] = float_to_bf16_bits(sum);
            }
            res[q] = pack2(bits2[0], bits2[1]);
          }
          *reinterpret_cast<uint2*>(yp) = make_uint2(res[0], res[1]);
        } else {
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            if (col + e >= p.N) continue;
            const float base = bf16_bits_to_float(yp[e]);
            const float acc = out[h][e];
            const float sum = MODE == kFp32
                                  ? base + si.scale * acc
                                  : base + bf16_bits_to_float(float_to_bf16_bits(acc * si.scale));
            yp[e] = uint16_t(float_to_bf16_bits(sum));
          }
        }
      }
    }
  }
}

// ------------------------------------------------------------------ segments
// Reads and validates segment `seg`; identical in every CTA that asks.
__device__ __forceinline__ bool load_segment(const FusedParams& p, int seg, SegmentInfo& si,
                                             int& start) {
  const int nseg = min(*p.seg_count, p.max_segments);
  if (seg >= nseg) return false;
  start = p.indptr[seg];
  si.n = p.indptr[seg + 1] - start;
  si.g = p.seg_slots[seg];
  if (si.n <= 0 || si.n > kSeg || si.g < 0 || si.g >= p.num_slots) return false;
  si.r = p.ranks[si.g];
  si.bucket = p.b_strides[si.g];
  if (si.r <= 0 || si.r > 64 || si.r > p.cap) return false;
  if (si.bucket < 1 || si.bucket > 64 || (si.bucket & (si.bucket - 1))) return false;
  si.kp = si.bucket < 8 ? 8 : si.bucket;
  si.scale = p.scales[si.g];
  si.boff = p.b_offsets[si.g];
  // B regions start at 8-element (16-byte) boundaries: the vector and bulk loads
  // below rely on it, so a misaligned region is skipped instead of being read.
  return si.boff >= 0 && (si.boff & 7) == 0;
}

// Token rows of the segment into shared memory; false if any index is out of range.
__device__ __forceinline__ bool load_tokens(const FusedParams& p, const SegmentInfo& si,
                                            int start, int* tok) {
  if (threadIdx.x < kSeg) tok[threadIdx.x] = threadIdx.x < si.n ? p.perm[start + threadIdx.x] : -1;
  __syncthreads();
  bool bad = false;
  for (int i = 0; i < si.n; ++i) bad |= tok[i] < 0 || tok[i] >= p.T;
  return !bad;
}

__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_launch_dependents() {
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}

// ------------------------------------------------------------------ shrink kernel
// grid (cluster_k, max_segments), cluster (cluster_k, 1, 1).  Each CTA stages its
// K slice of the segment's x rows (slots 0..15) and A rows (slots 16..) in shared
// memory with one burst of 16-byte cp.async copies (row pitch = kslice*2 + 64 bytes,
// so the fragment loads below are free of bank conflicts), then runs the MMAs from
// shared memory.  After the MMAs the tile region is reused for the partial sums.
__device__ __forceinline__ void cp_async16(void* dst, const void* src) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_u32(dst)), "l"(src)
               : "memory");
}
__device__ __forceinline__ void cp_async_wait_all() {
  asm volatile("cp.async.commit_group;\n cp.async.wait_group 0;" ::: "memory");
}
__device__ __forceinline__ uint4 lds16(const uint8_t* p) { return *reinterpret_cast<const uint4*>(p); }

__global__ void __launch_bounds__(kThreads, 3)
sgmv_shrink_kernel(const __grid_constant__ FusedParams p, int kslice) {
  extern __shared__ __align__(128) uint8_t tiles[];
  __shared__ int tok[kSeg];
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int g8 = lane >> 2, t4 = lane & 3;
  const int parts = gridDim.x, rank = blockIdx.x;
  SegmentInfo si;
  int start = 0;
  // Every CTA of a cluster shares the segment, so these exits are cluster-uniform.
  if (!load_segment(p, blockIdx.y, si, start) || !load_tokens(p, si, start, tok)) {
    pdl_launch_dependents();
    return;
  }
  const int kb = min(p.K, rank * kslice);
  const int klen = min(p.K, kb + kslice) - kb;  // a multiple of 8
  const int pitch = kslice * 2 + 64;
  const int R = p.S * si.r;
  // ---- stage x rows (m < n) and A rows (j < R) of this K slice
  const int chunks = klen / 8;
  const int rows = si.n + R;
  for (int idx = tid; idx < rows * chunks; idx += kThreads) {
    const int row = idx / chunks, c = idx - row * chunks;
    const uint16_t* src;
    int slot;
    if (row < si.n) {
      src = p.x + int64_t(tok[row]) * p.x_stride + kb + c * 8;
      slot = row;
    } else {
      const int j = row - si.n;
      src = p.a + (int64_t(si.g) * p.S * p.cap + j) * p.K + kb + c * 8;
      slot = kSeg + j;
    }
    cp_async16(tiles + slot * pitch + c * 16, src);
  }
  cp_async_wait_all();
  __syncthreads();
  // ---- MMAs: warps own 8-row tiles of A (and split K when there are few tiles)
  const int ntiles = (R + 7) / 8;
  const int kparts = ntiles >= kWarps ? 1 : kWarps / ntiles;
  const int my_tile0 = ntiles >= kWarps ? warp : warp % ntiles;
  const int my_kpart = ntiles >= kWarps ? 0 : warp / ntiles;
  const bool active = my_kpart < kparts;
  float acc[kMaxTilesPerWarp][4];
#pragma unroll
  for (int i = 0; i < kMaxTilesPerWarp; ++i)
#pragma unroll
    for (int e = 0; e < 4; ++e) acc[i][e] = 0.f;
  if (active) {
    const int kblocks = (klen + 31) / 32;
    const int b0 = kblocks * my_kpart / kparts, b1 = kblocks * (my_kpart + 1) / kparts;
    const uint8_t* xr0 = tiles + g8 * pitch;
    const uint8_t* xr1 = tiles + (g8 + 8) * pitch;
    const uint4 zero = make_uint4(0, 0, 0, 0);
#pragma unroll 4
    for (int b = b0; b < b1; ++b) {
      const int k = b * 32 + 8 * t4;
      const bool kin = k < klen;
      const uint4 x0 = kin ? lds16(xr0 + k * 2) : zero;
      const uint4 x1 = kin ? lds16(xr1 + k * 2) : zero;
#pragma unroll
      for (int i = 0; i < kMaxTilesPerWarp; ++i) {
        const int tile = my_tile0 + i * kWarps;
        if (tile < ntiles) {
          const uint4 av = kin ? lds16(tiles + (kSeg + tile * 8 + g8) * pitch + k * 2) : zero;
          mma16816(acc[i], x0.x, x1.x, x0.y, x1.y, av.x, av.y);
          mma16816(acc[i], x0.z, x1.z, x0.w, x1.w, av.z, av.w);
        }
      }
    }
  }
  __syncthreads();  // tiles are dead from here on: reuse them for the partial sums
  float* warp_part = reinterpret_cast<float*>(tiles);         // [kparts][16][8*ntiles]
  float* cta_part = reinterpret_cast<float*>(tiles) + kSeg * 64;  // [16][kMaxRows]
  if (kparts == 1) {
    // Warps beyond ntiles*kparts hold no tile (their accumulators are zero).
#pragma unroll
    for (int i = 0; i < kMaxTilesPerWarp; ++i) {
      const int tile = my_tile0 + i * kWarps;
      const int j = tile * 8 + 2 * t4;
      if (active && tile < ntiles && j < R) {
        cta_part[g8 * kMaxRows + j] = acc[i][0];
        cta_part[(g8 + 8) * kMaxRows + j] = acc[i][2];
      }
      if (active && tile < ntiles && j + 1 < R) {
        cta_part[g8 * kMaxRows + j + 1] = acc[i][1];
        cta_part[(g8 + 8) * kMaxRows + j + 1] = acc[i][3];
      }
    }
  } else {
    // ntiles < 8 and kparts * ntiles <= 8, so kparts * (8 * ntiles) <= 64.
    const int RP = 8 * ntiles;
    if (active) {
      const int j = my_tile0 * 8 + 2 * t4;
      float* wp = warp_part + my_kpart * kSeg * RP;
      wp[g8 * RP + j] = acc[0][0];
      wp[g8 * RP + j + 1] = acc[0][1];
      wp[(g8 + 8) * RP + j] = acc[0][2];
      wp[(g8 + 8) * RP + j + 1] = acc[0][3];
    }
    __syncthreads();
    for (int i = tid; i < kSeg * R; i += kThreads) {
      const int m = i / R, j = i - m * R;
      float sum = 0.f;
      for (int q = 0; q < kparts; ++q) sum += warp_part[(q * kSeg + m) * RP + j];
      cta_part[m * kMaxRows + j] = sum;
    }
  }
  if (parts == 1) {
    __syncthreads();
    for (int i = tid; i < si.n * R; i += kThreads) {
      const int m = i / R, j = i - m * R;
      p.z[int64_t(tok[m]) * p.z_stride + j] = cta_part[m * kMaxRows + j];
    }
  } else {
    // Rank 0 adds the cluster's partials in rank order and writes z.
    cg::cluster_group cluster = cg::this_cluster();
    cluster.sync();
    if (rank == 0) {
      for (int i = tid; i < si.n * R; i += kThreads) {
        const int m = i / R, j = i - m * R;
        float sum = 0.f;
        for (int c = 0; c < parts; ++c) sum += cluster.map_shared_rank(cta_part, c)[m * kMaxRows + j];
        p.z[int64_t(tok[m]) * p.z_stride + j] = sum;
      }
    }
    cluster.sync();  // keep every CTA's partial alive until rank 0 has read it
  }
  __syncthreads();
  pdl_launch_dependents();
}

// ------------------------------------------------------------------ expand kernel
// grid (column chunks, max_segments).
template <int MODE>
__global__ void __launch_bounds__(kThreads, 2) sgmv_expand_kernel(const __grid_constant__ FusedParams p) {
  __shared__ __align__(16) float zs[kSeg * kMaxSlices * kMaxKp];
  __shared__ int tok[kSeg];
  __shared__ int offs[kMaxSlices + 1];
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  pdl_wait();  // z is written by the preceding shrink grid
  SegmentInfo si;
  int start = 0;
  if (!load_segment(p, blockIdx.y, si, start)) return;
  if (tid <= p.S) offs[tid] = p.slice_offsets[tid];
  if (!load_tokens(p, si, start, tok)) return;
  const int live = min(si.r, si.bucket);
  for (int i = tid; i < kSeg * p.S * si.kp; i += kThreads) {
    const int m = i / (p.S * si.kp);
    const int rem = i - m * p.S * si.kp;
    const int s = rem / si.kp, k = rem - s * si.kp;
    float v = 0.f;
    if (k < live && m < si.n) v = p.z[int64_t(tok[m]) * p.z_stride + s * si.r + k];
    zs[(m * kMaxSlices + s) * kMaxKp + k] = v;
  }
  __syncthreads();
  const int units = (p.N + 15) / 16;
  const int u_begin = blockIdx.x * p.units_per_chunk;
  const int u_end = min(units, u_begin + p.units_per_chunk);
  switch (si.kp) {
    case 8: expand_units<8, MODE>(p, si, tok, zs, offs, u_begin, u_end, lane, warp); break;
    case 16: expand_units<16, MODE>(p, si, tok, zs, offs, u_begin, u_end, lane, warp); break;
    case 32: expand_units<32, MODE>(p, si, tok, zs, offs, u_begin, u_end, lane, warp); break;
    default: expand_units<64, MODE>(p, si, tok, zs, offs, u_begin, u_end, lane, warp); break;
  }
}

// ------------------------------------------------------------------ bulk-copy expand
// Persistent, warp-specialised expand.  The output columns of every segment are cut
// into 256-column items; CTA i owns a contiguous block of items, so it touches one or
// two segments and reads their metadata once.  Warp kConsumers is the producer: it
// merges consecutive items of one segment into a stage of up to kStageCols columns
// (at most 32 KB of B rows) and streams the stage's B rows and y rows into a
// kStages-deep shared-memory ring with cp.async.bulk, completion tracked by the
// stage's "full" mbarrier.  Warps 0..kConsumers-1 compute a stage on the tensor cores
// from shared memory and write y back into it; consumer thread 0 bulk-stores the y
// rows and releases the previous stage (whose stores have been read by then) through
// its "empty" mbarrier, so the stores of one stage overlap the next stage's compute.
// A header with ok = -1 ends the stream.
constexpr int kStages = 3;
constexpr int kItemCols = 256;
constexpr int kStageCols = 1024;
constexpr int kConsumers = 8;
constexpr int kTmaThreads = (kConsumers + 1) * 32;
constexpr int kYPitch = kStageCols * 2 + 16;  // bytes per y row in shared memory
constexpr int kBTileBytes = 32 * 1024;        // B rows of one stage
constexpr int kYTileBytes = kSeg * kYPitch;
constexpr int kZBufBytes = kSeg * kMaxRows * 4;  // the current segment's z, FP32

struct alignas(16) ItemHeader {
  int ok, seg, n, r, bucket, col0, ncols;
  float scale;
  int tok[kSeg];
};

constexpr int kStageBytes = (kBTileBytes + kYTileBytes + int(sizeof(ItemHeader)) + 127) / 128 * 128;
constexpr int kTmaSmem = kStages * kStageBytes + kZBufBytes + 2 * kStages * 8 + 64;

struct Stage {
  uint8_t* base;
  __device__ uint16_t* btile() const { return reinterpret_cast<uint16_t*>(base); }
  __device__ uint8_t* ytile() const { return base + kBTileBytes; }
  __device__ ItemHeader* header() const {
    return reinterpret_cast<ItemHeader*>(base + kBTileBytes + kYTileBytes);
  }
};

// One item on the consumer warps: units of 16 columns, warps round-robin.
// zbuf: the segment's z, FP32 [kSeg][kMaxRows], zero beyond each slice's live rank.
template <int KP, int MODE>
__device__ __forceinline__ void consume_item(const ItemHeader& h, const Stage& st, int S, int N,
                                             const int* offs, const float* zbuf, int lane,
                                             int warp) {
  constexpr int KSTEPS = KP >= 16 ? KP / 16 : 1;
  const int g = lane >> 2, t = lane & 3;
  const uint16_t* bt = st.btile();
  uint8_t* yt = st.ytile();
  int cached_slice = -1;
  uint32_t zf[KSTEPS][2][4];

  // Slice s of the z tile holds rank positions s*KP .. s*KP+KP-1 (zero padded).
  auto zval = [&](int m, int s, int k) -> float { return zbuf[m * kMaxRows + s * KP + k]; };
  auto load_z = [&](int s) {
#pragma unroll
    for (int ks = 0; ks < KSTEPS; ++ks) {
      if constexpr (KP == 8) {
        const float v0 = zval(g, s, 2 * t), v1 = zval(g, s, 2 * t + 1);
        const float w0 = zval(g + 8, s, 2 * t), w1 = zval(g + 8, s, 2 * t + 1);
        if (MODE == kFp32) {
          split2(v0, v1, zf[ks][0][0], zf[ks][1][0]);
          split2(w0, w1, zf[ks][0][1], zf[ks][1][1]);
        } else {
          zf[ks][0][0] = pack2(float_to_bf16_bits(v0), float_to_bf16_bits(v1));
          zf[ks][0][1] = pack2(float_to_bf16_bits(w0), float_to_bf16_bits(w1));
        }
      } else {
        const int k0 = KP == 16 ? 4 * t : (ks >> 1) * 32 + 8 * t + (ks & 1) * 4;
        float va[4], vb[4];
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          va[e] = zval(g, s, k0 + e);
          vb[e] = zval(g + 8, s, k0 + e);
        }
        if (MODE == kFp32) {
          split2(va[0], va[1], zf[ks][0][0], zf[ks][1][0]);
          split2(vb[0], vb[1], zf[ks][0][1], zf[ks][1][1]);
          split2(va[2], va[3], zf[ks][0][2], zf[ks][1][2]);
          split2(vb[2], vb[3], zf[ks][0][3], zf[ks][1][3]);
        } else {
          zf[ks][0][0] = pack2(float_to_bf16_bits(va[0]), float_to_bf16_bits(va[1]));
          zf[ks][0][1] = pack2(float_to_bf16_bits(vb[0]), float_to_bf16_bits(vb[1]));
          zf[ks][0][2] = pack2(float_to_bf16_bits(va[2]), float_to_bf16_bits(va[3]));
          zf[ks][0][3] = pack2(float_to_bf16_bits(vb[2]), float_to_bf16_bits(vb[3]));
        }
      }
    }
  };
  // B fragment of one 8-column tile; `row` is the column's index inside the chunk.
  auto load_b = [&](int row, bool ok, uint32_t (&bf)[KSTEPS][2]) {
    const uint16_t* rp = bt + row * h.bucket;
    if constexpr (KP == 8) {
      uint32_t v = 0;
      if (ok) {
        if (h.bucket >= 8 || 2 * t + 1 < h.bucket) {
          v = *reinterpret_cast<const uint32_t*>(rp + 2 * t);
        } else if (2 * t < h.bucket) {
          v = rp[2 * t];
        }
      }
      bf[0][0] = v;
      bf[0][1] = 0;
    } else if constexpr (KP == 16) {
      const uint2 v = ok ? *reinterpret_cast<const uint2*>(rp + 4 * t) : make_uint2(0, 0);
      bf[0][0] = v.x;
      bf[0][1] = v.y;
    } else {
#pragma unroll
      for (int kb = 0; kb < KP / 32; ++kb) {
        const uint4 v = ok ? *reinterpret_cast<const uint4*>(rp + kb * 32 + 8 * t)
                           : make_uint4(0, 0, 0, 0);
        bf[2 * kb][0] = v.x;
        bf[2 * kb][1] = v.y;
        bf[2 * kb + 1][0] = v.z;
        bf[2 * kb + 1][1] = v.w;
      }
    }
  };
  auto slice_of = [&](int col) {
    int s = 0;
    for (int i = 1; i < S; ++i)
      if (col >= offs[i]) s = i;
    return s;
  };

  const int units = (h.ncols + 15) / 16;
  for (int u = warp; u < units; u += kConsumers) {
    const int r0 = u * 16;  // first column of the unit, relative to col0
    const int n0 = h.col0 + r0;
    const int rb = r0 + 4 * (g >> 1) + (g & 1);
    uint32_t bfr[2][KSTEPS][2];
    load_b(rb, rb < h.ncols, bfr[0]);
    load_b(rb + 2, rb + 2 < h.ncols, bfr[1]);
    const int s_first = slice_of(n0);
    const int s_last = slice_of(min(n0 + 15, N - 1));
    float out[2][4];
    for (int s = s_first; s <= s_last; ++s) {
      if (s != cached_slice) {
        load_z(s);
        cached_slice = s;
      }
      float acc[2][4];
#pragma unroll
      for (int tile = 0; tile < 2; ++tile) {
#pragma unroll
        for (int i = 0; i < 4; ++i) acc[tile][i] = 0.f;
#pragma unroll
        for (int ks = 0; ks < KSTEPS; ++ks) {
#pragma unroll
          for (int part = 0; part < (MODE == kFp32 ? 2 : 1); ++part) {
            if constexpr (KP == 8) {
              mma1688(acc[tile], zf[ks][part][0], zf[ks][part][1], bfr[tile][ks][0]);
            } else {
              mma16816(acc[tile], zf[ks][part][0], zf[ks][part][1], zf[ks][part][2],
                       zf[ks][part][3], bfr[tile][ks][0], bfr[tile][ks][1]);
            }
          }
        }
      }
      const float v[2][4] = {{acc[0][0], acc[0][1], acc[1][0], acc[1][1]},
                             {acc[0][2], acc[0][3], acc[1][2], acc[1][3]}};
#pragma unroll
      for (int c = 0; c < 4; ++c) {
        const int col = n0 + 4 * t + c;
        if (s_first == s_last || (col < N && slice_of(col) == s)) {
          out[0][c] = v[0][c];
          out[1][c] = v[1][c];
        }
      }
    }
    const int rc = r0 + 4 * t;  // this lane's first column inside the chunk
    if (rc >= h.ncols) continue;  // ncols is a multiple of 8, so rc+3 < ncols otherwise
#pragma unroll
    for (int hh = 0; hh < 2; ++hh) {
      const int m = g + 8 * hh;
      if (m >= h.n) continue;
      uint2* yp = reinterpret_cast<uint2*>(yt + m * kYPitch + rc * 2);
      const uint2 old = *yp;
      const uint32_t w[2] = {old.x, old.y};
      uint32_t res[2];
#pragma unroll
      for (int q = 0; q < 2; ++q) {
        uint32_t bits2[2];
#pragma unroll
        for (int e = 0; e < 2; ++e) {
          const float base = bf16_bits_to_float((w[q] >> (16 * e)) & 0xffffu);
          const float acc = out[hh][2 * q + e];
          const float sum = MODE == kFp32
                                ? base + h.scale * acc
                                : base + bf16_bits_to_float(float_to_bf16_bits(acc * h.scale));
          bits2[e] = float_to_bf16_bits(sum);
        }
        res[q] = pack2(bits2[0], bits2[1]);
      }
      *yp = make_uint2(res[0], res[1]);
    }
  }
}

template <int MODE>
__global__ void __launch_bounds__(kTmaThreads, 1)
sgmv_expand_bulk_kernel(const __grid_constant__ FusedParams p) {
  extern __shared__ __align__(128) uint8_t smem[];
  float* zbuf = reinterpret_cast<float*>(smem + kStages * kStageBytes);
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + kStages * kStageBytes + kZBufBytes);
  uint64_t* empty = full + kStages;
  int* offs = reinterpret_cast<int*>(empty + kStages);
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  if (tid == 0) {
    for (int s = 0; s < kStages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    fence_mbar_init();
  }
  if (tid <= p.S) offs[tid] = p.slice_offsets[tid];
  __syncthreads();
  pdl_wait();  // z comes from the preceding shrink grid

  if (warp == kConsumers) {
    // ---------------- producer warp
    const int nseg = min(*p.seg_count, p.max_segments);
    const int chunks = (p.N + kItemCols - 1) / kItemCols;
    const int nitems = nseg * chunks;
    const int per_cta = (nitems + gridDim.x - 1) / gridDim.x;
    const int i0 = blockIdx.x * per_cta;
    const int i1 = min(nitems, i0 + per_cta);
    int cached = -1, tok = -1, start = 0;
    bool seg_ok = false;
    SegmentInfo si{};
    int k = 0;
    for (int it = i0;; ++k) {
      const int stage = k % kStages;
      const uint32_t phase = uint32_t(k / kStages) & 1u;
      bool go = true;
      if (lane == 0) go = mbar_wait(&empty[stage], phase ^ 1u);
      if (!__shfl_sync(0xffffffffu, go ? 1 : 0, 0)) break;  // timed out: stop producing
      const Stage st{smem + stage * kStageBytes};
      ItemHeader* h = st.header();
      if (it >= i1) {  // end of stream
        if (lane == 0) {
          h->ok = -1;
          mbar_arrive_expect_tx(&full[stage], 0u);
        }
        break;
      }
      const int seg = it / chunks, chunk = it - seg * chunks;
      if (seg != cached) {
        cached = seg;
        seg_ok = load_segment(p, seg, si, start);
        tok = (seg_ok && lane < si.n) ? p.perm[start + lane] : -1;
        const bool bad = seg_ok && lane < si.n && (tok < 0 || tok >= p.T);
        seg_ok = seg_ok && !__any_sync(0xffffffffu, bad);
      }
      // Merge consecutive items of this segment while the B rows fit the stage.
      const int max_cols = seg_ok ? min(kStageCols, kBTileBytes / (2 * si.bucket)) : kItemCols;
      const int take = min(min(max_cols / kItemCols, chunks - chunk), i1 - it);
      const int col0 = chunk * kItemCols;
      const int ncols = min(take * kItemCols, p.N - col0);
      it += take;
      if (lane < kSeg) h->tok[lane] = tok;
      if (lane == 0) {
        h->ok = seg_ok ? 1 : 0;
        h->seg = seg;
        h->n = si.n;
        h->r = si.r;
        h->bucket = si.bucket;
        h->col0 = col0;
        h->ncols = ncols;
        h->scale = si.scale;
      }
      __syncwarp();
      const uint32_t bbytes = uint32_t(ncols) * si.bucket * 2;
      const uint32_t ybytes = uint32_t(ncols) * 2;
      if (lane == 0) mbar_arrive_expect_tx(&full[stage], seg_ok ? bbytes + si.n * ybytes : 0u);
      __syncwarp();
      if (seg_ok) {
        if (lane == 0)
          bulk_g2s(st.btile(), p.b + si.boff + int64_t(col0) * si.bucket, bbytes, &full[stage]);
        if (lane < si.n)
          bulk_g2s(st.ytile() + lane * kYPitch, p.y + int64_t(tok) * p.y_stride + col0, ybytes,
                   &full[stage]);
      }
    }
  } else {
    // ---------------- consumer warps
    int zseg = -1, prev_stage = -1;
    for (int k = 0;; ++k) {
      const int stage = k % kStages;
      const uint32_t phase = uint32_t(k / kStages) & 1u;
      if (!mbar_wait(&full[stage], phase)) break;
      const Stage st{smem + stage * kStageBytes};
      const ItemHeader& h = *st.header();
      if (h.ok < 0) break;
      if (h.ok) {
        const int kp = h.bucket < 8 ? 8 : h.bucket;
        if (h.seg != zseg) {
          // New segment: its z rows, slice s at s*kp, zero beyond min(r, bucket).
          zseg = h.seg;
          const int live = min(h.r, h.bucket);
          for (int i = tid; i < kSeg * p.S * kp; i += kConsumers * 32) {
            const int m = i / (p.S * kp);
            const int rem = i - m * p.S * kp;
            const int s = rem / kp, kk = rem - s * kp;
            zbuf[m * kMaxRows + s * kp + kk] =
                (m < h.n && kk < live) ? p.z[int64_t(h.tok[m]) * p.z_stride + s * h.r + kk] : 0.f;
          }
          named_barrier(1, kConsumers * 32);
        }
        switch (kp) {
          case 8: consume_item<8, MODE>(h, st, p.S, p.N, offs, zbuf, lane, warp); break;
          case 16: consume_item<16, MODE>(h, st, p.S, p.N, offs, zbuf, lane, warp); break;
          case 32: consume_item<32, MODE>(h, st, p.S, p.N, offs, zbuf, lane, warp); break;
          default: consume_item<64, MODE>(h, st, p.S, p.N, offs, zbuf, lane, warp); break;
        }
        fence_async_smem();
      }
      named_barrier(1, kConsumers * 32);
      if (tid == 0) {
        if (h.ok) {
          for (int m = 0; m < h.n; ++m)
            bulk_s2g(p.y + int64_t(h.tok[m]) * p.y_stride + h.col0, st.ytile() + m * kYPitch,
                     uint32_t(h.ncols) * 2);
        }
        bulk_commit();
        // The previous stage's stores have been read once at most this stage's group
        // is pending; release it then.
        if (prev_stage >= 0) {
          asm volatile("cp.async.bulk.wait_group.read 1;" ::: "memory");
          mbar_arrive(&empty[prev_stage]);
        }
      }
      prev_stage = stage;
    }
    if (tid == 0) {
      bulk_wait_all();
      if (prev_stage >= 0) mbar_arrive(&empty[prev_stage]);
    }
  }
}

}  // namespace
}  // namespace lfb

using namespace lfb;

extern "C" int lf_fused_shrink_expand(
    const void* x, int64_t x_stride, const void* a, const void* b, const int64_t* b_offsets,
    const int32_t* b_strides, void* y, int64_t y_stride, const int32_t* segment_indptr,
    const int32_t* segment_slots, const int32_t* token_indices, const int32_t* ranks,
    const float* scales, const int32_t* slice_offsets, const int32_t* segment_count,
    float* workspace, int64_t workspace_stride, int64_t num_tokens, int64_t width,
    int32_t out_width, int32_t num_slices, int32_t capacity, int32_t num_slots,
    int32_t max_segments, int32_t numerics, void* stream) {
  if (num_tokens < 0 || num_tokens >= (int64_t(1) << 31) || width < 1 || width >= (int64_t(1) << 31))
    return fail(LF_E_INVALID, "fused_shrink_expand: invalid token count or width");
  if (out_width < 1 || num_slices < 1 || num_slices > kMaxSlices || capacity < 1 || num_slots < 1)
    return fail(LF_E_INVALID, "fused_shrink_expand: invalid output width, slices, capacity or slots");
  if (width % 8 || x_stride % 8 || x_stride < width || !aligned16(x) || !aligned16(a))
    return fail(LF_E_INVALID, "fused_shrink_expand: x/A must be 16-byte aligned with width and stride multiples of 8");
  if (!aligned16(b) || (reinterpret_cast<uintptr_t>(y) & 7) || y_stride % 4 || y_stride < out_width)
    return fail(LF_E_INVALID, "fused_shrink_expand: B must be 16-byte aligned, y 8-byte aligned with stride a multiple of 4");
  if (!workspace || workspace_stride < int64_t(num_slices) * capacity)
    return fail(LF_E_INVALID, "fused_shrink_expand: workspace rows must hold num_slices*capacity floats");
  if (numerics != kFp32 && numerics != kReference)
    return fail(LF_E_INVALID, "fused_shrink_expand: numerics must be 0 (fp32) or 1 (reference)");
  if (max_segments < 0) return fail(LF_E_INVALID, "fused_shrink_expand: negative segment capacity");
  if (num_tokens == 0 || max_segments == 0) return LF_OK;
  const int units = (out_width + 15) / 16;
  const int units_per_chunk = 64;  // 1024 output columns per expand CTA
  const int chunks = (units + units_per_chunk - 1) / units_per_chunk;
  if (chunks > 65535 && max_segments > 65535)
    return fail(LF_E_INVALID, "fused_shrink_expand: grid too large");
  FusedParams p{static_cast<const uint16_t*>(x), x_stride, static_cast<const uint16_t*>(a),
                static_cast<const uint16_t*>(b), b_offsets, b_strides, static_cast<uint16_t*>(y),
                y_stride, segment_indptr, segment_slots, token_indices, ranks, scales,
                slice_offsets, segment_count, workspace, workspace_stride, int(num_tokens),
                int(width), out_width, num_slices, capacity, num_slots, max_segments,
                units_per_chunk};
  // K is split over a cluster of `parts` CTAs (a power of two up to 16, non-portable
  // above 8); each stages 16 token rows + S*r A rows (rounded up to the 8-row MMA
  // tiles the fragment loads read) of its K slice.  Pick the smallest cluster whose
  // slice fits ~72 KB, i.e. three CTAs per SM.
  const int rows_max = kSeg + (num_slices * (capacity < 64 ? capacity : 64) + 7) / 8 * 8;
  int parts = 1, kslice = int((width + 31) / 32 * 32);
  while (parts < kMaxCluster && int64_t(rows_max) * (kslice * 2 + 64) > 72 * 1024) {
    parts *= 2;
    kslice = int(((width + parts - 1) / parts + 31) / 32 * 32);
  }
  const int tile_bytes = rows_max * (kslice * 2 + 64);
  int smem = tile_bytes > (kSeg * 64 + kSeg * kMaxRows) * 4 ? tile_bytes
                                                             : (kSeg * 64 + kSeg * kMaxRows) * 4;
  if (smem > 220 * 1024) return fail(LF_E_INVALID, "fused_shrink_expand: K slice too large");
  const cudaStream_t s = static_cast<cudaStream_t>(stream);
  {
    static int flags[64] = {};
    if (int rc = ensure_smem(sgmv_shrink_kernel, smem, flags)) return rc;
    if (parts > 8) {
      static unsigned long long np_flags = 0;
      int device = 0;
      cudaGetDevice(&device);
      if (!(np_flags & (1ull << (device & 63)))) {
        if (cudaFuncSetAttribute(sgmv_shrink_kernel, cudaFuncAttributeNonPortableClusterSizeAllowed,
                                 1) != cudaSuccess)
          return check_launch("fused_shrink_expand: non-portable cluster size");
        np_flags |= 1ull << (device & 63);
      }
    }
    // Shrink the cluster (and grow the slice) until the hardware can co-schedule it.
    while (parts > 1) {
      cudaLaunchConfig_t probe = {};
      probe.gridDim = dim3(parts, 1, 1);
      probe.blockDim = dim3(kThreads);
      probe.dynamicSmemBytes = smem;
      cudaLaunchAttribute cattr[1];
      cattr[0].id = cudaLaunchAttributeClusterDimension;
      cattr[0].val.clusterDim.x = parts;
      cattr[0].val.clusterDim.y = 1;
      cattr[0].val.clusterDim.z = 1;
      probe.attrs = cattr;
      probe.numAttrs = 1;
      int active = 0;
      if (cudaOccupancyMaxActiveClusters(&active, sgmv_shrink_kernel, &probe) == cudaSuccess &&
          active > 0)
        break;
      cudaGetLastError();
      parts /= 2;
      kslice = int(((width + parts - 1) / parts + 31) / 32 * 32);
      const int bytes = rows_max * (kslice * 2 + 64);
      if (bytes > smem) {
        smem = bytes;
        if (smem > 220 * 1024) return fail(LF_E_INVALID, "fused_shrink_expand: K slice too large");
        if (int rc = ensure_smem(sgmv_shrink_kernel, smem, flags)) return rc;
      }
    }
    cudaLaunchConfig_t config = {};
    config.gridDim = dim3(parts, max_segments, 1);
    config.blockDim = dim3(kThreads);
    config.dynamicSmemBytes = smem;
    config.stream = s;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = parts;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    config.attrs = attr;
    config.numAttrs = 1;
    const cudaError_t err = cudaLaunchKernelEx(&config, sgmv_shrink_kernel, p, kslice);
    if (err != cudaSuccess) {
      last_error() = std::string("fused_shrink_expand (shrink): ") + cudaGetErrorString(err);
      return LF_E_CUDA;
    }
  }
  // The bulk-copy expand needs 16-byte aligned y rows and 8-column multiples; other
  // layouts use the direct-load expand.
  const bool bulk = out_width % 8 == 0 && y_stride % 8 == 0 &&
                    (reinterpret_cast<uintptr_t>(y) & 15) == 0;
  if (bulk) {
    int device = 0, sms = 0;
    if (cudaGetDevice(&device) != cudaSuccess ||
        cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, device) != cudaSuccess)
      return check_launch("fused_shrink_expand: device query");
    auto kernel = numerics == kFp32 ? sgmv_expand_bulk_kernel<kFp32>
                                    : sgmv_expand_bulk_kernel<kReference>;
    static int flags[2][64] = {};
    if (int rc = ensure_smem(kernel, kTmaSmem, flags[numerics])) return rc;
    cudaLaunchConfig_t config = {};
    config.gridDim = dim3(sms);
    config.blockDim = dim3(kTmaThreads);
    config.dynamicSmemBytes = kTmaSmem;
    config.stream = s;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    config.attrs = attr;
    config.numAttrs = 1;
    const cudaError_t err = cudaLaunchKernelEx(&config, kernel, p);
    if (err != cudaSuccess) {
      last_error() = std::string("fused_shrink_expand (expand): ") + cudaGetErrorString(err);
      return LF_E_CUDA;
    }
    return LF_OK;
  }
  {
    cudaLaunchConfig_t config = {};
    config.gridDim = dim3(chunks, max_segments, 1);
    config.blockDim = dim3(kThreads);
    config.stream = s;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    config.attrs = attr;
    config.numAttrs = 1;
    auto kernel = numerics == kFp32 ? sgmv_expand_kernel<kFp32> : sgmv_expand_kernel<kReference>;
    const cudaError_t err = cudaLaunchKernelEx(&config, kernel, p);
    if (err != cudaSuccess) {
      last_error() = std::string("fused_shrink_expand (expand): ") + cudaGetErrorString(err);
      return LF_E_CUDA;
    }
  }
  return LF_OK;
}

extern "C" int lf_device_wait_timeouts(int32_t* count, int32_t reset) {
  unsigned int value = 0;
  if (cudaMemcpyFromSymbol(&value, g_lf_wait_timeouts, sizeof(value)) != cudaSuccess)
    return check_launch("device_wait_timeouts");
  if (count) *count = int32_t(value);
  if (reset) {
    const unsigned int zero = 0;
    if (cudaMemcpyToSymbol(g_lf_wait_timeouts, &zero, sizeof(zero)) != cudaSuccess)
      return check_launch("device_wait_timeouts");
  }
  return LF_OK;
}
