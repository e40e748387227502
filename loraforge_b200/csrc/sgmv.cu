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

namespace cg = cooperative_groups;

namespace lfb {
namespace {

constexpr int kMaxCluster = 8;
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
  return true;
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
// grid (cluster_k, max_segments), cluster (cluster_k, 1, 1).
__global__ void __launch_bounds__(kThreads, 2) sgmv_shrink_kernel(const __grid_constant__ FusedParams p) {
  __shared__ float cta_part[kSeg * kMaxRows];
  __shared__ float warp_part[kSeg * 64];
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
  const int kblocks = (p.K + 31) / 32;
  const int kb_begin = int(int64_t(kblocks) * rank / parts);
  const int kb_end = int(int64_t(kblocks) * (rank + 1) / parts);
  const int R = p.S * si.r;
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
    const int span = kb_end - kb_begin;
    const int kb0 = kb_begin + span * my_kpart / kparts;
    const int kb1 = kb_begin + span * (my_kpart + 1) / kparts;
    const uint16_t* xr0 = tok[g8] >= 0 ? p.x + int64_t(tok[g8]) * p.x_stride : nullptr;
    const uint16_t* xr1 = tok[g8 + 8] >= 0 ? p.x + int64_t(tok[g8 + 8]) * p.x_stride : nullptr;
    const uint16_t* ar[kMaxTilesPerWarp];
#pragma unroll
    for (int i = 0; i < kMaxTilesPerWarp; ++i) {
      const int tile = my_tile0 + i * kWarps;
      const int j = tile * 8 + g8;
      ar[i] = (tile < ntiles && j < R) ? p.a + (int64_t(si.g) * p.S * p.cap + j) * p.K : nullptr;
    }
    const uint4 zero = make_uint4(0, 0, 0, 0);
#pragma unroll 2
    for (int kb = kb0; kb < kb1; ++kb) {
      const int k = kb * 32 + 8 * t4;
      const bool kin = k < p.K;
      const uint4 x0 = (kin && xr0) ? ldg16(xr0 + k) : zero;
      const uint4 x1 = (kin && xr1) ? ldg16(xr1 + k) : zero;
      uint4 av[kMaxTilesPerWarp];
#pragma unroll
      for (int i = 0; i < kMaxTilesPerWarp; ++i) av[i] = (kin && ar[i]) ? ldg16(ar[i] + k) : zero;
#pragma unroll
      for (int i = 0; i < kMaxTilesPerWarp; ++i) {
        if (my_tile0 + i * kWarps < ntiles) {
          mma16816(acc[i], x0.x, x1.x, x0.y, x1.y, av[i].x, av[i].y);
          mma16816(acc[i], x0.z, x1.z, x0.w, x1.w, av[i].z, av[i].w);
        }
      }
    }
  }
  // Fixed-order reduction of the K parts inside the CTA.
  if (kparts == 1) {
#pragma unroll
    for (int i = 0; i < kMaxTilesPerWarp; ++i) {
      const int tile = my_tile0 + i * kWarps;
      const int j = tile * 8 + 2 * t4;
      if (tile < ntiles && j < R) {
        cta_part[g8 * kMaxRows + j] = acc[i][0];
        cta_part[(g8 + 8) * kMaxRows + j] = acc[i][2];
      }
      if (tile < ntiles && j + 1 < R) {
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
  // About 512 input columns per CTA along K, at most a cluster of 8.
  int parts = int((width + 511) / 512);
  parts = parts < 1 ? 1 : (parts > kMaxCluster ? kMaxCluster : parts);
  const cudaStream_t s = static_cast<cudaStream_t>(stream);
  {
    cudaLaunchConfig_t config = {};
    config.gridDim = dim3(parts, max_segments, 1);
    config.blockDim = dim3(kThreads);
    config.stream = s;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = parts;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    config.attrs = attr;
    config.numAttrs = 1;
    const cudaError_t err = cudaLaunchKernelEx(&config, sgmv_shrink_kernel, p);
    if (err != cudaSuccess) {
      last_error() = std::string("fused_shrink_expand (shrink): ") + cudaGetErrorString(err);
      return LF_E_CUDA;
    }
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
