// Grouped (SGMV) LoRA shrink -> expand over decode segments of <= 16 tokens (one slot each).
//
// Two streaming kernels per call, chained with programmatic dependent launch:
//
//   sgmv_shrink_kernel   partial z[c][t, j] = sum_{k in chunk c} x[t, k] * A_g[j, k] for
//                        every token t of a segment and j < S*r.  Persistent CTAs walk a
//                        contiguous range of (segment, K chunk) units; each unit's x rows
//                        and A rows are staged in shared memory by a 3-deep cp.async
//                        pipeline, so every A row is read from HBM once per segment.  The
//                        FP32 partials go to the workspace; no atomics.
//   sgmv_expand_*        y[t, n] += scale_g * sum_k z[t, slice(n)*r + k] * B_g[n, k], with
//                        z = sum over chunks of the partials, added in chunk order (so
//                        results are deterministic).  The bulk-copy kernel streams B rows
//                        and y rows through a shared-memory ring with cp.async.bulk; the
//                        direct kernel (outputs that are not 16-byte aligned) reads them
//                        with vector loads.
//
// The MMAs run on the tensor cores (mma.sync m16n8k16 / m16n8k8, BF16 operands, FP32
// accumulate) with the segment's tokens as the M dimension.  Inside each 32-element K
// block the fragment slots carry a permutation of k that is the same for both
// operands, so a lane's 16 contiguous bytes feed two MMAs.  Output columns are
// permuted the same way so that each lane owns four consecutive outputs.
//
// Numerics: kFp32 keeps z in FP32 (split into BF16 hi + lo for the expand MMAs, about
// 16 significant bits) and rounds the output once: y = bf16(y + scale*acc).
// kReference reproduces the retained-rank operators' contract: z rounded to BF16,
// delta = bf16(acc*scale), y = bf16(y + delta)
// (src/loraforge/ops/csrc/lora_rows.cu:64 and :113).
#include "launch.cuh"
#include "tma.cuh"

namespace lfb {
namespace {

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
  float* z;                // FP32 workspace: partial c of token t at z + c*z_chunk + t*z_stride
  int64_t z_stride;        // >= S * cap, a multiple of 4
  int64_t z_chunk;         // floats per chunk partial (T * z_stride)
  int T, K, N, S, cap, num_slots, max_segments;
  int nchunks;             // K chunks of the shrink (slots of partials per token)
  int shrink_ctas;         // grid size of the shrink (defines its per-CTA unit runs)
  int units_per_chunk;     // direct expand: 16-column units per CTA
};

// z[tok, j] for a token of segment `seg`: the sum, in chunk order, of the partials
// the shrink wrote.  The shrink gives each CTA a contiguous run of (segment, chunk)
// units and writes one partial per (segment, CTA run), at the slot of the run's first
// chunk; the run starts are the segment's first chunk and every CTA boundary inside
// the segment.
__device__ __forceinline__ float z_value(const FusedParams& p, int nseg, int seg, int tok, int j) {
  const int64_t nunits = int64_t(nseg) * p.nchunks;
  const int64_t per = (nunits + p.shrink_ctas - 1) / p.shrink_ctas;
  const int64_t first = int64_t(seg) * p.nchunks, last = first + p.nchunks;
  const float* zp = p.z + int64_t(tok) * p.z_stride + j;
  float sum = zp[0];
  for (int64_t b = (first / per + 1) * per; b < last; b += per) sum += zp[(b - first) * p.z_chunk];
  return sum;
}

__device__ __forceinline__ uint32_t cvt_bf16x2(float first, float second) {
  uint32_t r;
  asm("cvt.rn.bf16x2.f32 %0, %1, %2;" : "=r"(r) : "f"(second), "f"(first));
  return r;
}

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
constexpr int kShrinkStages = 3;

struct alignas(16) ShrinkHeader {
  int ok, chunk, n, g, r;
  int pad[3];
  int tok[kSeg];
};

__device__ __forceinline__ void cp_async16(void* dst, const void* src) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_u32(dst)), "l"(src)
               : "memory");
}
__device__ __forceinline__ void cp_async_commit() {
  asm volatile("cp.async.commit_group;" ::: "memory");
}
template <int N>
__device__ __forceinline__ void cp_async_wait() {
  asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}
__device__ __forceinline__ uint4 lds16(const uint8_t* p) { return *reinterpret_cast<const uint4*>(p); }

// Persistent grid over (segment, K chunk) units, segment-major, a contiguous range
// per CTA.  A stage holds one unit: x rows of the segment's tokens in slots 0..15 and
// the slot's S*r A rows from slot 16, each `kc` columns wide with a row pitch of
// kc*2 + 64 bytes (kc a multiple of 64, so the 16-byte fragment loads below hit
// distinct bank groups).
__global__ void __launch_bounds__(kThreads, 2)
sgmv_shrink_kernel(const __grid_constant__ FusedParams p, int kc, int stage_bytes) {
  extern __shared__ __align__(128) uint8_t smem[];
  ShrinkHeader* hdr = reinterpret_cast<ShrinkHeader*>(smem + kShrinkStages * stage_bytes);
  float* warp_part = reinterpret_cast<float*>(hdr + kShrinkStages);  // [kparts][16][8*ntiles]
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int g8 = lane >> 2, t4 = lane & 3;
  const int pitch = kc * 2 + 64;
  const int nseg = min(*p.seg_count, p.max_segments);
  const int nunits = nseg * p.nchunks;
  const int per = (nunits + gridDim.x - 1) / gridDim.x;
  const int u0 = min(nunits, int(blockIdx.x) * per);
  const int u1 = min(nunits, u0 + per);
  // Warp 0 keeps the metadata of the segment it described last.
  int cseg = -1, cstart = 0, ctok = -1;
  bool cok = false;
  SegmentInfo csi{};

  // Describe unit u in stage st and start its copies (one cp.async group per call).
  auto issue = [&](int u, int st) {
    if (warp == 0 && u < u1) {
      const int seg = u / p.nchunks;
      if (seg != cseg) {
        cseg = seg;
        cok = load_segment(p, seg, csi, cstart);
        ctok = (cok && lane < csi.n) ? p.perm[cstart + lane] : -1;
        const bool bad = cok && lane < csi.n && (ctok < 0 || ctok >= p.T);
        cok = cok && !__any_sync(0xffffffffu, bad);
      }
      if (lane < kSeg) hdr[st].tok[lane] = ctok;
      if (lane == 0) {
        hdr[st].ok = cok ? 1 : 0;
        hdr[st].chunk = u - seg * p.nchunks;
        hdr[st].n = csi.n;
        hdr[st].g = csi.g;
        hdr[st].r = csi.r;
      }
    }
    __syncthreads();
    if (u < u1 && hdr[st].ok) {
      const ShrinkHeader& h = hdr[st];
      const int kb = h.chunk * kc;
      const int c16 = (min(p.K, kb + kc) - kb) / 8;
      const int rows = h.n + p.S * h.r;
      uint8_t* base = smem + st * stage_bytes;
      for (int idx = tid; idx < rows * c16; idx += kThreads) {
        const int row = idx / c16, c = idx - row * c16;
        const uint16_t* src;
        int slot;
        if (row < h.n) {
          src = p.x + int64_t(h.tok[row]) * p.x_stride + kb + c * 8;
          slot = row;
        } else {
          const int j = row - h.n;
          src = p.a + (int64_t(h.g) * p.S * p.cap + j) * p.K + kb + c * 8;
          slot = kSeg + j;
        }
        cp_async16(base + slot * pitch + c * 16, src);
      }
    }
    cp_async_commit();
  };

  issue(u0, 0);
  issue(u0 + 1, 1);
  // Accumulators persist over consecutive units of one segment (a "run"); a run's
  // partial is written at the slot of its first chunk when the run ends.
  float acc[kMaxTilesPerWarp][4];
#pragma unroll
  for (int i = 0; i < kMaxTilesPerWarp; ++i)
#pragma unroll
    for (int e = 0; e < 4; ++e) acc[i][e] = 0.f;
  for (int u = u0, k = 0; u < u1; ++u, ++k) {
    const int st = k % kShrinkStages;
    issue(u + 2, (k + 2) % kShrinkStages);
    cp_async_wait<2>();  // unit u's group has landed
    __syncthreads();
    const ShrinkHeader& h = hdr[st];
    const int seg = u / p.nchunks;
    const bool run_end = u + 1 == u1 || (u + 1) / p.nchunks != seg;
    const int R = p.S * h.r;
    const int ntiles = (R + 7) / 8;
    const int kparts = ntiles >= kWarps ? 1 : kWarps / ntiles;
    const int my_tile0 = ntiles >= kWarps ? warp : warp % ntiles;
    const int my_kpart = ntiles >= kWarps ? 0 : warp / ntiles;
    const bool active = my_kpart < kparts;
    if (h.ok && active) {
      const uint8_t* base = smem + st * stage_bytes;
      const int klen = min(p.K, (h.chunk + 1) * kc) - h.chunk * kc;
      const int kblocks = (klen + 31) / 32;
      const int b0 = kblocks * my_kpart / kparts, b1 = kblocks * (my_kpart + 1) / kparts;
      const uint8_t* xr0 = base + g8 * pitch;
      const uint8_t* xr1 = base + (g8 + 8) * pitch;
      const uint4 zero = make_uint4(0, 0, 0, 0);
#pragma unroll 4
      for (int blk = b0; blk < b1; ++blk) {
        const int kk = blk * 32 + 8 * t4;
        const bool kin = kk < klen;
        const uint4 x0 = kin ? lds16(xr0 + kk * 2) : zero;
        const uint4 x1 = kin ? lds16(xr1 + kk * 2) : zero;
#pragma unroll
        for (int i = 0; i < kMaxTilesPerWarp; ++i) {
          const int tile = my_tile0 + i * kWarps;
          if (tile < ntiles) {
            const uint4 av = kin ? lds16(base + (kSeg + tile * 8 + g8) * pitch + kk * 2) : zero;
            mma16816(acc[i], x0.x, x1.x, x0.y, x1.y, av.x, av.y);
            mma16816(acc[i], x0.z, x1.z, x0.w, x1.w, av.z, av.w);
          }
        }
      }
    }
    if (run_end && h.ok) {
      const int slot = max(u0, seg * p.nchunks) - seg * p.nchunks;
      float* zc = p.z + int64_t(slot) * p.z_chunk;
      if (kparts == 1) {
        // Warps beyond ntiles hold no tile.  Rows m >= n belong to no token.
        if (active) {
#pragma unroll
          for (int i = 0; i < kMaxTilesPerWarp; ++i) {
            const int tile = my_tile0 + i * kWarps;
            const int j = tile * 8 + 2 * t4;
            if (tile >= ntiles) continue;
#pragma unroll
            for (int hh = 0; hh < 2; ++hh) {
              const int m = g8 + 8 * hh;
              if (m >= h.n) continue;
              float* zr = zc + int64_t(h.tok[m]) * p.z_stride;
              if (j < R) zr[j] = acc[i][2 * hh];
              if (j + 1 < R) zr[j + 1] = acc[i][2 * hh + 1];
            }
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
        for (int i = tid; i < h.n * R; i += kThreads) {
          const int m = i / R, j = i - m * R;
          float sum = 0.f;
          for (int q = 0; q < kparts; ++q) sum += warp_part[(q * kSeg + m) * RP + j];
          zc[int64_t(h.tok[m]) * p.z_stride + j] = sum;
        }
      }
    }
    if (run_end) {
#pragma unroll
      for (int i = 0; i < kMaxTilesPerWarp; ++i)
#pragma unroll
        for (int e = 0; e < 4; ++e) acc[i][e] = 0.f;
    }
    __syncthreads();  // stage st and the partial buffer are free again
  }
  cp_async_wait<0>();
  __syncthreads();
  pdl_launch_dependents();
}

// Shrink tiling for the host: K chunk width (a multiple of 64) and stage bytes such
// that three stages of (16 + S*r) rows fit two CTAs per SM.
struct ShrinkTiling {
  int kc, stage_bytes, smem, nchunks;
};

inline ShrinkTiling shrink_tiling(int64_t width, int num_slices, int capacity) {
  const int rows = kSeg + (num_slices * (capacity < 64 ? capacity : 64) + 7) / 8 * 8;
  int kc = int((36 * 1024 / rows - 64) / 2) / 64 * 64;
  if (kc > 512) kc = 512;
  if (kc < 64) kc = 64;
  const int64_t wpad = (width + 63) / 64 * 64;
  if (kc > wpad) kc = int(wpad);
  ShrinkTiling t;
  t.kc = kc;
  t.stage_bytes = (rows * (kc * 2 + 64) + 127) / 128 * 128;
  t.smem = kShrinkStages * t.stage_bytes + kShrinkStages * int(sizeof(ShrinkHeader)) + kSeg * 64 * 4;
  t.nchunks = int((width + kc - 1) / kc);
  return t;
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
  const int nseg = min(*p.seg_count, p.max_segments);
  if (tid <= p.S) offs[tid] = p.slice_offsets[tid];
  if (!load_tokens(p, si, start, tok)) return;
  const int live = min(si.r, si.bucket);
  for (int i = tid; i < kSeg * p.S * si.kp; i += kThreads) {
    const int m = i / (p.S * si.kp);
    const int rem = i - m * p.S * si.kp;
    const int s = rem / si.kp, k = rem - s * si.kp;
    float v = 0.f;
    if (k < live && m < si.n) v = z_value(p, nseg, blockIdx.y, tok[m], s * si.r + k);
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
// from shared memory, store the updated y values straight to global memory (8 bytes
// per lane, so the stage is free as soon as the compute is done) and release the
// stage through its "empty" mbarrier.  A header with ok = -1 ends the stream.
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
                                             const int* offs, const float* zbuf, uint16_t* y,
                                             int64_t y_stride, int lane, int warp) {
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
  // Usually the whole stage lies in one slice; then no per-unit slice lookups.
  const int stage_first = slice_of(h.col0);
  const int stage_slice = stage_first == slice_of(h.col0 + h.ncols - 1) ? stage_first : -1;
  for (int u = warp; u < units; u += kConsumers) {
    const int r0 = u * 16;  // first column of the unit, relative to col0
    const int n0 = h.col0 + r0;
    const int rb = r0 + 4 * (g >> 1) + (g & 1);
    uint32_t bfr[2][KSTEPS][2];
    load_b(rb, rb < h.ncols, bfr[0]);
    load_b(rb + 2, rb + 2 < h.ncols, bfr[1]);
    const int s_first = stage_slice >= 0 ? stage_slice : slice_of(n0);
    const int s_last = stage_slice >= 0 ? stage_slice : slice_of(min(n0 + 15, N - 1));
    float out[2][4];
    for (int s = s_first; s <= s_last; ++s) {
      if (s != cached_slice) {
        load_z(s);
        cached_slice = s;
      }
      // Separate accumulators per tile and per hi/lo part: four independent MMA chains.
      constexpr int PARTS = MODE == kFp32 ? 2 : 1;
      float accp[2][PARTS][4];
#pragma unroll
      for (int tile = 0; tile < 2; ++tile)
#pragma unroll
        for (int part = 0; part < PARTS; ++part)
#pragma unroll
          for (int i = 0; i < 4; ++i) accp[tile][part][i] = 0.f;
#pragma unroll
      for (int ks = 0; ks < KSTEPS; ++ks) {
#pragma unroll
        for (int tile = 0; tile < 2; ++tile) {
#pragma unroll
          for (int part = 0; part < PARTS; ++part) {
            if constexpr (KP == 8) {
              mma1688(accp[tile][part], zf[ks][part][0], zf[ks][part][1], bfr[tile][ks][0]);
            } else {
              mma16816(accp[tile][part], zf[ks][part][0], zf[ks][part][1], zf[ks][part][2],
                       zf[ks][part][3], bfr[tile][ks][0], bfr[tile][ks][1]);
            }
          }
        }
      }
      float acc[2][4];
#pragma unroll
      for (int tile = 0; tile < 2; ++tile)
#pragma unroll
        for (int i = 0; i < 4; ++i)
          acc[tile][i] = PARTS == 2 ? accp[tile][0][i] + accp[tile][PARTS - 1][i] : accp[tile][0][i];
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
      const uint2 old = *reinterpret_cast<const uint2*>(yt + m * kYPitch + rc * 2);
      uint2* yp = reinterpret_cast<uint2*>(y + int64_t(h.tok[m]) * y_stride + h.col0 + rc);
      const float b0 = __uint_as_float(old.x << 16), b1 = __uint_as_float(old.x & 0xffff0000u);
      const float b2 = __uint_as_float(old.y << 16), b3 = __uint_as_float(old.y & 0xffff0000u);
      float d[4];
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        d[e] = MODE == kFp32 ? h.scale * out[hh][e]
                             : bf16_bits_to_float(float_to_bf16_bits(out[hh][e] * h.scale));
      }
      uint32_t res[2];
      res[0] = cvt_bf16x2(b0 + d[0], b1 + d[1]);
      res[1] = cvt_bf16x2(b2 + d[2], b3 + d[3]);
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
    const int nseg = min(*p.seg_count, p.max_segments);
    int zseg = -1;
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
                (m < h.n && kk < live) ? z_value(p, nseg, h.seg, h.tok[m], s * h.r + kk) : 0.f;
          }
          named_barrier(1, kConsumers * 32);
        }
        switch (kp) {
          case 8: consume_item<8, MODE>(h, st, p.S, p.N, offs, zbuf, p.y, p.y_stride, lane, warp); break;
          case 16: consume_item<16, MODE>(h, st, p.S, p.N, offs, zbuf, p.y, p.y_stride, lane, warp); break;
          case 32: consume_item<32, MODE>(h, st, p.S, p.N, offs, zbuf, p.y, p.y_stride, lane, warp); break;
          default: consume_item<64, MODE>(h, st, p.S, p.N, offs, zbuf, p.y, p.y_stride, lane, warp); break;
        }
      }
      named_barrier(1, kConsumers * 32);  // every warp is done with this stage
      if (tid == 0) mbar_arrive(&empty[stage]);
    }
  }
}

}  // namespace
}  // namespace lfb

using namespace lfb;

extern "C" int64_t lf_fused_workspace_floats(int64_t num_tokens, int64_t width,
                                             int32_t num_slices, int32_t capacity) {
  if (num_tokens < 0 || width < 1 || num_slices < 1 || capacity < 1) return -1;
  const ShrinkTiling t = shrink_tiling(width, num_slices, capacity);
  const int64_t zstride = (int64_t(num_slices) * capacity + 3) / 4 * 4;
  return int64_t(t.nchunks) * (num_tokens > 0 ? num_tokens : 1) * zstride;
}

extern "C" int lf_fused_shrink_expand(
    const void* x, int64_t x_stride, const void* a, const void* b, const int64_t* b_offsets,
    const int32_t* b_strides, void* y, int64_t y_stride, const int32_t* segment_indptr,
    const int32_t* segment_slots, const int32_t* token_indices, const int32_t* ranks,
    const float* scales, const int32_t* slice_offsets, const int32_t* segment_count,
    float* workspace, int64_t workspace_floats, int64_t num_tokens, int64_t width,
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
  if (numerics != kFp32 && numerics != kReference)
    return fail(LF_E_INVALID, "fused_shrink_expand: numerics must be 0 (fp32) or 1 (reference)");
  if (max_segments < 0) return fail(LF_E_INVALID, "fused_shrink_expand: negative segment capacity");
  const int64_t need = lf_fused_workspace_floats(num_tokens, width, num_slices, capacity);
  if (!workspace || workspace_floats < need || (reinterpret_cast<uintptr_t>(workspace) & 15))
    return fail(LF_E_INVALID, "fused_shrink_expand: workspace too small or not 16-byte aligned "
                              "(see lf_fused_workspace_floats)");
  if (num_tokens == 0 || max_segments == 0) return LF_OK;
  const ShrinkTiling tiling = shrink_tiling(width, num_slices, capacity);
  const int units = (out_width + 15) / 16;
  const int units_per_chunk = 64;  // direct expand: 1024 output columns per CTA
  const int chunks = (units + units_per_chunk - 1) / units_per_chunk;
  if (chunks > 65535 && max_segments > 65535)
    return fail(LF_E_INVALID, "fused_shrink_expand: grid too large");
  const int64_t zstride = (int64_t(num_slices) * capacity + 3) / 4 * 4;
  FusedParams p{static_cast<const uint16_t*>(x), x_stride, static_cast<const uint16_t*>(a),
                static_cast<const uint16_t*>(b), b_offsets, b_strides, static_cast<uint16_t*>(y),
                y_stride, segment_indptr, segment_slots, token_indices, ranks, scales,
                slice_offsets, segment_count, workspace, zstride, zstride * num_tokens,
                int(num_tokens), int(width), out_width, num_slices, capacity, num_slots,
                max_segments, tiling.nchunks, 0, units_per_chunk};
  int device = 0, sms = 0;
  if (cudaGetDevice(&device) != cudaSuccess ||
      cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, device) != cudaSuccess)
    return check_launch("fused_shrink_expand: device query");
  const cudaStream_t s = static_cast<cudaStream_t>(stream);
  p.shrink_ctas = 2 * sms;
  {
    static int flags[64] = {};
    if (int rc = ensure_smem(sgmv_shrink_kernel, tiling.smem, flags)) return rc;
    sgmv_shrink_kernel<<<p.shrink_ctas, kThreads, tiling.smem, s>>>(p, tiling.kc, tiling.stage_bytes);
    if (int rc = check_launch("fused_shrink_expand (shrink)")) return rc;
  }
  // The bulk-copy expand needs 16-byte aligned y rows and 8-column multiples; other
  // layouts use the direct-load expand.
  const bool bulk = out_width % 8 == 0 && y_stride % 8 == 0 &&
                    (reinterpret_cast<uintptr_t>(y) & 15) == 0;
  cudaLaunchConfig_t config = {};
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  config.attrs = attr;
  config.numAttrs = 1;
  config.stream = s;
  cudaError_t err;
  if (bulk) {
    auto kernel = numerics == kFp32 ? sgmv_expand_bulk_kernel<kFp32>
                                    : sgmv_expand_bulk_kernel<kReference>;
    static int flags[2][64] = {};
    if (int rc = ensure_smem(kernel, kTmaSmem, flags[numerics])) return rc;
    config.gridDim = dim3(sms);
    config.blockDim = dim3(kTmaThreads);
    config.dynamicSmemBytes = kTmaSmem;
    err = cudaLaunchKernelEx(&config, kernel, p);
  } else {
    auto kernel = numerics == kFp32 ? sgmv_expand_kernel<kFp32> : sgmv_expand_kernel<kReference>;
    config.gridDim = dim3(chunks, max_segments, 1);
    config.blockDim = dim3(kThreads);
    config.dynamicSmemBytes = 0;
    err = cudaLaunchKernelEx(&config, kernel, p);
  }
  if (err != cudaSuccess) {
    last_error() = std::string("fused_shrink_expand (expand): ") + cudaGetErrorString(err);
    return LF_E_CUDA;
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

// ------------------------------------------------------------------ allocation-free entry
// lf_fused_shrink_expand_noalloc runs the same two kernels as lf_fused_shrink_expand
// but takes its scratch from a fixed buffer compiled into this library, for callers
// that are not allowed to allocate device memory themselves.
#include <mutex>

namespace {
// 4 Mi floats (16 MiB).  A static __device__ array is created on every GPU that loads
// this library and lives until the process exits.
constexpr int64_t kNoAllocScratchFloats = int64_t(4) << 20;
static __device__ __align__(256) float g_noalloc_scratch[kNoAllocScratchFloats];

std::mutex g_noalloc_mutex;
float* g_noalloc_address[64] = {};  // device address of the buffer, per device
}  // namespace

extern "C" int lf_fused_shrink_expand_noalloc(
    const void* x, int64_t x_stride, const void* a, const void* b, const int64_t* b_offsets,
    const int32_t* b_strides, void* y, int64_t y_stride, const int32_t* segment_indptr,
    const int32_t* segment_slots, const int32_t* token_indices, const int32_t* ranks,
    const float* scales, const int32_t* slice_offsets, const int32_t* segment_count,
    int64_t num_tokens, int64_t width, int32_t out_width, int32_t num_slices, int32_t capacity,
    int32_t num_slots, int32_t max_segments, int32_t numerics, void* stream) {
  const int64_t need = lf_fused_workspace_floats(num_tokens, width, num_slices, capacity);
  if (need < 0) return fail(LF_E_INVALID, "fused_shrink_expand_noalloc: invalid sizes");
  if (need > kNoAllocScratchFloats) {
    last_error() = "fused_shrink_expand_noalloc: these sizes need " + std::to_string(need) +
                   " floats of scratch, more than the built-in " +
                   std::to_string(kNoAllocScratchFloats) +
                   "-float (16 MiB) buffer; use lf_fused_shrink_expand with a workspace";
    return LF_E_INVALID;
  }
  int device = 0;
  if (cudaGetDevice(&device) != cudaSuccess) return check_launch("fused_shrink_expand_noalloc");
  if (device < 0 || device >= 64)
    return fail(LF_E_UNSUPPORTED, "fused_shrink_expand_noalloc: device index above 63");
  float* scratch = nullptr;
  {
    // First call on a device: look up the buffer's device address with that device
    // current.  The host-side name g_noalloc_scratch is not a device address.
    std::lock_guard<std::mutex> lock(g_noalloc_mutex);
    if (!g_noalloc_address[device]) {
      void* address = nullptr;
      const cudaError_t err = cudaGetSymbolAddress(&address, g_noalloc_scratch);
      if (err != cudaSuccess || !address) {
        last_error() = std::string("fused_shrink_expand_noalloc: cudaGetSymbolAddress: ") +
                       cudaGetErrorString(err);
        return LF_E_CUDA;
      }
      g_noalloc_address[device] = static_cast<float*>(address);
    }
    scratch = g_noalloc_address[device];
  }
  return lf_fused_shrink_expand(x, x_stride, a, b, b_offsets, b_strides, y, y_stride,
                                segment_indptr, segment_slots, token_indices, ranks, scales,
                                slice_offsets, segment_count, scratch, kNoAllocScratchFloats,
                                num_tokens, width, out_width, num_slices, capacity, num_slots,
                                max_segments, numerics, stream);
}
