// Prefill SGMV on the 5th-generation tensor cores (tcgen05 + TMEM): segments of 16 to 128
// tokens of one adapter slot each, as produced by group_tokens(chunk = 128).
//
//   prefill_shrink_kernel  z[seg] = X[seg] . A_g^T, one unit per (segment, K part).  Four
//                          producer warps stage the segment's x rows (gathered through
//                          token_indices) and the slot's A rows into 128-byte-swizzled
//                          K-major tiles with cp.async; one thread issues
//                          tcgen05.mma (M = 128 tokens, N = S*r rounded up to 16, K = 16 per
//                          instruction, BF16 in, FP32 accumulated in TMEM) and commits each
//                          stage back to the producers.  The same four warps then read the
//                          accumulator from TMEM (tcgen05.ld) and publish the K part's FP32
//                          partial; the CTA that completes a segment's counter adds the
//                          parts in order into z (deterministic, no floating-point atomics).
//   prefill_expand_kernel  y[seg, cols] += scale . z[seg] . B_g[cols]^T, one unit per
//                          (segment, slice, 256-column block).  Two producer warps build the
//                          segment's z tile (BF16 hi + lo of the FP32 z, scale folded in)
//                          and load the compact B rows of the block: TMA boxes in the
//                          bucket's own swizzled layout for buckets 16 / 32 / 64 (K = the
//                          bucket), else cp.async rows zero-padded to 64 (K = 64);
//                          one thread issues M = 128, N = 256, K = 16 MMAs into one of two
//                          TMEM accumulators; eight epilogue warps read the other one and
//                          update the y rows (prefetched before the MMA completes).
//
// Every segment of a prefill call runs on these tiles, short ones included: a tile's unused
// rows cost tensor-core cycles but no memory traffic (x and y rows are moved only for the
// segment's tokens, A and B once per tile either way), while sending the short segments
// to the decode kernels costs two more launches (measured on BASELINE config 3: 57 us for
// two segments of under 16 tokens, against 0 extra here).  Numerics follow lf_fused_shrink_expand: FP32
// keeps z in FP32 (hi + lo BF16 parts) and rounds y once; "reference" rounds z to BF16
// and the scaled delta to BF16 before the BF16 sum (src/loraforge/ops/csrc/lora_rows.cu:64
// and :113).
//
// Every wait is bounded (tma.cuh): an expired wait is counted and the thread carries on
// to the CTA's final barrier, where the TMEM allocation is always released.
#include <cuda.h>
#include <cudaTypedefs.h>

#include <mutex>
#include <string>

#include "launch.cuh"
#include "sgmv.cuh"
#include "tcgen05.cuh"
#include "tma.cuh"

namespace lfb {
namespace {

using namespace tc;

constexpr int kTileM = 128;                  // tokens per tile (UMMA M)
constexpr int kRowBytes = 128;               // one swizzled K-major row: 64 BF16
constexpr int kXTileBytes = kTileM * kRowBytes;  // 16 KiB
constexpr int kMaxTokens = 128;              // tokens per segment (one tile)
constexpr int kMaxSlices = 4;
constexpr int kMaxRank = 64;
constexpr int kShrinkStages = 4;
constexpr int kShrinkThreads = 160;          // 4 producer/epilogue warps + 1 MMA warp
constexpr int kNT = 128;                     // expand columns per unit (UMMA N)
constexpr int kBTileBytes = kNT * kRowBytes; // 16 KiB
constexpr int kYTileBytes = kTileM * kNT * 2;  // 32 KiB: two boxes of 128 rows x 64 columns
constexpr int kExpandThreads = 384;          // 8 epilogue, producer, 2 z, MMA warps
constexpr int kPartLen = 1024;               // K elements per shrink part, at least
constexpr int kMaxParts = 3;                 // K parts of a call, at most
constexpr int kEStages = 3;                  // expand B / y tile ring
constexpr int kIdentBytes = 64 * kRowBytes;  // 64 x 64 BF16 identity, K-major, 128-B swizzle

enum Numerics { kFp32 = 0, kReference = 1 };

struct PParams {
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
  float* partial;     // [kparts][T][rpad]: each K part's FP32 z rows (row = permuted position)
  int T, K, N, S, cap, num_slots, max_segments;
  int rpad;      // shrink UMMA N: S*min(cap, 64) rounded up to 16 (<= 256)
  int kparts;    // most K parts of a call (partial tables in the workspace)
  int shrink_ctas;  // CTAs of the shrink grid
  int numerics;  // kFp32 or kReference
  int y_mode;    // bit 0: y 16-byte aligned with stride a multiple of 8; bit 1: tmap_y valid
  CUtensorMap tmap_x[5];  // x as 2-D [T rows, K], boxes of 64 columns x 128 / 64 / 32 / 16 / 8 rows
  CUtensorMap tmap_a;  // A as 2-D [slots*S*cap rows, K], boxes of rpad rows x 64 columns
  // The compact B buffer as 2-D [rows, bucket] for bucket 16 / 32 / 64 ([0] / [1] / [2]),
  // boxes of 128 ([.][0]) or 16 ([.][1]) rows, swizzled by the row's size (32 / 64 / 128
  // bytes), so a box lands in the UMMA K-major layout of that bucket.  The row extent is
  // nominal (kBRowsNominal): loads address only the rows of a slot's region, as the
  // cp.async path does.
  CUtensorMap tmap_b[3][2];
  // y as 2-D [T rows, N], boxes of 64 columns x 128 / 64 / 32 / 16 / 8 rows, 128-B swizzle
  // (the expand's tile loads of one run of tokens).
  CUtensorMap tmap_y[5];
};

constexpr int64_t kBRowsNominal = (int64_t(1) << 31) - 1;

struct PSeg {
  int ok, g, n, r, bucket, pos0;
  float scale;
  int64_t boff;
};

__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_launch_dependents() {
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}

__device__ __forceinline__ int segment_total(const PParams& p) {
  const int n = *p.seg_count;
  return max(0, min(n, min(p.max_segments, p.T)));
}

// K split of the shrink: enough parts for the segments to fill the shrink grid in one
// wave (at most kMaxParts, and parts of at least kPartLen), each a multiple of 64 long
// and none empty.  The expand sums the parts' partial z rows in part order.
struct KSplit {
  int parts, len;
};
__device__ __forceinline__ KSplit k_split(const PParams& p, int nseg) {
  const int want = max(1, min(p.kparts, p.shrink_ctas / max(1, nseg)));
  const int len = ((p.K + want - 1) / want + 63) / 64 * 64;
  return KSplit{(p.K + len - 1) / len, len};
}

// Box height (index into the x / y maps: 128, 64, 32, 16, 8 rows) covering n rows.
__device__ __forceinline__ int box_rows_index(int n) {
  return n > 64 ? 0 : n > 32 ? 1 : n > 16 ? 2 : n > 8 ? 3 : 4;
}

// Segment metadata; ok only for segments of 1..128 tokens whose slot, rank, bucket and
// B offset are inside the contract (others are skipped by every role).
__device__ __forceinline__ PSeg prefill_segment(const PParams& p, int seg) {
  PSeg s{};
  const int lo = p.indptr[seg], hi = p.indptr[seg + 1];
  s.pos0 = lo;
  s.n = hi - lo;
  s.g = p.seg_slots[seg];
  bool ok = lo >= 0 && hi <= p.T && s.n >= 1 && s.n <= kMaxTokens && s.g >= 0 &&
            s.g < p.num_slots;
  if (ok) {
    s.r = p.ranks[s.g];
    s.bucket = p.b_strides[s.g];
    s.scale = p.scales[s.g];
    s.boff = p.b_offsets[s.g];
    ok = s.r >= 1 && s.r <= kMaxRank && s.r <= p.cap && s.bucket >= 1 && s.bucket <= kMaxRank &&
         (s.bucket & (s.bucket - 1)) == 0 && s.boff >= 0 && (s.boff & 7) == 0;
  }
  s.ok = ok ? 1 : 0;
  return s;
}

// 128 producer/epilogue threads of the shrink: true if any of them passed `v` (barrier 2).
__device__ __forceinline__ bool any128(bool v) {
  uint32_t r;
  asm volatile(
      "{\n .reg .pred p, q;\n setp.ne.u32 p, %1, 0;\n bar.red.or.pred q, 2, 128, p;\n"
      " selp.u32 %0, 1, 0, q;\n}\n"
      : "=r"(r)
      : "r"(v ? 1u : 0u)
      : "memory");
  return r != 0;
}

__device__ __forceinline__ uint32_t pack_bf16(float lo, float hi) {
  return (float_to_bf16_bits(lo) & 0xffffu) | (float_to_bf16_bits(hi) << 16);
}

// Round-to-nearest-even FP32 pair -> packed BF16 pair in one hardware conversion
// (`first` in the low half); identical to pack_bf16 for finite values.
__device__ __forceinline__ uint32_t cvt_bf16x2(float first, float second) {
  uint32_t r;
  asm("cvt.rn.bf16x2.f32 %0, %1, %2;" : "=r"(r) : "f"(second), "f"(first));
  return r;
}

// ====================================================================== shrink
// Stage: x tile (128 rows) then A tile (rpad rows), both K-major with 128-byte rows and
// 128-byte swizzle.  A arrives as one 2-D TMA box; x too when the chunk's tokens are one
// contiguous run of rows (the usual prefill case), else each producer thread gathers its
// row with cp.async.  The stage's "full" barrier takes 129 arrivals: thread 0's
// expect-tx arrive for the TMA bytes and one arrive per producer thread once its own
// copies (if any) have landed and been made visible to the tensor cores' proxy.
// Two CTAs per SM: their ten warps put three on some SM sub-partition (16 K registers
// each), so a thread may hold at most 168 registers.
__global__ void __maxnreg__(168) prefill_shrink_kernel(const __grid_constant__ PParams p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = align1024(smem_raw);
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int SB = kXTileBytes + p.rpad * kRowBytes;
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + kShrinkStages * SB);
  uint64_t* empty = full + kShrinkStages;
  uint64_t* acc_full = empty + kShrinkStages;
  uint64_t* acc_empty = acc_full + 1;
  uint64_t* fin = acc_empty + 1;  // the MMA thread's last commit (all MMAs retired)
  uint32_t* tslot = reinterpret_cast<uint32_t*>(fin + 1);
  volatile int* abort = reinterpret_cast<volatile int*>(tslot + 2);
  const uint32_t tcols = p.rpad <= 32 ? 32u : (p.rpad <= 64 ? 64u : (p.rpad <= 128 ? 128u : 256u));

  if (tid == 0) {
    for (int s = 0; s < kShrinkStages; ++s) {
      mbar_init(&full[s], kTileM + 1);
      mbar_init(&empty[s], 1);
    }
    mbar_init(acc_full, 1);
    mbar_init(acc_empty, kTileM);
    mbar_init(fin, 1);
    fence_mbar_init();
    *abort = 0;
  }
  if (warp == 4) tc_alloc(tslot, tcols);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tslot;
  pdl_wait();
  pdl_launch_dependents();  // only after this CTA holds its TMEM columns

  const KSplit ks = k_split(p, segment_total(p));
  const int total = segment_total(p) * ks.parts;
  if (warp < 4) {
    // ------------------------------------------- producers, then epilogue, per unit
    const int row = tid;  // tile row == TMEM lane
    int sidx = 0;         // stage uses so far (ring position)
    int units = 0;
    for (int u = blockIdx.x; u < total; u += gridDim.x) {
      const int seg = u / ks.parts, kp = u - seg * ks.parts;
      const PSeg si = prefill_segment(p, seg);
      if (!si.ok) continue;
      if (any128(*abort)) break;  // an expired wait: stop together (barriers below)
      const int k0 = kp * ks.len;
      const int kend = min(p.K, k0 + ks.len);
      const int nsteps = (kend - k0 + 63) / 64;
      int tok = -1;
      if (row < si.n) {
        tok = p.perm[si.pos0 + row];
        if (tok < 0 || tok >= p.T) tok = -1;
      }
      // token_indices is ascending inside a slot's group: equal spans mean one run.
      const int first = p.perm[si.pos0], last = p.perm[si.pos0 + si.n - 1];
      const bool run = first >= 0 && last < p.T && last - first == si.n - 1;
      const uint16_t* xrow = tok >= 0 ? p.x + int64_t(tok) * p.x_stride : p.x;
      const int arow0 = si.g * p.S * p.cap;
      int pend0 = -1, pend1 = -1;
      for (int s = 0; s < nsteps; ++s, ++sidx) {
        const int stage = sidx % kShrinkStages;
        const uint32_t phase = uint32_t(sidx / kShrinkStages) & 1u;
        wait_or_abort(&empty[stage], phase ^ 1u, abort);
        const uint32_t st = smem_u32(smem + stage * SB);
        const int kk = k0 + s * 64;
        if (tid == 0) {
          // x: a box of the smallest height covering the segment's rows (the rows past it
          // feed accumulator rows that are never stored).
          const int h = box_rows_index(si.n);
          mbar_arrive_expect_tx(&full[stage], uint32_t(p.rpad * kRowBytes + (run ? (kTileM >> h) * kRowBytes : 0)));
          tma_load_2d(st + kXTileBytes, &p.tmap_a, kk, arow0, &full[stage]);
          if (run) tma_load_2d(st, &p.tmap_x[h], kk, first, &full[stage]);
        }
        if (run) {
          mbar_arrive(&full[stage]);
          continue;
        }
#pragma unroll
        for (int c = 0; c < 8; ++c) {
          const int kc = kk + 8 * c;
          const bool v = tok >= 0 && kc < kend;
          cp16(st + swz(row, c), v ? static_cast<const void*>(xrow + kc) : p.x, v ? 16u : 0u);
        }
        cp_commit();
        // Arrive for a gathered stage two steps later, once its copies have landed and
        // are visible to the tensor cores' (async) proxy.
        if (pend1 >= 0) {
          cp_wait<2>();
          fence_async_smem();
          mbar_arrive(&full[pend0]);
          pend0 = pend1;
          pend1 = stage;
        } else if (pend0 >= 0) {
          pend1 = stage;
        } else {
          pend0 = stage;
        }
      }
      if (!run) {
        cp_wait<0>();
        fence_async_smem();
        if (pend0 >= 0) mbar_arrive(&full[pend0]);
        if (pend1 >= 0) mbar_arrive(&full[pend1]);
      }

      // Epilogue: accumulator rows -> this K part's partial.
      wait_or_abort(acc_full, uint32_t(units) & 1u, abort);
      ++units;
      tc_fence_after();
      const uint32_t tbase = tmem + (uint32_t(warp * 32) << 16);
      float* prow = p.partial + (int64_t(kp) * p.T + si.pos0 + row) * p.rpad;
      for (int c0 = 0; c0 < p.rpad; c0 += 16) {
        uint32_t v[16];
        tc_ld16(tbase + c0, v);
        if (row < si.n) {
#pragma unroll
          for (int j = 0; j < 16; j += 4)
            *reinterpret_cast<float4*>(prow + c0 + j) =
                make_float4(__uint_as_float(v[j]), __uint_as_float(v[j + 1]), __uint_as_float(v[j + 2]),
                            __uint_as_float(v[j + 3]));
        }
      }
      tc_fence_before();
      mbar_arrive(acc_empty);
    }
    // No box may still be landing when the CTA exits (the normal path has consumed every
    // stage already; after an expired wait this waits, bounded, for the last ones).
    if (tid == 0)
      for (int j = max(0, sidx - kShrinkStages); j < sidx; ++j)
        mbar_wait(&full[j % kShrinkStages], uint32_t(j / kShrinkStages) & 1u);
  } else if (warp == 4 && lane == 0) {
    // ------------------------------------------------------------ MMA thread
    const uint32_t idesc = idesc_bf16(kTileM, p.rpad);
    int sidx = 0, units = 0;
    for (int u = blockIdx.x; u < total; u += gridDim.x) {
      const int seg = u / ks.parts, kp = u - seg * ks.parts;
      const PSeg si = prefill_segment(p, seg);
      if (!si.ok) continue;
      if (*abort) break;
      const int k0 = kp * ks.len;
      const int nsteps = (min(p.K, k0 + ks.len) - k0 + 63) / 64;
      if (units > 0) wait_or_abort(acc_empty, uint32_t(units - 1) & 1u, abort);
      tc_fence_after();
      for (int s = 0; s < nsteps; ++s, ++sidx) {
        const int stage = sidx % kShrinkStages;
        wait_or_abort(&full[stage], uint32_t(sidx / kShrinkStages) & 1u, abort);
        tc_fence_after();
        const uint32_t st = smem_u32(smem + stage * SB);
        const uint64_t ad = sw128_desc(st), bd = sw128_desc(st + kXTileBytes);
#pragma unroll
        for (int k = 0; k < 4; ++k) tc_mma(tmem, ad + 2 * k, bd + 2 * k, idesc, (s > 0 || k > 0) ? 1u : 0u);
        tc_commit(&empty[stage]);
      }
      tc_commit(acc_full);
      ++units;
    }
    // Every MMA has retired before the TMEM columns are released.
    tc_commit(fin);
    mbar_wait(fin, 0);
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 4) {
    tc_fence_after();
    tc_dealloc(tmem, tcols);
  }
}

// ====================================================================== expand
// Unit u of a CTA: segment u / nb, block u % nb, where a segment's nb blocks cover every
// slice in 128-column pieces (no block straddles two slices).
struct Block {
  int slice, c0, width;  // slice, first column inside the slice, slice width
};

__device__ __forceinline__ Block block_of(const int* offs, int S, int b) {
  Block k{0, 0, 0};
  for (int s = 0; s < S; ++s) {
    const int w = offs[s + 1] - offs[s];
    const int nb = (w + kNT - 1) / kNT;
    if (b < nb) {
      k.slice = s;
      k.c0 = b * kNT;
      k.width = w;
      return k;
    }
    b -= nb;
  }
  k.slice = -1;
  return k;
}

// Bucket of a segment's B rows when they are loaded by TMA boxes (16, 32 or 64: rows of
// 32 / 64 / 128 bytes, B offset a whole number of rows, row coordinates inside int32),
// else 0: rows zero-padded to 64 elements and staged with cp.async.
__device__ __forceinline__ int b_box_bucket(const PSeg& s, const PParams& p) {
  const bool sized = s.bucket == 16 || s.bucket == 32 || s.bucket == 64;
  return sized && s.boff % s.bucket == 0 && s.boff / s.bucket + p.N <= kBRowsNominal ? s.bucket : 0;
}

// How a unit's y rows come in.  kYTma: the segment's tokens are one run (token_indices
// is ascending inside a slot's group, so equal spans mean a run) and y has tensor maps:
// TMA boxes.  kYGather: rows gathered through token_indices, or no tensor maps:
// coalesced cp.async.  Both stage the tile in shared memory, from where the epilogue
// stores it back coalesced, and need 16-byte aligned rows and a block that starts on a
// multiple of 8 columns; kYDirect (otherwise): the epilogue threads read and write their
// rows in global memory.
enum YMode { kYDirect = 0, kYGather = 1, kYTma = 2 };
struct YUnit {
  int mode, tok0;  // tok0: first token of a run, else -1
};
__device__ __forceinline__ YUnit y_unit(const PParams& p, int run, int gcol0) {
  YUnit r{kYDirect, -1};
  if (!(p.y_mode & 1) || (gcol0 & 7)) return r;
  r.mode = run >= 0 && (p.y_mode & 2) ? kYTma : kYGather;
  r.tok0 = run;
  return r;
}

// Segment metadata of a role's current unit, looked up again only when the segment
// changes (a CTA's units are consecutive blocks, mostly of one segment).  run: the first
// token when the segment's rows are one run of tokens, else -1.
struct SegCache {
  int seg = -1, run = -1;
  int kb = 0, brow = 0;  // b_box_bucket and the slot's first B row in bucket-wide rows
  PSeg si{};
  __device__ __forceinline__ const PSeg& get(const PParams& p, int s) {
    if (s != seg) {
      seg = s;
      si = prefill_segment(p, s);
      run = -1;
      kb = brow = 0;
      if (si.ok) {
        const int first = p.perm[si.pos0], last = p.perm[si.pos0 + si.n - 1];
        if (first >= 0 && last < p.T && last - first == si.n - 1) run = first;
        kb = b_box_bucket(si, p);
        if (kb) brow = int(si.boff / kb);
      }
    }
    return si;
  }
};

// Token of row m of a segment (-1 when token_indices holds an invalid entry).
__device__ __forceinline__ int row_token(const PParams& p, const PSeg& si, const YUnit& yu, int m) {
  if (yu.tok0 >= 0) return yu.tok0 + m;
  const int t = p.perm[si.pos0 + m];
  return t >= 0 && t < p.T ? t : -1;
}

// y + delta for 8 columns: old y (BF16 x 8) and 8 FP32 accumulator values.
template <int MODE>
__device__ __forceinline__ uint4 y_update(uint4 o, const uint32_t* d, float scale) {
  const uint32_t ow[4] = {o.x, o.y, o.z, o.w};
  uint32_t nw[4];
#pragma unroll
  for (int e = 0; e < 4; ++e) {
    const float d0 = __uint_as_float(d[2 * e]), d1 = __uint_as_float(d[2 * e + 1]);
    const float y0 = __uint_as_float(ow[e] << 16), y1 = __uint_as_float(ow[e] & 0xffff0000u);
    const float v0 = MODE == kFp32 ? y0 + d0 : y0 + round_through_bf16(d0 * scale);
    const float v1 = MODE == kFp32 ? y1 + d1 : y1 + round_through_bf16(d1 * scale);
    nw[e] = cvt_bf16x2(v0, v1);
  }
  return make_uint4(nw[0], nw[1], nw[2], nw[3]);
}

// Warp roles: 0-7 epilogue (TMEM lane quarter = warp & 3, 64-column half = warp >> 2;
// they also store the updated y tile), 8 producer (B and y tiles), 9-10 z tiles, 11 MMA
// thread (and the TMEM allocation).  Rings: B / y tiles in kEStages stages, z tiles and
// TMEM accumulators (128 columns each) in 2.
template <int MODE>
__global__ void __launch_bounds__(kExpandThreads, 1) prefill_expand_kernel(const __grid_constant__ PParams p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = align1024(smem_raw);
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  uint8_t* ytile = smem;                               // kEStages x 32 KiB (two 64-column boxes)
  uint8_t* btile = ytile + kEStages * kYTileBytes;     // kEStages x 16 KiB
  uint8_t* ztile = btile + kEStages * kBTileBytes;     // 2 buffers x (hi, lo) x 16 KiB
  uint8_t* ident = ztile + 4 * kXTileBytes;  // 64 x 64 BF16 identity (FP32 numerics: adds y)
  uint64_t* b_full = reinterpret_cast<uint64_t*>(ident + kIdentBytes);
  uint64_t* b_empty = b_full + kEStages;
  uint64_t* y_full = b_empty + kEStages;
  uint64_t* y_done = y_full + kEStages;   // every epilogue thread has updated its rows
  uint64_t* y_empty = y_done + kEStages;  // ... and stored its share of the tile
  uint64_t* z_full = y_empty + kEStages;
  uint64_t* z_empty = z_full + 2;
  uint64_t* t_full = z_empty + 2;
  uint64_t* t_empty = t_full + 2;
  uint64_t* fin = t_empty + 2;  // the MMA thread's last commit (all MMAs retired)
  uint32_t* tslot = reinterpret_cast<uint32_t*>(fin + 1);
  int* offs = reinterpret_cast<int*>(tslot + 4);
  volatile int* abort = reinterpret_cast<volatile int*>(offs + kMaxSlices + 2);
  int* tokrow = reinterpret_cast<int*>(reinterpret_cast<uint8_t*>(b_full) + 320);  // kEStages x 128 row tokens
  constexpr int kEpi = 256, kZ = 64;

  if (tid == 0) {
    for (int i = 0; i < kEStages; ++i) {
      mbar_init(&b_full[i], 32);  // the producer warp (lane 0 also expects the boxes' bytes)
      mbar_init(&b_empty[i], 1);
      mbar_init(&y_full[i], 32);  // the producer warp (lane 0 also expects the boxes' bytes)
      mbar_init(&y_done[i], kEpi);
      mbar_init(&y_empty[i], kEpi);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&z_full[i], kZ);
      mbar_init(&z_empty[i], 1);
      mbar_init(&t_full[i], 1);
      mbar_init(&t_empty[i], kEpi);
    }
    mbar_init(fin, 1);
    fence_mbar_init();
    *abort = 0;
  }
  if (tid <= p.S) offs[tid] = p.slice_offsets[tid];
  if (MODE == kFp32) {
    // Row n holds 1.0 at column n: y box j (128 tokens x 64 columns) times it adds y to
    // the accumulator's columns 64j..64j+63.
    for (int i = tid; i < 64 * 8; i += kExpandThreads) {
      const int r = i >> 3, c = i & 7;
      uint32_t w[4] = {0u, 0u, 0u, 0u};
      if ((r >> 3) == c) w[(r & 7) >> 1] = 0x3F80u << (16 * (r & 1));
      sts16(smem_u32(ident) + swz(r, c), make_uint4(w[0], w[1], w[2], w[3]));
    }
    fence_async_smem();
  }
  if (warp == 11) tc_alloc(tslot, 2 * kNT);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tslot;
  pdl_launch_dependents();  // only after this CTA holds its TMEM columns

  const int nseg = segment_total(p);
  const KSplit ks = k_split(p, nseg);  // the shrink's partial z tables
  int nb = 0;
  for (int s = 0; s < p.S; ++s) nb += (offs[s + 1] - offs[s] + kNT - 1) / kNT;
  const int total = nseg * nb;
  const int per = (total + int(gridDim.x) - 1) / int(gridDim.x);
  const int u0 = min(total, int(blockIdx.x) * per), u1 = min(total, u0 + per);

  if (warp == 8) {
    // ------------------------------------------------------------ producer
    // y tile: boxes of 128 token rows x 64 columns (rows past the segment and columns past
    // the slice are read but never stored; past the tensor they read as zero).  B rows:
    // buckets 16 / 32 / 64 in TMA boxes of 128 and 16 rows in the bucket's own swizzled
    // layout, cp.async for the last rows under 16; rows past the slice are left as they
    // are (they only feed accumulator columns nobody stores).  Other buckets and offsets:
    // every row zero-padded to 64 elements through cp.async.
    int it = 0, pend = -1;
    bool pend_b = false, pend_y = false;
    SegCache sc;
    for (int u = u0; u < u1; ++u) {
      const int seg = u / nb;
      const Block blk = block_of(offs, p.S, u - seg * nb);
      const PSeg& si = sc.get(p, seg);
      if (!si.ok || blk.slice < 0) continue;
      if (*abort) break;
      const int s = it % kEStages;
      const uint32_t ph = (uint32_t(it / kEStages) & 1u) ^ 1u;
      if (!wait_or_abort(&b_empty[s], ph, abort) || !wait_or_abort(&y_empty[s], ph, abort)) break;
      ++it;
      const int gcol0 = offs[blk.slice] + blk.c0;
      const int cols = min(kNT, blk.width - blk.c0);
      const YUnit yu = y_unit(p, sc.run, gcol0);
      const uint32_t yt = smem_u32(ytile + s * kYTileBytes);
      int* trow = tokrow + s * kTileM;
      if (yu.mode != kYDirect) {
        // The rows' tokens, for the copies below and the epilogue's stores (all four
        // loads of a lane are issued before any is used).
        int tk[4];
#pragma unroll
        for (int q = 0; q < 4; ++q) tk[q] = lane + 32 * q < si.n ? row_token(p, si, yu, lane + 32 * q) : -1;
#pragma unroll
        for (int q = 0; q < 4; ++q)
          if (lane + 32 * q < si.n) trow[lane + 32 * q] = tk[q];
        __syncwarp();
      }
      if (yu.mode == kYTma && lane == 0) {
        // Boxes of the smallest height of 128 / 64 / 32 / 16 / 8 rows that covers the
        // segment; expected bytes before any box can complete.
        const int h = box_rows_index(si.n);
        const int nbox = (cols + 63) >> 6;
        mbar_expect_tx(&y_full[s], uint32_t(nbox * (kTileM >> h) * kRowBytes));
        for (int j = 0; j < nbox; ++j)
          tma_load_2d(yt + uint32_t(j * kXTileBytes), &p.tmap_y[h], gcol0 + 64 * j, yu.tok0, &y_full[s]);
      }
      const bool ycp = yu.mode == kYGather;  // the y tile has cp.async copies
      if (ycp) {
        // Row m, 16-byte chunk cc of the block's 16 (box cc / 8): four rows per warp step.
        for (int i = lane; i < si.n * 16; i += 32) {
          const int m = i >> 4, cc = i & 15, col = 8 * cc;
          const int tok = trow[m];
          if (col >= cols || tok < 0) continue;
          const int left = p.N - (gcol0 + col);  // columns of y's row from here (> 0)
          cp16(yt + uint32_t((cc >> 3) * kXTileBytes) + swz(m, cc & 7), p.y + int64_t(tok) * p.y_stride + gcol0 + col,
               left >= 8 ? 16u : uint32_t(2 * left));
        }
      }
      const uint32_t bt = smem_u32(btile + s * kBTileBytes);
      const int kb = sc.kb;
      bool staged = true;  // the B tile has cp.async copies
      if (kb) {
        const int rb = 2 * kb, cpr = rb >> 4;
        const int n128 = cols >> 7, n16 = (cols & 127) >> 4, boxed = cols & ~15;
        const int row0 = sc.brow + gcol0;
        const int m = kb == 16 ? 0 : kb == 32 ? 1 : 2;
        if (lane == 0 && boxed > 0) {
          // Expected bytes before any box can complete; this lane arrives afterwards.
          mbar_expect_tx(&b_full[s], uint32_t(boxed * rb));
          for (int i = 0; i < n128; ++i)
            tma_load_2d(bt + uint32_t(128 * i * rb), &p.tmap_b[m][0], 0, row0 + 128 * i, &b_full[s]);
          for (int i = 0; i < n16; ++i) {
            const int r = 128 * n128 + 16 * i;
            tma_load_2d(bt + uint32_t(r * rb), &p.tmap_b[m][1], 0, row0 + r, &b_full[s]);
          }
        }
        staged = boxed < cols;
        for (int i = lane; i < (cols - boxed) * cpr; i += 32) {
          const int r = boxed + i / cpr, c = i % cpr;
          cp16(bt + swz_rows(r, c, rb), p.b + si.boff + int64_t(gcol0 + r) * kb + 8 * c, 16u);
        }
      } else {
        for (int i = lane; i < kNT * 8; i += 32) {
          const int r = i >> 3, c = i & 7, k = 8 * c;
          const bool live = r < cols && k < si.bucket;
          const uint16_t* src = p.b + si.boff + int64_t(gcol0 + r) * si.bucket + k;
          if (si.bucket >= 8) {
            cp16(bt + swz(r, c), live ? static_cast<const void*>(src) : p.b, live ? 16u : 0u);
          } else {
            uint32_t w[4] = {0u, 0u, 0u, 0u};
            if (live)
              for (int e = 0; e < si.bucket; ++e) w[e >> 1] |= uint32_t(src[e]) << (16 * (e & 1));
            sts16(bt + swz(r, c), make_uint4(w[0], w[1], w[2], w[3]));
          }
        }
      }
      cp_commit();
      // A tile with cp.async copies is handed over once they have landed (one unit of lag
      // keeps two in flight); a tile of boxes alone at once, since its barrier phase also
      // waits for the boxes' bytes.
      if (pend >= 0) {
        cp_wait<1>();
        fence_async_smem();
        if (pend_b) mbar_arrive(&b_full[pend]);
        if (pend_y) mbar_arrive(&y_full[pend]);
        pend = -1;
      }
      if (!staged) mbar_arrive(&b_full[s]);
      if (!ycp) mbar_arrive(&y_full[s]);
      if (staged || ycp) {
        pend = s;
        pend_b = staged;
        pend_y = ycp;
      }
    }
    if (pend >= 0) {
      cp_wait<0>();
      fence_async_smem();
      if (pend_b) mbar_arrive(&b_full[pend]);
      if (pend_y) mbar_arrive(&y_full[pend]);
    }
    // No box may still be landing when the CTA exits (the normal path has consumed every
    // stage already; after an expired wait this waits, bounded, for the last ones).
    if (lane == 0)
      for (int j = max(0, it - kEStages); j < it; ++j) {
        mbar_wait(&b_full[j % kEStages], uint32_t(j / kEStages) & 1u);
        mbar_wait(&y_full[j % kEStages], uint32_t(j / kEStages) & 1u);
      }
  } else if (warp == 9 || warp == 10) {
    // ------------------------------------------------------------ z tiles
    const int zt = tid - 9 * 32;
    bool waited = false;
    int zcount = 0, key = -1;
    SegCache sc;
    for (int u = u0; u < u1; ++u) {
      const int seg = u / nb;
      const Block blk = block_of(offs, p.S, u - seg * nb);
      const PSeg& si = sc.get(p, seg);
      if (!si.ok || blk.slice < 0) continue;
      if (*abort) break;
      const int k2 = seg * kMaxSlices + blk.slice;
      if (k2 == key) continue;
      key = k2;
      if (!waited) {
        pdl_wait();  // the z rows are written by the preceding shrink grid
        waited = true;
      }
      const int zb = zcount & 1;
      wait_or_abort(&z_empty[zb], (uint32_t(zcount >> 1) & 1u) ^ 1u, abort);
      ++zcount;
      // z = the shrink's partial rows summed in part order (from 0), then BF16 hi + lo of
      // scale * z (FP32 numerics) or bf16(z) (reference), zero beyond min(rank, bucket) and
      // past the segment's rows; 8 elements per item, four items per pass with every
      // part's loads of all four issued before any sum.
      const uint32_t zh = smem_u32(ztile + zb * 2 * kXTileBytes), zl = zh + kXTileBytes;
      const int live = min(si.r, si.bucket);
      const float mul = MODE == kFp32 ? si.scale : 1.f;
      const int col0 = blk.slice * si.r;
      const bool vec = (col0 & 3) == 0;
      const int64_t part_stride = int64_t(p.T) * p.rpad;
      constexpr int kItems = 4;
      for (int i0 = zt; i0 < kTileM * 8; i0 += kItems * kZ) {
        float v[kItems][8];
        float4 ld[kItems][kMaxParts][2];
#pragma unroll
        for (int q = 0; q < kItems; ++q) {
          const int i = i0 + q * kZ, m = i >> 3, c = i & 7;
          const float* src = p.partial + int64_t(si.pos0 + m) * p.rpad + col0 + 8 * c;
          const bool full8 = i < kTileM * 8 && m < si.n && vec && 8 * c + 8 <= live;
#pragma unroll
          for (int pp = 0; pp < kMaxParts; ++pp) {
            if (full8 && pp < ks.parts) {
              ld[q][pp][0] = __ldcg(reinterpret_cast<const float4*>(src + pp * part_stride));
              ld[q][pp][1] = __ldcg(reinterpret_cast<const float4*>(src + pp * part_stride) + 1);
            }
          }
        }
#pragma unroll
        for (int q = 0; q < kItems; ++q) {
          const int i = i0 + q * kZ, m = i >> 3, c = i & 7;
          const float* src = p.partial + int64_t(si.pos0 + m) * p.rpad + col0 + 8 * c;
          const bool full8 = i < kTileM * 8 && m < si.n && vec && 8 * c + 8 <= live;
#pragma unroll
          for (int e = 0; e < 8; ++e) v[q][e] = 0.f;
          if (full8) {
#pragma unroll
            for (int pp = 0; pp < kMaxParts; ++pp) {
              if (pp < ks.parts) {
                v[q][0] += ld[q][pp][0].x; v[q][1] += ld[q][pp][0].y; v[q][2] += ld[q][pp][0].z; v[q][3] += ld[q][pp][0].w;
                v[q][4] += ld[q][pp][1].x; v[q][5] += ld[q][pp][1].y; v[q][6] += ld[q][pp][1].z; v[q][7] += ld[q][pp][1].w;
              }
            }
          } else if (i < kTileM * 8 && m < si.n) {
            for (int e = 0; e < 8 && 8 * c + e < live; ++e)
              for (int pp = 0; pp < ks.parts; ++pp) v[q][e] += __ldcg(src + pp * part_stride + e);
          }
        }
#pragma unroll
        for (int q = 0; q < kItems; ++q) {
          const int i = i0 + q * kZ, m = i >> 3, c = i & 7;
          if (i >= kTileM * 8) break;
          uint32_t hw[4], lw[4];
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            const float v0 = mul * v[q][2 * e], v1 = mul * v[q][2 * e + 1];
            hw[e] = cvt_bf16x2(v0, v1);
            const float h0 = __uint_as_float(hw[e] << 16), h1 = __uint_as_float(hw[e] & 0xffff0000u);
            lw[e] = cvt_bf16x2(v0 - h0, v1 - h1);
          }
          sts16(zh + swz(m, c), make_uint4(hw[0], hw[1], hw[2], hw[3]));
          if (MODE == kFp32) sts16(zl + swz(m, c), make_uint4(lw[0], lw[1], lw[2], lw[3]));
        }
      }
      fence_async_smem();
      mbar_arrive(&z_full[zb]);
    }
    // Every CTA waits for the shrink grid, so this grid's completion implies the shrink's.
    if (!waited) pdl_wait();
  } else if (warp == 11) {
    // ------------------------------------------------------------ MMA thread
    if (lane == 0) {
      const uint32_t idesc = idesc_bf16(kTileM, kNT), idesc64 = idesc_bf16(kTileM, 64);
      int it = 0, zcount = 0, tcount = 0, key = -1, zb = 0;
      SegCache sc;
      for (int u = u0; u < u1; ++u) {
        const int seg = u / nb;
        const Block blk = block_of(offs, p.S, u - seg * nb);
        const PSeg& si = sc.get(p, seg);
        if (!si.ok || blk.slice < 0) continue;
        if (*abort) break;
        const int k2 = seg * kMaxSlices + blk.slice;
        if (k2 != key) {
          if (key >= 0) tc_commit(&z_empty[zb]);  // the previous z tile is free once read
          key = k2;
          zb = zcount & 1;
          wait_or_abort(&z_full[zb], uint32_t(zcount >> 1) & 1u, abort);
          ++zcount;
        }
        const int s = it % kEStages;
        const uint32_t sph = uint32_t(it / kEStages) & 1u;
        wait_or_abort(&b_full[s], sph, abort);
        ++it;
        // FP32 numerics with the y tile in shared memory: the tensor cores add y too.
        const bool add_y = MODE == kFp32 && y_unit(p, sc.run, offs[blk.slice] + blk.c0).mode != kYDirect;
        if (add_y) wait_or_abort(&y_full[s], sph, abort);
        const int tb = tcount & 1;
        wait_or_abort(&t_empty[tb], (uint32_t(tcount >> 1) & 1u) ^ 1u, abort);
        ++tcount;
        if (*abort) break;
        tc_fence_after();
        const uint32_t d = tmem + uint32_t(tb * kNT);
        const uint32_t zh = smem_u32(ztile + zb * 2 * kXTileBytes);
        // K steps of 16: the bucket's (boxed B rows) or 4 (rows padded to 64).
        const int kb = sc.kb, ksteps = kb ? kb >> 4 : 4;
        const uint32_t bsa = smem_u32(btile + s * kBTileBytes);
        const uint64_t bd = kb ? swrow_desc(bsa, 2 * kb) : sw128_desc(bsa);
        const uint64_t ah = sw128_desc(zh), al = sw128_desc(zh + kXTileBytes);
#pragma unroll
        for (int k = 0; k < 4; ++k)
          if (k < ksteps) tc_mma(d, ah + 2 * k, bd + 2 * k, idesc, k > 0 ? 1u : 0u);
        if (MODE == kFp32) {
#pragma unroll
          for (int k = 0; k < 4; ++k)
            if (k < ksteps) tc_mma(d, al + 2 * k, bd + 2 * k, idesc, 1u);
        }
        if (add_y) {
          // D[:, 64j + n] += sum_k Y_j[:, k] I[n, k]: M = 128, N = 64, K = 64 per box.
          const uint64_t id = sw128_desc(smem_u32(ident));
#pragma unroll
          for (int j = 0; j < 2; ++j) {
            const uint64_t yd = sw128_desc(smem_u32(ytile + s * kYTileBytes + j * kXTileBytes));
#pragma unroll
            for (int k = 0; k < 4; ++k) tc_mma(d + uint32_t(64 * j), yd + 2 * k, id + 2 * k, idesc64, 1u);
          }
        }
        tc_commit(&b_empty[s]);
        tc_commit(&t_full[tb]);
      }
      // Every MMA has retired before the TMEM columns are released.
      tc_commit(fin);
      mbar_wait(fin, 0);
    }
  } else {
    // ------------------------------------------------------------ epilogue warps
    const int quarter = warp & 3, half = warp >> 2;
    const int row = quarter * 32 + lane;
    const bool vec_ok = (reinterpret_cast<uintptr_t>(p.y) & 15) == 0 && (p.y_stride & 7) == 0;
    int it = 0, tcount = 0;
    SegCache sc;
    for (int u = u0; u < u1; ++u) {
      const int seg = u / nb;
      const Block blk = block_of(offs, p.S, u - seg * nb);
      const PSeg& si = sc.get(p, seg);
      if (!si.ok || blk.slice < 0) continue;
      const int s = it % kEStages;
      const uint32_t yph = uint32_t(it / kEStages) & 1u;
      ++it;
      const int tb = tcount & 1;
      const uint32_t tph = uint32_t(tcount >> 1) & 1u;
      ++tcount;
      const int gcol0 = offs[blk.slice] + blk.c0;
      const int cl = half * 64;                                // first column of this half
      const int ncols = min(64, min(kNT, blk.width - blk.c0) - cl);  // may be <= 0
      const YUnit yu = y_unit(p, sc.run, gcol0);
      const uint32_t tbase = tmem + (uint32_t(quarter * 32) << 16) + uint32_t(tb * kNT + cl);
      bool ok;
      if (yu.mode != kYDirect) {
        // y tile in shared memory: row `row`, 16-byte chunks 0..7 of box `half`, updated in
        // place.  FP32 numerics: the accumulator already holds y + delta (the MMA thread
        // added the y tile) and only its BF16 rounding goes back.  Reference numerics: the
        // eight old chunks are read before the accumulator is.
        const bool live = row < si.n && ncols > 0;
        const uint32_t ybox = smem_u32(ytile + s * kYTileBytes + half * kXTileBytes);
        if (MODE == kFp32) {
          ok = __all_sync(0xffffffffu, wait_or_abort(&t_full[tb], tph, abort));  // tcgen05.ld is warp-wide
          if (ok) {
            tc_fence_after();
#pragma unroll
            for (int ch = 0; ch < 2; ++ch) {
              uint32_t r[32];
              tc_ld32(tbase + 32 * ch, r);
              if (live) {
#pragma unroll
                for (int i = 0; i < 4; ++i) {
                  const uint32_t* q = r + 8 * i;
                  sts16(ybox + swz(row, 4 * ch + i),
                        make_uint4(cvt_bf16x2(__uint_as_float(q[0]), __uint_as_float(q[1])),
                                   cvt_bf16x2(__uint_as_float(q[2]), __uint_as_float(q[3])),
                                   cvt_bf16x2(__uint_as_float(q[4]), __uint_as_float(q[5])),
                                   cvt_bf16x2(__uint_as_float(q[6]), __uint_as_float(q[7]))));
                }
              }
            }
            fence_async_smem();  // before a later TMA load rewrites the stage
          }
        } else {
          ok = wait_or_abort(&y_full[s], yph, abort);
          uint4 yv[8];
          if (ok && live) {
#pragma unroll
            for (int c = 0; c < 8; ++c) yv[c] = lds16(ybox + swz(row, c));
          }
          ok = wait_or_abort(&t_full[tb], tph, abort) && ok;
          ok = __all_sync(0xffffffffu, ok);  // tcgen05.ld is warp-wide
          if (ok) {
            tc_fence_after();
#pragma unroll
            for (int ch = 0; ch < 2; ++ch) {
              uint32_t r[32];
              tc_ld32(tbase + 32 * ch, r);
              if (live) {
#pragma unroll
                for (int i = 0; i < 4; ++i)
                  sts16(ybox + swz(row, 4 * ch + i), y_update<MODE>(yv[4 * ch + i], r + 8 * i, si.scale));
              }
            }
            fence_async_smem();  // before a later TMA load rewrites the stage
          }
        }
        tc_fence_before();
        mbar_arrive(&t_empty[tb]);
        // Once every row is updated, the tile goes back to y: thread i of 256 stores the
        // 16-byte chunks i, i + 256, ... (rows of 16 chunks, so a warp writes two rows'
        // 256 contiguous bytes per step).
        mbar_arrive(&y_done[s]);
        ok = wait_or_abort(&y_done[s], yph, abort) && ok;
        // Thread tid's chunk column is tid & 15 and its rows (tid >> 4) + 16k; the
        // tokens and the chunks are all read before the first store.
        const int cols = min(kNT, blk.width - blk.c0);
        const int cc = tid & 15, col = 8 * cc;
        bool released = false;
        if (ok && col < cols) {
          const int* trow = tokrow + s * kTileM;
          const uint32_t ysrc = smem_u32(ytile + s * kYTileBytes + (cc >> 3) * kXTileBytes);
          int tk[8];
          uint4 v[8];
#pragma unroll
          for (int k = 0; k < 8; ++k) {
            const int m = (tid >> 4) + 16 * k;
            tk[k] = m < si.n ? trow[m] : -1;
          }
#pragma unroll
          for (int k = 0; k < 8; ++k)
            if (tk[k] >= 0) v[k] = lds16(ysrc + swz((tid >> 4) + 16 * k, cc & 7));
          mbar_arrive(&y_empty[s]);  // the stage is free once its chunks are in registers
          released = true;
#pragma unroll
          for (int k = 0; k < 8; ++k) {
            if (tk[k] < 0) continue;
            uint16_t* dst = p.y + int64_t(tk[k]) * p.y_stride + gcol0 + col;
            if (col + 8 <= cols) {
              *reinterpret_cast<uint4*>(dst) = v[k];
            } else {
              const uint32_t w[4] = {v[k].x, v[k].y, v[k].z, v[k].w};
              for (int e = 0; e < cols - col; ++e) dst[e] = uint16_t(w[e >> 1] >> (16 * (e & 1)));
            }
          }
        }
        if (!released) mbar_arrive(&y_empty[s]);
      } else {
        // Rows gathered through token_indices: old y straight from global memory, fetched
        // before the MMA completes.
        int tok = -1;
        if (row < si.n) {
          tok = p.perm[si.pos0 + row];
          if (tok < 0 || tok >= p.T) tok = -1;
        }
        const int gcol = gcol0 + cl;
        uint16_t* yrow = tok >= 0 && ncols > 0 ? p.y + int64_t(tok) * p.y_stride + gcol : nullptr;
        const bool vec = yrow && ncols == 64 && vec_ok && (gcol & 7) == 0;
        uint4 yv[8];
        if (vec) {
#pragma unroll
          for (int i = 0; i < 8; ++i) yv[i] = *reinterpret_cast<const uint4*>(yrow + 8 * i);
        }
        ok = __all_sync(0xffffffffu, wait_or_abort(&t_full[tb], tph, abort));
        if (ok) {
          tc_fence_after();
#pragma unroll
          for (int ch = 0; ch < 2; ++ch) {
            uint32_t r[32];
            tc_ld32(tbase + 32 * ch, r);
            if (vec) {
#pragma unroll
              for (int i = 0; i < 4; ++i)
                *reinterpret_cast<uint4*>(yrow + 32 * ch + 8 * i) = y_update<MODE>(yv[4 * ch + i], r + 8 * i, si.scale);
            } else if (yrow) {
              for (int j = 0; j < 32; ++j) {
                const int c = 32 * ch + j;
                if (c >= ncols) break;
                const float d = __uint_as_float(r[j]);
                const float y0 = bf16_bits_to_float(yrow[c]);
                const float v = MODE == kFp32 ? y0 + d : y0 + round_through_bf16(d * si.scale);
                yrow[c] = uint16_t(float_to_bf16_bits(v));
              }
            }
          }
        }
      }
      if (yu.mode == kYDirect) {
        // The stage's barriers complete their phase for this unit all the same.
        tc_fence_before();
        mbar_arrive(&t_empty[tb]);
        mbar_arrive(&y_done[s]);
        mbar_arrive(&y_empty[s]);
      }
      if (!ok) break;
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 11) {
    tc_fence_after();
    tc_dealloc(tmem, 2 * kNT);
  }
}

// ====================================================================== z rows by token
// For the base GEMM with the LoRA delta in its mainloop (base_gemm.cu): z_tok[t][c] = the
// shrink's K parts summed in part order (as the expand sums them) for every token of a
// valid segment, c < rpad.  One CTA per segment; CTAs past the live count exit.
__global__ void __launch_bounds__(256) prefill_z_gather_kernel(const __grid_constant__ PParams p, float* z_tok) {
  pdl_wait();  // the partial rows come from the shrink grid
  pdl_launch_dependents();
  const int nseg = segment_total(p);
  const int seg = blockIdx.x;
  if (seg >= nseg) return;
  const PSeg si = prefill_segment(p, seg);
  if (!si.ok) return;
  const KSplit ks = k_split(p, nseg);
  const int64_t part_stride = int64_t(p.T) * p.rpad;
  const int q = p.rpad >> 2;  // float4 per row
  for (int i = threadIdx.x; i < si.n * q; i += blockDim.x) {
    const int m = i / q, c = (i - m * q) * 4;
    const int t = p.perm[si.pos0 + m];
    if (t < 0 || t >= p.T) continue;
    const float* src = p.partial + int64_t(si.pos0 + m) * p.rpad + c;
    float4 sum = make_float4(0.f, 0.f, 0.f, 0.f);
    for (int pp = 0; pp < ks.parts; ++pp) {
      const float4 v = __ldcg(reinterpret_cast<const float4*>(src + pp * part_stride));
      sum.x += v.x;
      sum.y += v.y;
      sum.z += v.z;
      sum.w += v.w;
    }
    *reinterpret_cast<float4*>(z_tok + int64_t(t) * p.rpad + c) = sum;
  }
}

// ====================================================================== host side
struct PrefillLayout {
  int rpad, kparts;
  int64_t partial, total;  // offsets in floats
};

inline PrefillLayout prefill_layout(int64_t tokens, int64_t width, int num_slices, int capacity) {
  PrefillLayout l{};
  const int64_t T = tokens > 0 ? tokens : 1;
  const int cap = capacity < kMaxRank ? capacity : kMaxRank;
  l.rpad = (num_slices * cap + 15) / 16 * 16;
  l.kparts = int((width + kPartLen - 1) / kPartLen);
  l.kparts = l.kparts < kMaxParts ? l.kparts : kMaxParts;
  l.partial = 0;
  l.total = l.partial + int64_t(l.kparts) * T * l.rpad;
  return l;
}

// cuTensorMapEncodeTiled through the runtime's driver entry point (no libcuda link).
inline PFN_cuTensorMapEncodeTiled_v12000 prefill_tensor_map_encoder() {
  static std::mutex mutex;
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  std::lock_guard<std::mutex> lock(mutex);
  if (!fn) {
    void* ptr = nullptr;
    cudaDriverEntryPointQueryResult status;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &ptr, cudaEnableDefault, &status) ==
            cudaSuccess &&
        status == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(ptr);
  }
  return fn;
}

template <typename Kernel, typename... Extra>
int launch_pdl(Kernel kernel, int grid, int block, int smem, cudaStream_t stream, const PParams& p,
               const char* what, Extra... extra) {
  cudaLaunchConfig_t config = {};
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  config.attrs = attr;
  config.numAttrs = 1;
  config.gridDim = dim3(grid);
  config.blockDim = dim3(block);
  config.dynamicSmemBytes = smem;
  config.stream = stream;
  const cudaError_t err = cudaLaunchKernelEx(&config, kernel, p, extra...);
  if (err != cudaSuccess) {
    last_error() = std::string(what) + ": " + cudaGetErrorString(err);
    return LF_E_CUDA;
  }
  return LF_OK;
}

}  // namespace
}  // namespace lfb

namespace lfb {
// This translation unit's expired-wait counter (each unit has its own copy).
int prefill_wait_timeouts(unsigned int* value, int reset) {
  if (cudaMemcpyFromSymbol(value, g_lf_wait_timeouts, sizeof(*value)) != cudaSuccess)
    return check_launch("device_wait_timeouts (prefill)");
  if (reset) {
    const unsigned int zero = 0;
    if (cudaMemcpyToSymbol(g_lf_wait_timeouts, &zero, sizeof(zero)) != cudaSuccess)
      return check_launch("device_wait_timeouts (prefill)");
  }
  return LF_OK;
}
}  // namespace lfb

using namespace lfb;

extern "C" int64_t lf_sgmv_prefill_workspace_floats(int64_t num_tokens, int64_t width,
                                                    int32_t num_slices, int32_t capacity) {
  if (num_tokens < 0 || width < 1 || num_slices < 1 || num_slices > kMaxSlices || capacity < 1)
    return -1;
  return prefill_layout(num_tokens, width, num_slices, capacity).total;
}

namespace lfb {
int prefill_launch(
    const void* x, int64_t x_stride, const void* a, const void* b, const int64_t* b_offsets,
    const int32_t* b_strides, void* y, int64_t y_stride, const int32_t* segment_indptr,
    const int32_t* segment_slots, const int32_t* token_indices, const int32_t* ranks,
    const float* scales, const int32_t* slice_offsets, const int32_t* segment_count,
    float* workspace, int64_t workspace_floats, int64_t num_tokens, int64_t width,
    int32_t out_width, int32_t num_slices, int32_t capacity, int32_t num_slots,
    int32_t max_segments, int32_t numerics, void* stream, float* z_tok) {
  if (num_tokens < 0 || num_tokens >= (int64_t(1) << 31) || width < 1 || width >= (int64_t(1) << 31))
    return fail(LF_E_INVALID, "sgmv_prefill: invalid token count or width");
  if (out_width < 1 || num_slices < 1 || num_slices > kMaxSlices || capacity < 1 || num_slots < 1)
    return fail(LF_E_INVALID, "sgmv_prefill: invalid output width, slices, capacity or slots");
  if (width % 8 || x_stride % 8 || x_stride < width || !aligned16(x) || !aligned16(a) || !aligned16(b))
    return fail(LF_E_INVALID, "sgmv_prefill: x/A/B must be 16-byte aligned with width and stride multiples of 8");
  if ((reinterpret_cast<uintptr_t>(y) & 7) || y_stride % 4 || y_stride < out_width)
    return fail(LF_E_INVALID, "sgmv_prefill: y must be 8-byte aligned with stride a multiple of 4");
  if (numerics != kFp32 && numerics != kReference)
    return fail(LF_E_INVALID, "sgmv_prefill: numerics must be 0 (fp32) or 1 (reference)");
  if (max_segments < 0) return fail(LF_E_INVALID, "sgmv_prefill: negative segment capacity");
  const PrefillLayout l = prefill_layout(num_tokens, width, num_slices, capacity);
  if (!workspace || workspace_floats < l.total || (reinterpret_cast<uintptr_t>(workspace) & 15))
    return fail(LF_E_INVALID, "sgmv_prefill: workspace too small or not 16-byte aligned "
                              "(see lf_sgmv_prefill_workspace_floats)");
  if (num_tokens == 0 || max_segments == 0) return LF_OK;
  int device = 0, sms = 0;
  if (cudaGetDevice(&device) != cudaSuccess ||
      cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, device) != cudaSuccess)
    return check_launch("sgmv_prefill: device query");
  const int64_t T = num_tokens;
  const int64_t seg_cap = max_segments < T ? max_segments : T;
  const int64_t nb_max = (out_width + kNT - 1) / kNT + num_slices;
  if (seg_cap * l.kparts >= (int64_t(1) << 31) || seg_cap * nb_max >= (int64_t(1) << 31))
    return fail(LF_E_INVALID, "sgmv_prefill: too many units");
  PParams p{static_cast<const uint16_t*>(x), x_stride, static_cast<const uint16_t*>(a),
            static_cast<const uint16_t*>(b), b_offsets, b_strides, static_cast<uint16_t*>(y),
            y_stride, segment_indptr, segment_slots, token_indices, ranks, scales, slice_offsets,
            segment_count, workspace + l.partial, int(T), int(width), out_width, num_slices, capacity,
            num_slots, max_segments, l.rpad, l.kparts, 2 * sms, numerics, 0};
  {
    // x [T, K] and A [slots*S*cap, K] as 2-D tensors for the shrink's TMA boxes.
    const PFN_cuTensorMapEncodeTiled_v12000 encode = prefill_tensor_map_encoder();
    if (!encode) return fail(LF_E_CUDA, "sgmv_prefill: cuTensorMapEncodeTiled unavailable");
    const cuuint32_t estr[2] = {1, 1};
    const cuuint64_t xdims[2] = {cuuint64_t(width), cuuint64_t(T)};
    const cuuint64_t xstrides[1] = {cuuint64_t(x_stride) * 2};
    const cuuint64_t adims[2] = {cuuint64_t(width), cuuint64_t(num_slots) * num_slices * capacity};
    const cuuint64_t astrides[1] = {cuuint64_t(width) * 2};
    const cuuint32_t abox[2] = {64, cuuint32_t(l.rpad)};
    CUresult r = CUDA_SUCCESS;
    for (int h = 0; h < 5 && r == CUDA_SUCCESS; ++h) {
      const cuuint32_t xbox[2] = {64u, cuuint32_t(kTileM >> h)};
      r = encode(&p.tmap_x[h], CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(x), xdims, xstrides, xbox,
                 estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                 CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    }
    if (r == CUDA_SUCCESS)
      r = encode(&p.tmap_a, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(a), adims, astrides,
                 abox, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                 CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    // The compact B per bucket 16 / 32 / 64, boxes of 128 and 16 rows.
    for (int m = 0; m < 3 && r == CUDA_SUCCESS; ++m) {
      const int kb = 16 << m;
      const cuuint64_t bdims[2] = {cuuint64_t(kb), cuuint64_t(kBRowsNominal)};
      const cuuint64_t bstrides[1] = {cuuint64_t(kb) * 2};
      const CUtensorMapSwizzle sw =
          m == 0 ? CU_TENSOR_MAP_SWIZZLE_32B : m == 1 ? CU_TENSOR_MAP_SWIZZLE_64B : CU_TENSOR_MAP_SWIZZLE_128B;
      for (int h = 0; h < 2 && r == CUDA_SUCCESS; ++h) {
        const cuuint32_t bbox[2] = {cuuint32_t(kb), h == 0 ? 128u : 16u};
        r = encode(&p.tmap_b[m][h], CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(b), bdims, bstrides,
                   bbox, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, sw, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                   CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
      }
    }
    // y [T, N] for the expand's tile loads and stores, when its layout allows TMA.
    if (aligned16(y) && y_stride % 8 == 0) p.y_mode = 1;
    if (r == CUDA_SUCCESS && p.y_mode && out_width >= 64 && T >= kTileM) {
      const cuuint64_t ydims[2] = {cuuint64_t(out_width), cuuint64_t(T)};
      const cuuint64_t ystrides[1] = {cuuint64_t(y_stride) * 2};
      for (int h = 0; h < 5 && r == CUDA_SUCCESS; ++h) {
        const cuuint32_t ybox[2] = {64u, cuuint32_t(kTileM >> h)};
        r = encode(&p.tmap_y[h], CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, y, ydims, ystrides, ybox, estr,
                   CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                   CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
      }
      p.y_mode |= 2;
    }
    if (r != CUDA_SUCCESS) return fail(LF_E_CUDA, "sgmv_prefill: cuTensorMapEncodeTiled failed");
  }
  const cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (z_tok && cudaMemsetAsync(z_tok, 0, sizeof(float) * size_t(T) * l.rpad, s) != cudaSuccess)
    return check_launch("sgmv_prefill (z by token): cudaMemsetAsync");
  // Shrink (2 CTAs per SM), then expand (1 per SM), all segments on the tensor cores.
  {
    const int smem = kShrinkStages * (kXTileBytes + l.rpad * kRowBytes) + 1024 + 128;
    static int flags[64] = {};
    if (int rc = ensure_smem(prefill_shrink_kernel, smem, flags)) return rc;
    const int64_t units = seg_cap * l.kparts;
    const int grid = int(units < 2 * sms ? units : 2 * sms);
    if (int rc = launch_pdl(prefill_shrink_kernel, grid, kShrinkThreads, smem, s, p,
                            "sgmv_prefill (shrink)"))
      return rc;
  }
  if (z_tok) {
    // Shrink only: the z rows by token for the fused base GEMM (zeroed first, so tokens
    // outside every valid segment carry no LoRA term).
    const int grid = int(seg_cap < 1 ? 1 : seg_cap);
    return launch_pdl(prefill_z_gather_kernel, grid, 256, 0, s, p, "sgmv_prefill (z by token)", z_tok);
  }
  {
    // Tiles and the identity, then 24 barriers, TMEM slot, slice offsets and abort word
    // (< 320 bytes), then the stages' row tokens.
    const int smem =
        kEStages * (kYTileBytes + kBTileBytes) + 4 * kXTileBytes + kIdentBytes + 1024 + 320 + kEStages * kTileM * 4;
    auto kernel = numerics == kFp32 ? prefill_expand_kernel<kFp32> : prefill_expand_kernel<kReference>;
    static int flags[2][64] = {};
    if (int rc = ensure_smem(kernel, smem, flags[numerics])) return rc;
    const int grid = sms;
    if (int rc = launch_pdl(kernel, grid, kExpandThreads, smem, s, p, "sgmv_prefill (expand)")) return rc;
  }
  return LF_OK;
}
}  // namespace lfb

extern "C" int lf_sgmv_prefill(
    const void* x, int64_t x_stride, const void* a, const void* b, const int64_t* b_offsets,
    const int32_t* b_strides, void* y, int64_t y_stride, const int32_t* segment_indptr,
    const int32_t* segment_slots, const int32_t* token_indices, const int32_t* ranks,
    const float* scales, const int32_t* slice_offsets, const int32_t* segment_count,
    float* workspace, int64_t workspace_floats, int64_t num_tokens, int64_t width,
    int32_t out_width, int32_t num_slices, int32_t capacity, int32_t num_slots,
    int32_t max_segments, int32_t numerics, void* stream) {
  return prefill_launch(x, x_stride, a, b, b_offsets, b_strides, y, y_stride, segment_indptr, segment_slots,
                        token_indices, ranks, scales, slice_offsets, segment_count, workspace, workspace_floats,
                        num_tokens, width, out_width, num_slices, capacity, num_slots, max_segments, numerics,
                        stream, nullptr);
}
