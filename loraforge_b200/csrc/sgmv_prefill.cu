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
//                          and stage the compact B rows of the block, zero-padded to 64;
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
#include "tma.cuh"

namespace lfb {
namespace {

constexpr int kTileM = 128;                  // tokens per tile (UMMA M)
constexpr int kRowBytes = 128;               // one swizzled K-major row: 64 BF16
constexpr int kXTileBytes = kTileM * kRowBytes;  // 16 KiB
constexpr int kMaxTokens = 128;              // tokens per segment (one tile)
constexpr int kMaxSlices = 4;
constexpr int kMaxRank = 64;
constexpr int kShrinkStages = 4;
constexpr int kShrinkThreads = 160;          // 4 producer/epilogue warps + 1 MMA warp
constexpr int kNT = 256;                     // expand columns per unit (UMMA N)
constexpr int kBTileBytes = kNT * kRowBytes; // 32 KiB
constexpr int kExpandThreads = 352;          // 8 epilogue, 2 producer, 1 MMA warp
constexpr int kPartLen = 1024;               // K elements per shrink part
constexpr int kBStages = 3;                  // expand B-tile ring

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
  float* partial;     // [kparts][T][rpad]
  float* zfinal;      // [T][rpad]: z of each token (row = permuted position)
  int* counters;      // [T], zero between calls
  int T, K, N, S, cap, num_slots, max_segments;
  int rpad;      // shrink UMMA N: S*min(cap, 64) rounded up to 16 (<= 256)
  int kparts;    // K parts of kPartLen
  int numerics;  // kFp32 or kReference
  int pad;
  CUtensorMap tmap_x;  // x as 2-D [T rows, K], boxes of 128 rows x 64 columns, 128-B swizzle
  CUtensorMap tmap_a;  // A as 2-D [slots*S*cap rows, K], boxes of rpad rows x 64 columns
};

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

// ------------------------------------------------------------------ tcgen05 wrappers
__device__ __forceinline__ void tc_alloc(uint32_t* slot, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(slot)),
               "r"(ncols)
               : "memory");
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tc_dealloc(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}
__device__ __forceinline__ void tc_fence_before() {
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tc_fence_after() {
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}
// D[tmem] (+)= A[smem desc] . B[smem desc]^T, kind::f16 (BF16 in, FP32 accumulate).
__device__ __forceinline__ void tc_mma(uint32_t d, uint64_t a, uint64_t b, uint32_t idesc,
                                       uint32_t accumulate) {
  asm volatile(
      "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
      " tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n}\n" ::"r"(d),
      "l"(a), "l"(b), "r"(idesc), "r"(accumulate)
      : "memory");
}
// Arrive once on `bar` when every tcgen05 operation this thread issued has completed.
__device__ __forceinline__ void tc_commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
                   smem_u32(bar))
               : "memory");
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

// Bounded mbarrier wait that records an expiry in the CTA's abort word; later waits are
// skipped once the word is set, so a broken pipeline ends in bounded time.
__device__ __forceinline__ bool wait_or_abort(uint64_t* bar, uint32_t parity, volatile int* abort) {
  if (*abort) return false;
  if (mbar_wait(bar, parity)) return true;
  *abort = 1;
  return false;
}

// Thread i of the warp receives TMEM lane (lane field of taddr) + i, 16 / 32 columns;
// the load is waited for inside the same asm block, so the registers are final on exit.
__device__ __forceinline__ void tc_ld16(uint32_t taddr, uint32_t (&r)[16]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];\n"
      "tcgen05.wait::ld.sync.aligned;"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
      : "r"(taddr));
}
__device__ __forceinline__ void tc_ld32(uint32_t taddr, uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
      "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];\n"
      "tcgen05.wait::ld.sync.aligned;"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]),
        "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]),
        "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr));
}

// Shared-memory descriptor of a K-major tile with 128-byte rows, 128-byte swizzle and
// 8-row groups 1024 bytes apart (tile base 1024-byte aligned).  Advancing the start
// address by 32 bytes selects the next 16-element K step.
__device__ __forceinline__ uint64_t sw128_desc(uint32_t saddr) {
  return uint64_t((saddr & 0x3FFFFu) >> 4) | (uint64_t(16 >> 4) << 16) | (uint64_t(1024 >> 4) << 32) |
         (uint64_t(1) << 46) | (uint64_t(2) << 61);
}

// Instruction descriptor, kind::f16: BF16 A and B (K-major), FP32 D, M x N.
__host__ __device__ constexpr uint32_t idesc_bf16(int m, int n) {
  return (1u << 4) | (1u << 7) | (1u << 10) | (uint32_t(n >> 3) << 17) | (uint32_t(m >> 4) << 24);
}

// Byte offset of 16-byte chunk c (elements 8c..8c+7) of row r in a swizzled tile.
__device__ __forceinline__ uint32_t swz(int r, int c) {
  return uint32_t(r) * kRowBytes + (uint32_t((c ^ (r & 7)) & 7) << 4);
}

// 16-byte cp.async; bytes beyond src_bytes (0 or 16 here) are zero-filled.
__device__ __forceinline__ void cp16(uint32_t dst, const void* src, uint32_t src_bytes) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(dst), "l"(src), "r"(src_bytes)
               : "memory");
}
__device__ __forceinline__ void cp_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_wait() {
  asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}
__device__ __forceinline__ void sts16(uint32_t dst, uint4 v) {
  asm volatile("st.shared.v4.b32 [%0], {%1, %2, %3, %4};" ::"r"(dst), "r"(v.x), "r"(v.y), "r"(v.z), "r"(v.w)
               : "memory");
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

__device__ __forceinline__ uint8_t* align1024(uint8_t* p) {
  return p + ((1024u - (smem_u32(p) & 1023u)) & 1023u);
}

// ====================================================================== shrink
__device__ __forceinline__ void tma_load_2d(uint32_t dst, const CUtensorMap* map, int c0, int c1,
                                            uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, "
      "{%2, %3}], [%4];" ::"r"(dst),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(c0), "r"(c1), "r"(smem_u32(bar))
      : "memory");
}

// Stage: x tile (128 rows) then A tile (rpad rows), both K-major with 128-byte rows and
// 128-byte swizzle.  A arrives as one 2-D TMA box; x too when the chunk's tokens are one
// contiguous run of rows (the usual prefill case), else each producer thread gathers its
// row with cp.async.  The stage's "full" barrier takes 129 arrivals: thread 0's
// expect-tx arrive for the TMA bytes and one arrive per producer thread once its own
// copies (if any) have landed and been made visible to the tensor cores' proxy.
__global__ void __launch_bounds__(kShrinkThreads, 1) prefill_shrink_kernel(const __grid_constant__ PParams p) {
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
  int* flag = reinterpret_cast<int*>(tslot + 1);
  volatile int* abort = reinterpret_cast<volatile int*>(flag + 1);
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

  const int total = segment_total(p) * p.kparts;
  if (warp < 4) {
    // ------------------------------------------- producers, then epilogue, per unit
    const int row = tid;  // tile row == TMEM lane
    int sidx = 0;         // stage uses so far (ring position)
    int units = 0;
    for (int u = blockIdx.x; u < total; u += gridDim.x) {
      const int seg = u / p.kparts, kp = u - seg * p.kparts;
      const PSeg si = prefill_segment(p, seg);
      if (!si.ok) continue;
      if (any128(*abort)) break;  // an expired wait: stop together (barriers below)
      const int k0 = kp * kPartLen;
      const int kend = min(p.K, k0 + kPartLen);
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
          mbar_arrive_expect_tx(&full[stage], uint32_t(p.rpad * kRowBytes + (run ? kXTileBytes : 0)));
          tma_load_2d(st + kXTileBytes, &p.tmap_a, kk, arow0, &full[stage]);
          if (run) tma_load_2d(st, &p.tmap_x, kk, first, &full[stage]);
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
      // The CTA that completes the segment's count adds the parts in order into z.
      __threadfence();
      named_barrier(1, kTileM);
      if (tid == 0) {
        const int old = atomicAdd(&p.counters[seg], 1);
        *flag = old == p.kparts - 1 ? 1 : 0;
      }
      named_barrier(1, kTileM);
      if (*flag) {
        __threadfence();
        if (row < si.n) {
          const int64_t pos = si.pos0 + row;
          for (int jb = 0; jb < p.rpad; jb += 64) {
            const int nv = min(64, p.rpad - jb) / 4;  // float4s in this block (rpad % 16 == 0)
            float4 acc[16];
#pragma unroll
            for (int i = 0; i < 16; ++i) acc[i] = make_float4(0.f, 0.f, 0.f, 0.f);
            for (int q = 0; q < p.kparts; ++q) {
              const float4* src = reinterpret_cast<const float4*>(p.partial + (int64_t(q) * p.T + pos) * p.rpad + jb);
              float4 v[16];
#pragma unroll
              for (int i = 0; i < 16; ++i) v[i] = i < nv ? __ldcg(src + i) : make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
              for (int i = 0; i < 16; ++i) {
                acc[i].x += v[i].x;
                acc[i].y += v[i].y;
                acc[i].z += v[i].z;
                acc[i].w += v[i].w;
              }
            }
            float4* dst = reinterpret_cast<float4*>(p.zfinal + pos * p.rpad + jb);
#pragma unroll
            for (int i = 0; i < 16; ++i)
              if (i < nv) dst[i] = acc[i];
          }
        }
        if (tid == 0) p.counters[seg] = 0;
      }
      named_barrier(1, kTileM);  // *flag is rewritten by the next unit
    }
  } else if (warp == 4 && lane == 0) {
    // ------------------------------------------------------------ MMA thread
    const uint32_t idesc = idesc_bf16(kTileM, p.rpad);
    int sidx = 0, units = 0;
    for (int u = blockIdx.x; u < total; u += gridDim.x) {
      const int seg = u / p.kparts, kp = u - seg * p.kparts;
      const PSeg si = prefill_segment(p, seg);
      if (!si.ok) continue;
      if (*abort) break;
      const int k0 = kp * kPartLen;
      const int nsteps = (min(p.K, k0 + kPartLen) - k0 + 63) / 64;
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
// slice in 256-column pieces (no block straddles two slices).
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

template <int MODE>
__global__ void __launch_bounds__(kExpandThreads, 1) prefill_expand_kernel(const __grid_constant__ PParams p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = align1024(smem_raw);
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  uint8_t* btile = smem;                           // kBStages x 32 KiB
  uint8_t* ztile = smem + kBStages * kBTileBytes;  // 2 buffers x (hi, lo) x 16 KiB
  uint64_t* b_full = reinterpret_cast<uint64_t*>(ztile + 4 * kXTileBytes);
  uint64_t* b_empty = b_full + kBStages;
  uint64_t* z_full = b_empty + kBStages;
  uint64_t* z_empty = z_full + 2;
  uint64_t* t_full = z_empty + 2;
  uint64_t* t_empty = t_full + 2;
  uint64_t* fin = t_empty + 2;  // the MMA thread's last commit (all MMAs retired)
  uint32_t* tslot = reinterpret_cast<uint32_t*>(fin + 1);
  int* offs = reinterpret_cast<int*>(tslot + 4);
  volatile int* abort = reinterpret_cast<volatile int*>(offs + kMaxSlices + 2);
  constexpr int kEpi = 256, kProd = 64;

  if (tid == 0) {
    for (int i = 0; i < kBStages; ++i) {
      mbar_init(&b_full[i], kProd);
      mbar_init(&b_empty[i], 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&z_full[i], kProd);
      mbar_init(&z_empty[i], 1);
      mbar_init(&t_full[i], 1);
      mbar_init(&t_empty[i], kEpi);
    }
    mbar_init(fin, 1);
    fence_mbar_init();
    *abort = 0;
  }
  if (tid <= p.S) offs[tid] = p.slice_offsets[tid];
  if (warp == 10) tc_alloc(tslot, 512);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tslot;
  pdl_launch_dependents();  // only after this CTA holds its TMEM columns

  const int nseg = segment_total(p);
  int nb = 0;
  for (int s = 0; s < p.S; ++s) nb += (offs[s + 1] - offs[s] + kNT - 1) / kNT;
  const int total = nseg * nb;
  const int per = (total + int(gridDim.x) - 1) / int(gridDim.x);
  const int u0 = min(total, int(blockIdx.x) * per), u1 = min(total, u0 + per);

  if (warp == 8 || warp == 9) {
    // ------------------------------------------------------------ producers
    const int pt = tid - kEpi;
    bool waited = false;
    int bidx = 0, zcount = 0, key = -1, pend = -1;
    for (int u = u0; u < u1; ++u) {
      const int seg = u / nb;
      const Block blk = block_of(offs, p.S, u - seg * nb);
      const PSeg si = prefill_segment(p, seg);
      if (!si.ok || blk.slice < 0) continue;
      if (*abort) break;
      // B rows of the block, zero-padded to 64 elements (3-stage ring).
      const int bs = bidx % kBStages;
      wait_or_abort(&b_empty[bs], (uint32_t(bidx / kBStages) & 1u) ^ 1u, abort);
      ++bidx;
      const uint32_t bt = smem_u32(btile + bs * kBTileBytes);
      const int gcol0 = offs[blk.slice] + blk.c0;
      for (int i = pt; i < kNT * 8; i += kProd) {
        const int r = i >> 3, c = i & 7, k = 8 * c;
        const bool live = blk.c0 + r < blk.width && k < si.bucket;
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
      cp_commit();
      // The previous block is handed over once its copies have landed (one block of
      // lag keeps two in flight).
      if (pend >= 0) {
        cp_wait<1>();
        fence_async_smem();
        mbar_arrive(&b_full[pend]);
      }
      pend = bs;
      // z tile of (segment, slice): the shrink's BF16 hi / lo rows, swizzled.
      const int k2 = seg * kMaxSlices + blk.slice;
      if (k2 != key) {
        key = k2;
        if (!waited) {
          pdl_wait();  // the z rows are written by the preceding shrink grid
          waited = true;
        }
        const int zb = zcount & 1;
        wait_or_abort(&z_empty[zb], (uint32_t(zcount >> 1) & 1u) ^ 1u, abort);
        ++zcount;
        // BF16 hi + lo of scale * z (FP32 numerics) or bf16(z) (reference), zero beyond
        // min(rank, bucket) and past the segment's rows; 8 elements per thread step.
        const uint32_t zh = smem_u32(ztile + zb * 2 * kXTileBytes), zl = zh + kXTileBytes;
        const int live = min(si.r, si.bucket);
        const float mul = MODE == kFp32 ? si.scale : 1.f;
        const int col0 = blk.slice * si.r;
        const bool vec = (col0 & 3) == 0;
        // Four items per pass: all their loads are issued before any conversion.
        for (int i0 = pt; i0 < kTileM * 8; i0 += 4 * kProd) {
          float v[4][8];
#pragma unroll
          for (int q = 0; q < 4; ++q) {
            const int i = i0 + q * kProd, m = i >> 3, c = i & 7;
            const float* src = p.zfinal + int64_t(si.pos0 + m) * p.rpad + col0 + 8 * c;
            if (i < kTileM * 8 && m < si.n && vec && 8 * c + 8 <= live) {
              const float4 a0 = __ldcg(reinterpret_cast<const float4*>(src));
              const float4 a1 = __ldcg(reinterpret_cast<const float4*>(src) + 1);
              v[q][0] = a0.x; v[q][1] = a0.y; v[q][2] = a0.z; v[q][3] = a0.w;
              v[q][4] = a1.x; v[q][5] = a1.y; v[q][6] = a1.z; v[q][7] = a1.w;
            } else {
#pragma unroll
              for (int e = 0; e < 8; ++e)
                v[q][e] = (i < kTileM * 8 && m < si.n && 8 * c + e < live) ? __ldcg(src + e) : 0.f;
            }
          }
#pragma unroll
          for (int q = 0; q < 4; ++q) {
            const int i = i0 + q * kProd, m = i >> 3, c = i & 7;
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
        cp_commit();
        cp_wait<0>();
        fence_async_smem();
        mbar_arrive(&b_full[pend]);
        pend = -1;
        mbar_arrive(&z_full[zb]);
      }
    }
    if (pend >= 0) {
      cp_wait<0>();
      fence_async_smem();
      mbar_arrive(&b_full[pend]);
    }
    // Every CTA waits for the shrink grid, so this grid's completion implies the shrink's.
    if (!waited) pdl_wait();
  } else if (warp == 10) {
    // ------------------------------------------------------------ MMA thread
    if (lane == 0) {
      const uint32_t idesc = idesc_bf16(kTileM, kNT);
      int bidx = 0, zcount = 0, tcount = 0, key = -1, zb = 0;
      for (int u = u0; u < u1; ++u) {
        const int seg = u / nb;
        const Block blk = block_of(offs, p.S, u - seg * nb);
        const PSeg si = prefill_segment(p, seg);
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
        const int bs = bidx % kBStages;
        wait_or_abort(&b_full[bs], uint32_t(bidx / kBStages) & 1u, abort);
        ++bidx;
        const int tb = tcount & 1;
        wait_or_abort(&t_empty[tb], (uint32_t(tcount >> 1) & 1u) ^ 1u, abort);
        ++tcount;
        if (*abort) break;
        tc_fence_after();
        const uint32_t d = tmem + uint32_t(tb * kNT);
        const uint32_t zh = smem_u32(ztile + zb * 2 * kXTileBytes);
        const uint64_t bd = sw128_desc(smem_u32(btile + bs * kBTileBytes));
        const uint64_t ah = sw128_desc(zh), al = sw128_desc(zh + kXTileBytes);
#pragma unroll
        for (int k = 0; k < 4; ++k) tc_mma(d, ah + 2 * k, bd + 2 * k, idesc, k > 0 ? 1u : 0u);
        if (MODE == kFp32) {
#pragma unroll
          for (int k = 0; k < 4; ++k) tc_mma(d, al + 2 * k, bd + 2 * k, idesc, 1u);
        }
        tc_commit(&b_empty[bs]);
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
    int tcount = 0;
    for (int u = u0; u < u1; ++u) {
      const int seg = u / nb;
      const Block blk = block_of(offs, p.S, u - seg * nb);
      const PSeg si = prefill_segment(p, seg);
      if (!si.ok || blk.slice < 0) continue;
      const int tb = tcount & 1;
      const uint32_t tph = uint32_t(tcount >> 1) & 1u;
      ++tcount;
      int tok = -1;
      if (row < si.n) {
        tok = p.perm[si.pos0 + row];
        if (tok < 0 || tok >= p.T) tok = -1;
      }
      const int cl = blk.c0 + half * 128;            // first column of this half, in the slice
      const int ncols = min(128, blk.width - cl);    // columns of this half (may be <= 0)
      const int gcol = offs[blk.slice] + cl;
      uint16_t* yrow = tok >= 0 ? p.y + int64_t(tok) * p.y_stride + gcol : nullptr;
      const bool vec = yrow && ncols == 128 && vec_ok && (gcol & 7) == 0;
      // The old y of this half row is fetched before the MMA completes.
      uint4 yv[16];
      if (vec) {
#pragma unroll
        for (int i = 0; i < 16; ++i) yv[i] = *reinterpret_cast<const uint4*>(yrow + 8 * i);
      }
      if (!wait_or_abort(&t_full[tb], tph, abort)) break;
      tc_fence_after();
      const uint32_t tbase = tmem + (uint32_t(quarter * 32) << 16) + uint32_t(tb * kNT + half * 128);
#pragma unroll
      for (int ch = 0; ch < 4; ++ch) {
        uint32_t r[32];
        tc_ld32(tbase + 32 * ch, r);
        if (vec) {
#pragma unroll
          for (int i = 0; i < 4; ++i) {
            const uint4 o = yv[4 * ch + i];
            const uint32_t ow[4] = {o.x, o.y, o.z, o.w};
            uint32_t nw[4];
#pragma unroll
            for (int e = 0; e < 4; ++e) {
              const float d0 = __uint_as_float(r[8 * i + 2 * e]), d1 = __uint_as_float(r[8 * i + 2 * e + 1]);
              const float y0 = __uint_as_float(ow[e] << 16), y1 = __uint_as_float(ow[e] & 0xffff0000u);
              const float v0 = MODE == kFp32 ? y0 + d0 : y0 + round_through_bf16(d0 * si.scale);
              const float v1 = MODE == kFp32 ? y1 + d1 : y1 + round_through_bf16(d1 * si.scale);
              nw[e] = cvt_bf16x2(v0, v1);
            }
            *reinterpret_cast<uint4*>(yrow + 32 * ch + 8 * i) = make_uint4(nw[0], nw[1], nw[2], nw[3]);
          }
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
      tc_fence_before();
      mbar_arrive(&t_empty[tb]);
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 10) {
    tc_fence_after();
    tc_dealloc(tmem, 512);
  }
}

// ====================================================================== host side
struct PrefillLayout {
  int rpad, kparts;
  int64_t partial, zfinal, counters, total;  // offsets in floats
};

inline PrefillLayout prefill_layout(int64_t tokens, int64_t width, int num_slices, int capacity) {
  PrefillLayout l{};
  const int64_t T = tokens > 0 ? tokens : 1;
  const int cap = capacity < kMaxRank ? capacity : kMaxRank;
  l.rpad = (num_slices * cap + 15) / 16 * 16;
  l.kparts = int((width + kPartLen - 1) / kPartLen);
  l.partial = 0;
  l.zfinal = l.partial + int64_t(l.kparts) * T * l.rpad;
  l.counters = l.zfinal + T * l.rpad;
  l.total = l.counters + (T + 3) / 4 * 4;
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

template <typename Kernel>
int launch_pdl(Kernel kernel, int grid, int block, int smem, cudaStream_t stream, const PParams& p,
               const char* what) {
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
  const cudaError_t err = cudaLaunchKernelEx(&config, kernel, p);
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

extern "C" int lf_sgmv_prefill(
    const void* x, int64_t x_stride, const void* a, const void* b, const int64_t* b_offsets,
    const int32_t* b_strides, void* y, int64_t y_stride, const int32_t* segment_indptr,
    const int32_t* segment_slots, const int32_t* token_indices, const int32_t* ranks,
    const float* scales, const int32_t* slice_offsets, const int32_t* segment_count,
    float* workspace, int64_t workspace_floats, int64_t num_tokens, int64_t width,
    int32_t out_width, int32_t num_slices, int32_t capacity, int32_t num_slots,
    int32_t max_segments, int32_t numerics, void* stream) {
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
            segment_count, workspace + l.partial, workspace + l.zfinal,
            reinterpret_cast<int*>(workspace + l.counters), int(T), int(width), out_width,
            num_slices, capacity, num_slots, max_segments, l.rpad, l.kparts, numerics, 0};
  {
    // x [T, K] and A [slots*S*cap, K] as 2-D tensors for the shrink's TMA boxes.
    const PFN_cuTensorMapEncodeTiled_v12000 encode = prefill_tensor_map_encoder();
    if (!encode) return fail(LF_E_CUDA, "sgmv_prefill: cuTensorMapEncodeTiled unavailable");
    const cuuint32_t estr[2] = {1, 1};
    const cuuint64_t xdims[2] = {cuuint64_t(width), cuuint64_t(T)};
    const cuuint64_t xstrides[1] = {cuuint64_t(x_stride) * 2};
    const cuuint32_t xbox[2] = {64, kTileM};
    const cuuint64_t adims[2] = {cuuint64_t(width), cuuint64_t(num_slots) * num_slices * capacity};
    const cuuint64_t astrides[1] = {cuuint64_t(width) * 2};
    const cuuint32_t abox[2] = {64, cuuint32_t(l.rpad)};
    CUresult r = encode(&p.tmap_x, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(x), xdims,
                        xstrides, xbox, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                        CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r == CUDA_SUCCESS)
      r = encode(&p.tmap_a, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(a), adims, astrides,
                 abox, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                 CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) return fail(LF_E_CUDA, "sgmv_prefill: cuTensorMapEncodeTiled failed");
  }
  const cudaStream_t s = static_cast<cudaStream_t>(stream);
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
  {
    const int smem = kBStages * kBTileBytes + 4 * kXTileBytes + 1024 + 256;
    auto kernel = numerics == kFp32 ? prefill_expand_kernel<kFp32> : prefill_expand_kernel<kReference>;
    static int flags[2][64] = {};
    if (int rc = ensure_smem(kernel, smem, flags[numerics])) return rc;
    const int grid = sms;
    if (int rc = launch_pdl(kernel, grid, kExpandThreads, smem, s, p, "sgmv_prefill (expand)")) return rc;
  }
  return LF_OK;
}
