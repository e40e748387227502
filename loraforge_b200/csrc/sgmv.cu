// Grouped (SGMV) LoRA shrink -> expand over decode segments of <= 16 tokens (one slot each).
//
// Two persistent kernels per call, one CTA per SM, chained with programmatic dependent
// launch (PDL).  Both are bandwidth kernels: every byte they need is streamed into a
// multi-stage shared-memory ring by a producer warp with cp.async.bulk (the TMA
// engine's 1-D bulk copy), completion tracked by per-stage "full" mbarriers, while
// eight consumer warps compute the previous stages on the tensor cores and release
// them through "empty" mbarriers.
//
//   sgmv_shrink_kernel   units (segment, K chunk), segment-major, a contiguous run of
//                        units per CTA.  A stage holds the segment's x rows (16 slots)
//                        and the slot's S*r live A rows for one K chunk.  Consumer warp w
//                        takes the chunk's 32-column k blocks w, w+8, ...; the eight
//                        per-warp partial products are summed in shared memory in warp
//                        order and added to a per-run accumulator.  At the end of a run
//                        (the CTA's last unit of a segment) the accumulator is written to
//                        the FP32 partials and the run is counted on the segment's
//                        counter; the CTA that completes the count sums the runs'
//                        partials in chunk order into z[segment] and resets the counter.
//                        The summation order depends only on the grid size, so results
//                        are deterministic (no floating-point atomics).
//   sgmv_expand_kernel   units (segment, 128-column block), split over the CTAs by an
//                        estimated cost that weighs the slot's B bucket (expand_split).
//                        A stage holds the slot's compact B rows of one or more blocks
//                        and the segment's y rows.  The
//                        producer never waits for the shrink (B and y do not depend on
//                        it), so the first stages are in flight while the shrink
//                        finishes; consumers wait for it (griddepcontrol.wait) before
//                        reading z.  Each consumer warp owns 32 output columns of the
//                        stage; y is written straight from registers (16 bytes a lane).
//
// MMAs: mma.sync m16n8k16 / m16n8k8 with BF16 operands and FP32 accumulation, the
// segment's (up to) 16 tokens as the M dimension.  Inside each 32-element k block the
// fragment slots carry a permutation of k that is the same for both operands, so one
// 16-byte shared-memory load per lane feeds two MMAs.  The expand permutes the
// output columns of four n8 tiles so that each lane owns 8 consecutive outputs.
//
// Numerics: kFp32 keeps z in FP32 (split into BF16 hi + lo for the expand MMAs, about
// 16 significant bits) and rounds the output once: y = bf16(y + scale*acc).
// kReference reproduces the retained-rank operators' contract: z rounded to BF16,
// delta = bf16(acc*scale), y = bf16(y + delta)
// (src/loraforge/ops/csrc/lora_rows.cu:64 and :113).
//
// Every mbarrier wait is bounded (tma.cuh); consumers agree on an expired wait with a
// barrier vote before leaving their loop, so no thread is left at a named barrier.
#include <cooperative_groups.h>
#include <cuda.h>
#include <cudaTypedefs.h>

#include <algorithm>
#include <mutex>
#include <string>

#include "launch.cuh"
#include "sgmv.cuh"
#include "tma.cuh"

namespace cg = cooperative_groups;

namespace lfb {
namespace {

constexpr int kSeg = 16;  // tokens per segment (one m16 tile)
constexpr int kMaxSlices = 4;
constexpr int kMaxRank = 64;
constexpr int kConsumerWarps = 8;
constexpr int kConsumers = kConsumerWarps * 32;
constexpr int kThreads = kConsumers + 32;  // + one producer warp
constexpr int kRowPad = 64;                // bytes after each staged row (bank spread)
constexpr int kExpandCols = 128;           // output columns per expand unit
constexpr int kRedPitch = 72;  // floats per row of the cross-warp reduction buffer
constexpr int kRedBytes = kConsumerWarps * kSeg * kRedPitch * 4;
constexpr int kHeaderBytes = 128;
constexpr int kMaxStages = 8;
constexpr int kStageBudget = 110 * 1024;  // per CTA: two CTAs share an SM (228 KiB, 1 KiB reserved each)

enum Numerics { kFp32 = 0, kReference = 1 };

struct Params {
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
  float* partial;  // [nchunks][T][rstride]: per-run partial sums of z
  float* zfinal;   // [T][rstride]: z of each segment's tokens (row = permuted position)
  int* counters;   // [T]: chunks completed per segment (zero between calls)
  int T, K, N, S, cap, num_slots, max_segments;
  int rstride;  // row stride of partial / zfinal: S*min(cap, 64) rounded up to 8
  int kc, nchunks;
  int stages, stage_bytes;  // of the kernel being launched
  int max_tokens;           // longer segments are left to the prefill (tcgen05) kernels
  int bstage;               // expand: bytes of B rows per stage (16 or 32 KiB)
  CUtensorMap tmap_a;  // A as 2-D [slots*S*cap rows, K], boxes of 8 rows x min(kc, 256)
  // The same with boxes of 64 / 32 / 16 rows: for kc <= 256 the 8-row groups of a stage are
  // plain row-major, so fewer, taller boxes fill the same layout.
  CUtensorMap tmap_a_rows[3];
};

// Producer -> consumer description of one stage (lives at the end of the stage).
struct alignas(16) Header {
  int ok;  // 1 live, 0 skipped segment, -1 end of stream
  int seg, n, r, bucket, pos0, col0, ncols, len, rows;
  float scale;
  int pad;
  int tok[kSeg];
};
static_assert(sizeof(Header) <= kHeaderBytes, "stage header");

struct Seg {
  int ok, g, n, r, bucket, pos0;
  float scale;
  int64_t boff;
};

__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_launch_dependents() {
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}

// Position in a ring of NS stages: stage index and the parity of its current use.
struct Ring {
  int stage = 0;
  uint32_t phase = 0;
  __device__ __forceinline__ void next(int NS) {
    if (++stage == NS) {
      stage = 0;
      phase ^= 1u;
    }
  }
};

__device__ __forceinline__ int segment_total(const Params& p) {
  const int n = *p.seg_count;
  return max(0, min(n, min(p.max_segments, p.T)));
}

// Whole warp: the metadata of segment `seg` and this lane's token (lane < n, else -1).
// A segment is skipped (ok = 0) when its slot, rank, bucket, B offset or any token
// index is outside the contract, so no load or bulk copy ever leaves its buffer.
__device__ __forceinline__ Seg load_segment_warp(const Params& p, int seg, int lane, int& tok) {
  Seg s{};
  tok = -1;
  const int lo = p.indptr[seg], hi = p.indptr[seg + 1];
  s.pos0 = lo;
  s.n = hi - lo;
  s.g = p.seg_slots[seg];
  bool ok = lo >= 0 && hi <= p.T && s.n >= 1 && s.n <= p.max_tokens && s.g >= 0 && s.g < p.num_slots;
  if (ok) {
    s.r = p.ranks[s.g];
    s.bucket = p.b_strides[s.g];
    s.scale = p.scales[s.g];
    s.boff = p.b_offsets[s.g];
    ok = s.r >= 1 && s.r <= kMaxRank && s.r <= p.cap && s.bucket >= 1 && s.bucket <= kMaxRank &&
         (s.bucket & (s.bucket - 1)) == 0 && s.boff >= 0 && (s.boff & 7) == 0;
  }
  if (ok && lane < s.n) tok = p.perm[lo + lane];
  const bool bad = ok && lane < s.n && (tok < 0 || tok >= p.T);
  ok = ok && !__any_sync(0xffffffffu, bad);
  s.ok = ok ? 1 : 0;
  if (!ok) tok = -1;
  return s;
}

// All consumer threads: true iff every one of them passed `ok` (barrier 1).
__device__ __forceinline__ bool consumers_all(bool ok) {
  uint32_t r;
  asm volatile(
      "{\n .reg .pred p, q;\n setp.ne.u32 p, %1, 0;\n bar.red.and.pred q, 1, %2, p;\n"
      " selp.u32 %0, 1, 0, q;\n}\n"
      : "=r"(r)
      : "r"(ok ? 1u : 0u), "n"(kConsumers)
      : "memory");
  return r != 0;
}

__device__ __forceinline__ void consumers_sync() { named_barrier(1, kConsumers); }

__device__ __forceinline__ uint4 lds16(const uint8_t* p) { return *reinterpret_cast<const uint4*>(p); }

__device__ __forceinline__ uint32_t cvt_bf16x2(float first, float second) {
  uint32_t r;
  asm("cvt.rn.bf16x2.f32 %0, %1, %2;" : "=r"(r) : "f"(second), "f"(first));
  return r;
}

__device__ __forceinline__ uint32_t pack2(uint32_t lo_bits, uint32_t hi_bits) {
  return (lo_bits & 0xffffu) | (hi_bits << 16);
}

// z (FP32) pair -> BF16 "hi" pair and the BF16 residual "lo" pair.
__device__ __forceinline__ void split2(float v0, float v1, uint32_t& hi, uint32_t& lo) {
  const uint32_t h0 = float_to_bf16_bits(v0), h1 = float_to_bf16_bits(v1);
  hi = pack2(h0, h1);
  lo = pack2(float_to_bf16_bits(v0 - bf16_bits_to_float(h0)),
             float_to_bf16_bits(v1 - bf16_bits_to_float(h1)));
}

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

// ====================================================================== shrink
// Stage layout: x rows (16 slots, pitch kc*2 + 64 bytes, one bulk copy per token), then
// the A rows as 2-D TMA boxes of 8 rows x bw columns (bw = min(kc, 256)), box-major:
// element (j, c) of the chunk at ((j/8)*(kc/bw) + c/bw) * 8*bw*2 + (j%8)*bw*2 + (c%bw)*2.
// kc is a power of two of at least 64 (shrink_config), so bw is one too and the address
// takes shifts and masks, not the integer divisions that would sit in front of every load.
__device__ __forceinline__ const uint8_t* a_frag(const uint8_t* abase, int kc, int j, int kb, int t) {
  const int lbw = kc < 256 ? 31 - __clz(kc) : 8;  // log2(bw)
  const int c = kb * 32;
  return abase + (((j >> 3) * (kc >> lbw) + (c >> lbw)) << (lbw + 4)) + ((j & 7) << (lbw + 1)) +
         ((c & ((1 << lbw) - 1)) << 1) + 16 * t;
}

__device__ __forceinline__ void tma_load_2d(void* dst, const CUtensorMap* map, int c0, int c1,
                                            uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, "
      "{%2, %3}], [%4];" ::"r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(c0), "r"(c1), "r"(smem_u32(bar))
      : "memory");
}

// Register path (at most 8 n tiles, S*r <= 64): warp w owns n tile w / kparts and the
// k blocks kb = w % kparts (mod kparts) of every unit, kparts = 8 / ntiles.
__device__ __forceinline__ void shrink_unit_regs(const uint8_t* st, int xpitch, int kc, int len,
                                                 int tile, int kpart, int kparts, int g, int t,
                                                 float (&d)[4]) {
  const int nkb = (len + 31) >> 5;
  const uint8_t* abase = st + kSeg * xpitch;
  for (int kb = kpart; kb < nkb; kb += kparts) {
    const bool live = kb * 32 + 8 * t < len;
    uint4 xa = make_uint4(0, 0, 0, 0), xb = xa, w = xa;
    if (live) {
      const int koff = kb * 64 + 16 * t;
      xa = lds16(st + g * xpitch + koff);
      xb = lds16(st + (g + 8) * xpitch + koff);
      w = lds16(a_frag(abase, kc, tile * 8 + g, kb, t));
    }
    mma16816(d, xa.x, xb.x, xa.y, xb.y, w.x, w.y);
    mma16816(d, xa.z, xb.z, xa.w, xb.w, w.z, w.w);
  }
}

// Runs of one segment end at the segment's last chunk or at the CTA's last unit.
// The run's partial (rows of `n` tokens, R columns) is given by `sum(m, j)`; publish
// it, count it on the segment's counter, and let the CTA that completes the count add
// the runs in chunk order into z.  All consumer threads call this together.
template <typename Sum>
__device__ __forceinline__ void publish_run(const Params& p, int* flag, int tid, int seg, int chunk,
                                            int u0, int per, int n, int R, int pos0, Sum sum) {
  const int seg_first = seg * p.nchunks;
  const int run_first = max(u0, seg_first) - seg_first;
  const int run_len = chunk - run_first + 1;
  float* part = p.partial + (int64_t(run_first) * p.T + pos0) * p.rstride;
  for (int e = tid; e < n * R; e += kConsumers) {
    const int m = e / R, j = e - m * R;
    part[int64_t(m) * p.rstride + j] = sum(m, j);
  }
  __threadfence();
  consumers_sync();
  if (tid == 0) {
    const int old = atomicAdd(&p.counters[seg], run_len);
    *flag = old + run_len == p.nchunks ? 1 : 0;
  }
  consumers_sync();
  if (*flag) {
    // Runs start at chunk 0 and at every CTA boundary (multiples of `per`).
    __threadfence();
    const int64_t cstride = int64_t(p.T) * p.rstride;
    for (int e = tid; e < n * R; e += kConsumers) {
      const int m = e / R, j = e - m * R;
      const float* src = p.partial + int64_t(pos0 + m) * p.rstride + j;
      // Runs in chunk order; up to eight partials are loaded before they are added, so
      // their L2 round trips overlap (the order of the additions does not change).
      float s = 0.f;
      for (int c = 0; c < p.nchunks;) {
        float v[8];
        int cs[8], k = 0;
        for (; k < 8 && c < p.nchunks; ++k, c = ((seg_first + c) / per + 1) * per - seg_first) cs[k] = c;
#pragma unroll
        for (int i = 0; i < 8; ++i) v[i] = i < k ? __ldcg(src + cs[i] * cstride) : 0.f;
#pragma unroll
        for (int i = 0; i < 8; ++i)
          if (i < k) s += v[i];
      }
      p.zfinal[int64_t(pos0 + m) * p.rstride + j] = s;
    }
    if (tid == 0) p.counters[seg] = 0;
  }
  // *flag is rewritten only after the next run's first consumers_sync, which every
  // consumer reaches after having read it here.
}

// After an expired wait the consumers leave their loop at unit u of segment `seg` with the
// units [max(u0, seg * nchunks), u1) unpublished.  One thread counts them on their segments'
// counters anyway, and the CTA that completes a count returns it to zero without writing z:
// those segments' outputs are invalid (the expiry is counted in g_lf_wait_timeouts), but the
// workspace's counters stay consistent, so the next call on the same workspace (or on the
// library's built-in scratch) is correct again.
__device__ __forceinline__ void abandon_runs(const Params& p, int seg, int u0, int u1) {
  for (int s = seg; s * p.nchunks < u1; ++s) {
    const int first = max(u0, s * p.nchunks), last = min(u1, (s + 1) * p.nchunks);
    if (last <= first) continue;
    const int old = atomicAdd(&p.counters[s], last - first);
    if (old + (last - first) == p.nchunks) atomicExch(&p.counters[s], 0);
  }
}

template <bool REGS>
__global__ void __launch_bounds__(kThreads, REGS ? 2 : 1)
    sgmv_shrink_kernel(const __grid_constant__ Params p) {
  extern __shared__ __align__(128) uint8_t smem[];
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int NS = p.stages, SB = p.stage_bytes;
  const int xpitch = p.kc * 2 + kRowPad;
  const int hoff = SB - kHeaderBytes;
  float* red = reinterpret_cast<float*>(smem + NS * SB);
  float* acc = red + (REGS ? kConsumerWarps * kSeg * 8 : kConsumerWarps * kSeg * kRedPitch);
  uint64_t* full = reinterpret_cast<uint64_t*>(acc + (REGS ? 0 : kSeg * p.rstride));
  uint64_t* empty = full + kMaxStages;
  int* flag = reinterpret_cast<int*>(empty + kMaxStages);

  if (tid == 0) {
    for (int s = 0; s < NS; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], kConsumerWarps);
    }
    fence_mbar_init();
  }
  if (!REGS)
    for (int i = tid; i < kSeg * p.rstride; i += kThreads) acc[i] = 0.f;
  // The A tensor map lives in kernel parameter space: fetch it while the preceding grid
  // finishes, so the first TMA issue does not wait for it.
  if (tid == kConsumers) {
    asm volatile("prefetch.tensormap [%0];" ::"l"(&p.tmap_a) : "memory");
    for (int h = 0; h < 3; ++h) asm volatile("prefetch.tensormap [%0];" ::"l"(&p.tmap_a_rows[h]) : "memory");
  }
  __syncthreads();
  pdl_wait();  // x, metadata and the workspace may come from the preceding grid
  pdl_launch_dependents();

  // Unit counts fit int32 (checked on the host).
  const int nseg = segment_total(p);
  const int total = nseg * p.nchunks;
  const int per = (total + int(gridDim.x) - 1) / int(gridDim.x);
  const int u0 = int(blockIdx.x) * per;
  const int u1 = min(total, u0 + per);
  if (u0 >= u1) return;

  if (warp == kConsumerWarps) {
    // ------------------------------------------------------------ producer warp
    const int bw = p.kc < 256 ? p.kc : 256;
    int cur = -1, tok = -1;
    Seg si{};
    Ring ring;
    int seg = u0 / p.nchunks, chunk = u0 - seg * p.nchunks;
    for (int u = u0; u < u1; ++u, ring.next(NS), chunk = chunk + 1 == p.nchunks ? (++seg, 0) : chunk + 1) {
      const int stage = ring.stage;
      int ok = 1;
      if (lane == 0) ok = mbar_wait(&empty[stage], ring.phase ^ 1u) ? 1 : 0;
      if (!__shfl_sync(0xffffffffu, ok, 0)) break;  // consumers gone: stop producing
      if (seg != cur) {
        cur = seg;
        si = load_segment_warp(p, seg, lane, tok);
      }
      uint8_t* st = smem + stage * SB;
      Header* h = reinterpret_cast<Header*>(st + hoff);
      const int k0 = chunk * p.kc;
      const int len = min(p.kc, p.K - k0);
      const int R = si.ok ? p.S * si.r : 0;
      const int boxes = (len + bw - 1) / bw;  // boxes past the end of K are not issued
      const int groups = (R + 7) >> 3;
      if (lane == 0) {
        h->ok = si.ok;
        h->seg = seg;
        h->n = si.n;
        h->r = si.r;
        h->pos0 = si.pos0;
        h->len = len;
        h->rows = R;
      }
      const uint32_t row_bytes = uint32_t(len) * 2;
      const uint32_t tx = si.ok ? uint32_t(si.n) * row_bytes + uint32_t(groups * boxes) * (8 * bw * 2) : 0u;
      __syncwarp();
      if (lane == 0) mbar_arrive_expect_tx(&full[stage], tx);
      __syncwarp();
      if (si.ok) {
        if (lane < si.n)
          bulk_g2s(st + lane * xpitch, p.x + int64_t(tok) * p.x_stride + k0, row_bytes, &full[stage]);
        const int row0 = si.g * p.S * p.cap;
        uint8_t* abase = st + kSeg * xpitch;
        if (p.kc <= 256) {
          // One box per 64 / 32 / 16 / 8 rows of the groups' rows: a copy costs the copy
          // engine about the same whatever its size up to a few KiB.
          if (lane == 0)
            for (int r0 = 0, left = groups * 8; left > 0;) {
              const int h = left >= 64 ? 64 : left >= 32 ? 32 : left >= 16 ? 16 : 8;
              const CUtensorMap* map = h == 64   ? &p.tmap_a_rows[0]
                                       : h == 32 ? &p.tmap_a_rows[1]
                                       : h == 16 ? &p.tmap_a_rows[2]
                                                 : &p.tmap_a;
              tma_load_2d(abase + r0 * bw * 2, map, k0, row0 + r0, &full[stage]);
              r0 += h;
              left -= h;
            }
        } else {
          for (int i = lane; i < groups * boxes; i += 32) {
            const int grp = i / boxes, box = i - grp * boxes;
            tma_load_2d(abase + (grp * (p.kc / bw) + box) * (8 * bw * 2), &p.tmap_a, k0 + box * bw,
                        row0 + grp * 8, &full[stage]);
          }
        }
      }
    }
    return;
  }

  // -------------------------------------------------------------- consumer warps
  const int g = lane >> 2, t = lane & 3;
  if constexpr (REGS) {
    // Each warp keeps its share of the run in registers; warps meet once per run.
    float d[4] = {0.f, 0.f, 0.f, 0.f};
    bool aborted = false;
    Ring ring;
    int seg = u0 / p.nchunks, chunk = u0 - seg * p.nchunks;
    for (int u = u0; u < u1; ++u, ring.next(NS), chunk = chunk + 1 == p.nchunks ? (++seg, 0) : chunk + 1) {
      const int stage = ring.stage;
      const bool got = !aborted && mbar_wait(&full[stage], ring.phase);
      aborted = !got;
      const uint8_t* st = smem + stage * SB;
      const Header* hp = reinterpret_cast<const Header*>(st + hoff);
      int ok = 0, n = 0, R = 0, pos0 = 0;
      int kparts = 1;
      if (got) {
        ok = hp->ok;
        n = hp->n;
        R = hp->rows;
        pos0 = hp->pos0;
        const int ntiles = (R + 7) >> 3;
        kparts = ntiles > 0 ? kConsumerWarps / ntiles : 1;
        const int tile = warp / kparts;
        if (ok && tile < ntiles)
          shrink_unit_regs(st, xpitch, p.kc, hp->len, tile, warp - tile * kparts, kparts, g, t, d);
        __syncwarp();
        if (lane == 0) mbar_arrive(&empty[stage]);
      }
      if (!(u + 1 == u1 || chunk + 1 == p.nchunks)) continue;  // run continues
      if (!consumers_all(!aborted)) {
        if (tid == 0) abandon_runs(p, seg, u0, u1);
        break;
      }
      if (!ok) continue;
      float* rw = red + warp * kSeg * 8;  // [warp][16 rows][8 cols]
      *reinterpret_cast<float2*>(rw + g * 8 + 2 * t) = make_float2(d[0], d[1]);
      *reinterpret_cast<float2*>(rw + (g + 8) * 8 + 2 * t) = make_float2(d[2], d[3]);
      d[0] = d[1] = d[2] = d[3] = 0.f;
      consumers_sync();
      publish_run(p, flag, tid, seg, chunk, u0, per, n, R, pos0, [&](int m, int j) {
        float s = 0.f;
        for (int q = 0; q < kparts; ++q) s += red[(((j >> 3) * kparts + q) * kSeg + m) * 8 + (j & 7)];
        return s;
      });
    }
  } else {
    // Wide path (S*r > 64): the unit's product is summed over warps in shared memory
    // per group of 8 n tiles and added to a per-run accumulator.
    Ring ring;
    int seg = u0 / p.nchunks, chunk = u0 - seg * p.nchunks;
    for (int u = u0; u < u1; ++u, ring.next(NS), chunk = chunk + 1 == p.nchunks ? (++seg, 0) : chunk + 1) {
      const int stage = ring.stage;
      const bool got = mbar_wait(&full[stage], ring.phase);
      if (!consumers_all(got)) {
        if (tid == 0) abandon_runs(p, seg, u0, u1);
        break;
      }
      const uint8_t* st = smem + stage * SB;
      const Header h = *reinterpret_cast<const Header*>(st + hoff);
      if (h.ok) {
        const uint8_t* abase = st + kSeg * xpitch;
        const int ntiles = (h.rows + 7) >> 3;
        const int nkb = (h.len + 31) >> 5;
        for (int ng = 0; ng < ntiles; ng += 8) {
          float d[8][4];
#pragma unroll
          for (int i = 0; i < 8; ++i)
#pragma unroll
            for (int e = 0; e < 4; ++e) d[i][e] = 0.f;
          for (int kb = warp; kb < nkb; kb += kConsumerWarps) {
            const int koff = kb * 64 + 16 * t;
            const bool live = kb * 32 + 8 * t < h.len;
            uint4 xa = make_uint4(0, 0, 0, 0), xb = xa;
            if (live) {
              xa = lds16(st + g * xpitch + koff);
              xb = lds16(st + (g + 8) * xpitch + koff);
            }
#pragma unroll
            for (int i = 0; i < 8; ++i) {
              if (ng + i < ntiles) {
                uint4 w = make_uint4(0, 0, 0, 0);
                if (live) w = lds16(a_frag(abase, p.kc, (ng + i) * 8 + g, kb, t));
                mma16816(d[i], xa.x, xb.x, xa.y, xb.y, w.x, w.y);
                mma16816(d[i], xa.z, xb.z, xa.w, xb.w, w.z, w.w);
              }
            }
          }
          if (ng + 8 >= ntiles) {  // this warp's last read of the stage
            __syncwarp();
            if (lane == 0) mbar_arrive(&empty[stage]);
          }
          float* rw = red + warp * kSeg * kRedPitch;
#pragma unroll
          for (int i = 0; i < 8; ++i) {
            *reinterpret_cast<float2*>(rw + g * kRedPitch + i * 8 + 2 * t) = make_float2(d[i][0], d[i][1]);
            *reinterpret_cast<float2*>(rw + (g + 8) * kRedPitch + i * 8 + 2 * t) =
                make_float2(d[i][2], d[i][3]);
          }
          consumers_sync();
          for (int e = tid; e < kSeg * 64; e += kConsumers) {
            const int m = e >> 6, jl = e & 63, j = ng * 8 + jl;
            float s = 0.f;
#pragma unroll
            for (int w = 0; w < kConsumerWarps; ++w) s += red[(w * kSeg + m) * kRedPitch + jl];
            if (j < p.rstride) acc[m * p.rstride + j] += s;
          }
          consumers_sync();
        }
      } else {
        __syncwarp();
        if (lane == 0) mbar_arrive(&empty[stage]);
      }
      if (!h.ok || !(u + 1 == u1 || chunk + 1 == p.nchunks)) continue;
      publish_run(p, flag, tid, seg, chunk, u0, per, h.n, h.rows, h.pos0,
                  [&](int m, int j) { return acc[m * p.rstride + j]; });
      for (int e = tid; e < kSeg * p.rstride; e += kConsumers) acc[e] = 0.f;
      consumers_sync();
    }
  }
}

// ====================================================================== expand
constexpr int kStageCols = 512;                  // output columns per expand stage (max)
constexpr int kYStagePitch = kStageCols * 2 + kRowPad;

struct alignas(16) ExpandHeader {
  int ok;  // 1 live, -1 end of stream
  int seg, n, r, bucket, pos0, col0, ncols;
  int slice;  // the stage's slice when all its columns are in one, else -1
  float scale;
  int pad[2];
  int tok[kSeg];
};
static_assert(sizeof(ExpandHeader) <= kHeaderBytes, "expand stage header");

__device__ __forceinline__ int slice_of(const int* offs, int S, int col) {
  int s = 0;
  for (int i = 1; i < S; ++i)
    if (col >= offs[i]) s = i;
  return s;
}

// z fragments of slice s for this lane, multiplied by `mul`: [mma q][hi, lo][4 regs].
// Every z value of the lane is loaded before the first is converted, so the loads
// overlap instead of paying one L2 round trip each.
// ZS: z is the CTA's own shared-memory copy `zsm` (rows of kZsPitch floats, the segment's
// token m at row m) instead of the workspace's z rows, read with plain loads.
constexpr int kZsPitch = 64;

template <int KP, int MODE, bool ZS = false>
__device__ __forceinline__ void load_z(const Params& p, const ExpandHeader& h, int s, float mul,
                                       int g, int t, uint32_t (&zf)[4][2][4],
                                       const float* zsm = nullptr) {
  const int live = min(h.r, h.bucket);
  constexpr int NV = KP == 8 ? 4 : KP / 16 * 8;
  const float* zr0 = ZS ? zsm + g * kZsPitch + s * h.r : p.zfinal + int64_t(h.pos0 + g) * p.rstride + s * h.r;
  const float* zr1 = zr0 + (ZS ? int64_t(8) * kZsPitch : int64_t(8) * p.rstride);
  float v[NV];
#pragma unroll
  for (int i = 0; i < NV; ++i) {
    // Value i: row half m (token g or g + 8) and rank index kk of fragment register
    // i / 2 of MMA i / 8, in the k order the B fragments use.
    int m, kk;
    if constexpr (KP == 8) {
      m = i >> 1;
      kk = 2 * t + (i & 1);
    } else {
      const int q = i >> 3, j = i & 7;
      const int base = KP == 16 ? 4 * t : 32 * (q >> 1) + 8 * t + 4 * (q & 1);
      m = (j >> 1) & 1;
      kk = base + ((j >> 2) << 1) + (j & 1);
    }
    const float* zp = (m ? zr1 : zr0) + kk;
    v[i] = (g + 8 * m < h.n && kk < live) ? (ZS ? *zp : __ldcg(zp)) : 0.f;
  }
#pragma unroll
  for (int i = 0; i < NV; i += 2) {
    const int q = KP == 8 ? 0 : i >> 3, reg = KP == 8 ? i >> 1 : (i & 7) >> 1;
    const float v0 = mul * v[i], v1 = mul * v[i + 1];
    if (MODE == kFp32) {
      split2(v0, v1, zf[q][0][reg], zf[q][1][reg]);
    } else {
      zf[q][0][reg] = pack2(float_to_bf16_bits(v0), float_to_bf16_bits(v1));
    }
  }
}

// B fragment of the tile column at row `cb` of the stage's B block (bucket elements
// per row): [mma q][2 regs], slots matching load_z's k permutation.
template <int KP>
__device__ __forceinline__ void load_b(const uint8_t* bt, int cb, int bucket, int t,
                                       uint32_t (&bf)[4][2]) {
  const uint8_t* row = bt + cb * bucket * 2;
  if constexpr (KP == 8) {
    uint32_t v = 0;
    if (bucket >= 8 || 2 * t + 1 < bucket) {
      v = *reinterpret_cast<const uint32_t*>(row + 4 * t);
    } else if (2 * t < bucket) {
      v = *reinterpret_cast<const uint16_t*>(row + 4 * t);
    }
    bf[0][0] = v;
    bf[0][1] = 0;
  } else if constexpr (KP == 16) {
    const uint2 v = *reinterpret_cast<const uint2*>(row + 8 * t);
    bf[0][0] = v.x;
    bf[0][1] = v.y;
  } else {
#pragma unroll
    for (int kb = 0; kb < KP / 32; ++kb) {
      const uint4 v = lds16(row + kb * 64 + 16 * t);
      bf[2 * kb][0] = v.x;
      bf[2 * kb][1] = v.y;
      bf[2 * kb + 1][0] = v.z;
      bf[2 * kb + 1][1] = v.w;
    }
  }
}

// One consumer warp, every 32-column group grp = warp, warp + 8, ... of a stage.
// Tile j of a group holds the columns 8*(nu>>1) + 2j + (nu&1) for its n index nu, so
// lane (g, t) ends up owning the 8 consecutive columns 8t..8t+7 of rows g and g+8.
template <int KP, int MODE, bool STAGED, bool ZS = false>
__device__ __forceinline__ void expand_stage(const Params& p, const ExpandHeader& h,
                                             const uint8_t* st, const int* offs,
                                             uint32_t (&zf)[4][2][4], int& zseg, int& zslice,
                                             int lane, int warp, const float* zsm = nullptr) {
  constexpr int Q = KP >= 16 ? KP / 16 : 1;
  constexpr int PARTS = MODE == kFp32 ? 2 : 1;
  const int g = lane >> 2, t = lane & 3;
  const float mul = MODE == kFp32 ? h.scale : 1.f;  // fp32: scale folded into z
  const int groups = (h.ncols + 31) >> 5;
  for (int grp = warp; grp < groups; grp += kConsumerWarps) {
    const int c_rel = grp * 32;
    const int my = c_rel + 8 * t;  // this lane's first column inside the stage
    const bool mine = my < h.ncols;
    int s_first = h.slice, s_last = h.slice;
    if (s_first < 0) {
      s_first = slice_of(offs, p.S, h.col0 + c_rel);
      s_last = slice_of(offs, p.S, h.col0 + min(c_rel + 32, h.ncols) - 1);
    }
    // Old y of rows g and g+8 (zero past the segment's rows or the stage's columns).
    auto y_old = [&](int hh, float (&v)[8]) {
      const int m = g + 8 * hh;
      if constexpr (STAGED) {
        uint4 w = make_uint4(0, 0, 0, 0);
        if (mine && m < h.n) w = lds16(st + p.bstage + m * kYStagePitch + my * 2);
        unpack_bf16x8(w, v);
      } else {
#pragma unroll
        for (int c = 0; c < 8; ++c)
          v[c] = (m < h.n && my + c < h.ncols)
                     ? bf16_bits_to_float(p.y[int64_t(h.tok[m]) * p.y_stride + h.col0 + my + c])
                     : 0.f;
      }
    };
    for (int s = s_first; s <= s_last; ++s) {
      if (h.seg != zseg || s != zslice) {
        load_z<KP, MODE, ZS>(p, h, s, mul, g, t, zf, zsm);
        zseg = h.seg;
        zslice = s;
      }
      // fp32: the accumulator starts at the old y, so it ends at y + scale * B z.
      float d[4][4];
      if (MODE == kFp32) {
        float v0[8], v1[8];
        y_old(0, v0);
        y_old(1, v1);
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          d[j][0] = v0[2 * j];
          d[j][1] = v0[2 * j + 1];
          d[j][2] = v1[2 * j];
          d[j][3] = v1[2 * j + 1];
        }
      } else {
#pragma unroll
        for (int j = 0; j < 4; ++j) d[j][0] = d[j][1] = d[j][2] = d[j][3] = 0.f;
      }
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        uint32_t bf[4][2];
        load_b<KP>(st, c_rel + 8 * (g >> 1) + 2 * j + (g & 1), h.bucket, t, bf);
#pragma unroll
        for (int part = 0; part < PARTS; ++part)
#pragma unroll
          for (int q = 0; q < Q; ++q) {
            if constexpr (KP == 8) {
              mma1688(d[j], zf[0][part][0], zf[0][part][1], bf[0][0]);
            } else {
              mma16816(d[j], zf[q][part][0], zf[q][part][1], zf[q][part][2], zf[q][part][3],
                       bf[q][0], bf[q][1]);
            }
          }
      }
#pragma unroll
      for (int hh = 0; hh < 2; ++hh) {
        const int m = g + 8 * hh;
        if (m >= h.n || !mine) continue;
        float v[8];
#pragma unroll
        for (int c = 0; c < 8; ++c) v[c] = d[c >> 1][2 * hh + (c & 1)];
        if (MODE != kFp32) {
          float yv[8];
          y_old(hh, yv);
#pragma unroll
          for (int c = 0; c < 8; ++c) v[c] = yv[c] + round_through_bf16(v[c] * h.scale);
        }
        uint16_t* yrow = p.y + int64_t(h.tok[m]) * p.y_stride + h.col0 + my;
        if (STAGED && s_first == s_last) {
          *reinterpret_cast<uint4*>(yrow) = make_uint4(cvt_bf16x2(v[0], v[1]), cvt_bf16x2(v[2], v[3]),
                                                       cvt_bf16x2(v[4], v[5]), cvt_bf16x2(v[6], v[7]));
        } else {
          // Ragged edge or a group that straddles slices: the columns of slice s only.
          const int cols = min(8, h.ncols - my);
          for (int c = 0; c < cols; ++c)
            if (s_first == s_last || slice_of(offs, p.S, h.col0 + my + c) == s)
              yrow[c] = uint16_t(float_to_bf16_bits(v[c]));
        }
      }
    }
  }
}

// Stages whose columns lie in one slice, with y staged: each warp runs two of its
// 32-column groups side by side (same arithmetic as expand_stage), so the y loads, MMA
// chains and stores of one group overlap the latencies of the other.  Measured per bucket:
// 16 (config 1, where it was introduced), 32 (config 4 365 -> 360 us/step) and 64
// (config 2 68.8 -> 66.1).
template <int KP, int MODE, bool ZS = false>
__device__ __forceinline__ void expand_stage_pair(const Params& p, const ExpandHeader& h,
                                                  const uint8_t* st, uint32_t (&zf)[4][2][4],
                                                  int& zseg, int& zslice, int lane, int warp,
                                                  const float* zsm = nullptr) {
  constexpr int PARTS = MODE == kFp32 ? 2 : 1;
  const int g = lane >> 2, t = lane & 3;
  const float mul = MODE == kFp32 ? h.scale : 1.f;  // fp32: scale folded into z
  if (h.seg != zseg || h.slice != zslice) {
    load_z<KP, MODE, ZS>(p, h, h.slice, mul, g, t, zf, zsm);
    zseg = h.seg;
    zslice = h.slice;
  }
  const int groups = (h.ncols + 31) >> 5;
  for (int grp0 = warp; grp0 < groups; grp0 += 2 * kConsumerWarps) {
    float d[2][4][4];
    int my[2];
    bool mine[2];
#pragma unroll
    for (int q = 0; q < 2; ++q) {
      my[q] = (grp0 + q * kConsumerWarps) * 32 + 8 * t;
      mine[q] = my[q] < h.ncols;
#pragma unroll
      for (int hh = 0; hh < 2; ++hh) {
        const int m = g + 8 * hh;
        float v[8];
        uint4 w = make_uint4(0, 0, 0, 0);
        if (MODE == kFp32 && mine[q] && m < h.n) w = lds16(st + p.bstage + m * kYStagePitch + my[q] * 2);
        unpack_bf16x8(w, v);
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          d[q][j][2 * hh] = v[2 * j];
          d[q][j][2 * hh + 1] = v[2 * j + 1];
        }
      }
    }
#pragma unroll
    for (int q = 0; q < 2; ++q) {
      if (grp0 + q * kConsumerWarps >= groups) break;
      const int c_rel = (grp0 + q * kConsumerWarps) * 32;
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        uint32_t bf[4][2];
        load_b<KP>(st, c_rel + 8 * (g >> 1) + 2 * j + (g & 1), h.bucket, t, bf);
#pragma unroll
        for (int part = 0; part < PARTS; ++part) {
          if constexpr (KP == 8) {
            mma1688(d[q][j], zf[0][part][0], zf[0][part][1], bf[0][0]);
          } else {
#pragma unroll
            for (int k16 = 0; k16 < KP / 16; ++k16)
              mma16816(d[q][j], zf[k16][part][0], zf[k16][part][1], zf[k16][part][2], zf[k16][part][3],
                       bf[k16][0], bf[k16][1]);
          }
        }
      }
    }
#pragma unroll
    for (int q = 0; q < 2; ++q) {
#pragma unroll
      for (int hh = 0; hh < 2; ++hh) {
        const int m = g + 8 * hh;
        if (m >= h.n || !mine[q]) continue;
        float v[8];
#pragma unroll
        for (int c = 0; c < 8; ++c) v[c] = d[q][c >> 1][2 * hh + (c & 1)];
        if (MODE != kFp32) {
          float yv[8];
          unpack_bf16x8(lds16(st + p.bstage + m * kYStagePitch + my[q] * 2), yv);
#pragma unroll
          for (int c = 0; c < 8; ++c) v[c] = yv[c] + round_through_bf16(v[c] * h.scale);
        }
        uint16_t* yrow = p.y + int64_t(h.tok[m]) * p.y_stride + h.col0 + my[q];
        *reinterpret_cast<uint4*>(yrow) = make_uint4(cvt_bf16x2(v[0], v[1]), cvt_bf16x2(v[2], v[3]),
                                                     cvt_bf16x2(v[4], v[5]), cvt_bf16x2(v[6], v[7]));
      }
    }
  }
}

// Estimated cost of one expand unit (segment s, 128 columns) in units of one token row
// (about 25 SM cycles): a base by the slot's B bucket plus one per token row.  Per-stage
// clock64 counts on BASELINE configs 1 and 2 put a unit at about 470-630 cycles for
// buckets up to 16 (stages of 512 columns), 780 for 32 (256 columns) and 1840 for 64 (128
// columns, half the consumer warps idle), plus about 25 cycles per token row.
constexpr int kUnitCost = 24;
__device__ __forceinline__ int expand_unit_cost(int bucket, int n) {
  return (bucket <= 16 ? kUnitCost : bucket <= 32 ? 30 : 72) + n;
}

// Whole CTA (kThreads threads, before the warp roles split): this CTA's expand units
// [bounds[0], bounds[1]).  Each thread sums the costs of a contiguous range of segments
// (ncb units of expand_unit_cost each; a segment outside the contract costs as a bucket-16
// one, its units are skipped by the producer), a block scan gives each range's start, and
// the thread whose range holds a boundary (total * part / parts) places it inside its
// segment.  When every segment has the same bucket and the CTAs get fewer than 32 units
// each, the units split by count instead: a cost split would add a z reload at every
// segment change to the light CTAs, which costs more than it balances (BASELINE config 1
// qkv and down).  `ws` holds kThreads / 32 + 2 int64 values of shared memory.
__device__ void expand_split(const Params& p, int nseg, int ncb, long long* ws, int* bounds) {
  constexpr int kWarps = kThreads / 32;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int span = (nseg + kThreads - 1) / kThreads;
  const int s0 = min(nseg, tid * span), s1 = min(nseg, s0 + span);
  auto bucket_of = [&](int s) {
    const int g = p.seg_slots[s];
    return g >= 0 && g < p.num_slots ? p.b_strides[g] : 16;
  };
  auto unit_cost = [&](int s, int bucket) {
    const int n = p.indptr[s + 1] - p.indptr[s];
    return expand_unit_cost(bucket, n < 0 ? 0 : n > kSeg ? kSeg : n);
  };
  long long mine = 0;
  int lo = 1 << 30, hi = -1;
  for (int s = s0; s < s1; ++s) {
    const int b = bucket_of(s);
    lo = min(lo, b);
    hi = max(hi, b);
    mine += (long long)ncb * unit_cost(s, b);
  }
  long long inc = mine;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const long long v = __shfl_up_sync(0xffffffffu, inc, o);
    if (lane >= o) inc += v;
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    lo = min(lo, __shfl_xor_sync(0xffffffffu, lo, o));
    hi = max(hi, __shfl_xor_sync(0xffffffffu, hi, o));
  }
  if (tid == 0) {
    ws[kWarps] = 1 << 30;  // min bucket
    ws[kWarps + 1] = -1;   // max bucket
  }
  __syncthreads();
  if (lane == 31) ws[warp] = inc;
  if (lane == 0) {
    atomicMin(&ws[kWarps], (long long)lo);
    atomicMax(&ws[kWarps + 1], (long long)hi);
  }
  __syncthreads();
  long long before = inc - mine, total = 0;
#pragma unroll
  for (int w = 0; w < kWarps; ++w) {
    before += w < warp ? ws[w] : 0;
    total += ws[w];
  }
  const int units = nseg * ncb;
  const bool by_count = ws[kWarps] == ws[kWarps + 1] && units < 32 * int(gridDim.x);
  for (int k = 0; k < 2; ++k) {
    const int part = int(blockIdx.x) + k, parts = int(gridDim.x);
    if (by_count) {
      const int per = (units + parts - 1) / parts;
      if (tid == 0) bounds[k] = min(units, part * per);
      continue;
    }
    if (part <= 0 || part >= parts || total <= 0) {
      if (tid == 0) bounds[k] = part <= 0 ? 0 : units;
      continue;
    }
    const long long target = total * part / parts;  // < total: exactly one range holds it
    if (before <= target && target < before + mine) {
      long long acc = before;
      for (int s = s0; s < s1; ++s) {
        const int c = unit_cost(s, bucket_of(s));
        if (target < acc + (long long)ncb * c) {
          const long long unit = (target - acc) / c;
          bounds[k] = s * ncb + (unit < ncb ? int(unit) : ncb);
          break;
        }
        acc += (long long)ncb * c;
      }
    }
  }
  __syncthreads();
}

template <int MODE, bool STAGED>
__global__ void __launch_bounds__(kThreads, 2) sgmv_expand_kernel(const __grid_constant__ Params p) {
  extern __shared__ __align__(128) uint8_t smem[];
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int NS = p.stages, SB = p.stage_bytes;
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + NS * SB);
  uint64_t* empty = full + kMaxStages;
  int* offs = reinterpret_cast<int*>(empty + kMaxStages);
  const int hoff = SB - kHeaderBytes;  // header offset inside a stage

  if (tid == 0) {
    for (int s = 0; s < NS; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], kConsumerWarps);
    }
    fence_mbar_init();
  }
  if (tid <= p.S) offs[tid] = p.slice_offsets[tid];
  __syncthreads();
  pdl_launch_dependents();

  const int nseg = segment_total(p);
  const int ncb = (p.N + kExpandCols - 1) / kExpandCols;
  // The metadata read here comes from the grid before the shrink, which the shrink waited
  // for (griddepcontrol.wait) before it let this grid launch.
  __shared__ long long split_ws[kThreads / 32 + 2];
  __shared__ int split_bounds[2];
  expand_split(p, nseg, ncb, split_ws, split_bounds);

  if (warp == kConsumerWarps) {
    // ------------------------------------------------------------ producer warp
    // B rows and y rows do not depend on the shrink: no griddepcontrol.wait here.
    const int u0 = split_bounds[0], u1 = split_bounds[1];
    // Consecutive 128-column units of one segment are merged into a stage while its
    // B rows fit p.bstage and its columns kStageCols.
    int cur = -1, tok = -1;
    Seg si{};
    Ring ring;
    bool alive = true;
    for (int u = u0; u < u1 && alive;) {
      const int seg = u / ncb;
      const int cb = u - seg * ncb;
      if (seg != cur) {
        cur = seg;
        si = load_segment_warp(p, seg, lane, tok);
      }
      if (!si.ok) {  // skip the rest of this segment's units
        u = min(u1, (seg + 1) * ncb);
        continue;
      }
      const int max_cols = min(kStageCols, p.bstage / (2 * si.bucket));  // >= kExpandCols
      const int take = min(min(max_cols / kExpandCols, ncb - cb), u1 - u);
      const int c0 = cb * kExpandCols;
      const int nc = min(p.N, (cb + take) * kExpandCols) - c0;
      u += take;
      const int stage = ring.stage;
      const uint32_t phase = ring.phase;
      ring.next(NS);
      int ok = 1;
      if (lane == 0) ok = mbar_wait(&empty[stage], phase ^ 1u) ? 1 : 0;
      if (!__shfl_sync(0xffffffffu, ok, 0)) {
        alive = false;
        break;
      }
      uint8_t* st = smem + stage * SB;
      ExpandHeader* h = reinterpret_cast<ExpandHeader*>(st + hoff);
      if (lane == 0) {
        const int s0 = slice_of(offs, p.S, c0), s1 = slice_of(offs, p.S, c0 + nc - 1);
        h->ok = 1;
        h->seg = seg;
        h->n = si.n;
        h->r = si.r;
        h->bucket = si.bucket;
        h->pos0 = si.pos0;
        h->col0 = c0;
        h->ncols = nc;
        h->slice = s0 == s1 ? s0 : -1;
        h->scale = si.scale;
      }
      if (lane < kSeg) h->tok[lane] = tok;
      // B block: bulk-copy whole 16-byte units; the last < 16 bytes (only when the
      // output width is not a multiple of 8) are copied here with plain loads.
      const uint16_t* bsrc = p.b + si.boff + int64_t(c0) * si.bucket;
      const uint32_t bbytes = uint32_t(nc) * si.bucket * 2;
      const uint32_t bbulk = bbytes & ~15u;
      for (uint32_t i = bbulk / 2 + lane; i < bbytes / 2; i += 32)
        reinterpret_cast<uint16_t*>(st)[i] = bsrc[i];
      const uint32_t ybytes = STAGED ? uint32_t(nc) * 2 : 0u;
      __syncwarp();
      if (lane == 0) mbar_arrive_expect_tx(&full[stage], bbulk + uint32_t(si.n) * ybytes);
      __syncwarp();
      if (lane == 31 && bbulk) bulk_g2s(st, bsrc, bbulk, &full[stage]);
      if (STAGED && lane < si.n)
        bulk_g2s(st + p.bstage + lane * kYStagePitch, p.y + int64_t(tok) * p.y_stride + c0, ybytes,
                 &full[stage]);
    }
    if (alive) {  // end of stream
      const int stage = ring.stage;
      int ok = 1;
      if (lane == 0) ok = mbar_wait(&empty[stage], ring.phase ^ 1u) ? 1 : 0;
      if (__shfl_sync(0xffffffffu, ok, 0) && lane == 0) {
        reinterpret_cast<ExpandHeader*>(smem + stage * SB + hoff)->ok = -1;
        mbar_arrive(&full[stage]);
      }
    }
    return;
  }

  // -------------------------------------------------------------- consumer warps
  // Warps run independently (no CTA barrier in this loop): each waits for a stage,
  // computes its column groups and releases the stage.
  pdl_wait();  // z is written by the preceding shrink grid
  uint32_t zf[4][2][4];
  int zseg = -1, zslice = -1;
  for (Ring ring;; ring.next(NS)) {
    const int stage = ring.stage;
    if (!mbar_wait(&full[stage], ring.phase)) break;
    const uint8_t* st = smem + stage * SB;
    const ExpandHeader& h = *reinterpret_cast<const ExpandHeader*>(st + hoff);
    if (h.ok < 0) break;
    if (STAGED && h.slice >= 0) {
      if (h.bucket == 64) expand_stage_pair<64, MODE>(p, h, st, zf, zseg, zslice, lane, warp);
      else if (h.bucket == 32) expand_stage_pair<32, MODE>(p, h, st, zf, zseg, zslice, lane, warp);
      else if (h.bucket == 16) expand_stage_pair<16, MODE>(p, h, st, zf, zseg, zslice, lane, warp);
      else expand_stage_pair<8, MODE>(p, h, st, zf, zseg, zslice, lane, warp);
    } else switch (h.bucket < 8 ? 8 : h.bucket) {
      case 8: expand_stage<8, MODE, STAGED>(p, h, st, offs, zf, zseg, zslice, lane, warp); break;
      case 16: expand_stage<16, MODE, STAGED>(p, h, st, offs, zf, zseg, zslice, lane, warp); break;
      case 32: expand_stage<32, MODE, STAGED>(p, h, st, offs, zf, zseg, zslice, lane, warp); break;
      default: expand_stage<64, MODE, STAGED>(p, h, st, offs, zf, zseg, zslice, lane, warp); break;
    }
    __syncwarp();
    if (lane == 0) mbar_arrive(&empty[stage]);
  }
}

// ====================================================================== one-launch decode
// sgmv_cluster_kernel: a whole decode shrink -> expand in one launch, z kept in shared
// memory (S*r <= 64).  One thread-block cluster of C CTAs per segment, CTA rank q of
// segment s at blockIdx.x = s*C + q:
//   1. the producer streams chunks [q*cpp, (q+1)*cpp) of K through the stage ring (the
//      segment's x rows and its S*r live A rows, laid out as the shrink kernel's stages)
//      and the consumers accumulate the CTA's part of z in registers (the shrink's
//      register path);
//   2. the CTA's partial goes to its shared memory; after a cluster barrier every CTA
//      adds the C partials in rank order from the cluster's distributed shared memory, so
//      all C CTAs hold the same z (deterministic, no workspace, no counters);
//   3. rank q expands the output columns [q*upp, (q+1)*upp) x 128 of the segment with the
//      expand kernel's stages and consumers, reading z from shared memory.
// The producer issues its expand stages (B rows, y rows) as soon as its shrink stages are
// issued, so they are in flight while the cluster sums z.  Every thread of the cluster
// passes two cluster barriers exactly once, also after an expired wait: #1 between the
// partials and their sum (the producer arrives as soon as its shrink stages are issued),
// #2 at the end, so that no CTA leaves while a peer may still read its partial.
__device__ __forceinline__ void cluster_arrive() { asm volatile("barrier.cluster.arrive;" ::: "memory"); }
__device__ __forceinline__ void cluster_wait() { asm volatile("barrier.cluster.wait;" ::: "memory"); }

template <int MODE, bool STAGED>
__global__ void __launch_bounds__(kThreads, 2) sgmv_cluster_kernel(const __grid_constant__ Params p) {
  extern __shared__ __align__(128) uint8_t smem[];
  __shared__ Seg seg_s;
  __shared__ int tok_s[kSeg];
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int NS = p.stages, SB = p.stage_bytes;
  const int hoff = SB - kHeaderBytes;
  const int xpitch = p.kc * 2 + kRowPad;
  float* red = reinterpret_cast<float*>(smem + NS * SB);  // [warp][16 rows][8 cols]
  float* zpart = red + kConsumerWarps * kSeg * 8;         // [16][kZsPitch]: this CTA's K part
  float* zs = zpart + kSeg * kZsPitch;                    // [16][kZsPitch]: the segment's z
  uint64_t* full = reinterpret_cast<uint64_t*>(zs + kSeg * kZsPitch);
  uint64_t* empty = full + kMaxStages;
  int* offs = reinterpret_cast<int*>(empty + kMaxStages);

  if (tid == 0) {
    for (int s = 0; s < NS; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], kConsumerWarps);
    }
    fence_mbar_init();
  }
  if (tid <= p.S) offs[tid] = p.slice_offsets[tid];
  if (tid == kConsumers) {
    asm volatile("prefetch.tensormap [%0];" ::"l"(&p.tmap_a) : "memory");
    for (int h = 0; h < 3; ++h) asm volatile("prefetch.tensormap [%0];" ::"l"(&p.tmap_a_rows[h]) : "memory");
  }
  __syncthreads();
  pdl_wait();  // x, y and the metadata may come from the preceding grid
  pdl_launch_dependents();

  cg::cluster_group cluster = cg::this_cluster();
  const int C = int(cluster.num_blocks());
  const int q = int(cluster.block_rank());
  const int seg = int(blockIdx.x) / C;
  if (seg >= segment_total(p)) return;  // the whole cluster: one segment, one count
  if (warp == kConsumerWarps) {
    int tok;
    const Seg s = load_segment_warp(p, seg, lane, tok);
    if (lane < kSeg) tok_s[lane] = tok;
    if (lane == 0) seg_s = s;
  }
  __syncthreads();
  const Seg si = seg_s;
  if (!si.ok) return;  // every CTA of the cluster read the same metadata
  const int R = p.S * si.r;
  const int cpp = (p.nchunks + C - 1) / C;
  const int c0 = min(p.nchunks, q * cpp), c1 = min(p.nchunks, c0 + cpp);
  const int ncb = (p.N + kExpandCols - 1) / kExpandCols;
  const int upp = (ncb + C - 1) / C;
  const int u0 = min(ncb, q * upp), u1 = min(ncb, u0 + upp);

  if (warp == kConsumerWarps) {
    // ------------------------------------------------------------ producer warp
    Ring ring;
    bool alive = true;
    const int bw = p.kc < 256 ? p.kc : 256;
    const int groups = (R + 7) >> 3;
    const int row0 = si.g * p.S * p.cap;
    const int tok = lane < kSeg ? tok_s[lane] : -1;
    for (int c = c0; c < c1; ++c) {
      const int stage = ring.stage;
      const uint32_t phase = ring.phase;
      ring.next(NS);
      int ok = 1;
      if (lane == 0) ok = mbar_wait(&empty[stage], phase ^ 1u) ? 1 : 0;
      if (!__shfl_sync(0xffffffffu, ok, 0)) {
        alive = false;
        break;
      }
      uint8_t* st = smem + stage * SB;
      const int k0 = c * p.kc;
      const int len = min(p.kc, p.K - k0);
      const int boxes = (len + bw - 1) / bw;
      const uint32_t row_bytes = uint32_t(len) * 2;
      const uint32_t tx = uint32_t(si.n) * row_bytes + uint32_t(groups * boxes) * (8 * bw * 2);
      __syncwarp();
      if (lane == 0) mbar_arrive_expect_tx(&full[stage], tx);
      __syncwarp();
      if (lane < si.n)
        bulk_g2s(st + lane * xpitch, p.x + int64_t(tok) * p.x_stride + k0, row_bytes, &full[stage]);
      uint8_t* abase = st + kSeg * xpitch;
      if (p.kc <= 256) {
        if (lane == 0)
          for (int r0 = 0, left = groups * 8; left > 0;) {
            const int h = left >= 64 ? 64 : left >= 32 ? 32 : left >= 16 ? 16 : 8;
            const CUtensorMap* map = h == 64   ? &p.tmap_a_rows[0]
                                     : h == 32 ? &p.tmap_a_rows[1]
                                     : h == 16 ? &p.tmap_a_rows[2]
                                               : &p.tmap_a;
            tma_load_2d(abase + r0 * bw * 2, map, k0, row0 + r0, &full[stage]);
            r0 += h;
            left -= h;
          }
      } else {
        for (int i = lane; i < groups * boxes; i += 32) {
          const int grp = i / boxes, box = i - grp * boxes;
          tma_load_2d(abase + (grp * (p.kc / bw) + box) * (8 * bw * 2), &p.tmap_a, k0 + box * bw,
                      row0 + grp * 8, &full[stage]);
        }
      }
    }
    __syncwarp();
    cluster_arrive();  // #1: the producer takes no part in the z sum
    // Expand stages: consecutive 128-column units merged while B rows fit p.bstage.
    for (int u = u0; u < u1 && alive;) {
      const int cb = u;
      const int max_cols = min(kStageCols, p.bstage / (2 * si.bucket));  // >= kExpandCols
      const int take = min(max_cols / kExpandCols, u1 - u);
      const int cc0 = cb * kExpandCols;
      const int nc = min(p.N, (cb + take) * kExpandCols) - cc0;
      u += take;
      const int stage = ring.stage;
      const uint32_t phase = ring.phase;
      ring.next(NS);
      int ok = 1;
      if (lane == 0) ok = mbar_wait(&empty[stage], phase ^ 1u) ? 1 : 0;
      if (!__shfl_sync(0xffffffffu, ok, 0)) {
        alive = false;
        break;
      }
      uint8_t* st = smem + stage * SB;
      ExpandHeader* h = reinterpret_cast<ExpandHeader*>(st + hoff);
      if (lane == 0) {
        const int s0 = slice_of(offs, p.S, cc0), s1 = slice_of(offs, p.S, cc0 + nc - 1);
        h->ok = 1;
        h->seg = seg;
        h->n = si.n;
        h->r = si.r;
        h->bucket = si.bucket;
        h->pos0 = si.pos0;
        h->col0 = cc0;
        h->ncols = nc;
        h->slice = s0 == s1 ? s0 : -1;
        h->scale = si.scale;
      }
      if (lane < kSeg) h->tok[lane] = tok;
      const uint16_t* bsrc = p.b + si.boff + int64_t(cc0) * si.bucket;
      const uint32_t bbytes = uint32_t(nc) * si.bucket * 2;
      const uint32_t bbulk = bbytes & ~15u;
      for (uint32_t i = bbulk / 2 + lane; i < bbytes / 2; i += 32)
        reinterpret_cast<uint16_t*>(st)[i] = bsrc[i];
      const uint32_t ybytes = STAGED ? uint32_t(nc) * 2 : 0u;
      __syncwarp();
      if (lane == 0) mbar_arrive_expect_tx(&full[stage], bbulk + uint32_t(si.n) * ybytes);
      __syncwarp();
      if (lane == 31 && bbulk) bulk_g2s(st, bsrc, bbulk, &full[stage]);
      if (STAGED && lane < si.n)
        bulk_g2s(st + p.bstage + lane * kYStagePitch, p.y + int64_t(tok) * p.y_stride + cc0, ybytes,
                 &full[stage]);
    }
    if (alive) {  // end of stream
      const int stage = ring.stage;
      int ok = 1;
      if (lane == 0) ok = mbar_wait(&empty[stage], ring.phase ^ 1u) ? 1 : 0;
      if (__shfl_sync(0xffffffffu, ok, 0) && lane == 0) {
        reinterpret_cast<ExpandHeader*>(smem + stage * SB + hoff)->ok = -1;
        mbar_arrive(&full[stage]);
      }
    }
    __syncwarp();
    cluster_wait();  // #1
    cluster_arrive();
    cluster_wait();  // #2
    return;
  }

  // -------------------------------------------------------------- consumer warps
  const int g = lane >> 2, t = lane & 3;
  const int ntiles = (R + 7) >> 3;  // 1..8 (S*r <= 64)
  const int kparts = kConsumerWarps / ntiles;
  const int tile = warp / kparts, kpart = warp - tile * kparts;
  float d[4] = {0.f, 0.f, 0.f, 0.f};
  bool aborted = false;
  Ring ring;
  for (int c = c0; c < c1; ++c, ring.next(NS)) {
    const int stage = ring.stage;
    if (!mbar_wait(&full[stage], ring.phase)) {
      aborted = true;
      break;
    }
    const uint8_t* st = smem + stage * SB;
    const int len = min(p.kc, p.K - c * p.kc);
    if (tile < ntiles) shrink_unit_regs(st, xpitch, p.kc, len, tile, kpart, kparts, g, t, d);
    __syncwarp();
    if (lane == 0) mbar_arrive(&empty[stage]);
  }
  aborted = !consumers_all(!aborted);
  // This CTA's part of z: warps of one n tile hold interleaved k blocks; add them in
  // warp order.  Rows past the segment's tokens are never read.
  float* rw = red + warp * kSeg * 8;
  *reinterpret_cast<float2*>(rw + g * 8 + 2 * t) = make_float2(d[0], d[1]);
  *reinterpret_cast<float2*>(rw + (g + 8) * 8 + 2 * t) = make_float2(d[2], d[3]);
  consumers_sync();
  for (int e = tid; e < kSeg * kZsPitch; e += kConsumers) {
    const int m = e / kZsPitch, j = e - m * kZsPitch;
    float s = 0.f;
    if (j < R)
      for (int k = 0; k < kparts; ++k) s += red[(((j >> 3) * kparts + k) * kSeg + m) * 8 + (j & 7)];
    zpart[e] = s;
  }
  cluster_arrive();
  cluster_wait();  // #1: every CTA's partial is written
  for (int e = tid; e < kSeg * kZsPitch; e += kConsumers) {
    float s = 0.f;
    for (int r = 0; r < C; ++r) s += cluster.map_shared_rank(zpart, r)[e];
    zs[e] = s;
  }
  consumers_sync();
  if (!aborted) {
    uint32_t zf[4][2][4];
    int zseg = -1, zslice = -1;
    for (;; ring.next(NS)) {
      const int stage = ring.stage;
      if (!mbar_wait(&full[stage], ring.phase)) break;
      const uint8_t* st = smem + stage * SB;
      const ExpandHeader& h = *reinterpret_cast<const ExpandHeader*>(st + hoff);
      if (h.ok < 0) break;
      if (STAGED && h.slice >= 0) {
        if (h.bucket == 64) expand_stage_pair<64, MODE, true>(p, h, st, zf, zseg, zslice, lane, warp, zs);
        else if (h.bucket == 32) expand_stage_pair<32, MODE, true>(p, h, st, zf, zseg, zslice, lane, warp, zs);
        else if (h.bucket == 16) expand_stage_pair<16, MODE, true>(p, h, st, zf, zseg, zslice, lane, warp, zs);
        else expand_stage_pair<8, MODE, true>(p, h, st, zf, zseg, zslice, lane, warp, zs);
      } else switch (h.bucket < 8 ? 8 : h.bucket) {
        case 8: expand_stage<8, MODE, STAGED, true>(p, h, st, offs, zf, zseg, zslice, lane, warp, zs); break;
        case 16: expand_stage<16, MODE, STAGED, true>(p, h, st, offs, zf, zseg, zslice, lane, warp, zs); break;
        case 32: expand_stage<32, MODE, STAGED, true>(p, h, st, offs, zf, zseg, zslice, lane, warp, zs); break;
        default: expand_stage<64, MODE, STAGED, true>(p, h, st, offs, zf, zseg, zslice, lane, warp, zs); break;
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(&empty[stage]);
    }
  }
  cluster_arrive();
  cluster_wait();  // #2: no peer reads this CTA's partial any more
}

// ====================================================================== host side
struct ShrinkConfig {
  int rstride, kc, nchunks, stages, stage_bytes, smem;
};

inline int round_up(int v, int m) { return (v + m - 1) / m * m; }

inline int shrink_stage_bytes(int rstride, int kc) {
  return round_up(kSeg * (kc * 2 + kRowPad) + rstride * kc * 2 + kHeaderBytes, 128);
}

// Register path (S*r <= 64): two CTAs per SM.  Wide path: one.  The K chunk is the widest
// of 512 / 256 / 128 columns whose stage fits 52 KiB: each unit reads a chunk-wide piece of
// every live A row, and 1 KiB pieces (kc = 512) stream from HBM markedly faster than 512-byte
// ones when a projection's rows are long (rank 32, K = 27648: 148.8 -> 128.8 us per call).
inline ShrinkConfig shrink_config(int64_t width, int num_slices, int capacity) {
  ShrinkConfig c{};
  c.rstride = round_up(num_slices * (capacity < kMaxRank ? capacity : kMaxRank), 8);
  const bool regs = c.rstride <= 64;
  int kc = 64;
  for (int cand : {512, 256, 128}) {
    if (shrink_stage_bytes(c.rstride, cand) <= 52 * 1024) {
      kc = cand;
      break;
    }
  }
  while (kc > 64 && kc / 2 >= width) kc /= 2;
  c.kc = kc;
  c.nchunks = int((width + kc - 1) / kc);
  c.stage_bytes = shrink_stage_bytes(c.rstride, kc);
  const int fixed = (regs ? kConsumerWarps * kSeg * 8 * 4 : kRedBytes + kSeg * c.rstride * 4) +
                    2 * kMaxStages * 8 + 16;
  const int budget = regs ? kStageBudget : 2 * kStageBudget;
  int stages = (budget - fixed) / c.stage_bytes;
  c.stages = stages < 2 ? 2 : (stages > 4 ? 4 : stages);
  c.smem = c.stages * c.stage_bytes + fixed;
  return c;
}

// cuTensorMapEncodeTiled through the runtime's driver entry point (no libcuda link).
inline PFN_cuTensorMapEncodeTiled_v12000 tensor_map_encoder() {
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

struct ExpandConfig {
  int stages, stage_bytes, smem;
};

// B rows per stage: 32 KiB when a slot's bucket can reach 32 (a 512-column stage of rank-32
// rows: half as many stages, each moving twice the bytes; config 4 390 -> 371 us/step,
// config 2 71.0 -> 68.0), else 16 KiB, which keeps three stages in flight for rank-16 and
// smaller buckets (their 512 columns fit 16 KiB; 32 KiB stages measured 102.7 -> 108.7 us/step
// on config 1).
inline int expand_bstage(int capacity) {
  return (capacity > 16 ? 32 : 16) * 1024;
}

inline ExpandConfig expand_config(bool staged, int bstage) {
  ExpandConfig c{};
  c.stage_bytes = round_up(bstage + (staged ? kSeg * kYStagePitch : 0) + kHeaderBytes, 128);
  int stages = kStageBudget / c.stage_bytes;
  c.stages = stages < 2 ? 2 : (stages > kMaxStages ? kMaxStages : stages);
  c.smem = c.stages * c.stage_bytes + 2 * kMaxStages * 8 + (kMaxSlices + 4) * 4;
  return c;
}

// The one-launch kernel (sgmv_cluster_kernel): the register path only (S*r <= 64); one
// stage size for both phases (the larger of a shrink stage and an expand stage), at least
// two stages in the two-CTA budget; the widest K chunk that allows that.  Cluster size C:
// the segment's A and B bytes (at the capacity's rank and bucket) over 256 KiB, rounded up
// to a power of two, at most 8.  Taken only when a segment's B rows are no more bytes than
// its A rows: BASELINE config 1 measured qkv 31.6 -> 29.7 us and down 29.2 -> 29.7 us with
// it, but gate_up (B 3.5x A) 48.1 -> 73.8 us, its expand spread over a cluster per segment
// in two waves instead of the persistent expand's balanced split.
struct ClusterConfig {
  bool ok;
  int C, kc, nchunks, stages, stage_bytes, smem;
};

inline ClusterConfig cluster_config(int64_t width, int out_width, int num_slices, int capacity,
                                    bool staged, int bstage) {
  ClusterConfig c{};
  const int cap = capacity < kMaxRank ? capacity : kMaxRank;
  const int rstride = round_up(num_slices * cap, 8);
  if (rstride > 64) return c;
  const int fixed = kConsumerWarps * kSeg * 8 * 4 + 2 * kSeg * kZsPitch * 4 + 2 * kMaxStages * 8 +
                    (kMaxSlices + 4) * 4;
  const int ebytes = round_up(bstage + (staged ? kSeg * kYStagePitch : 0) + kHeaderBytes, 128);
  int kc = 0;
  for (int cand : {512, 256, 128, 64}) {
    const int sb = std::max(shrink_stage_bytes(rstride, cand), ebytes);
    if (2 * sb + fixed <= kStageBudget) {
      kc = cand;
      break;
    }
  }
  if (kc == 0) return c;
  while (kc > 64 && kc / 2 >= width) kc /= 2;
  c.kc = kc;
  c.nchunks = int((width + kc - 1) / kc);
  c.stage_bytes = std::max(shrink_stage_bytes(rstride, kc), ebytes);
  const int stages = (kStageBudget - fixed) / c.stage_bytes;
  c.stages = stages > kMaxStages ? kMaxStages : stages;
  c.smem = c.stages * c.stage_bytes + fixed;
  int bucket = 1;
  while (bucket < cap) bucket *= 2;
  const int64_t seg_bytes = int64_t(rstride) * width * 2 + int64_t(out_width) * bucket * 2;
  int C = 1;
  while (C < 8 && seg_bytes > int64_t(C) * 256 * 1024) C *= 2;
  c.C = C;
  c.ok = int64_t(out_width) * bucket <= int64_t(rstride) * width;
  return c;
}

inline int64_t scratch_floats(int64_t tokens, const ShrinkConfig& c) {
  const int64_t T = tokens > 0 ? tokens : 1;
  return (int64_t(c.nchunks) + 1) * T * c.rstride + (T + 3) / 4 * 4;
}

template <typename Kernel>
int launch_pdl(Kernel kernel, int grid, int smem, cudaStream_t stream, const Params& p,
               const char* what) {
  cudaLaunchConfig_t config = {};
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  config.attrs = attr;
  config.numAttrs = 1;
  config.gridDim = dim3(grid);
  config.blockDim = dim3(kThreads);
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

using namespace lfb;

extern "C" int64_t lf_fused_workspace_floats(int64_t num_tokens, int64_t width,
                                             int32_t num_slices, int32_t capacity) {
  if (num_tokens < 0 || width < 1 || num_slices < 1 || num_slices > kMaxSlices || capacity < 1)
    return -1;
  return scratch_floats(num_tokens, shrink_config(width, num_slices, capacity));
}

namespace lfb {
int64_t decode_scratch_floats(int64_t num_tokens, int64_t width, int num_slices, int capacity) {
  return scratch_floats(num_tokens, shrink_config(width, num_slices, capacity));
}

Scratch decode_scratch(float* region, int64_t num_tokens, int64_t width, int num_slices,
                       int capacity) {
  const ShrinkConfig sc = shrink_config(width, num_slices, capacity);
  const int64_t T = num_tokens > 0 ? num_tokens : 1;
  return Scratch{region, reinterpret_cast<int*>(region + (int64_t(sc.nchunks) + 1) * T * sc.rstride)};
}
}  // namespace lfb

namespace {
// Validates a caller-provided workspace and runs the requested phases.
int workspace_launch(
    const void* x, int64_t x_stride, const void* a, const void* b, const int64_t* b_offsets,
    const int32_t* b_strides, void* y, int64_t y_stride, const int32_t* segment_indptr,
    const int32_t* segment_slots, const int32_t* token_indices, const int32_t* ranks,
    const float* scales, const int32_t* slice_offsets, const int32_t* segment_count,
    float* workspace, int64_t workspace_floats, int64_t num_tokens, int64_t width,
    int32_t out_width, int32_t num_slices, int32_t capacity, int32_t num_slots,
    int32_t max_segments, int32_t numerics, void* stream, int phases) {
  if (num_tokens < 0 || num_tokens >= (int64_t(1) << 31) || width < 1 || width >= (int64_t(1) << 31))
    return fail(LF_E_INVALID, "fused_shrink_expand: invalid token count or width");
  if (num_slices < 1 || num_slices > kMaxSlices || capacity < 1)
    return fail(LF_E_INVALID, "fused_shrink_expand: invalid slices or capacity");
  const ShrinkConfig sc = shrink_config(width, num_slices, capacity);
  const int64_t need = scratch_floats(num_tokens, sc);
  if (!workspace || workspace_floats < need || (reinterpret_cast<uintptr_t>(workspace) & 15))
    return fail(LF_E_INVALID, "fused_shrink_expand: workspace too small or not 16-byte aligned "
                              "(see lf_fused_workspace_floats)");
  const Scratch scratch = decode_scratch(workspace, num_tokens, width, num_slices, capacity);
  return fused_launch(x, x_stride, a, b, b_offsets, b_strides, y, y_stride, segment_indptr,
                      segment_slots, token_indices, ranks, scales, slice_offsets, segment_count,
                      scratch, num_tokens, width, out_width, num_slices, capacity, num_slots,
                      max_segments, numerics, kSeg, stream, phases);
}
}  // namespace

extern "C" int lf_fused_shrink_expand(
    const void* x, int64_t x_stride, const void* a, const void* b, const int64_t* b_offsets,
    const int32_t* b_strides, void* y, int64_t y_stride, const int32_t* segment_indptr,
    const int32_t* segment_slots, const int32_t* token_indices, const int32_t* ranks,
    const float* scales, const int32_t* slice_offsets, const int32_t* segment_count,
    float* workspace, int64_t workspace_floats, int64_t num_tokens, int64_t width,
    int32_t out_width, int32_t num_slices, int32_t capacity, int32_t num_slots,
    int32_t max_segments, int32_t numerics, void* stream) {
  return workspace_launch(x, x_stride, a, b, b_offsets, b_strides, y, y_stride, segment_indptr,
                          segment_slots, token_indices, ranks, scales, slice_offsets, segment_count,
                          workspace, workspace_floats, num_tokens, width, out_width, num_slices,
                          capacity, num_slots, max_segments, numerics, stream,
                          kPhaseShrink | kPhaseExpand);
}

// The two halves of lf_fused_shrink_expand, for callers that combine z across devices
// between them (row-parallel LoRA): z rows are left in the workspace by the shrink and
// read by the expand; lf_fused_z_rows tells where.
extern "C" int lf_sgmv_shrink(
    const void* x, int64_t x_stride, const void* a, const void* b, const int64_t* b_offsets,
    const int32_t* b_strides, void* y, int64_t y_stride, const int32_t* segment_indptr,
    const int32_t* segment_slots, const int32_t* token_indices, const int32_t* ranks,
    const float* scales, const int32_t* slice_offsets, const int32_t* segment_count,
    float* workspace, int64_t workspace_floats, int64_t num_tokens, int64_t width,
    int32_t out_width, int32_t num_slices, int32_t capacity, int32_t num_slots,
    int32_t max_segments, int32_t numerics, void* stream) {
  return workspace_launch(x, x_stride, a, b, b_offsets, b_strides, y, y_stride, segment_indptr,
                          segment_slots, token_indices, ranks, scales, slice_offsets, segment_count,
                          workspace, workspace_floats, num_tokens, width, out_width, num_slices,
                          capacity, num_slots, max_segments, numerics, stream, kPhaseShrink);
}

extern "C" int lf_sgmv_expand(
    const void* x, int64_t x_stride, const void* a, const void* b, const int64_t* b_offsets,
    const int32_t* b_strides, void* y, int64_t y_stride, const int32_t* segment_indptr,
    const int32_t* segment_slots, const int32_t* token_indices, const int32_t* ranks,
    const float* scales, const int32_t* slice_offsets, const int32_t* segment_count,
    float* workspace, int64_t workspace_floats, int64_t num_tokens, int64_t width,
    int32_t out_width, int32_t num_slices, int32_t capacity, int32_t num_slots,
    int32_t max_segments, int32_t numerics, void* stream) {
  return workspace_launch(x, x_stride, a, b, b_offsets, b_strides, y, y_stride, segment_indptr,
                          segment_slots, token_indices, ranks, scales, slice_offsets, segment_count,
                          workspace, workspace_floats, num_tokens, width, out_width, num_slices,
                          capacity, num_slots, max_segments, numerics, stream, kPhaseExpand);
}

extern "C" int lf_fused_z_rows(int64_t num_tokens, int64_t width, int32_t num_slices,
                               int32_t capacity, int64_t* offset, int64_t* row_floats) {
  if (num_tokens < 0 || width < 1 || num_slices < 1 || num_slices > kMaxSlices || capacity < 1 ||
      !offset || !row_floats)
    return fail(LF_E_INVALID, "fused_z_rows: invalid sizes");
  const ShrinkConfig sc = shrink_config(width, num_slices, capacity);
  const int64_t T = num_tokens > 0 ? num_tokens : 1;
  *offset = int64_t(sc.nchunks) * T * sc.rstride;
  *row_floats = sc.rstride;
  return LF_OK;
}

namespace lfb {
int fused_launch(const void* x, int64_t x_stride, const void* a, const void* b,
                 const int64_t* b_offsets, const int32_t* b_strides, void* y, int64_t y_stride,
                 const int32_t* segment_indptr, const int32_t* segment_slots,
                 const int32_t* token_indices, const int32_t* ranks, const float* scales,
                 const int32_t* slice_offsets, const int32_t* segment_count, const Scratch& scratch,
                 int64_t num_tokens, int64_t width, int32_t out_width, int32_t num_slices,
                 int32_t capacity, int32_t num_slots, int32_t max_segments, int32_t numerics,
                 int max_tokens, void* stream, int phases) {
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
  const ShrinkConfig sc = shrink_config(width, num_slices, capacity);
  if (num_tokens == 0 || max_segments == 0) return LF_OK;
  const bool staged = out_width % 8 == 0 && y_stride % 8 == 0 &&
                      (reinterpret_cast<uintptr_t>(y) & 15) == 0;
  const int bstage = expand_bstage(capacity);
  const ExpandConfig ec = expand_config(staged, bstage);
  const int64_t T = num_tokens;
  Params p{static_cast<const uint16_t*>(x), x_stride, static_cast<const uint16_t*>(a),
           static_cast<const uint16_t*>(b), b_offsets, b_strides, static_cast<uint16_t*>(y),
           y_stride, segment_indptr, segment_slots, token_indices, ranks, scales, slice_offsets,
           segment_count, scratch.data, scratch.data + int64_t(sc.nchunks) * T * sc.rstride,
           scratch.counters, int(T), int(width), out_width, num_slices, capacity, num_slots, max_segments,
           sc.rstride, sc.kc, sc.nchunks, sc.stages, sc.stage_bytes, max_tokens};
  // Both phases in one call and the register path: one launch, z in shared memory.
  const ClusterConfig cc = cluster_config(width, out_width, num_slices, capacity, staged, bstage);
  const bool one_launch = phases == (kPhaseShrink | kPhaseExpand) && cc.ok;
  if (one_launch) {
    p.kc = cc.kc;
    p.nchunks = cc.nchunks;
  }
  {
    // A as a 2-D tensor [num_slots*S*cap rows, K columns] for the shrink's TMA boxes.
    const PFN_cuTensorMapEncodeTiled_v12000 encode = tensor_map_encoder();
    if (!encode) return fail(LF_E_CUDA, "fused_shrink_expand: cuTensorMapEncodeTiled unavailable");
    const cuuint64_t dims[2] = {cuuint64_t(width), cuuint64_t(num_slots) * num_slices * capacity};
    const cuuint64_t strides[1] = {cuuint64_t(width) * 2};
    const cuuint32_t box[2] = {cuuint32_t(p.kc < 256 ? p.kc : 256), 8};
    const cuuint32_t estr[2] = {1, 1};
    CUresult r = encode(&p.tmap_a, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(a), dims, strides, box,
                        estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE,
                        CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    for (int h = 0; h < 3 && r == CUDA_SUCCESS; ++h) {
      const cuuint32_t tall[2] = {box[0], cuuint32_t(64 >> h)};
      r = encode(&p.tmap_a_rows[h], CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(a), dims, strides, tall,
                 estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                 CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    }
    if (r != CUDA_SUCCESS) return fail(LF_E_CUDA, "fused_shrink_expand: cuTensorMapEncodeTiled failed");
  }
  int device = 0, sms = 0;
  if (cudaGetDevice(&device) != cudaSuccess ||
      cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, device) != cudaSuccess)
    return check_launch("fused_shrink_expand: device query");
  const cudaStream_t s = static_cast<cudaStream_t>(stream);
  const int64_t seg_cap = max_segments < num_tokens ? max_segments : num_tokens;
  if (seg_cap * sc.nchunks >= (int64_t(1) << 31) ||
      seg_cap * ((out_width + kExpandCols - 1) / kExpandCols) >= (int64_t(1) << 31))
    return fail(LF_E_INVALID, "fused_shrink_expand: too many (segment, chunk) units");
  if (one_launch) {
    p.stages = cc.stages;
    p.stage_bytes = cc.stage_bytes;
    p.bstage = bstage;
    auto kernel = numerics == kFp32
                      ? (staged ? sgmv_cluster_kernel<kFp32, true> : sgmv_cluster_kernel<kFp32, false>)
                      : (staged ? sgmv_cluster_kernel<kReference, true>
                                : sgmv_cluster_kernel<kReference, false>);
    static int flags[4][64] = {};
    if (int rc = ensure_smem(kernel, cc.smem, flags[numerics * 2 + (staged ? 1 : 0)])) return rc;
    if (seg_cap * cc.C >= (int64_t(1) << 31)) return fail(LF_E_INVALID, "fused_shrink_expand: too many segments");
    cudaLaunchConfig_t config = {};
    cudaLaunchAttribute attr[2];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = unsigned(cc.C);
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[1].val.programmaticStreamSerializationAllowed = 1;
    config.attrs = attr;
    config.numAttrs = 2;
    config.gridDim = dim3(unsigned(seg_cap * cc.C));
    config.blockDim = dim3(kThreads);
    config.dynamicSmemBytes = cc.smem;
    config.stream = s;
    const cudaError_t err = cudaLaunchKernelEx(&config, kernel, p);
    if (err != cudaSuccess) {
      last_error() = std::string("fused_shrink_expand (one launch): ") + cudaGetErrorString(err);
      return LF_E_CUDA;
    }
    return LF_OK;
  }
  if (phases & kPhaseShrink) {
    // Up to 8 n tiles (S*r <= 64) the warps accumulate in registers.
    const bool regs = sc.rstride <= 64;
    auto shrink = regs ? sgmv_shrink_kernel<true> : sgmv_shrink_kernel<false>;
    static int flags[2][64] = {};
    if (int rc = ensure_smem(shrink, sc.smem, flags[regs ? 1 : 0])) return rc;
    const int64_t units = seg_cap * sc.nchunks;
    const int64_t ctas = int64_t(regs ? 2 : 1) * sms;
    const int grid = int(units < ctas ? units : ctas);
    if (int rc = launch_pdl(shrink, grid, sc.smem, s, p, "fused_shrink_expand (shrink)")) return rc;
  }
  if (!(phases & kPhaseExpand)) return LF_OK;
  p.stages = ec.stages;
  p.stage_bytes = ec.stage_bytes;
  p.bstage = bstage;
  const int64_t units = seg_cap * ((out_width + kExpandCols - 1) / kExpandCols);
  const int grid = int(units < 2 * sms ? units : 2 * sms);
  auto kernel = numerics == kFp32
                    ? (staged ? sgmv_expand_kernel<kFp32, true> : sgmv_expand_kernel<kFp32, false>)
                    : (staged ? sgmv_expand_kernel<kReference, true>
                              : sgmv_expand_kernel<kReference, false>);
  static int flags[4][64] = {};
  if (int rc = ensure_smem(kernel, ec.smem, flags[numerics * 2 + (staged ? 1 : 0)])) return rc;
  return launch_pdl(kernel, grid, ec.smem, s, p, "fused_shrink_expand (expand)");
}
}  // namespace lfb

extern "C" int lf_device_wait_timeouts(int32_t* count, int32_t reset) {
  unsigned int value = 0;
  if (cudaMemcpyFromSymbol(&value, g_lf_wait_timeouts, sizeof(value)) != cudaSuccess)
    return check_launch("device_wait_timeouts");
  unsigned int prefill = 0;
  if (int rc = prefill_wait_timeouts(&prefill, reset)) return rc;
  if (count) *count = int32_t(value + prefill);
  if (reset) {
    const unsigned int zero = 0;
    if (cudaMemcpyToSymbol(g_lf_wait_timeouts, &zero, sizeof(zero)) != cudaSuccess)
      return check_launch("device_wait_timeouts");
  }
  return LF_OK;
}

// ------------------------------------------------------------------ allocation-free entry
// lf_fused_shrink_expand_noalloc runs the same two kernels as lf_fused_shrink_expand
// but takes its scratch from fixed buffers compiled into this library, for callers
// that are not allowed to allocate device memory themselves.
namespace {
// 4 Mi floats (16 MiB) of partial sums and z rows, and one completion counter for each
// of up to kNoAllocTokens segments at a fixed position (so calls of different sizes
// may follow one another).  Static __device__ arrays are created on every GPU that
// loads this library, zero-filled, and live until the process exits.
constexpr int64_t kNoAllocScratchFloats = int64_t(4) << 20;
constexpr int64_t kNoAllocTokens = 16384;
static __device__ __align__(256) float g_noalloc_scratch[kNoAllocScratchFloats];
static __device__ __align__(256) int g_noalloc_counters[kNoAllocTokens];

// Device addresses of the two arrays, per device index, with the context they were
// looked up in: after a context is torn down and created again (cudaDeviceReset) the
// module is loaded at new addresses, so an entry whose context is no longer current is
// looked up again.
struct NoAllocAddress {
  void* context = nullptr;
  float* scratch = nullptr;
  int* counters = nullptr;
};
std::mutex g_noalloc_mutex;
NoAllocAddress g_noalloc[64];

using CtxGetCurrent = CUresult (*)(CUcontext*);
CtxGetCurrent ctx_get_current() {
  static CtxGetCurrent fn = nullptr;
  static bool tried = false;
  if (!tried) {  // called under g_noalloc_mutex
    tried = true;
    void* ptr = nullptr;
    cudaDriverEntryPointQueryResult status;
    if (cudaGetDriverEntryPoint("cuCtxGetCurrent", &ptr, cudaEnableDefault, &status) == cudaSuccess &&
        status == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<CtxGetCurrent>(ptr);
  }
  return fn;
}

// The built-in arrays' device addresses on the current device (looked up with it current).
int noalloc_scratch(const char* what, Scratch* out) {
  int device = 0;
  if (cudaGetDevice(&device) != cudaSuccess) return check_launch(what);
  if (device < 0 || device >= 64) return fail(LF_E_UNSUPPORTED, "noalloc: device index above 63");
  std::lock_guard<std::mutex> lock(g_noalloc_mutex);
  CtxGetCurrent get = ctx_get_current();
  CUcontext ctx = nullptr;
  if (get && get(&ctx) != CUDA_SUCCESS) ctx = nullptr;
  NoAllocAddress& entry = g_noalloc[device];
  if (!entry.scratch || !ctx || entry.context != static_cast<void*>(ctx)) {
    // cudaGetSymbolAddress makes the device's primary context current if none is yet.
    void* address = nullptr;
    void* counters = nullptr;
    cudaError_t err = cudaGetSymbolAddress(&address, g_noalloc_scratch);
    if (err == cudaSuccess) err = cudaGetSymbolAddress(&counters, g_noalloc_counters);
    if (err != cudaSuccess || !address || !counters) {
      last_error() = std::string(what) + ": cudaGetSymbolAddress: " + cudaGetErrorString(err);
      return LF_E_CUDA;
    }
    if (get && get(&ctx) != CUDA_SUCCESS) ctx = nullptr;
    entry.context = ctx;
    entry.scratch = static_cast<float*>(address);
    entry.counters = static_cast<int*>(counters);
  }
  *out = Scratch{entry.scratch, entry.counters};
  return LF_OK;
}
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
  if (need > kNoAllocScratchFloats || num_tokens > kNoAllocTokens) {
    last_error() = "fused_shrink_expand_noalloc: these sizes need " + std::to_string(need) +
                   " floats of scratch for " + std::to_string(num_tokens) +
                   " tokens, more than the built-in " + std::to_string(kNoAllocScratchFloats) +
                   "-float (16 MiB) buffer or " + std::to_string(kNoAllocTokens) +
                   " tokens; use lf_fused_shrink_expand with a workspace";
    return LF_E_INVALID;
  }
  Scratch scratch{};
  if (int rc = noalloc_scratch("fused_shrink_expand_noalloc", &scratch)) return rc;
  return fused_launch(x, x_stride, a, b, b_offsets, b_strides, y, y_stride, segment_indptr,
                      segment_slots, token_indices, ranks, scales, slice_offsets, segment_count,
                      scratch, num_tokens, width, out_width, num_slices, capacity, num_slots,
                      max_segments, numerics, kSeg, stream, kPhaseShrink | kPhaseExpand);
}

// Zero the completion counters of the library's built-in scratch on the current device
// (cudaMemsetAsync on the stream; allocates nothing).
extern "C" int lf_fused_noalloc_reset(void* stream) {
  Scratch scratch{};
  if (int rc = noalloc_scratch("fused_noalloc_reset", &scratch)) return rc;
  if (cudaMemsetAsync(scratch.counters, 0, sizeof(int) * kNoAllocTokens,
                      static_cast<cudaStream_t>(stream)) != cudaSuccess)
    return check_launch("fused_noalloc_reset");
  return LF_OK;
}

// Zero the completion counters of a caller-owned decode workspace (cudaMemsetAsync).
extern "C" int lf_fused_workspace_reset(float* workspace, int64_t workspace_floats, int64_t num_tokens,
                                        int64_t width, int32_t num_slices, int32_t capacity,
                                        void* stream) {
  const int64_t need = lf_fused_workspace_floats(num_tokens, width, num_slices, capacity);
  if (need < 0) return fail(LF_E_INVALID, "fused_workspace_reset: invalid sizes");
  if (!workspace || workspace_floats < need)
    return fail(LF_E_INVALID, "fused_workspace_reset: workspace too small for these sizes");
  const Scratch scratch = decode_scratch(workspace, num_tokens, width, num_slices, capacity);
  const int64_t T = num_tokens > 0 ? num_tokens : 1;
  if (cudaMemsetAsync(scratch.counters, 0, sizeof(int) * size_t(T),
                      static_cast<cudaStream_t>(stream)) != cudaSuccess)
    return check_launch("fused_workspace_reset");
  return LF_OK;
}
