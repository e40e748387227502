// Device-side stable grouping of decode/prefill tokens by adapter slot.
//
// One CTA of 1024 threads: a shared-memory histogram of slot ids, two block-wide
// exclusive scans (token offsets per slot and segment offsets per slot) and a
// stable scatter done by one warp with __match_any_sync ranks.  The result is the
// routing table SGLang's prepare_lora_batch produces for the reference
// (seg_indptr / weight_indices / permutation, consumed at
// src/loraforge/integrations/_sglang_fleet.py:390-407), computed without a host
// round trip so it can live inside a CUDA graph.
#include <string>

#include "launch.cuh"

namespace lfb {
namespace {

constexpr int kGroupThreads = 1024;
constexpr int kGroupWarps = kGroupThreads / 32;

// Exclusive scan of two int arrays of length n in shared memory, in place, with all
// 1024 threads.  Returns the totals through *total_a / *total_b (shared).
__device__ void block_exclusive_scan2(int* a, int* b, int n, int* warp_a, int* warp_b,
                                      int* total_a, int* total_b) {
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int per = (n + kGroupThreads - 1) / kGroupThreads;
  const int begin = min(n, tid * per), end = min(n, begin + per);
  int sa = 0, sb = 0;
  for (int i = begin; i < end; ++i) {
    sa += a[i];
    sb += b[i];
  }
  int ia = sa, ib = sb;  // warp inclusive scan
#pragma unroll
  for (int d = 1; d < 32; d <<= 1) {
    const int va = __shfl_up_sync(0xffffffffu, ia, d);
    const int vb = __shfl_up_sync(0xffffffffu, ib, d);
    if (lane >= d) {
      ia += va;
      ib += vb;
    }
  }
  if (lane == 31) {
    warp_a[warp] = ia;
    warp_b[warp] = ib;
  }
  __syncthreads();
  if (warp == 0) {
    int wa = warp_a[lane], wb = warp_b[lane];
    int xa = wa, xb = wb;
#pragma unroll
    for (int d = 1; d < 32; d <<= 1) {
      const int va = __shfl_up_sync(0xffffffffu, xa, d);
      const int vb = __shfl_up_sync(0xffffffffu, xb, d);
      if (lane >= d) {
        xa += va;
        xb += vb;
      }
    }
    warp_a[lane] = xa - wa;  // exclusive warp offsets
    warp_b[lane] = xb - wb;
    if (lane == 31) {
      *total_a = xa;
      *total_b = xb;
    }
  }
  __syncthreads();
  int ra = warp_a[warp] + ia - sa, rb = warp_b[warp] + ib - sb;
  for (int i = begin; i < end; ++i) {
    const int va = a[i], vb = b[i];
    a[i] = ra;
    b[i] = rb;
    ra += va;
    rb += vb;
  }
  __syncthreads();
}

// Block-wide scans of one int per thread (all kGroupThreads threads call them).
__device__ int block_exclusive_sum(int v, int* wtmp, int* total) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  int x = v;
#pragma unroll
  for (int d = 1; d < 32; d <<= 1) {
    const int y = __shfl_up_sync(0xffffffffu, x, d);
    if (lane >= d) x += y;
  }
  if (lane == 31) wtmp[warp] = x;
  __syncthreads();
  if (warp == 0) {
    const int w = wtmp[lane];
    int xs = w;
#pragma unroll
    for (int d = 1; d < 32; d <<= 1) {
      const int y = __shfl_up_sync(0xffffffffu, xs, d);
      if (lane >= d) xs += y;
    }
    wtmp[lane] = xs - w;
    if (lane == 31) *total = xs;
  }
  __syncthreads();
  const int r = wtmp[warp] + x - v;
  __syncthreads();
  return r;
}

// Largest v of the threads before this one (-1 if none is larger).
__device__ int block_exclusive_max(int v, int* wtmp) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  int x = v;
#pragma unroll
  for (int d = 1; d < 32; d <<= 1) {
    const int y = __shfl_up_sync(0xffffffffu, x, d);
    if (lane >= d) x = max(x, y);
  }
  int ex = __shfl_up_sync(0xffffffffu, x, 1);
  if (lane == 0) ex = -1;
  if (lane == 31) wtmp[warp] = x;
  __syncthreads();
  if (warp == 0) {
    int xs = wtmp[lane];
#pragma unroll
    for (int d = 1; d < 32; d <<= 1) {
      const int y = __shfl_up_sync(0xffffffffu, xs, d);
      if (lane >= d) xs = max(xs, y);
    }
    int pex = __shfl_up_sync(0xffffffffu, xs, 1);
    if (lane == 0) pex = -1;
    wtmp[lane] = pex;
  }
  __syncthreads();
  const int r = max(wtmp[warp], ex);
  __syncthreads();
  return r;
}

// Index of position p in a code array padded by one int every 32: a thread walking its
// own stretch of 8 positions then meets 32 different banks across the warp.
__device__ __forceinline__ int code_at(int p) { return p + (p >> 5); }
// Ints of a padded code array for n positions.
__host__ __device__ constexpr int code_ints(int n) { return n + (n >> 5) + 1; }

// The segments of a slot-ordered grouping cut at every gap in token order, from
// code[code_at(p)] for the n active positions: bit 0 = a run starts at p, bits 1.. = slot + 1 where
// a slot's range starts (0 elsewhere).  Each run is cut into pieces of at most `chunk`
// (chunk <= 0: one piece per run).  Thread i walks a contiguous stretch of positions
// three times (its last run / slot start, its segment count, then its segments), with
// block scans carrying the run start and slot in from the left.  All kGroupThreads
// threads of the CTA call it.
__device__ void cut_runs(const int* code, int n, int chunk, int32_t* out_indptr, int32_t* out_slots,
                         int32_t* out_count, int* wtmp, int* total) {
  const int tid = threadIdx.x;
  const int per = (n + kGroupThreads - 1) / kGroupThreads;
  const int b = min(n, tid * per), e = min(n, b + per);
  int last_run = -1, last_slot = -1;
  for (int p = b; p < e; ++p) {
    const int c = code[code_at(p)];
    if (c & 1) last_run = p;
    if (c >> 1) last_slot = p;
  }
  const int carry = block_exclusive_max(last_run, wtmp);  // last run start before b
  const int from = block_exclusive_max(last_slot, wtmp);  // last slot start before b
  int cur = from >= 0 ? (code[code_at(from)] >> 1) - 1 : -1;
  int start = carry, pieces = 0;
  for (int p = b; p < e; ++p) {
    const bool run_start = (code[code_at(p)] & 1) != 0;
    if (run_start) start = p;
    if (run_start || (chunk > 0 && (p - start) % chunk == 0)) ++pieces;
  }
  int id = block_exclusive_sum(pieces, wtmp, total);
  start = carry;
  for (int p = b; p < e; ++p) {
    const int c = code[code_at(p)];
    if (c >> 1) cur = (c >> 1) - 1;
    if (c & 1) start = p;
    if ((c & 1) || (chunk > 0 && (p - start) % chunk == 0)) {
      out_indptr[id] = p;
      out_slots[id] = cur;
      ++id;
    }
  }
  if (tid == 0) {
    out_indptr[*total] = n;
    *out_count = *total;
  }
}

// The runs of a batch in token order: a run is a maximal stretch of consecutive tokens
// with one slot in [0, num_slots), cut into pieces of at most `chunk` tokens from its own
// start (chunk <= 0: one piece per run); token_indices lists the active tokens in token
// order, then the others.  One CTA: thread i takes a contiguous stretch of tokens and walks
// it three times (active count and last run start, its pieces, then its writes), with
// block scans carrying the counts and the run start in from the left.
__global__ void __launch_bounds__(kGroupThreads)
token_runs_kernel(const int32_t* __restrict__ slots, int T, int num_slots, int chunk,
                  int32_t* __restrict__ indptr, int32_t* __restrict__ seg_slots,
                  int32_t* __restrict__ perm, int32_t* __restrict__ seg_count) {
  __shared__ int wtmp[kGroupWarps];
  __shared__ int total_active, total_pieces;
  const int tid = threadIdx.x;
  const int per = (T + kGroupThreads - 1) / kGroupThreads;
  const int b = min(T, tid * per), e = min(T, b + per);
  auto slot_at = [&](int t) {
    const int s = slots[t];
    return (s >= 0 && s < num_slots) ? s : -1;
  };
  const int before = b > 0 ? slot_at(b - 1) : -1;
  int active = 0, last_run = -1, prev = before;
  for (int t = b; t < e; ++t) {
    const int s = slot_at(t);
    if (s >= 0) {
      ++active;
      if (s != prev) last_run = t;
    }
    prev = s;
  }
  const int apos = block_exclusive_sum(active, wtmp, &total_active);  // active tokens before b
  const int carry = block_exclusive_max(last_run, wtmp);              // last run start before b
  int start = carry, pieces = 0;
  prev = before;
  for (int t = b; t < e; ++t) {
    const int s = slot_at(t);
    if (s >= 0) {
      if (s != prev) start = t;
      if (s != prev || (chunk > 0 && (t - start) % chunk == 0)) ++pieces;
    }
    prev = s;
  }
  int id = block_exclusive_sum(pieces, wtmp, &total_pieces);
  int pos = apos, ipos = total_active + (b - apos);  // next active / inactive position
  start = carry;
  prev = before;
  for (int t = b; t < e; ++t) {
    const int s = slot_at(t);
    if (s >= 0) {
      if (s != prev) start = t;
      if (s != prev || (chunk > 0 && (t - start) % chunk == 0)) {
        indptr[id] = pos;
        seg_slots[id] = s;
        ++id;
      }
      perm[pos++] = t;
    } else {
      perm[ipos++] = t;
    }
    prev = s;
  }
  if (tid == 0) {
    indptr[total_pieces] = total_active;
    *seg_count = total_pieces;
  }
}

// Shared memory: start[num_slots + 2] (bucket num_slots collects inactive tokens,
// num_slots + 1 is a dummy for padding lanes), segbase[num_slots + 1], scan scratch,
// and, when it fits, a cache of the tokens' bucket ids.
__global__ void __launch_bounds__(kGroupThreads)
group_tokens_kernel(const int32_t* __restrict__ slots, int T, int num_slots, int chunk,
                    int32_t* __restrict__ indptr, int32_t* __restrict__ seg_slots,
                    int32_t* __restrict__ perm, int32_t* __restrict__ seg_count,
                    int cache_tokens, int blocked) {
  extern __shared__ int smem[];
  int* start = smem;                       // num_slots + 2
  int* segbase = start + num_slots + 2;    // num_slots + 1
  int* warp_a = segbase + num_slots + 1;   // 32
  int* warp_b = warp_a + kGroupWarps;      // 32
  int* totals = warp_b + kGroupWarps;      // 2
  int* cache = totals + 2;                 // T when cache_tokens
  // Blocked scatter: per-warp bucket counts [32][num_slots + 2] and per-token ranks [T].
  uint16_t* wcount = reinterpret_cast<uint16_t*>(cache + (cache_tokens ? T : 0));
  uint16_t* rank = wcount + kGroupWarps * (num_slots + 2);
  const int tid = threadIdx.x;

  for (int s = tid; s < num_slots + 2; s += kGroupThreads) start[s] = 0;
  __syncthreads();
  // One shared atomic per bucket and warp step (the lanes of a bucket counted together);
  // a thread's eight slot ids of a pass are all loaded before the first is used.
  for (int t0 = tid & ~31; t0 < T; t0 += 8 * kGroupThreads) {
    int sv[8];
#pragma unroll
    for (int q = 0; q < 8; ++q) {
      const int t = t0 + q * kGroupThreads + (tid & 31);
      sv[q] = t < T ? slots[t] : 0;
    }
#pragma unroll
    for (int q = 0; q < 8; ++q) {
      const int t = t0 + q * kGroupThreads + (tid & 31);
      int bucket = num_slots + 1;
      if (t < T) {
        bucket = (sv[q] >= 0 && sv[q] < num_slots) ? sv[q] : num_slots;
        if (cache_tokens) cache[t] = bucket;
      }
      const unsigned same = __match_any_sync(0xffffffffu, bucket);
      if (t < T && (tid & 31) == __ffs(same) - 1) atomicAdd(&start[bucket], __popc(same));
    }
  }
  __syncthreads();
  for (int s = tid; s < num_slots; s += kGroupThreads) {
    const int c = start[s];
    segbase[s] = chunk > 0 ? (c + chunk - 1) / chunk : (c > 0 ? 1 : 0);
  }
  if (tid == 0) segbase[num_slots] = 0;
  __syncthreads();
  // Scan buckets 0..num_slots (the inactive bucket starts at n_active) and the
  // per-slot segment counts.
  block_exclusive_scan2(start, segbase, num_slots + 1, warp_a, warp_b, &totals[0], &totals[1]);
  const int n_active = start[num_slots];
  const int nseg = segbase[num_slots];
  for (int s = tid; s < num_slots; s += kGroupThreads) {
    const int begin = start[s];
    const int first = segbase[s];
    const int pieces = segbase[s + 1] - first;
    for (int j = 0; j < pieces; ++j) {
      indptr[first + j] = begin + (chunk > 0 ? j * chunk : 0);
      seg_slots[first + j] = s;
    }
  }
  if (tid == 0) {
    indptr[nseg] = n_active;
    *seg_count = nseg;
  }
  __syncthreads();
  auto bucket_of = [&](int t) {
    if (t >= T) return num_slots + 1;
    if (cache_tokens) return cache[t];
    const int sl = slots[t];
    return (sl >= 0 && sl < num_slots) ? sl : num_slots;
  };
  const int lane = tid & 31, warp = tid >> 5;
  const unsigned lower = (1u << lane) - 1u;
  if (blocked) {
    // Stable scatter in three parallel passes.  (1) Warp w ranks the tokens of its
    // contiguous block in order (32 at a time, lanes of one bucket numbered by
    // __match_any_sync) and counts them per bucket.  (2) Per bucket, the warps' counts
    // become exclusive offsets in warp order.  (3) Every token lands at
    // bucket start + its warp's offset + its rank inside the warp's block.
    const int nb = num_slots + 2;
    for (int i = tid; i < kGroupWarps * nb; i += kGroupThreads) wcount[i] = 0;
    __syncthreads();
    const int per = (T + kGroupWarps - 1) / kGroupWarps;
    const int b0 = warp * per, b1 = min(T, b0 + per);
    uint16_t* mine = wcount + warp * nb;
    for (int base = b0; base < b1; base += 32) {
      const int t = base + lane;
      const int bucket = t < b1 ? bucket_of(t) : num_slots + 1;
      const unsigned same = __match_any_sync(0xffffffffu, bucket);
      const int r = mine[bucket] + __popc(same & lower);
      __syncwarp();
      if (lane == __ffs(same) - 1) mine[bucket] = uint16_t(mine[bucket] + __popc(same));
      __syncwarp();
      if (t < b1) rank[t] = uint16_t(r);
    }
    __syncthreads();
    for (int k = tid; k < nb; k += kGroupThreads) {
      int run = 0;
      for (int w = 0; w < kGroupWarps; ++w) {
        const int c = wcount[w * nb + k];
        wcount[w * nb + k] = uint16_t(run);
        run += c;
      }
    }
    __syncthreads();
    for (int t = tid; t < T; t += kGroupThreads) {
      const int bucket = bucket_of(t);
      perm[start[bucket] + wcount[(t / per) * nb + bucket] + rank[t]] = t;
    }
    return;
  }
  // Stable scatter: warp 0 walks the tokens in order, 32 at a time; lanes with the
  // same bucket get consecutive positions in token order.
  if (tid < 32) {
    for (int base = 0; base < T; base += 32) {
      const int t = base + lane;
      const int bucket = bucket_of(t);
      const unsigned same = __match_any_sync(0xffffffffu, bucket);
      const int pos = start[bucket] + __popc(same & lower);
      __syncwarp();
      if (lane == __ffs(same) - 1) start[bucket] += __popc(same);
      __syncwarp();
      if (t < T) perm[pos] = t;
    }
  }
}

// Re-chunks a grouping so that no segment spans a gap in token order: inside each slot's
// range of token_indices, a run is a maximal stretch of consecutive tokens, and each run
// is cut into pieces of at most `chunk` tokens from its own start (chunk <= 0: one piece
// per run).  token_indices is unchanged; the new segments go to out_*.  One CTA.
//
// First every position p gets its cut_runs code in shared memory (coalesced, in
// parallel; a run starts where a slot starts or token_indices[p] != token_indices[p-1] + 1),
// then cut_runs makes the segments.  Without room for the codes (cached == 0) the same
// three walks read the tables in global memory.
__global__ void __launch_bounds__(kGroupThreads)
split_runs_kernel(const int32_t* __restrict__ in_indptr, const int32_t* __restrict__ in_slots,
                  const int32_t* __restrict__ perm, const int32_t* __restrict__ in_count, int T,
                  int chunk, int cached, int32_t* __restrict__ out_indptr,
                  int32_t* __restrict__ out_slots, int32_t* __restrict__ out_count) {
  extern __shared__ int code[];  // [T] when cached
  __shared__ int wtmp[kGroupWarps];
  __shared__ int total;
  const int tid = threadIdx.x;
  const int count = max(0, min(*in_count, T));
  const int n = count > 0 ? max(0, min(in_indptr[count], T)) : 0;
  if (cached) {
    // Four positions (and then four segments) per thread and pass, all loads first.
    for (int p0 = tid; p0 < n; p0 += 4 * kGroupThreads) {
      int cur[4], prev[4];
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        const int p = p0 + q * kGroupThreads;
        cur[q] = p < n ? perm[p] : 0;
        prev[q] = p < n && p > 0 ? perm[p - 1] : 0;
      }
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        const int p = p0 + q * kGroupThreads;
        if (p < n) code[code_at(p)] = (p == 0 || cur[q] != prev[q] + 1) ? 1 : 0;
      }
    }
    __syncthreads();
    for (int k0 = tid; k0 < count; k0 += 4 * kGroupThreads) {
      int slot[4], before[4], at[4];
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        const int k = k0 + q * kGroupThreads;
        slot[q] = k < count ? in_slots[k] : 0;
        before[q] = k < count && k > 0 ? in_slots[k - 1] : -1;
        at[q] = k < count ? in_indptr[k] : -1;
      }
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        const int k = k0 + q * kGroupThreads;
        if (k < count && (k == 0 || before[q] != slot[q]) && at[q] >= 0 && at[q] < n)
          code[code_at(at[q])] = 1 | ((slot[q] + 1) << 1);
      }
    }
    __syncthreads();
    cut_runs(code, n, chunk, out_indptr, out_slots, out_count, wtmp, &total);
    return;
  }
  const int per = (n + kGroupThreads - 1) / kGroupThreads;
  const int b = min(n, tid * per), e = min(n, b + per);
  // Global-memory walks: the input segment holding position b (last k with indptr <= b).
  int k0 = 0;
  if (b < e) {
    int lo = 0, hi = count - 1;
    while (lo < hi) {
      const int mid = (lo + hi + 1) >> 1;
      if (in_indptr[mid] <= b) lo = mid;
      else hi = mid - 1;
    }
    k0 = lo;
  }
  // visit(p, slot or -1 when unchanged, run_start)
  auto walk = [&](auto&& visit) {
    int k = k0;
    for (int p = b; p < e; ++p) {
      while (k + 1 < count && in_indptr[k + 1] <= p) ++k;
      const int slot = in_slots[k];
      const bool slot_start = p == in_indptr[k] && (k == 0 || in_slots[k - 1] != slot);
      visit(p, (slot_start || p == b) ? slot : -1, slot_start || p == 0 || perm[p] != perm[p - 1] + 1);
    }
  };
  int last_run = -1;
  walk([&](int p, int, bool run_start) {
    if (run_start) last_run = p;
  });
  const int carry = block_exclusive_max(last_run, wtmp);  // last run start before b
  int cur = -1;  // set at the stretch's first position by the walk
  int start = carry, pieces = 0;
  walk([&](int p, int, bool run_start) {
    if (run_start) start = p;
    if (run_start || (chunk > 0 && (p - start) % chunk == 0)) ++pieces;
  });
  int id = block_exclusive_sum(pieces, wtmp, &total);
  start = carry;
  walk([&](int p, int slot, bool run_start) {
    if (slot >= 0) cur = slot;
    if (run_start) start = p;
    if (run_start || (chunk > 0 && (p - start) % chunk == 0)) {
      out_indptr[id] = p;
      out_slots[id] = cur;
      ++id;
    }
  });
  if (tid == 0) {
    out_indptr[total] = n;
    *out_count = total;
  }
}

// routes[token_indices[i]] = segment_slots[s] for every i in segment s's range; one warp
// per segment, grid-stride over segments.  Segments past *segment_count (or
// max_segments), index entries outside [0, num_indices) and token positions outside
// [0, T) are ignored, so padded routing tables of captured graphs are safe.
__global__ void segment_routes_kernel(const int32_t* __restrict__ indptr,
                                      const int32_t* __restrict__ seg_slots,
                                      const int32_t* __restrict__ token_indices,
                                      const int32_t* __restrict__ segment_count,
                                      int max_segments, int num_indices, int T,
                                      int32_t* __restrict__ routes) {
  const int lane = threadIdx.x & 31;
  const int nseg = min(max_segments, max(0, *segment_count));
  const int warps = gridDim.x * (blockDim.x >> 5);
  for (int s = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5); s < nseg; s += warps) {
    const int begin = max(0, indptr[s]), end = min(num_indices, indptr[s + 1]);
    const int slot = seg_slots[s];
    for (int i = begin + lane; i < end; i += 32) {
      const int t = token_indices[i];
      if (t >= 0 && t < T) routes[t] = slot;
    }
  }
}

}  // namespace
}  // namespace lfb

extern "C" int lf_segment_routes(const int32_t* segment_indptr, const int32_t* segment_slots,
                                 const int32_t* token_indices, const int32_t* segment_count,
                                 int32_t max_segments, int64_t num_indices, int64_t num_tokens,
                                 int32_t* routes, void* stream) {
  using namespace lfb;
  if (num_tokens < 0 || num_tokens >= (int64_t(1) << 31) || num_indices < 0 ||
      num_indices >= (int64_t(1) << 31) || max_segments < 0)
    return fail(LF_E_INVALID, "segment_routes: sizes must fit signed int32");
  if (num_tokens == 0) return LF_OK;
  if (!routes || !segment_count || (max_segments && (!segment_indptr || !segment_slots)) ||
      (num_indices && !token_indices))
    return fail(LF_E_INVALID, "segment_routes: null buffer");
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  // 0xff bytes make every int32 route -1 (no adapter) before the scatter.
  if (cudaMemsetAsync(routes, 0xff, sizeof(int32_t) * size_t(num_tokens), s) != cudaSuccess)
    return check_launch("segment_routes memset");
  if (max_segments == 0) return LF_OK;
  const int threads = 256, per_block = threads / 32;
  const int blocks = min((max_segments + per_block - 1) / per_block, 4 * 148);
  segment_routes_kernel<<<blocks, threads, 0, s>>>(segment_indptr, segment_slots, token_indices,
                                                  segment_count, max_segments, int(num_indices),
                                                  int(num_tokens), routes);
  return check_launch("segment_routes");
}

extern "C" int lf_split_runs(const int32_t*, const int32_t*, const int32_t*, const int32_t*, int64_t, int32_t,
                             int32_t*, int32_t*, int32_t*, void*);

namespace lfb {
namespace {
// Launch plan of group_tokens_kernel for T tokens: shared bytes, token cache, blocked
// scatter.
struct GroupPlan {
  size_t bytes;
  int cache, blocked;
};
constexpr size_t kGroupSmemLimit = 200 * 1024;
inline GroupPlan group_plan(int T, int num_slots) {
  GroupPlan g{};
  const size_t fixed = sizeof(int) * (size_t(num_slots) * 2 + 3 + 2 * kGroupWarps + 2);
  g.cache = fixed + sizeof(int) * size_t(T) <= kGroupSmemLimit ? 1 : 0;
  g.bytes = fixed + (g.cache ? sizeof(int) * size_t(T) : 0);
  // The parallel blocked scatter needs 16-bit per-warp counts and ranks in shared memory.
  const size_t blocked_extra = sizeof(uint16_t) * (size_t(kGroupWarps) * (num_slots + 2) + size_t(T) + 1);
  g.blocked = T >= 64 && T <= 65535 && g.bytes + blocked_extra + 16 <= kGroupSmemLimit ? 1 : 0;
  if (g.blocked) g.bytes += blocked_extra + 16;
  return g;
}

int check_group_args(const int32_t* slots, int64_t num_tokens, int32_t num_slots, const int32_t* segment_indptr,
                     const int32_t* segment_slots, const int32_t* token_indices, const int32_t* segment_count,
                     const char* what) {
  if (num_tokens < 0 || num_tokens >= (int64_t(1) << 31))
    return fail(LF_E_INVALID, (std::string(what) + ": token count must fit signed int32").c_str());
  if (num_slots < 1 || num_slots > 16384) return fail(LF_E_INVALID, (std::string(what) + ": num_slots must be in 1..16384").c_str());
  if (!segment_indptr || !segment_count || (num_tokens && (!slots || !segment_slots || !token_indices)))
    return fail(LF_E_INVALID, (std::string(what) + ": null buffer").c_str());
  if (sizeof(int) * (size_t(num_slots) * 2 + 3 + 2 * kGroupWarps + 2) > kGroupSmemLimit)
    return fail(LF_E_INVALID, (std::string(what) + ": too many slots").c_str());
  return LF_OK;
}

int launch_group(const int32_t* slots, int T, int32_t num_slots, int32_t chunk, int32_t* indptr, int32_t* seg_slots,
                 int32_t* perm, int32_t* count, const GroupPlan& g, cudaStream_t stream) {
  static int flags[64] = {};
  if (int rc = ensure_smem(group_tokens_kernel, int(kGroupSmemLimit), flags)) return rc;
  group_tokens_kernel<<<1, kGroupThreads, g.bytes, stream>>>(slots, T, num_slots, chunk, indptr, seg_slots, perm,
                                                            count, g.cache, g.blocked);
  return check_launch("group_tokens");
}
}  // namespace
}  // namespace lfb

extern "C" int lf_group_tokens(const int32_t* slots, int64_t num_tokens, int32_t num_slots,
                               int32_t chunk, int32_t* segment_indptr,
                               int32_t* segment_slots, int32_t* token_indices,
                               int32_t* segment_count, void* stream) {
  using namespace lfb;
  if (int rc = check_group_args(slots, num_tokens, num_slots, segment_indptr, segment_slots, token_indices,
                                segment_count, "group_tokens"))
    return rc;
  const int T = static_cast<int>(num_tokens);
  return launch_group(slots, T, num_slots, chunk, segment_indptr, segment_slots, token_indices, segment_count,
                      group_plan(T, num_slots), static_cast<cudaStream_t>(stream));
}

extern "C" int lf_group_token_runs(const int32_t* slots, int64_t num_tokens, int32_t num_slots,
                                   int32_t chunk, int32_t* segment_indptr, int32_t* segment_slots,
                                   int32_t* token_indices, int32_t* segment_count, void* stream) {
  using namespace lfb;
  if (int rc = check_group_args(slots, num_tokens, num_slots, segment_indptr, segment_slots, token_indices,
                                segment_count, "group_token_runs"))
    return rc;
  token_runs_kernel<<<1, kGroupThreads, 0, static_cast<cudaStream_t>(stream)>>>(
      slots, int(num_tokens), num_slots, chunk, segment_indptr, segment_slots, token_indices, segment_count);
  return check_launch("group_token_runs");
}

extern "C" int lf_split_runs(const int32_t* segment_indptr, const int32_t* segment_slots,
                             const int32_t* token_indices, const int32_t* segment_count,
                             int64_t num_tokens, int32_t chunk, int32_t* out_indptr,
                             int32_t* out_slots, int32_t* out_count, void* stream) {
  using namespace lfb;
  if (num_tokens < 0 || num_tokens >= (int64_t(1) << 31))
    return fail(LF_E_INVALID, "split_runs: token count must fit signed int32");
  if (!segment_indptr || !segment_count || !out_indptr || !out_count ||
      (num_tokens && (!segment_slots || !token_indices || !out_slots)))
    return fail(LF_E_INVALID, "split_runs: null buffer");
  if (out_indptr == segment_indptr || out_slots == segment_slots || out_count == segment_count)
    return fail(LF_E_INVALID, "split_runs: output tables must not alias the input tables");
  // One int of shared memory per position when the batch fits (up to 51200 tokens).
  const size_t limit = 200 * 1024;
  const int cached = sizeof(int) * size_t(code_ints(int(num_tokens))) <= limit ? 1 : 0;
  static int flags[64] = {};
  if (int rc = ensure_smem(split_runs_kernel, int(limit), flags)) return rc;
  split_runs_kernel<<<1, kGroupThreads, cached ? sizeof(int) * size_t(code_ints(int(num_tokens))) : 0,
                      static_cast<cudaStream_t>(stream)>>>(segment_indptr, segment_slots, token_indices,
                                                           segment_count, int(num_tokens), chunk, cached,
                                                           out_indptr, out_slots, out_count);
  return check_launch("split_runs");
}
