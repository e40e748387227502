// Base projection GEMM with the LoRA delta in its mainloop, on tcgen05 + TMEM:
//
//   y[t, n] = sum_k x[t, k] W[n, k]  +  scale_g(t) . sum_j z[t, s(n)*r + j] B_g(t)[n, j]
//
// The reference adds the LoRA delta to the base projection's output in a separate pass
// (lora_expand(..., base=) in src/loraforge/ops/gemv.py:130-238, and the base output the
// fleet backend passes through, src/loraforge/integrations/_sglang_fleet.py:340-347), which
// reads and writes y once more.  Here the delta is more K steps of the same accumulator:
// for a tile of 128 tokens x 256 output columns, after the K loop over x . W^T, every slot
// present among the tile's tokens adds Z_g . B_g^T, where Z_g holds scale_g . z of the
// tile's tokens routed to g (BF16 hi + lo of the FP32 z) and zero rows elsewhere.  y is
// written once, from the FP32 accumulator, with one rounding; it is never read.
//
// z comes from the prefill shrink (rows by token, FP32).  Persistent CTAs walk the output
// tiles (token-tile major, so a tile row of x is shared by consecutive CTAs in L2); per CTA:
//   warp 0  producer: x [128 x 64] and W [256 x 64] boxes (TMA, 128-byte swizzle) into a
//           3-stage ring, and per LoRA slot the B_g rows of the tile's columns (TMA boxes in
//           the bucket's own swizzled layout, or cp.async rows zero-padded to 64);
//   warp 1  MMA thread (M = 128, N = 256, K = 16 per instruction; FP32 in TMEM) and the
//           TMEM allocation: two 256-column accumulators, so the epilogue of one tile
//           overlaps the mainloop of the next;
//   warps 2-3 the Z_g tiles (BF16 hi + lo, scale folded in, 128-byte swizzle);
//   warps 4-7 epilogue: TMEM lane quarter = warp & 3, one token row per thread, BF16 out.
// Every mbarrier wait is bounded (tma.cuh); an expiry stops every role at its next wait
// and the TMEM columns are always released.
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

constexpr int kBM = 128;                 // tokens per tile (UMMA M)
constexpr int kBN = 256;                 // output columns per tile (UMMA N)
constexpr int kBK = 64;                  // K per stage: one 128-byte swizzled row
constexpr int kStages = 3;
constexpr int kXBytes = kBM * 128;       // 16 KiB
constexpr int kWBytes = kBN * 128;       // 32 KiB
constexpr int kStageBytes = kXBytes + kWBytes;
constexpr int kZBytes = kBM * 128;       // one Z tile (hi or lo), 16 KiB
constexpr int kLBBytes = kBN * 128;      // B_g rows of a tile, 32 KiB
constexpr int kThreads = 256;
constexpr int kMaxRank = 64;
constexpr int kMaxList = kBM;            // distinct slots in a tile, at most
constexpr int64_t kBRows = (int64_t(1) << 31) - 1;  // nominal row extent of the B tensor maps

struct GParams {
  uint16_t* y;
  int64_t y_stride;
  const uint16_t* b;
  const int64_t* b_offsets;
  const int32_t* b_strides;
  const int32_t* ranks;
  const float* scales;
  const int32_t* routes;      // [T] slot of each token (-1: none)
  const float* ztok;          // [T][zpitch] FP32 z by token, columns s*r + k
  const int32_t* lists;       // [mtiles][1 + kMaxList]: distinct slots of each token tile
  const int32_t* slice_offsets;
  int T, K, N, S, cap, num_slots, zpitch, mtiles, ntiles;
  CUtensorMap tmap_x;     // x [T, K], boxes of 64 columns x 128 rows, 128-byte swizzle
  CUtensorMap tmap_w;     // W [N, K], boxes of 64 columns x 256 rows, 128-byte swizzle
  CUtensorMap tmap_b[3];  // compact B as [rows, bucket] for bucket 16 / 32 / 64, boxes of 256 rows
};

// One LoRA term of a tile: slot g with its metadata, or ok = 0 (skipped by every role).
struct Lora {
  int ok, g, r, bucket, kb, brow;
  float scale;
  int64_t boff;
};

__device__ __forceinline__ Lora lora_of(const GParams& p, int g) {
  Lora l{};
  l.g = g;
  if (g < 0 || g >= p.num_slots) return l;
  l.r = p.ranks[g];
  l.bucket = p.b_strides[g];
  l.scale = p.scales[g];
  l.boff = p.b_offsets[g];
  l.ok = l.r >= 1 && l.r <= kMaxRank && l.r <= p.cap && l.bucket >= 1 && l.bucket <= kMaxRank &&
         (l.bucket & (l.bucket - 1)) == 0 && l.boff >= 0 && (l.boff & 7) == 0;
  // TMA boxes in the bucket's own layout when the rows are whole rows of that width.
  const bool sized = l.bucket == 16 || l.bucket == 32 || l.bucket == 64;
  l.kb = l.ok && sized && l.boff % l.bucket == 0 && l.boff / l.bucket + p.N <= kBRows ? l.bucket : 0;
  l.brow = l.kb ? int(l.boff / l.kb) : 0;
  return l;
}

__device__ __forceinline__ int slice_of_col(const int* offs, int S, int col) {
  int s = 0;
  for (int i = 1; i < S; ++i)
    if (col >= offs[i]) s = i;
  return s;
}

__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_launch_dependents() {
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}

__device__ __forceinline__ uint32_t cvt_bf16x2_pair(float first, float second) {
  uint32_t r;
  asm("cvt.rn.bf16x2.f32 %0, %1, %2;" : "=r"(r) : "f"(second), "f"(first));
  return r;
}

// Distinct slots of each 128-token tile, in order of first appearance: lists[mt][0] =
// count, then the slots.  One CTA (128 threads) per token tile.
__global__ void __launch_bounds__(kBM) tile_slot_lists_kernel(const int32_t* routes, int T, int num_slots,
                                                              int32_t* lists) {
  __shared__ int slot[kBM];
  __shared__ int first[kBM];
  pdl_wait();  // routes come from the preceding grid
  const int t = threadIdx.x, m0 = blockIdx.x * kBM;
  const int g = m0 + t < T ? routes[m0 + t] : -1;
  slot[t] = g >= 0 && g < num_slots ? g : -1;
  __syncthreads();
  bool is_first = slot[t] >= 0;
  for (int u = 0; u < t && is_first; ++u)
    if (slot[u] == slot[t]) is_first = false;
  first[t] = is_first ? 1 : 0;
  __syncthreads();
  int before = 0;
  for (int u = 0; u < t; ++u) before += first[u];
  int32_t* out = lists + int64_t(blockIdx.x) * (1 + kMaxList);
  if (is_first) out[1 + before] = slot[t];
  if (t == kBM - 1) out[0] = before + first[t];
  pdl_launch_dependents();
}

__global__ void __launch_bounds__(kThreads, 1) base_lora_gemm_kernel(const __grid_constant__ GParams p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = align1024(smem_raw);
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  uint8_t* ring = smem;                               // kStages x (x 16 KiB, W 32 KiB)
  uint8_t* ztile = ring + kStages * kStageBytes;      // hi 16 KiB, lo 16 KiB
  uint8_t* lbtile = ztile + 2 * kZBytes;              // 32 KiB
  uint64_t* full = reinterpret_cast<uint64_t*>(lbtile + kLBBytes);
  uint64_t* empty = full + kStages;
  uint64_t* z_full = empty + kStages;
  uint64_t* z_empty = z_full + 1;
  uint64_t* lb_full = z_empty + 1;
  uint64_t* lb_empty = lb_full + 1;
  uint64_t* acc_full = lb_empty + 1;
  uint64_t* acc_empty = acc_full + 2;
  uint64_t* fin = acc_empty + 2;
  uint32_t* tslot = reinterpret_cast<uint32_t*>(fin + 1);
  int* offs = reinterpret_cast<int*>(tslot + 4);
  volatile int* abort = reinterpret_cast<volatile int*>(offs + 8);

  if (tid == 0) {
    for (int i = 0; i < kStages; ++i) {
      mbar_init(&full[i], 1);
      mbar_init(&empty[i], 1);
    }
    mbar_init(z_full, 64);
    mbar_init(z_empty, 1);
    mbar_init(lb_full, 32);  // the producer warp (lane 0 also expects the boxes' bytes)
    mbar_init(lb_empty, 1);
    for (int i = 0; i < 2; ++i) {
      mbar_init(&acc_full[i], 1);
      mbar_init(&acc_empty[i], 128);
    }
    mbar_init(fin, 1);
    fence_mbar_init();
    *abort = 0;
  }
  if (tid <= p.S) offs[tid] = p.slice_offsets[tid];
  if (warp == 1) tc_alloc(tslot, 2 * kBN);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tslot;

  const int tiles = p.mtiles * p.ntiles;
  const int ksteps = (p.K + kBK - 1) / kBK;

  if (warp == 0) {
    // ------------------------------------------------------------ producer
    int sidx = 0, lcount = 0;
    bool waited = false;
    for (int tile = blockIdx.x; tile < tiles; tile += gridDim.x) {
      const int mt = tile / p.ntiles, nt = tile - mt * p.ntiles;
      const int m0 = mt * kBM, n0 = nt * kBN;
      for (int ks = 0; ks < ksteps; ++ks, ++sidx) {
        const int st = sidx % kStages;
        if (!wait_or_abort(&empty[st], (uint32_t(sidx / kStages) & 1u) ^ 1u, abort)) break;
        if (lane == 0) {
          const uint32_t sa = smem_u32(ring + st * kStageBytes);
          mbar_arrive_expect_tx(&full[st], uint32_t(kStageBytes));
          tma_load_2d(sa, &p.tmap_x, ks * kBK, m0, &full[st]);
          tma_load_2d(sa + kXBytes, &p.tmap_w, ks * kBK, n0, &full[st]);
        }
      }
      if (*abort) break;
      // LoRA B rows of this tile's columns, one slot at a time.
      if (!waited) {
        pdl_wait();  // the slot lists come from the preceding grid
        waited = true;
      }
      const int32_t* list = p.lists + int64_t(mt) * (1 + kMaxList);
      const int count = list[0];
      const int cols = min(kBN, p.N - n0);
      for (int i = 0; i < count; ++i) {
        const Lora l = lora_of(p, list[1 + i]);
        if (!l.ok) continue;
        if (!wait_or_abort(lb_empty, (uint32_t(lcount) & 1u) ^ 1u, abort)) break;
        ++lcount;
        const uint32_t bt = smem_u32(lbtile);
        bool staged = true;
        // A tile of fewer than 256 columns takes the padded path: a 256-row box would read
        // rows past the slot's block (and, for the last slot, past the buffer).
        if (l.kb && cols == kBN) {
          const int rb = 2 * l.kb;
          const int m = l.kb == 16 ? 0 : l.kb == 32 ? 1 : 2;
          if (lane == 0) {
            mbar_expect_tx(lb_full, uint32_t(kBN * rb));
            tma_load_2d(bt, &p.tmap_b[m], 0, l.brow + n0, lb_full);
          }
          staged = false;
        } else {
          for (int q = lane; q < kBN * 8; q += 32) {
            const int r = q >> 3, c = q & 7, k = 8 * c;
            const bool live = r < cols && k < l.bucket;
            const uint16_t* src = p.b + l.boff + int64_t(n0 + r) * l.bucket + k;
            if (l.bucket >= 8) {
              cp16(bt + swz(r, c), live ? static_cast<const void*>(src) : p.b, live ? 16u : 0u);
            } else {
              uint32_t wv[4] = {0u, 0u, 0u, 0u};
              if (live)
                for (int e = 0; e < l.bucket; ++e) wv[e >> 1] |= uint32_t(src[e]) << (16 * (e & 1));
              sts16(bt + swz(r, c), make_uint4(wv[0], wv[1], wv[2], wv[3]));
            }
          }
          cp_commit();
        }
        if (staged) {
          cp_wait<0>();
          fence_async_smem();
        }
        mbar_arrive(lb_full);
      }
      if (*abort) break;
    }
    if (!waited) pdl_wait();
    // No box may still be landing when the CTA exits.
    if (lane == 0)
      for (int j = max(0, sidx - kStages); j < sidx; ++j) mbar_wait(&full[j % kStages], uint32_t(j / kStages) & 1u);
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA thread
    if (lane == 0) {
      const uint32_t idesc = idesc_bf16(kBM, kBN);
      int sidx = 0, zcount = 0, lcount = 0, tcount = 0;
      pdl_wait();  // the tiles' slot lists come from the preceding grid
      for (int tile = blockIdx.x; tile < tiles; tile += gridDim.x) {
        const int mt = tile / p.ntiles, nt = tile - mt * p.ntiles;
        const int ab = tcount & 1;
        if (!wait_or_abort(&acc_empty[ab], (uint32_t(tcount >> 1) & 1u) ^ 1u, abort)) break;
        ++tcount;
        tc_fence_after();
        const uint32_t d = tmem + uint32_t(ab * kBN);
        for (int ks = 0; ks < ksteps; ++ks, ++sidx) {
          const int st = sidx % kStages;
          if (!wait_or_abort(&full[st], uint32_t(sidx / kStages) & 1u, abort)) break;
          tc_fence_after();
          const uint32_t sa = smem_u32(ring + st * kStageBytes);
          const uint64_t ad = sw128_desc(sa), bd = sw128_desc(sa + kXBytes);
#pragma unroll
          for (int k = 0; k < 4; ++k) tc_mma(d, ad + 2 * k, bd + 2 * k, idesc, (ks > 0 || k > 0) ? 1u : 0u);
          tc_commit(&empty[st]);
        }
        if (*abort) break;
        const int32_t* list = p.lists + int64_t(mt) * (1 + kMaxList);
        const int count = list[0];
        for (int i = 0; i < count; ++i) {
          const Lora l = lora_of(p, list[1 + i]);
          if (!l.ok) continue;
          if (!wait_or_abort(z_full, uint32_t(zcount) & 1u, abort)) break;
          ++zcount;
          if (!wait_or_abort(lb_full, uint32_t(lcount) & 1u, abort)) break;
          ++lcount;
          tc_fence_after();
          const int kb = l.kb && min(kBN, p.N - nt * kBN) == kBN ? l.kb : 0;  // as the producer loaded it
          const int kst = kb ? kb >> 4 : 4;
          const uint32_t bt = smem_u32(lbtile);
          const uint64_t bd = kb ? swrow_desc(bt, 2 * kb) : sw128_desc(bt);
          const uint64_t zh = sw128_desc(smem_u32(ztile)), zl = sw128_desc(smem_u32(ztile + kZBytes));
#pragma unroll
          for (int k = 0; k < 4; ++k)
            if (k < kst) tc_mma(d, zh + 2 * k, bd + 2 * k, idesc, 1u);
#pragma unroll
          for (int k = 0; k < 4; ++k)
            if (k < kst) tc_mma(d, zl + 2 * k, bd + 2 * k, idesc, 1u);
          tc_commit(z_empty);
          tc_commit(lb_empty);
        }
        tc_commit(&acc_full[ab]);
        if (*abort) break;
      }
      // Every MMA has retired before the TMEM columns are released.
      tc_commit(fin);
      mbar_wait(fin, 0);
    }
  } else if (warp == 2 || warp == 3) {
    // ------------------------------------------------------------ Z tiles
    const int zt = tid - 64;
    pdl_wait();  // the z rows and slot lists come from the preceding grids
    int zcount = 0;
    for (int tile = blockIdx.x; tile < tiles; tile += gridDim.x) {
      const int mt = tile / p.ntiles, nt = tile - mt * p.ntiles;
      const int m0 = mt * kBM, n0 = nt * kBN;
      const int slice = slice_of_col(offs, p.S, n0);
      const int32_t* list = p.lists + int64_t(mt) * (1 + kMaxList);
      const int count = list[0];
      for (int i = 0; i < count; ++i) {
        const Lora l = lora_of(p, list[1 + i]);
        if (!l.ok) continue;
        if (!wait_or_abort(z_empty, (uint32_t(zcount) & 1u) ^ 1u, abort)) break;
        ++zcount;
        // Row m: scale . z of token m0 + m when it is routed to this slot, else zero;
        // elements beyond min(rank, bucket) and past 64 are zero.
        const int live = min(l.r, l.bucket);
        const int col0 = slice * l.r;
        const uint32_t zh = smem_u32(ztile), zl = zh + kZBytes;
        for (int item = zt; item < kBM * 8; item += 64) {
          const int m = item >> 3, c = item & 7;
          const int t = m0 + m;
          float v[8];
#pragma unroll
          for (int e = 0; e < 8; ++e) v[e] = 0.f;
          if (t < p.T && p.routes[t] == l.g) {
            const float* src = p.ztok + int64_t(t) * p.zpitch + col0 + 8 * c;
            for (int e = 0; e < 8 && 8 * c + e < live; ++e) v[e] = l.scale * __ldcg(src + e);
          }
          uint32_t hw[4], lw[4];
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            hw[e] = cvt_bf16x2_pair(v[2 * e], v[2 * e + 1]);
            const float h0 = __uint_as_float(hw[e] << 16), h1 = __uint_as_float(hw[e] & 0xffff0000u);
            lw[e] = cvt_bf16x2_pair(v[2 * e] - h0, v[2 * e + 1] - h1);
          }
          sts16(zh + swz(m, c), make_uint4(hw[0], hw[1], hw[2], hw[3]));
          sts16(zl + swz(m, c), make_uint4(lw[0], lw[1], lw[2], lw[3]));
        }
        fence_async_smem();
        mbar_arrive(z_full);
      }
      if (*abort) break;
    }
  } else {
    // ------------------------------------------------------------ epilogue
    const int quarter = warp & 3;
    const int row = quarter * 32 + lane;
    const bool vec = (reinterpret_cast<uintptr_t>(p.y) & 15) == 0 && (p.y_stride & 7) == 0;
    int tcount = 0;
    for (int tile = blockIdx.x; tile < tiles; tile += gridDim.x) {
      const int mt = tile / p.ntiles, nt = tile - mt * p.ntiles;
      const int m0 = mt * kBM, n0 = nt * kBN;
      const int ab = tcount & 1;
      const bool ok = __all_sync(0xffffffffu, wait_or_abort(&acc_full[ab], uint32_t(tcount >> 1) & 1u, abort));
      ++tcount;
      if (!ok) break;
      tc_fence_after();
      const int t = m0 + row;
      uint16_t* yrow = p.y + int64_t(t) * p.y_stride + n0;
      const int cols = min(kBN, p.N - n0);
      for (int c0 = 0; c0 < kBN; c0 += 32) {
        uint32_t r[32];
        tc_ld32(tmem + (uint32_t(quarter * 32) << 16) + uint32_t(ab * kBN + c0), r);
        if (t >= p.T || c0 >= cols) continue;
        if (vec && c0 + 32 <= cols) {
#pragma unroll
          for (int q = 0; q < 4; ++q) {
            const uint32_t* v = r + 8 * q;
            *reinterpret_cast<uint4*>(yrow + c0 + 8 * q) =
                make_uint4(cvt_bf16x2_pair(__uint_as_float(v[0]), __uint_as_float(v[1])),
                           cvt_bf16x2_pair(__uint_as_float(v[2]), __uint_as_float(v[3])),
                           cvt_bf16x2_pair(__uint_as_float(v[4]), __uint_as_float(v[5])),
                           cvt_bf16x2_pair(__uint_as_float(v[6]), __uint_as_float(v[7])));
          }
        } else {
          for (int j = 0; j < 32 && c0 + j < cols; ++j) yrow[c0 + j] = uint16_t(float_to_bf16_bits(__uint_as_float(r[j])));
        }
      }
      tc_fence_before();
      mbar_arrive(&acc_empty[ab]);
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tc_dealloc(tmem, 2 * kBN);
  }
}

// cuTensorMapEncodeTiled through the runtime's driver entry point (no libcuda link).
PFN_cuTensorMapEncodeTiled_v12000 gemm_tensor_map_encoder() {
  static std::mutex mutex;
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  std::lock_guard<std::mutex> lock(mutex);
  if (!fn) {
    void* ptr = nullptr;
    cudaDriverEntryPointQueryResult status;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &ptr, cudaEnableDefault, &status) == cudaSuccess &&
        status == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(ptr);
  }
  return fn;
}

template <typename Kernel, typename... Args>
int launch_pdl_ex(Kernel kernel, dim3 grid, dim3 block, int smem, cudaStream_t stream, const char* what,
                  Args... args) {
  cudaLaunchConfig_t config = {};
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  config.attrs = attr;
  config.numAttrs = 1;
  config.gridDim = grid;
  config.blockDim = block;
  config.dynamicSmemBytes = smem;
  config.stream = stream;
  const cudaError_t err = cudaLaunchKernelEx(&config, kernel, args...);
  if (err != cudaSuccess) {
    last_error() = std::string(what) + ": " + cudaGetErrorString(err);
    return LF_E_CUDA;
  }
  return LF_OK;
}

struct GemmLayout {
  int64_t prefill, ztok, routes, lists, total;  // offsets in floats (4-byte words)
  int zpitch, mtiles;
};

GemmLayout gemm_layout(int64_t tokens, int64_t width, int num_slices, int capacity) {
  GemmLayout l{};
  const int64_t T = tokens > 0 ? tokens : 1;
  l.prefill = 0;
  const int64_t pf = lf_sgmv_prefill_workspace_floats(tokens, width, num_slices, capacity);
  const int cap = capacity < kMaxRank ? capacity : kMaxRank;
  l.zpitch = (num_slices * cap + 15) / 16 * 16;
  l.mtiles = int((T + kBM - 1) / kBM);
  l.ztok = (pf + 3) / 4 * 4;
  l.routes = l.ztok + T * l.zpitch;
  l.lists = l.routes + (T + 3) / 4 * 4;
  l.total = l.lists + int64_t(l.mtiles) * (1 + kMaxList);
  return l;
}

}  // namespace
}  // namespace lfb

using namespace lfb;

extern "C" int64_t lf_lora_base_gemm_workspace_floats(int64_t num_tokens, int64_t width, int32_t num_slices,
                                                      int32_t capacity) {
  if (num_tokens < 0 || width < 1 || num_slices < 1 || num_slices > 4 || capacity < 1) return -1;
  return gemm_layout(num_tokens, width, num_slices, capacity).total;
}

extern "C" int lf_lora_base_gemm(
    const void* x, int64_t x_stride, const void* w, int64_t w_stride, const void* a, const void* b,
    const int64_t* b_offsets, const int32_t* b_strides, void* y, int64_t y_stride,
    const int32_t* segment_indptr, const int32_t* segment_slots, const int32_t* token_indices,
    const int32_t* ranks, const float* scales, const int32_t* slice_offsets, const int32_t* segment_count,
    float* workspace, int64_t workspace_floats, int64_t num_tokens, int64_t width, int32_t out_width,
    int32_t num_slices, int32_t capacity, int32_t num_slots, int32_t max_segments, void* stream) {
  if (num_tokens < 0 || num_tokens >= (int64_t(1) << 31) || width < 1 || width >= (int64_t(1) << 31) ||
      out_width < 1 || num_slices < 1 || num_slices > 4 || capacity < 1 || num_slots < 1 || max_segments < 0)
    return fail(LF_E_INVALID, "lora_base_gemm: invalid sizes");
  if (width % 8 || x_stride % 8 || x_stride < width || w_stride % 8 || w_stride < width || !aligned16(x) ||
      !aligned16(w) || !aligned16(a) || !aligned16(b))
    return fail(LF_E_INVALID, "lora_base_gemm: x/W/A/B must be 16-byte aligned with width and strides multiples of 8");
  if (!aligned16(y) || y_stride % 8 || y_stride < out_width)
    return fail(LF_E_INVALID, "lora_base_gemm: y must be 16-byte aligned with a stride multiple of 8");
  const GemmLayout l = gemm_layout(num_tokens, width, num_slices, capacity);
  if (!workspace || workspace_floats < l.total || (reinterpret_cast<uintptr_t>(workspace) & 15))
    return fail(LF_E_INVALID, "lora_base_gemm: workspace too small or not 16-byte aligned "
                              "(see lf_lora_base_gemm_workspace_floats)");
  if (num_tokens == 0) return LF_OK;
  const cudaStream_t s = static_cast<cudaStream_t>(stream);
  float* ztok = workspace + l.ztok;
  int32_t* routes = reinterpret_cast<int32_t*>(workspace + l.routes);
  int32_t* lists = reinterpret_cast<int32_t*>(workspace + l.lists);
  // 1. The LoRA z rows by token: the prefill shrink over the segments (tcgen05 tiles).
  if (int rc = prefill_launch(x, x_stride, a, b, b_offsets, b_strides, y, y_stride, segment_indptr, segment_slots,
                              token_indices, ranks, scales, slice_offsets, segment_count, workspace + l.prefill,
                              l.ztok, num_tokens, width, out_width, num_slices, capacity, num_slots, max_segments,
                              0, stream, ztok))
    return rc;
  // 2. Each token's slot, and the distinct slots of every 128-token tile.
  if (int rc = lf_segment_routes(segment_indptr, segment_slots, token_indices, segment_count, max_segments,
                                 num_tokens, num_tokens, routes, stream))
    return rc;
  if (int rc = launch_pdl_ex(tile_slot_lists_kernel, dim3(l.mtiles), dim3(kBM), 0, s, "lora_base_gemm (slot lists)",
                             static_cast<const int32_t*>(routes), int(num_tokens), int(num_slots), lists))
    return rc;
  // 3. The GEMM with the LoRA terms in its mainloop.
  GParams p{static_cast<uint16_t*>(y), y_stride, static_cast<const uint16_t*>(b), b_offsets, b_strides, ranks,
            scales, routes, ztok, lists, slice_offsets, int(num_tokens), int(width), out_width, num_slices,
            capacity, num_slots, l.zpitch, l.mtiles, (out_width + kBN - 1) / kBN};
  {
    const PFN_cuTensorMapEncodeTiled_v12000 encode = gemm_tensor_map_encoder();
    if (!encode) return fail(LF_E_CUDA, "lora_base_gemm: cuTensorMapEncodeTiled unavailable");
    const cuuint32_t estr[2] = {1, 1};
    const cuuint64_t xdims[2] = {cuuint64_t(width), cuuint64_t(num_tokens)};
    const cuuint64_t xstr[1] = {cuuint64_t(x_stride) * 2};
    const cuuint32_t xbox[2] = {64u, cuuint32_t(kBM)};
    const cuuint64_t wdims[2] = {cuuint64_t(width), cuuint64_t(out_width)};
    const cuuint64_t wstr[1] = {cuuint64_t(w_stride) * 2};
    const cuuint32_t wbox[2] = {64u, cuuint32_t(kBN)};
    CUresult r = encode(&p.tmap_x, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(x), xdims, xstr, xbox, estr,
                        CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                        CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r == CUDA_SUCCESS)
      r = encode(&p.tmap_w, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(w), wdims, wstr, wbox, estr,
                 CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                 CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    for (int m = 0; m < 3 && r == CUDA_SUCCESS; ++m) {
      const int kb = 16 << m;
      const cuuint64_t bdims[2] = {cuuint64_t(kb), cuuint64_t(kBRows)};
      const cuuint64_t bstr[1] = {cuuint64_t(kb) * 2};
      const cuuint32_t bbox[2] = {cuuint32_t(kb), cuuint32_t(kBN)};
      const CUtensorMapSwizzle sw =
          m == 0 ? CU_TENSOR_MAP_SWIZZLE_32B : m == 1 ? CU_TENSOR_MAP_SWIZZLE_64B : CU_TENSOR_MAP_SWIZZLE_128B;
      r = encode(&p.tmap_b[m], CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(b), bdims, bstr, bbox, estr,
                 CU_TENSOR_MAP_INTERLEAVE_NONE, sw, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                 CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    }
    if (r != CUDA_SUCCESS) return fail(LF_E_CUDA, "lora_base_gemm: cuTensorMapEncodeTiled failed");
  }
  int device = 0, sms = 0;
  if (cudaGetDevice(&device) != cudaSuccess ||
      cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, device) != cudaSuccess)
    return check_launch("lora_base_gemm: device query");
  const int smem = kStages * kStageBytes + 2 * kZBytes + kLBBytes + 1024 + 256;
  static int flags[64] = {};
  if (int rc = ensure_smem(base_lora_gemm_kernel, smem, flags)) return rc;
  const int tiles = p.mtiles * p.ntiles;
  return launch_pdl_ex(base_lora_gemm_kernel, dim3(tiles < sms ? tiles : sms), dim3(kThreads), smem, s,
                       "lora_base_gemm", p);
}
