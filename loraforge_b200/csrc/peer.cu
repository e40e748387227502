// One-shot sum of the row-parallel LoRA intermediate over NVLink peer memory.
//
// Row-parallel projections (A's input columns sharded over G ranks) leave every rank with
// a partial FP32 z of [tokens, S*r] rows; the expand needs their sum.  At decode sizes
// this is tens of KiB, so the cost is latency, not bandwidth.  Instead of a library
// all-reduce, each rank owns one symmetric buffer (cudaMalloc + CUDA IPC, mapped by every
// peer) and a single kernel does the exchange in one pass:
//
//   1. each of kPeerCtas CTAs copies its slice of the local partial into the rank's own
//      buffer (slot = epoch & 1, double-buffered across calls);
//   2. after a CTA barrier over its copies, one thread per peer stores the epoch into the
//      CTA's flag in that peer's buffer with st.release.sys (release is cumulative: the
//      barrier orders the other threads' copies before it, so a peer that acquires the
//      flag sees the whole slice), then waits until every peer's flag for this CTA index
//      in its own buffer has reached the epoch (ld.acquire.sys, bounded);
//   3. it sums the slice over the G peers' buffers in rank order (P2P loads over NVLink)
//      into the local z rows, so every rank gets the same bits.
//
// The epoch is a per-CTA counter in the rank's own buffer, advanced by the kernel, so a
// CUDA graph that captured the call replays correctly.  Double buffering makes one
// barrier per call enough: a peer can only overwrite slot e & 1 in call e + 2, after the
// barrier of call e + 1, which this rank joins only when its call e has finished reading.
// Every wait is bounded; on expiry the kernel sets the status word of the rank's buffer,
// leaves its z rows partial and returns (lf_peer_status reads the word).
#include <cstring>

#include "common.cuh"

namespace lfb {
namespace {

constexpr int kPeerCtas = 16;
constexpr int kPeerThreads = 256;
constexpr int kPeerMaxWorld = 16;
// Symmetric buffer layout (bytes): flags [kPeerCtas][kPeerMaxWorld] u32, then one epoch
// counter per CTA, then the status word, then two slots of `capacity` floats.
constexpr int kFlagsBytes = kPeerCtas * kPeerMaxWorld * 4;
constexpr int kCounterOffset = kFlagsBytes;
constexpr int kStatusOffset = kCounterOffset + kPeerCtas * 4;
constexpr int kSlotOffset = 2048;
constexpr long long kSpinLimit = 1ll << 22;  // polls of a local word (~0.2-0.4 us each): under 2 s

__device__ __forceinline__ void store_release_sys(uint32_t* p, uint32_t v) {
  asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ uint32_t load_acquire_sys(const uint32_t* p) {
  uint32_t v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

__global__ void __launch_bounds__(kPeerThreads) peer_sum_kernel(const uint64_t* __restrict__ bases,
                                                                int rank, int world, float* z,
                                                                int64_t floats, int64_t capacity,
                                                                long long spin_limit) {
  __shared__ uint32_t epoch_s;
  __shared__ int ok_s;
  const int tid = threadIdx.x, cta = blockIdx.x;
  uint8_t* own = reinterpret_cast<uint8_t*>(bases[rank]);
  if (tid == 0) {
    uint32_t* ctr = reinterpret_cast<uint32_t*>(own + kCounterOffset) + cta;
    epoch_s = *ctr + 1u;
    *ctr = epoch_s;
    ok_s = 1;
  }
  __syncthreads();
  const uint32_t epoch = epoch_s;
  const int64_t slot_off = kSlotOffset + int64_t(epoch & 1u) * capacity * 4;
  // This CTA's slice of the rows, in float4 units when the size allows.
  const bool vec = (floats & 3) == 0;
  const int64_t units = vec ? floats / 4 : floats;
  const int64_t per = (units + kPeerCtas - 1) / kPeerCtas;
  const int64_t u0 = min(units, cta * per), u1 = min(units, u0 + per);
  float* mine = reinterpret_cast<float*>(own + slot_off);
  for (int64_t u = u0 + tid; u < u1; u += kPeerThreads) {
    if (vec) reinterpret_cast<float4*>(mine)[u] = reinterpret_cast<const float4*>(z)[u];
    else mine[u] = z[u];
  }
  __syncthreads();
  if (tid < world) {
    // The barrier above orders the CTA's copies before this thread's release store, and
    // a release is cumulative: the peer that acquires the flag sees the whole slice.
    uint8_t* peer = reinterpret_cast<uint8_t*>(bases[tid]);
    store_release_sys(reinterpret_cast<uint32_t*>(peer) + cta * kPeerMaxWorld + rank, epoch);
    const uint32_t* flag = reinterpret_cast<const uint32_t*>(own) + cta * kPeerMaxWorld + tid;
    long long it = 0;
    while (int32_t(load_acquire_sys(flag) - epoch) < 0) {
      if (++it > spin_limit) {
        ok_s = 0;
        atomicOr(reinterpret_cast<int*>(own + kStatusOffset), 1);
        break;
      }
    }
  }
  __syncthreads();
  if (!ok_s) return;  // a peer never arrived: z keeps this rank's partial
  for (int64_t u = u0 + tid; u < u1; u += kPeerThreads) {
    if (vec) {
      float4 s = make_float4(0.f, 0.f, 0.f, 0.f);
      for (int g = 0; g < world; ++g) {
        const float4 v = __ldcv(reinterpret_cast<const float4*>(reinterpret_cast<const uint8_t*>(bases[g]) + slot_off) + u);
        s.x += v.x;
        s.y += v.y;
        s.z += v.z;
        s.w += v.w;
      }
      reinterpret_cast<float4*>(z)[u] = s;
    } else {
      float s = 0.f;
      for (int g = 0; g < world; ++g)
        s += __ldcv(reinterpret_cast<const float*>(reinterpret_cast<const uint8_t*>(bases[g]) + slot_off) + u);
      z[u] = s;
    }
  }
}

}  // namespace
}  // namespace lfb

using namespace lfb;

extern "C" int64_t lf_peer_buffer_bytes(int64_t capacity_floats) {
  if (capacity_floats < 1) return -1;
  return kSlotOffset + 2 * capacity_floats * 4;
}

extern "C" int lf_peer_alloc(int64_t capacity_floats, void** buffer, void* ipc_handle) {
  const int64_t bytes = lf_peer_buffer_bytes(capacity_floats);
  if (bytes < 0 || !buffer || !ipc_handle) return fail(LF_E_INVALID, "peer_alloc: invalid arguments");
  *buffer = nullptr;
  if (cudaMalloc(buffer, size_t(bytes)) != cudaSuccess) return check_launch("peer_alloc: cudaMalloc");
  if (cudaMemset(*buffer, 0, size_t(bytes)) != cudaSuccess ||
      cudaIpcGetMemHandle(static_cast<cudaIpcMemHandle_t*>(ipc_handle), *buffer) != cudaSuccess) {
    const int rc = check_launch("peer_alloc: cudaMemset / cudaIpcGetMemHandle");
    cudaFree(*buffer);
    *buffer = nullptr;
    return rc;
  }
  return LF_OK;
}

extern "C" int lf_peer_handle_bytes(void) { return int(sizeof(cudaIpcMemHandle_t)); }

extern "C" int lf_peer_open(const void* ipc_handle, void** buffer) {
  if (!ipc_handle || !buffer) return fail(LF_E_INVALID, "peer_open: null argument");
  cudaIpcMemHandle_t h;
  memcpy(&h, ipc_handle, sizeof(h));
  if (cudaIpcOpenMemHandle(buffer, h, cudaIpcMemLazyEnablePeerAccess) != cudaSuccess)
    return check_launch("peer_open: cudaIpcOpenMemHandle");
  return LF_OK;
}

extern "C" int lf_peer_close(void* buffer) {
  if (buffer && cudaIpcCloseMemHandle(buffer) != cudaSuccess) return check_launch("peer_close");
  return LF_OK;
}

extern "C" int lf_peer_free(void* buffer) {
  if (buffer && cudaFree(buffer) != cudaSuccess) return check_launch("peer_free");
  return LF_OK;
}

extern "C" int lf_peer_status(void* own_buffer, int32_t* status, int32_t reset) {
  if (!own_buffer || !status) return fail(LF_E_INVALID, "peer_status: null argument");
  int32_t v = 0;
  if (cudaMemcpy(&v, static_cast<uint8_t*>(own_buffer) + kStatusOffset, 4, cudaMemcpyDeviceToHost) != cudaSuccess)
    return check_launch("peer_status");
  *status = v;
  if (reset) {
    const int32_t zero = 0;
    if (cudaMemcpy(static_cast<uint8_t*>(own_buffer) + kStatusOffset, &zero, 4, cudaMemcpyHostToDevice) != cudaSuccess)
      return check_launch("peer_status");
  }
  return LF_OK;
}

extern "C" int lf_peer_sum(const uint64_t* bases, int32_t rank, int32_t world, float* z, int64_t floats,
                           int64_t capacity_floats, int64_t spin_limit, void* stream) {
  if (world < 1 || world > kPeerMaxWorld || rank < 0 || rank >= world)
    return fail(LF_E_INVALID, "peer_sum: world must be 1..16 and rank in [0, world)");
  if (floats < 0 || floats > capacity_floats) return fail(LF_E_INVALID, "peer_sum: more floats than the buffer holds");
  if (!bases || (floats && !z)) return fail(LF_E_INVALID, "peer_sum: null pointer");
  if ((reinterpret_cast<uintptr_t>(z) & 15) != 0) return fail(LF_E_INVALID, "peer_sum: z must be 16-byte aligned");
  const long long limit = spin_limit > 0 && spin_limit < kSpinLimit ? spin_limit : kSpinLimit;
  peer_sum_kernel<<<kPeerCtas, kPeerThreads, 0, static_cast<cudaStream_t>(stream)>>>(bases, rank, world, z, floats,
                                                                                     capacity_floats, limit);
  return check_launch("peer_sum");
}
