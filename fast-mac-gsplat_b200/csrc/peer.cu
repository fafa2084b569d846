// Sum of a float buffer across the GPUs of one node over NVLink peer memory
// (replaces the NCCL all-reduce of the shared-Gaussian gradients; the
// reference is single-device and has no counterpart).
//
// Every rank owns one buffer, cudaMalloc'ed here and mapped into the other
// ranks' processes through CUDA IPC: GSB_PEER_FLAG_BYTES of flags, then the
// data. Flag words (uint32): [0, 8) start-barrier slots, [8, 16) end-barrier
// slots and [16, 24) abort slots, one per source rank, written by the peers;
// word 32 counts finished CTAs of the local kernel and word 33 records that one
// of them gave up.
//
// One kernel per call and rank (two-shot all-reduce):
//   start barrier  every rank's data is final when its kernel starts, so each
//                  CTA announces it in every peer's slot (idempotent stores,
//                  release at system scope) and waits for all ranks' slots;
//   reduce         rank r owns shard r of the data: it loads that shard from
//                  all ranks' buffers (peer loads over NVLink), adds, and
//                  stores the sum into all ranks' buffers (peer stores);
//   end barrier    the last CTA to finish (fence + counter) announces the end
//                  and waits for every rank's, so when the kernel ends every
//                  shard of the local buffer holds the sum.
// Waits are bounded by the global timer (wait_ns per barrier). A rank whose
// wait runs out, or that finds a peer already past this call's epoch, gives up
// the call: it writes the epoch into its abort slot of every peer's buffer,
// raises GSB_DEVERR_PEER_TIMEOUT, skips its share of the sum and the end
// barrier, and returns. A rank
// that finds such an abort mark while it waits gives up the same way, and the
// end barrier reports a peer's abort of this epoch even when the wait itself
// was satisfied, so a rank that arrives late after a peer gave up never
// reports a clean sum (its peer may already have moved its buffer on). The
// host must not use the buffer after a call that raised the flag. The data
// moves by plain 16-byte loads and stores to peer memory.
#include <algorithm>
#include <cstring>

#include "gsb_common.cuh"
#include "gsb_host.cuh"

namespace gsb {
namespace {

constexpr int kPeerThreads = 256;
constexpr int kPeerUnroll = 4;  // float4 per thread per round, per rank
constexpr unsigned long long kPeerDefaultWaitNs = 10ull * 1000ull * 1000ull * 1000ull;
// Flag words: start slots, end slots and abort slots (one per source rank),
// the local kernel's finished-CTA counter and its failure word.
constexpr int kFlagStart = 0, kFlagEnd = 8, kFlagAbort = 16, kFlagCounter = 32, kFlagFail = 33;

struct PeerArgs {
  float4* data[GSB_PEER_MAX_RANKS];
  uint32_t* flags[GSB_PEER_MAX_RANKS];
};

__device__ __forceinline__ unsigned long long global_ns() {
  unsigned long long t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}
__device__ __forceinline__ void st_release_sys(uint32_t* p, uint32_t v) {
  asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ uint32_t ld_acquire_sys(const uint32_t* p) {
  uint32_t v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

// True when some peer wrote an abort mark for this epoch (or a later one:
// wrap-safe comparison; 0 means never) into this rank's buffer.
__device__ bool peer_aborted(const uint32_t* own, int world, uint32_t epoch) {
  for (int p = 0; p < world; ++p) {
    const uint32_t a = ld_acquire_sys(&own[kFlagAbort + p]);
    if (a != 0u && (int32_t)(a - epoch) >= 0) return true;
  }
  return false;
}

// Waits until slots[0 .. world) (in this rank's own buffer) equal `epoch`.
// False when the wait ran past wait_ns, when a peer aborted this epoch, or when
// a slot is already past it (that peer has left this call without us).
__device__ bool wait_slots(const uint32_t* own, int first_slot, int world, uint32_t epoch,
                           unsigned long long wait_ns) {
  const unsigned long long t0 = global_ns();
  for (int p = 0; p < world; ++p) {
    for (;;) {
      const int32_t d = (int32_t)(ld_acquire_sys(&own[first_slot + p]) - epoch);
      if (d > 0) return false;
      if (d == 0) break;
      if (peer_aborted(own, world, epoch) || global_ns() - t0 > wait_ns) return false;
      __nanosleep(100);
    }
  }
  return !peer_aborted(own, world, epoch);
}

// Gives up this call: marks the epoch in this rank's abort slot of every
// buffer (so the peers stop waiting) and raises the error flag.
__device__ void abort_call(const PeerArgs& a, int rank, int world, uint32_t epoch, uint32_t* status, uint32_t site) {
  __threadfence_system();
  for (int p = 0; p < world; ++p) st_release_sys(&a.flags[p][kFlagAbort + rank], epoch);
  raise_error(status, GSB_DEVERR_PEER_TIMEOUT, site);
}

__device__ __forceinline__ float4 add4(float4 a, float4 b) {
  return make_float4(a.x + b.x, a.y + b.y, a.z + b.z, a.w + b.w);
}

__global__ void __launch_bounds__(kPeerThreads)
    k_peer_allreduce(PeerArgs a, int rank, int world, int64_t lo, int64_t hi, uint32_t epoch,
                     unsigned long long wait_ns, uint32_t* __restrict__ status) {
  pdl_wait();
  pdl_trigger();
  __shared__ int s_ok, s_last;
  uint32_t* own = a.flags[rank];
  if ((int)threadIdx.x < world) {
    __threadfence_system();
    st_release_sys(&a.flags[threadIdx.x][kFlagStart + rank], epoch);
  }
  if (threadIdx.x == 0) {
    s_ok = wait_slots(own, kFlagStart, world, epoch, wait_ns);
    if (!s_ok) {
      atomicOr(&own[kFlagFail], 1u);
      abort_call(a, rank, world, epoch, status, kSitePeerStart);
    }
  }
  __syncthreads();
  if (s_ok) {
    const int64_t step = (int64_t)gridDim.x * kPeerThreads * kPeerUnroll;
    for (int64_t base = lo + (int64_t)blockIdx.x * kPeerThreads * kPeerUnroll + threadIdx.x; base < hi;
         base += step) {
      float4 acc[kPeerUnroll];
#pragma unroll
      for (int u = 0; u < kPeerUnroll; ++u) {
        const int64_t i = base + (int64_t)u * kPeerThreads;
        acc[u] = i < hi ? a.data[0][i] : make_float4(0.f, 0.f, 0.f, 0.f);
      }
      for (int p = 1; p < world; ++p) {
        float4 v[kPeerUnroll];
#pragma unroll
        for (int u = 0; u < kPeerUnroll; ++u) {
          const int64_t i = base + (int64_t)u * kPeerThreads;
          v[u] = i < hi ? a.data[p][i] : make_float4(0.f, 0.f, 0.f, 0.f);
        }
#pragma unroll
        for (int u = 0; u < kPeerUnroll; ++u) acc[u] = add4(acc[u], v[u]);
      }
      for (int p = 0; p < world; ++p) {
#pragma unroll
        for (int u = 0; u < kPeerUnroll; ++u) {
          const int64_t i = base + (int64_t)u * kPeerThreads;
          if (i < hi) a.data[p][i] = acc[u];
        }
      }
    }
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    __threadfence_system();  // this CTA's stores (seen through the barrier) before the count
    s_last = atomicAdd(&own[kFlagCounter], 1u) == gridDim.x - 1;
  }
  __syncthreads();
  if (s_last && threadIdx.x == 0) {
    // Every CTA of this kernel has counted itself: the failure word is final.
    const bool failed = ld_volatile_u32(&own[kFlagFail]) != 0u;
    if (!failed) {
      __threadfence_system();
      for (int p = 0; p < world; ++p) st_release_sys(&a.flags[p][kFlagEnd + rank], epoch);
      if (!wait_slots(own, kFlagEnd, world, epoch, wait_ns)) abort_call(a, rank, world, epoch, status, kSitePeerEnd);
    }
    own[kFlagCounter] = 0;  // the next call starts after this kernel has ended
    own[kFlagFail] = 0;
  }
}

}  // namespace
}  // namespace gsb

using namespace gsb;

static_assert(sizeof(cudaIpcMemHandle_t) == GSB_PEER_HANDLE_BYTES, "IPC handle size");

extern "C" int gsb_peer_buffer_alloc(size_t data_bytes, void** base) {
  if (base == nullptr) return GSB_ERR_INVALID_ARGUMENT;
  void* p = nullptr;
  if (cudaMalloc(&p, GSB_PEER_FLAG_BYTES + data_bytes) != cudaSuccess) return GSB_ERR_CUDA;
  if (cudaMemset(p, 0, GSB_PEER_FLAG_BYTES) != cudaSuccess) {
    cudaFree(p);
    return GSB_ERR_CUDA;
  }
  *base = p;
  return GSB_OK;
}

extern "C" int gsb_peer_buffer_free(void* base) { return cuda_status(cudaFree(base)); }

extern "C" int gsb_peer_handle(const void* base, void* handle) {
  if (base == nullptr || handle == nullptr) return GSB_ERR_INVALID_ARGUMENT;
  return cuda_status(cudaIpcGetMemHandle(static_cast<cudaIpcMemHandle_t*>(handle), const_cast<void*>(base)));
}

extern "C" int gsb_peer_open(const void* handle, void** base) {
  if (base == nullptr || handle == nullptr) return GSB_ERR_INVALID_ARGUMENT;
  cudaIpcMemHandle_t h;
  memcpy(&h, handle, sizeof(h));
  return cuda_status(cudaIpcOpenMemHandle(base, h, cudaIpcMemLazyEnablePeerAccess));
}

extern "C" int gsb_peer_close(void* base) { return cuda_status(cudaIpcCloseMemHandle(base)); }

extern "C" int gsb_peer_allreduce_sum(int32_t rank, int32_t world, void* const* bases, int64_t n_floats,
                                      uint32_t epoch, uint64_t wait_ns, uint32_t* status, void* stream) {
  if (world < 1 || world > GSB_PEER_MAX_RANKS || rank < 0 || rank >= world || bases == nullptr || n_floats < 0 ||
      (n_floats & 3) != 0 || epoch == 0u || status == nullptr)
    return GSB_ERR_INVALID_ARGUMENT;
  if (wait_ns == 0) wait_ns = kPeerDefaultWaitNs;
  if (world == 1) return GSB_OK;  // the sum over one rank is the buffer itself
  PeerArgs a;
  for (int r = 0; r < GSB_PEER_MAX_RANKS; ++r) {
    char* b = r < world ? static_cast<char*>(bases[r]) : nullptr;
    if (r < world && b == nullptr) return GSB_ERR_INVALID_ARGUMENT;
    a.flags[r] = reinterpret_cast<uint32_t*>(b);
    a.data[r] = b ? reinterpret_cast<float4*>(b + GSB_PEER_FLAG_BYTES) : nullptr;
  }
  const int64_t n4 = n_floats / 4;
  const int64_t shard = (n4 + world - 1) / world;
  const int64_t lo = std::min<int64_t>(n4, (int64_t)rank * shard);
  const int64_t hi = std::min<int64_t>(n4, lo + shard);
  int sms = 148, dev = 0;
  if (cudaGetDevice(&dev) == cudaSuccess) cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  const int64_t per_cta = (int64_t)kPeerThreads * kPeerUnroll;
  const int grid = (int)std::max<int64_t>(1, std::min<int64_t>(2 * (int64_t)sms, (hi - lo + per_cta - 1) / per_cta));
  const cudaError_t e = launch_pdl(k_peer_allreduce, grid, kPeerThreads, 0, static_cast<cudaStream_t>(stream), a,
                                   (int)rank, (int)world, lo, hi, epoch, (unsigned long long)wait_ns, status);
  note_launches(1);
  return cuda_status(e);
}
