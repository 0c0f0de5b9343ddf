// peer.cu -- gathering per-rank outputs into every rank's memory over NVLink, without a
// collective library call.
//
// Sequence-sharded decode has one exchange per step: every rank needs the attention
// outputs of all ranks' sequences, in rank order.  Each rank owns one peer buffer in its
// own HBM, mapped into every other rank's address space through CUDA IPC:
//
//     [0, 256)            flags: uint32 per source rank, the last epoch it published
//     [256, 512)          this rank's push counters: uint32 per destination rank
//     [512, ...)          slot 0, then slot 1: world x bytes_per_rank each
//
// A step's push kernel copies this rank's output (bytes_per_rank) into slot s of every
// rank's buffer at offset rank * bytes_per_rank with plain 16-byte stores (through NVLink
// for peers), kPushCtas CTAs per destination so that enough SMs feed each link.  The CTA
// that finishes a destination last (a counter in this rank's own header) publishes the
// step's epoch in that rank's flag for this rank (system-scope release).  The wait kernel spins, bounded, until this
// rank's flags all carry the epoch (system-scope acquire); once it completes, slot s holds
// every rank's rows.  Slots alternate by step: a rank pushes step N + 2 into slot s only
// after its own wait for step N + 1, i.e. after every rank pushed step N + 1, which each
// did after finishing its work on step N's data (stream order).
//
// Waits never spin forever: after the timeout the kernel records INFERD_ERR_DEVICE_TIMEOUT
// and returns, so a rank that stopped publishing leaves the others with an error instead
// of a hung GPU.  No TMA or multicast touches peer memory; the stores are ordinary ones.
#include <cstring>

#include "common.cuh"
#include "runtime.cuh"

namespace inferd {
namespace {

constexpr int kPushThreads = 256;
constexpr int kPushCtas = 16;  // CTAs per destination
constexpr int kMaxWorld = 64;
constexpr int kCounterOffset = 256;  // bytes: the push counters in this rank's own header

__device__ __forceinline__ void st_release_sys(uint32_t* p, uint32_t v) {
  asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ uint32_t ld_acquire_sys(const uint32_t* p) {
  uint32_t v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

// CTA (d, c) copies part c of src into dst[d] + rank * bytes; the last of destination d's
// CTAs to finish publishes epoch in flags[d][rank].  counters: this rank's own header.
__global__ void __launch_bounds__(kPushThreads) gather_push_kernel(
    const uint8_t* __restrict__ src, int64_t bytes, uint8_t* const* __restrict__ dst,
    uint32_t* const* __restrict__ flags, uint32_t* __restrict__ counters, int32_t rank,
    uint32_t epoch) {
  __shared__ int last;
  const int d = blockIdx.x / kPushCtas, part = blockIdx.x % kPushCtas;
  uint8_t* out = dst[d] + static_cast<int64_t>(rank) * bytes;
  const int64_t n16 = bytes / 16;  // bytes is a multiple of 16
  const int64_t lo = n16 * part / kPushCtas, hi = n16 * (part + 1) / kPushCtas;
  const uint4* s4 = reinterpret_cast<const uint4*>(src);
  uint4* o4 = reinterpret_cast<uint4*>(out);
  int64_t i = lo + threadIdx.x;
  for (; i + kPushThreads < hi; i += 2 * kPushThreads) {  // two 16-byte loads in flight
    const uint4 a = __ldg(s4 + i), b = __ldg(s4 + i + kPushThreads);
    o4[i] = a;
    o4[i + kPushThreads] = b;
  }
  for (; i < hi; i += kPushThreads) o4[i] = __ldg(s4 + i);
  __threadfence_system();  // this thread's stores before the counter, at system scope
  __syncthreads();
  if (threadIdx.x == 0) {
    // counters only grow: every push adds kPushCtas per destination
    last = (atomicAdd(counters + d, 1u) + 1u) % kPushCtas == 0;
  }
  __syncthreads();
  if (threadIdx.x == 0 && last) {
    __threadfence_system();  // the other CTAs' stores, seen through their counter updates
    st_release_sys(flags[d] + rank, epoch);
  }
}

// Thread d < world publishes epoch in flags[d][rank]: the rows of this epoch were stored
// into every rank's slot by the grids before this one on the stream (the attention kernel's
// fused epilogue), which completed before this grid started.
__global__ void __launch_bounds__(kMaxWorld) gather_publish_kernel(uint32_t* const* flags, int32_t rank,
                                                                   int32_t world, uint32_t epoch) {
  const int d = threadIdx.x;
  if (d < world) {
    __threadfence_system();
    st_release_sys(flags[d] + rank, epoch);
  }
}

// Lane r < world waits until flags[r] has reached epoch (wrap-safe compare).
__global__ void __launch_bounds__(kMaxWorld) gather_wait_kernel(const uint32_t* flags, int32_t world,
                                                                uint32_t epoch, uint64_t timeout_ns,
                                                                int32_t* error_word) {
  const int r = threadIdx.x;
  if (r < world) {
    const uint64_t t0 = globaltimer();
    uint32_t iters = 0;
    while (static_cast<int32_t>(ld_acquire_sys(flags + r) - epoch) < 0) {
      if (++iters >= kWaitMaxIters || globaltimer() - t0 > timeout_ns) {
        report_error(error_word, INFERD_ERR_DEVICE_TIMEOUT);
        break;
      }
      __nanosleep(64);
    }
  }
  __syncthreads();
}

inline bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

}  // namespace
}  // namespace inferd

using namespace inferd;

extern "C" INFERD_API int inferd_peer_alloc(size_t bytes, void** ptr, void* ipc_handle) {
  if (bytes == 0 || ptr == nullptr || ipc_handle == nullptr) return INFERD_ERR_INVALID_ARGUMENT;
  void* p = nullptr;
  int st = cuda_status(cudaMalloc(&p, bytes));
  if (st != INFERD_OK) return st;
  st = cuda_status(cudaMemset(p, 0, bytes));
  cudaIpcMemHandle_t h;
  if (st == INFERD_OK) st = cuda_status(cudaIpcGetMemHandle(&h, p));
  if (st != INFERD_OK) {
    cudaFree(p);
    return st;
  }
  static_assert(sizeof(cudaIpcMemHandle_t) == INFERD_IPC_HANDLE_BYTES, "IPC handle size");
  memcpy(ipc_handle, &h, sizeof(h));
  *ptr = p;
  return INFERD_OK;
}

extern "C" INFERD_API int inferd_peer_open(const void* ipc_handle, void** ptr) {
  if (ipc_handle == nullptr || ptr == nullptr) return INFERD_ERR_INVALID_ARGUMENT;
  cudaIpcMemHandle_t h;
  memcpy(&h, ipc_handle, sizeof(h));
  return cuda_status(cudaIpcOpenMemHandle(ptr, h, cudaIpcMemLazyEnablePeerAccess));
}

extern "C" INFERD_API int inferd_peer_close(void* ptr) {
  if (ptr == nullptr) return INFERD_ERR_INVALID_ARGUMENT;
  return cuda_status(cudaIpcCloseMemHandle(ptr));
}

extern "C" INFERD_API int inferd_peer_free(void* ptr) {
  if (ptr == nullptr) return INFERD_ERR_INVALID_ARGUMENT;
  return cuda_status(cudaFree(ptr));
}

extern "C" INFERD_API int inferd_gather_push(const void* src, int64_t bytes, void* const* dst,
                                             uint32_t* const* flags, uint32_t* counters, int32_t rank,
                                             int32_t world, uint32_t epoch, void* stream) {
  if (bytes < 0 || world <= 0 || world > kMaxWorld || rank < 0 || rank >= world)
    return INFERD_ERR_INVALID_ARGUMENT;
  if (dst == nullptr || flags == nullptr || (bytes > 0 && src == nullptr)) return INFERD_ERR_INVALID_ARGUMENT;
  if (!aligned16(src) || bytes % 16 != 0) return INFERD_ERR_INVALID_ARGUMENT;  // rows are 16-byte multiples
  if (counters == nullptr) return INFERD_ERR_INVALID_ARGUMENT;
  gather_push_kernel<<<world * kPushCtas, kPushThreads, 0, static_cast<cudaStream_t>(stream)>>>(
      static_cast<const uint8_t*>(src), bytes, reinterpret_cast<uint8_t* const*>(dst), flags, counters, rank,
      epoch);
  return launch_status();
}

extern "C" INFERD_API int inferd_gather_wait(const uint32_t* flags, int32_t world, uint32_t epoch,
                                             uint64_t timeout_ns, int32_t* error_word, void* stream) {
  if (flags == nullptr || world <= 0 || world > kMaxWorld) return INFERD_ERR_INVALID_ARGUMENT;
  if (timeout_ns == 0 || timeout_ns > kWaitTimeoutNs) timeout_ns = kWaitTimeoutNs;
  gather_wait_kernel<<<1, kMaxWorld, 0, static_cast<cudaStream_t>(stream)>>>(flags, world, epoch,
                                                                            timeout_ns, error_word);
  return launch_status();
}

extern "C" INFERD_API int inferd_gather_publish(uint32_t* const* flags, int32_t rank, int32_t world,
                                                uint32_t epoch, void* stream) {
  if (flags == nullptr || world <= 0 || world > kMaxWorld || rank < 0 || rank >= world)
    return INFERD_ERR_INVALID_ARGUMENT;
  gather_publish_kernel<<<1, kMaxWorld, 0, static_cast<cudaStream_t>(stream)>>>(flags, rank, world, epoch);
  return launch_status();
}
