// paged_attention_noalloc.cu -- paged attention for callers that cannot allocate.
//
// Some callers of this library cannot allocate device memory when they call it: hosts
// that bind the C ABI through an FFI (Go, Java, Node) and have no device allocator of
// their own, and serving loops that fix their device-memory budget at start-up and
// treat any allocation during a decode step as an error.  inferd_paged_attention needs
// a caller-provided workspace for its split partials and ticket counters; this entry
// point instead uses a fixed scratch area that lives in the library itself.
//
// The scratch is one file-scope __device__ array of kNoAllocScratchBytes (32 MiB).
// Every GPU that loads the library holds it until the process exits.  All calls on a
// device share it and it keeps the previous call's contents, so:
//   * each call clears the ticket counters at its head before launching;
//   * calls whose executions overlap on the GPU (different streams, no ordering) race
//     on the scratch and give wrong results -- order them on one stream.
// Only the tensor-core path uses scratch; shapes that run on the generic path (fp32,
// head_dim != 128, block_size != 16, more than 32 query rows per kv head) need none and
// are never refused for their size.
// The scratch's device address is looked up on a device's first call and kept for the
// life of the process.  It is not looked up again after cudaDeviceReset() or anything
// else that replaces the device's primary context, so such a process must not call this
// entry point again on that device.
#include <mutex>

#include "common.cuh"
#include "runtime.cuh"

namespace inferd {
namespace {

constexpr size_t kNoAllocScratchBytes = size_t{32} << 20;  // 32 MiB
constexpr int kMaxDevices = 64;

static __device__ __align__(256) uint8_t g_noalloc_scratch[kNoAllocScratchBytes];

// Device address of g_noalloc_scratch per device.  In host code the symbol is only a
// host-side stand-in, so the real address is looked up once per device with the device
// current (cudaGetSymbolAddress) and passed to the kernels as a plain pointer.
std::mutex g_scratch_mu;
void* g_scratch_ptr[kMaxDevices] = {nullptr};

int scratch_for_current_device(void** out) {
  const int dev = current_device();
  if (dev < 0 || dev >= kMaxDevices) return INFERD_ERR_UNSUPPORTED;
  std::lock_guard<std::mutex> lock(g_scratch_mu);
  if (g_scratch_ptr[dev] == nullptr) {
    void* p = nullptr;
    const cudaError_t e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
    if (e != cudaSuccess || p == nullptr) return cuda_status(e != cudaSuccess ? e : cudaErrorUnknown);
    g_scratch_ptr[dev] = p;
  }
  *out = g_scratch_ptr[dev];
  return INFERD_OK;
}

}  // namespace
}  // namespace inferd

using namespace inferd;

extern "C" int inferd_paged_attention_noalloc(
    void* out, const void* query, const void* key_cache, const void* value_cache,
    const void* block_tables, int32_t block_table_bytes, int64_t block_table_stride,
    const int32_t* context_lens, int32_t num_seqs, int32_t q_len, int32_t num_q_heads,
    int32_t num_kv_heads, int32_t head_dim, int32_t block_size, int64_t num_blocks,
    int32_t max_context_len, float scale, int32_t dtype, int32_t* error_word, void* stream) {
  if (num_seqs < 0 || q_len <= 0 || num_q_heads <= 0 || num_kv_heads <= 0 || head_dim <= 0)
    return INFERD_ERR_INVALID_ARGUMENT;
  if (num_seqs == 0) return INFERD_OK;
  if (num_q_heads % num_kv_heads != 0) return INFERD_ERR_INVALID_ARGUMENT;
  const int32_t nq = q_len * (num_q_heads / num_kv_heads);
  const bool fast = paged_attention_fast_path(dtype, head_dim, block_size, nq, num_blocks,
                                              num_kv_heads, key_cache, value_cache, query, out);
  if (fast) {
    const size_t need = inferd_paged_attention_workspace_bytes(
        num_seqs, q_len, num_q_heads, num_kv_heads, head_dim, current_device());
    if (need > kNoAllocScratchBytes) return INFERD_ERR_WORKSPACE;  // beyond the static area
  }
  void* scratch = nullptr;
  int st = scratch_for_current_device(&scratch);
  if (st != INFERD_OK) return st;
  if (fast) {
    // The ticket counters must start at zero; an earlier call that did not complete
    // could have left them otherwise, so clear them on the caller's stream every time.
    // The counter size is that of one launch chunk (the function clamps to it).
    const size_t counters = inferd_paged_attention_counter_bytes(num_seqs, num_kv_heads);
    st = cuda_status(cudaMemsetAsync(scratch, 0, counters, static_cast<cudaStream_t>(stream)));
    if (st != INFERD_OK) return st;
  }
  return inferd_paged_attention(out, query, key_cache, value_cache, block_tables,
                                block_table_bytes, block_table_stride, context_lens, num_seqs,
                                q_len, num_q_heads, num_kv_heads, head_dim, block_size,
                                num_blocks, max_context_len, scale, dtype, scratch,
                                kNoAllocScratchBytes, error_word, stream);
}
