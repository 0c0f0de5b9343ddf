// runtime.cuh -- host-side helpers shared by the C-ABI entry points.
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>
#include <stdint.h>

namespace inferd {

// Records the CUDA error string for inferd_last_cuda_error() and maps it to a status.
int cuda_status(cudaError_t err);

// Launch-error check after a <<<>>> launch.
inline int launch_status() { return cuda_status(cudaGetLastError()); }

// Streaming-multiprocessor count of the current device (cached per device).
int current_sm_count();
int current_device();

// cuTensorMapEncodeTiled obtained through the runtime's driver entry point, so the
// library does not link libcuda directly.  Returns nullptr if unavailable.
typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*,
                                  const cuuint64_t*, const cuuint64_t*, const cuuint32_t*,
                                  const cuuint32_t*, CUtensorMapInterleave, CUtensorMapSwizzle,
                                  CUtensorMapL2promotion, CUtensorMapFloatOOBfill);
EncodeTiledFn encode_tiled_fn();

// True when inferd_paged_attention runs these arguments on its tensor-core fast path,
// the only path that uses the workspace (nq = q_len * q_heads / kv_heads).
bool paged_attention_fast_path(int32_t dtype, int32_t head_dim, int32_t block_size, int32_t nq,
                               int64_t num_blocks, int32_t num_kv_heads, const void* key_cache,
                               const void* value_cache, const void* query, const void* out);

}  // namespace inferd
