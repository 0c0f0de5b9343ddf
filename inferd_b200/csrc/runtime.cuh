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

}  // namespace inferd
