// runtime.cu -- status strings, error capture, device queries and the driver entry
// point used to build TMA tensor maps.
#include <mutex>

#include "common.cuh"
#include "runtime.cuh"

namespace inferd {

namespace {
thread_local char g_last_cuda_error[256] = {0};
std::mutex g_mu;
int g_sm_count[64] = {0};
EncodeTiledFn g_encode = nullptr;
bool g_encode_tried = false;
}  // namespace

int cuda_status(cudaError_t err) {
  if (err == cudaSuccess) return INFERD_OK;
  const char* s = cudaGetErrorString(err);
  size_t i = 0;
  for (; s != nullptr && s[i] != '\0' && i + 1 < sizeof(g_last_cuda_error); ++i)
    g_last_cuda_error[i] = s[i];
  g_last_cuda_error[i] = '\0';
  return INFERD_ERR_CUDA;
}

int current_device() {
  int dev = 0;
  cudaGetDevice(&dev);
  return dev;
}

int current_sm_count() {
  int dev = current_device();
  if (dev < 0 || dev >= 64) return 148;
  std::lock_guard<std::mutex> lock(g_mu);
  if (g_sm_count[dev] == 0) {
    int n = 0;
    if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n <= 0)
      n = 148;
    g_sm_count[dev] = n;
  }
  return g_sm_count[dev];
}

EncodeTiledFn encode_tiled_fn() {
  std::lock_guard<std::mutex> lock(g_mu);
  if (!g_encode_tried) {
    g_encode_tried = true;
    void* fn = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &fn, cudaEnableDefault, &q) ==
            cudaSuccess &&
        q == cudaDriverEntryPointSuccess) {
      g_encode = reinterpret_cast<EncodeTiledFn>(fn);
    }
  }
  return g_encode;
}

}  // namespace inferd

extern "C" {

int inferd_version(void) { return 100; }

const char* inferd_status_string(int status) {
  switch (status) {
    case INFERD_OK: return "ok";
    case INFERD_ERR_INVALID_ARGUMENT: return "invalid argument";
    case INFERD_ERR_UNSUPPORTED: return "unsupported dtype or size combination";
    case INFERD_ERR_WORKSPACE: return "workspace missing, misaligned or too small";
    case INFERD_ERR_CUDA: return "CUDA launch or runtime failure";
    case INFERD_ERR_DEVICE_INDEX: return "block id or slot outside the KV pool";
    case INFERD_ERR_DEVICE_TIMEOUT: return "a bounded device-side wait expired";
    default: return "unknown status";
  }
}

const char* inferd_last_cuda_error(void) { return inferd::g_last_cuda_error; }

int inferd_host_device_pointer(const void* host, void** device_ptr) {
  if (host == nullptr || device_ptr == nullptr) return INFERD_ERR_INVALID_ARGUMENT;
  void* d = nullptr;
  const cudaError_t e = cudaHostGetDevicePointer(&d, const_cast<void*>(host), 0);
  if (e != cudaSuccess) {
    const int st = inferd::cuda_status(e);
    cudaGetLastError();  // not sticky: leave no error for the next launch check
    return st;
  }
  *device_ptr = d;
  return INFERD_OK;
}

}  // extern "C"
