// Host-side plumbing of the C ABI: device binding, SM counts, the device-side error
// word that bounded waits set, and status strings.
#include <mutex>

#include "h3_common.cuh"

namespace h3host {

namespace {
constexpr int kMaxDevices = 64;
std::mutex g_mutex;
int g_sm_count[kMaxDevices] = {0};
int* g_error_word[kMaxDevices] = {nullptr};
}  // namespace

int bind_device_of(const void* ptr, int* device) {
  cudaPointerAttributes attr;
  cudaError_t e = cudaPointerGetAttributes(&attr, ptr);
  if (e != cudaSuccess) {
    cudaGetLastError();
    return H3_ERR_INVALID;
  }
  if (attr.type != cudaMemoryTypeDevice && attr.type != cudaMemoryTypeManaged)
    return H3_ERR_INVALID;  // host pointers are rejected: the path has no CPU fallback
  if (attr.device < 0 || attr.device >= kMaxDevices) return H3_ERR_INVALID;
  int cur = -1;
  if (cudaGetDevice(&cur) != cudaSuccess || cur != attr.device) {
    if (cudaSetDevice(attr.device) != cudaSuccess) return H3_ERR_CUDA;
  }
  *device = attr.device;
  return H3_OK;
}

int sm_count(int device) {
  if (device < 0 || device >= kMaxDevices) return 148;
  if (g_sm_count[device] == 0) {
    int n = 0;
    cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, device);
    g_sm_count[device] = n > 0 ? n : 148;
  }
  return g_sm_count[device];
}

int* error_word(int device) {
  if (device < 0 || device >= kMaxDevices) return nullptr;
  std::lock_guard<std::mutex> lock(g_mutex);
  if (g_error_word[device] == nullptr) {
    int* p = nullptr;
    if (cudaMalloc(&p, sizeof(int)) != cudaSuccess) return nullptr;
    if (cudaMemset(p, 0, sizeof(int)) != cudaSuccess) return nullptr;
    g_error_word[device] = p;
  }
  return g_error_word[device];
}

int check_launch() {
  cudaError_t e = cudaGetLastError();
  return e == cudaSuccess ? H3_OK : H3_ERR_CUDA;
}

}  // namespace h3host

extern "C" int h3_abi_version(void) { return 1; }

extern "C" const char* h3_status_string(int status) {
  switch (status) {
    case H3_OK: return "ok";
    case H3_ERR_INVALID: return "invalid argument or unsupported geometry";
    case H3_ERR_CUDA: return "CUDA runtime error";
    case H3_ERR_TIMEOUT: return "bounded device wait timed out";
    case H3_ERR_UNSUPPORTED: return "device is not sm_100";
    default: return "unknown status";
  }
}

extern "C" int h3_device_error(int device, int* code) {
  if (code == nullptr) return H3_ERR_INVALID;
  *code = 0;
  int cur = -1;
  cudaGetDevice(&cur);
  if (cur != device && cudaSetDevice(device) != cudaSuccess) return H3_ERR_CUDA;
  int* w = h3host::error_word(device);
  if (w == nullptr) return H3_ERR_CUDA;
  if (cudaDeviceSynchronize() != cudaSuccess) return H3_ERR_CUDA;
  int v = 0;
  if (cudaMemcpy(&v, w, sizeof(int), cudaMemcpyDeviceToHost) != cudaSuccess) return H3_ERR_CUDA;
  if (cudaMemset(w, 0, sizeof(int)) != cudaSuccess) return H3_ERR_CUDA;
  *code = v;
  return H3_OK;
}
