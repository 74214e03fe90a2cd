// Host-side plumbing of the C ABI: device binding, SM counts, the device-side error
// word that bounded waits set, and status strings.
#include <cudaTypedefs.h>

#include <mutex>

#include "h3_common.cuh"

namespace h3host {

namespace {
constexpr int kMaxDevices = 64;
std::mutex g_mutex;
int g_sm_count[kMaxDevices] = {0};
int* g_error_word[kMaxDevices] = {nullptr};  // device view of the mapped word
int* g_error_host[kMaxDevices] = {nullptr};  // host view of the same word
}  // namespace

DeviceScope::~DeviceScope() {
  if (prev_ >= 0) cudaSetDevice(prev_);
}

int DeviceScope::bind_index(int device) {
  if (device < 0 || device >= kMaxDevices) return H3_ERR_INVALID;
  int cur = -1;
  if (cudaGetDevice(&cur) != cudaSuccess) {
    cudaGetLastError();
    return H3_ERR_CUDA;
  }
  if (cur != device) {
    if (cudaSetDevice(device) != cudaSuccess) return H3_ERR_CUDA;
    if (prev_ < 0) prev_ = cur;
  }
  return H3_OK;
}

int DeviceScope::bind(const void* ptr, int* device) {
  cudaPointerAttributes attr;
  cudaError_t e = cudaPointerGetAttributes(&attr, ptr);
  if (e != cudaSuccess) {
    cudaGetLastError();
    return H3_ERR_INVALID;
  }
  if (attr.type != cudaMemoryTypeDevice && attr.type != cudaMemoryTypeManaged)
    return H3_ERR_INVALID;  // host pointers are rejected: the path has no CPU fallback
  if (int s = bind_index(attr.device)) return s;
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

// The error word of a device: one int of host-mapped, page-locked memory, written by
// kernels with a system-scope store and read by the host directly (h3_device_error_peek
// needs no synchronisation).  Created on first use with the device current.
int* error_word(int device) {
  if (device < 0 || device >= kMaxDevices) return nullptr;
  std::lock_guard<std::mutex> lock(g_mutex);
  if (g_error_word[device] == nullptr) {
    int* host = nullptr;
    if (cudaHostAlloc(reinterpret_cast<void**>(&host), sizeof(int),
                      cudaHostAllocMapped | cudaHostAllocPortable) != cudaSuccess) {
      cudaGetLastError();
      return nullptr;
    }
    *reinterpret_cast<volatile int*>(host) = 0;
    int* dev = nullptr;
    if (cudaHostGetDevicePointer(reinterpret_cast<void**>(&dev), host, 0) != cudaSuccess) {
      cudaGetLastError();
      cudaFreeHost(host);
      return nullptr;
    }
    g_error_host[device] = host;
    g_error_word[device] = dev;
  }
  return g_error_word[device];
}

int* error_word_host(int device) {
  if (device < 0 || device >= kMaxDevices) return nullptr;
  std::lock_guard<std::mutex> lock(g_mutex);
  return g_error_host[device];
}

static PFN_cuTensorMapEncodeTiled_v12000 tiled_encoder() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) ==
            cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
    else
      cudaGetLastError();
  });
  return fn;
}

bool encode_row_map(CUtensorMap* map, const void* base, int64_t rows, int64_t row_bytes,
                    int box_lines) {
  auto fn = tiled_encoder();
  if (fn == nullptr || rows <= 0 || row_bytes <= 0 || row_bytes % 128 != 0 || box_lines < 1 ||
      box_lines > 256 || (row_bytes / 128) % box_lines != 0 || !aligned(base, 16))
    return false;
  cuuint64_t dims[3] = {128, (cuuint64_t)(row_bytes / 128), (cuuint64_t)rows};
  cuuint64_t strides[2] = {128, (cuuint64_t)row_bytes};
  cuuint32_t box[3] = {128, (cuuint32_t)box_lines, 1};
  cuuint32_t estr[3] = {1, 1, 1};
  return fn(map, CU_TENSOR_MAP_DATA_TYPE_UINT8, 3, const_cast<void*>(base), dims, strides, box,
            estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
            CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
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
  h3host::DeviceScope scope;
  if (int s = scope.bind_index(device)) return s;
  if (h3host::error_word(device) == nullptr) return H3_ERR_CUDA;
  volatile int* w = h3host::error_word_host(device);
  if (cudaDeviceSynchronize() != cudaSuccess) return H3_ERR_CUDA;
  *code = *w;
  *w = 0;
  return H3_OK;
}

extern "C" int h3_device_error_peek(int device, int* code) {
  if (code == nullptr || device < 0) return H3_ERR_INVALID;
  volatile int* w = h3host::error_word_host(device);
  *code = w == nullptr ? 0 : *w;
  return H3_OK;
}

// ---------------------------------------------------------------------------
// SM clock probe.  One thread that reads %clock64 and %globaltimer, sleeps in 1 us steps
// until `ns` nanoseconds have passed and reads both again: cycles / time is the SM clock
// over that interval.  Launched beside other kernels (one 32-thread CTA, no shared
// memory, so it fits on an SM next to a GEMM CTA) it gives the clock those kernels ran
// at, which sampled nvidia-smi readings taken between kernels miss.  Bounded by design.
// ---------------------------------------------------------------------------
namespace h3host {
__global__ void clock_probe_kernel(unsigned long long ns, unsigned long long* out) {
  if (threadIdx.x != 0) return;
  unsigned long long g0, g;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(g0));
  const long long c0 = clock64();
  g = g0;
  while (g - g0 < ns) {
    __nanosleep(1000);
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(g));
  }
  const long long c1 = clock64();
  out[0] = g - g0;
  out[1] = (unsigned long long)(c1 - c0);
}
}  // namespace h3host

extern "C" int h3_sm_clock_probe(unsigned long long ns, unsigned long long* out, void* stream) {
  if (out == nullptr || ns == 0 || ns > 10000000000ull) return H3_ERR_INVALID;
  int dev;
  h3host::DeviceScope scope;
  if (int s = scope.bind(out, &dev)) return s;
  h3host::clock_probe_kernel<<<1, 32, 0, (cudaStream_t)stream>>>(ns, out);
  return h3host::check_launch();
}
