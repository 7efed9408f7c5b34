// Library-wide C-ABI helpers: status strings, error capture, device checks,
// tensor-map encoding through the runtime's driver entry point (so the library
// does not link libcuda directly and loads on hosts without a driver).
#include <atomic>
#include <cstdio>
#include <cstring>
#include <mutex>
#include <set>
#include <utility>

#include "common.cuh"

namespace mt {

static thread_local char g_last_error[512] = "";

void set_last_error(const char* where, cudaError_t err) {
  snprintf(g_last_error, sizeof(g_last_error), "%s: %s (%s)", where, cudaGetErrorName(err), cudaGetErrorString(err));
}

void set_last_error_text(const char* text) { snprintf(g_last_error, sizeof(g_last_error), "%s", text); }

// Kernels this library has launched in the process (every launch is followed
// by exactly one check_launch).
std::atomic<long long> g_launches{0};

int check_launch(const char* where) {
  cudaError_t err = cudaGetLastError();
  if (err != cudaSuccess) {
    set_last_error(where, err);
    return MT_ERR_LAUNCH;
  }
  g_launches.fetch_add(1, std::memory_order_relaxed);
  return MT_OK;
}

namespace {
constexpr int kMaxDevices = 64;
int g_cc_major[kMaxDevices];
int g_sm_count[kMaxDevices];
bool g_dev_ready[kMaxDevices];
std::mutex g_mutex;
std::set<std::pair<int, const void*>> g_smem_set;

int device_info(int* dev_out) {
  int dev = 0;
  cudaError_t err = cudaGetDevice(&dev);
  if (err != cudaSuccess) {
    set_last_error("cudaGetDevice", err);
    return MT_ERR_LAUNCH;
  }
  if (dev < 0 || dev >= kMaxDevices) return MT_ERR_INVALID_ARGUMENT;
  if (!g_dev_ready[dev]) {
    std::lock_guard<std::mutex> lock(g_mutex);
    if (!g_dev_ready[dev]) {
      cudaDeviceProp prop;
      err = cudaGetDeviceProperties(&prop, dev);
      if (err != cudaSuccess) {
        set_last_error("cudaGetDeviceProperties", err);
        return MT_ERR_LAUNCH;
      }
      g_cc_major[dev] = prop.major * 10 + prop.minor;
      g_sm_count[dev] = prop.multiProcessorCount;
      g_dev_ready[dev] = true;
    }
  }
  *dev_out = dev;
  return MT_OK;
}

typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                  const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                  CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);
EncodeTiledFn g_encode = nullptr;
}  // namespace

typedef CUresult (*CtxGetCurrentFn)(CUcontext*);
CtxGetCurrentFn g_ctx_get_current = nullptr;

// Timing events of the calling thread (driver handles owned by the caller).
typedef CUresult (*EventRecordFn)(CUevent, CUstream);
EventRecordFn g_event_record = nullptr;
thread_local CUevent t_timing_events[2] = {nullptr, nullptr};

void record_timing_event(int which, cudaStream_t stream) {
  CUevent ev = t_timing_events[which & 1];
  if (ev == nullptr || g_event_record == nullptr) return;
  g_event_record(ev, reinterpret_cast<CUstream>(stream));
}

int bind_device_of(const void* ptr) {
  // A thread that has not touched CUDA yet (e.g. PyTorch's autograd worker
  // for device 0) may have no current context; the driver-API tensor-map
  // encoder needs one.  Bind the primary context of the device owning `ptr`.
  if (g_ctx_get_current == nullptr) {
    std::lock_guard<std::mutex> lock(g_mutex);
    if (g_ctx_get_current == nullptr) {
      void* fn = nullptr;
      cudaDriverEntryPointQueryResult q;
      if (cudaGetDriverEntryPoint("cuCtxGetCurrent", &fn, cudaEnableDefault, &q) != cudaSuccess || fn == nullptr)
        return MT_ERR_LAUNCH;
      g_ctx_get_current = reinterpret_cast<CtxGetCurrentFn>(fn);
    }
  }
  CUcontext ctx = nullptr;
  if (g_ctx_get_current(&ctx) == CUDA_SUCCESS && ctx != nullptr) return MT_OK;
  cudaPointerAttributes attr;
  cudaError_t err = cudaPointerGetAttributes(&attr, ptr);
  if (err != cudaSuccess || attr.type != cudaMemoryTypeDevice) {
    set_last_error("cudaPointerGetAttributes", err);
    return MT_ERR_INVALID_ARGUMENT;
  }
  err = cudaSetDevice(attr.device);
  if (err != cudaSuccess) {
    set_last_error("cudaSetDevice", err);
    return MT_ERR_LAUNCH;
  }
  return MT_OK;
}

int check_arch() {
  int dev;
  int st = device_info(&dev);
  if (st != MT_OK) return st;
  if (g_cc_major[dev] != 100) {
    snprintf(g_last_error, sizeof(g_last_error), "device compute capability %d.%d is not sm_100",
             g_cc_major[dev] / 10, g_cc_major[dev] % 10);
    return MT_ERR_UNSUPPORTED_ARCH;
  }
  return MT_OK;
}

int get_sm_count() {
  int dev;
  if (device_info(&dev) != MT_OK) return 148;
  return g_sm_count[dev];
}

int set_smem_limit(const void* func, int bytes) {
  int dev;
  int st = device_info(&dev);
  if (st != MT_OK) return st;
  if (bytes <= 48 * 1024) return MT_OK;
  std::lock_guard<std::mutex> lock(g_mutex);
  const auto key = std::make_pair(dev, func);
  if (g_smem_set.count(key)) return MT_OK;
  // Raise to the largest opt-in size once; later launches of any size fit.
  cudaError_t err = cudaFuncSetAttribute(func, cudaFuncAttributeMaxDynamicSharedMemorySize, 227 * 1024);
  if (err != cudaSuccess) {
    set_last_error("cudaFuncSetAttribute", err);
    return MT_ERR_LAUNCH;
  }
  g_smem_set.insert(key);
  return MT_OK;
}

int encode_tensor_map(CUtensorMap* map, CUtensorMapDataType dtype, int rank, void* base, const uint64_t* dims,
                      const uint64_t* strides_bytes, const uint32_t* box, CUtensorMapSwizzle swizzle) {
  if (g_encode == nullptr) {
    std::lock_guard<std::mutex> lock(g_mutex);
    if (g_encode == nullptr) {
      void* fn = nullptr;
      cudaDriverEntryPointQueryResult q;
      cudaError_t err = cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &fn, cudaEnableDefault, &q);
      if (err != cudaSuccess || fn == nullptr || q != cudaDriverEntryPointSuccess) {
        set_last_error("cudaGetDriverEntryPoint(cuTensorMapEncodeTiled)", err);
        return MT_ERR_TENSOR_MAP;
      }
      g_encode = reinterpret_cast<EncodeTiledFn>(fn);
    }
  }
  cuuint64_t d[5];
  cuuint64_t s[4];
  cuuint32_t b[5];
  cuuint32_t e[5];
  for (int i = 0; i < rank; ++i) {
    d[i] = dims[i];
    b[i] = box[i];
    e[i] = 1;
  }
  for (int i = 0; i + 1 < rank; ++i) s[i] = strides_bytes[i];
  CUresult r = g_encode(map, dtype, (cuuint32_t)rank, base, d, s, b, e, CU_TENSOR_MAP_INTERLEAVE_NONE, swizzle,
                        CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) {
    snprintf(g_last_error, sizeof(g_last_error), "cuTensorMapEncodeTiled failed with CUresult %d (rank %d)", (int)r,
             rank);
    return MT_ERR_TENSOR_MAP;
  }
  return MT_OK;
}

}  // namespace mt

extern "C" {

const char* mt_status_string(int status) {
  switch (status) {
    case MT_OK: return "ok";
    case MT_ERR_INVALID_ARGUMENT: return "invalid argument";
    case MT_ERR_UNSUPPORTED_DTYPE: return "unsupported dtype";
    case MT_ERR_UNSUPPORTED_LAYOUT: return "unsupported layout or alignment";
    case MT_ERR_UNSUPPORTED_ARCH: return "unsupported GPU architecture (needs sm_100)";
    case MT_ERR_LAUNCH: return "CUDA launch error";
    case MT_ERR_DEVICE_TIMEOUT: return "device-side wait timed out";
    case MT_ERR_WORKSPACE: return "workspace missing or too small";
    case MT_ERR_TENSOR_MAP: return "tensor map encoding failed";
    default: return "unknown status";
  }
}

int mt_version(void) { return 1; }
int mt_built_arch(void) { return 100; }
const char* mt_last_error(void) { return mt::g_last_error; }
int64_t mt_launch_count(void) { return mt::g_launches.load(std::memory_order_relaxed); }

}  // extern "C"

extern "C" int mt_set_timing_events(void* before_main, void* after_main) {
  using namespace mt;
  if ((before_main == nullptr) != (after_main == nullptr)) return MT_ERR_INVALID_ARGUMENT;
  if (before_main != nullptr && g_event_record == nullptr) {
    std::lock_guard<std::mutex> lock(g_mutex);
    if (g_event_record == nullptr) {
      void* fn = nullptr;
      cudaDriverEntryPointQueryResult q;
      if (cudaGetDriverEntryPoint("cuEventRecord", &fn, cudaEnableDefault, &q) != cudaSuccess || fn == nullptr)
        return MT_ERR_LAUNCH;
      g_event_record = reinterpret_cast<EventRecordFn>(fn);
    }
  }
  t_timing_events[0] = static_cast<CUevent>(before_main);
  t_timing_events[1] = static_cast<CUevent>(after_main);
  return MT_OK;
}

