// The runtime half of the C ABI (include/drift_runtime.h): the CUDA-side twin
// of the libamdhip64 calls the runner binds through FFM
// (runner/src/drift/runner/native/HipRuntime.scala:73-120), the by-name kernel
// table, and the library's error reporting.
#include <cuda_runtime.h>

#include <cstdarg>
#include <cstdio>
#include <cstring>
#include <mutex>
#include <vector>

#include "common.cuh"
#include "registry.cuh"

namespace drift {

// ---- errors ----------------------------------------------------------------------
static thread_local char error_message[1024] = "";

void set_error(const char* format, ...) {
  va_list args;
  va_start(args, format);
  vsnprintf(error_message, sizeof(error_message), format, args);
  va_end(args);
}

const char* last_error() { return error_message; }

int invalid(const char* format, ...) {
  va_list args;
  va_start(args, format);
  vsnprintf(error_message, sizeof(error_message), format, args);
  va_end(args);
  return DRIFT_ERROR_INVALID_ARGUMENT;
}

int cuda_status(cudaError_t status, const char* call) {
  if (status == cudaSuccess) return 0;
  set_error("%s failed with CUDA error %d: %s", call, int(status), cudaGetErrorString(status));
  return int(status);
}

// ---- storage types -------------------------------------------------------------------
int block_elements(int dtype) {
  switch (dtype) {
    case DRIFT_F32:
    case DRIFT_F16:
    case DRIFT_BF16:
    case DRIFT_I32: return 1;
    case DRIFT_Q4_0:
    case DRIFT_Q4_1:
    case DRIFT_Q8_0: return 32;
    case DRIFT_Q4_K:
    case DRIFT_Q6_K: return 256;
    default: return -1;
  }
}

int block_bytes(int dtype) {
  switch (dtype) {
    case DRIFT_F32:
    case DRIFT_I32: return 4;
    case DRIFT_F16:
    case DRIFT_BF16: return 2;
    case DRIFT_Q4_0: return 18;
    case DRIFT_Q4_1: return 20;
    case DRIFT_Q8_0: return 34;
    case DRIFT_Q4_K: return 144;
    case DRIFT_Q6_K: return 210;
    default: return -1;
  }
}

const char* dtype_name(int dtype) {
  switch (dtype) {
    case DRIFT_F32: return "F32";
    case DRIFT_F16: return "F16";
    case DRIFT_BF16: return "BF16";
    case DRIFT_I32: return "I32";
    case DRIFT_Q4_0: return "Q4_0";
    case DRIFT_Q4_1: return "Q4_1";
    case DRIFT_Q8_0: return "Q8_0";
    case DRIFT_Q4_K: return "Q4_K";
    case DRIFT_Q6_K: return "Q6_K";
    default: return "an unknown type";
  }
}

int64_t byte_size(int dtype, int64_t elements) {
  const int per = block_elements(dtype);
  if (per <= 0 || elements % per != 0) return -1;
  return elements / per * block_bytes(dtype);
}

int sm_count() {
  static int counts[64] = {0};
  int device = 0;
  if (cudaGetDevice(&device) != cudaSuccess || device < 0 || device >= 64) return 148;
  if (counts[device] == 0) {
    int count = 0;
    if (cudaDeviceGetAttribute(&count, cudaDevAttrMultiProcessorCount, device) != cudaSuccess)
      count = 148;
    counts[device] = count;
  }
  return counts[device];
}

// ---- the kernel table -------------------------------------------------------------------
static std::vector<KernelEntry>& kernel_table() {
  static std::vector<KernelEntry> table;
  return table;
}

int register_kernel(const char* name, const void* function) {
  kernel_table().push_back(KernelEntry{name, function});
  return int(kernel_table().size()) - 1;
}

int kernel_count() { return int(kernel_table().size()); }

const KernelEntry* kernel_at(int index) {
  if (index < 0 || index >= kernel_count()) return nullptr;
  return &kernel_table()[size_t(index)];
}

const KernelEntry* find_kernel(const char* name) {
  for (const KernelEntry& e : kernel_table())
    if (std::strcmp(e.name, name) == 0) return &e;
  return nullptr;
}

// A function handle: a kernel of this library, or one of a loaded image.
struct Function {
  const void* launchable;  // what cudaLaunchKernel takes
  std::string name;
};

}  // namespace drift

using namespace drift;

extern "C" {

int drift_init(int flags) {
  if (flags != 0) return invalid("drift_init takes flags 0, not %d", flags);
  return cuda_status(cudaFree(nullptr), "cudaFree(0)");  // creates the primary context
}

int drift_set_device(int device) { return cuda_status(cudaSetDevice(device), "cudaSetDevice"); }

int drift_get_device(int* device) { return cuda_status(cudaGetDevice(device), "cudaGetDevice"); }

int drift_get_device_count(int* count) {
  return cuda_status(cudaGetDeviceCount(count), "cudaGetDeviceCount");
}

int drift_set_device_flags(int flags) {
  unsigned cuda_flags;
  switch (flags) {
    case 1: cuda_flags = cudaDeviceScheduleSpin; break;
    case 2: cuda_flags = cudaDeviceScheduleYield; break;
    case 4: cuda_flags = cudaDeviceScheduleBlockingSync; break;
    default: return invalid("device flags %d: 1 spin, 2 yield or 4 blocking sync", flags);
  }
  return cuda_status(cudaSetDeviceFlags(cuda_flags), "cudaSetDeviceFlags");
}

int drift_device_get_name(char* name, int length, int device) {
  if (!name || length <= 0) return invalid("no room for the device name");
  cudaDeviceProp properties;
  DRIFT_CUDA(cudaGetDeviceProperties(&properties, device));
  std::snprintf(name, size_t(length), "%s", properties.name);
  return 0;
}

int drift_device_synchronize(void) {
  return cuda_status(cudaDeviceSynchronize(), "cudaDeviceSynchronize");
}

int drift_mem_get_info(size_t* free_bytes, size_t* total_bytes) {
  return cuda_status(cudaMemGetInfo(free_bytes, total_bytes), "cudaMemGetInfo");
}

const char* drift_get_error_string(int status) {
  if (status == DRIFT_ERROR_INVALID_ARGUMENT || status == DRIFT_ERROR_TIMEOUT) return last_error();
  return cudaGetErrorString(cudaError_t(status));
}

const char* drift_last_error_message(void) { return last_error(); }

int drift_malloc(void** pointer, size_t bytes) {
  if (!pointer) return invalid("drift_malloc: no slot for the pointer");
  return cuda_status(cudaMalloc(pointer, bytes), "cudaMalloc");
}

int drift_free(void* pointer) { return cuda_status(cudaFree(pointer), "cudaFree"); }

int drift_memset(void* pointer, int value, size_t bytes) {
  return cuda_status(cudaMemset(pointer, value, bytes), "cudaMemset");
}

int drift_memcpy(void* target, const void* source, size_t bytes, int kind) {
  if (kind < 0 || kind > 4) return invalid("memcpy kind %d", kind);
  return cuda_status(cudaMemcpy(target, source, bytes, cudaMemcpyKind(kind)), "cudaMemcpy");
}

int drift_memcpy_async(void* target, const void* source, size_t bytes, int kind,
                       drift_stream_t stream) {
  if (kind < 0 || kind > 4) return invalid("memcpy kind %d", kind);
  return cuda_status(
      cudaMemcpyAsync(target, source, bytes, cudaMemcpyKind(kind), cudaStream_t(stream)),
      "cudaMemcpyAsync");
}

int drift_host_register(void* host, size_t bytes, int flags) {
  unsigned cuda_flags = 0;
  if (flags & 0x2) cuda_flags |= cudaHostRegisterMapped;
  if (flags & 0x8) cuda_flags |= cudaHostRegisterReadOnly;
  return cuda_status(cudaHostRegister(host, bytes, cuda_flags), "cudaHostRegister");
}

int drift_host_unregister(void* host) {
  return cuda_status(cudaHostUnregister(host), "cudaHostUnregister");
}

int drift_host_get_device_pointer(void** device, void* host, int flags) {
  return cuda_status(cudaHostGetDevicePointer(device, host, unsigned(flags)),
                     "cudaHostGetDevicePointer");
}

int drift_stream_create(drift_stream_t* stream) {
  return cuda_status(cudaStreamCreateWithFlags(reinterpret_cast<cudaStream_t*>(stream),
                                               cudaStreamNonBlocking),
                     "cudaStreamCreate");
}

int drift_stream_destroy(drift_stream_t stream) {
  return cuda_status(cudaStreamDestroy(cudaStream_t(stream)), "cudaStreamDestroy");
}

int drift_stream_synchronize(drift_stream_t stream) {
  return cuda_status(cudaStreamSynchronize(cudaStream_t(stream)), "cudaStreamSynchronize");
}

int drift_event_create(drift_event_t* event) {
  return cuda_status(cudaEventCreate(reinterpret_cast<cudaEvent_t*>(event)), "cudaEventCreate");
}

int drift_event_destroy(drift_event_t event) {
  return cuda_status(cudaEventDestroy(cudaEvent_t(event)), "cudaEventDestroy");
}

int drift_event_record(drift_event_t event, drift_stream_t stream) {
  return cuda_status(cudaEventRecord(cudaEvent_t(event), cudaStream_t(stream)), "cudaEventRecord");
}

int drift_stream_wait_event(drift_stream_t stream, drift_event_t event) {
  return cuda_status(cudaStreamWaitEvent(cudaStream_t(stream), cudaEvent_t(event), 0),
                     "cudaStreamWaitEvent");
}

int drift_event_synchronize(drift_event_t event) {
  return cuda_status(cudaEventSynchronize(cudaEvent_t(event)), "cudaEventSynchronize");
}

int drift_event_elapsed_time(float* milliseconds, drift_event_t start, drift_event_t end) {
  return cuda_status(cudaEventElapsedTime(milliseconds, cudaEvent_t(start), cudaEvent_t(end)),
                     "cudaEventElapsedTime");
}

int drift_module_load_data(drift_module_t* module, const void* image) {
  if (!module || !image) return invalid("drift_module_load_data: no image");
  cudaLibrary_t library;
  DRIFT_CUDA(cudaLibraryLoadData(&library, image, nullptr, nullptr, 0, nullptr, nullptr, 0));
  *module = reinterpret_cast<drift_module_t>(library);
  return 0;
}

int drift_module_unload(drift_module_t module) {
  if (!module) return invalid("this library's own kernels cannot be unloaded");
  return cuda_status(cudaLibraryUnload(reinterpret_cast<cudaLibrary_t>(module)),
                     "cudaLibraryUnload");
}

int drift_module_get_function(drift_function_t* function, drift_module_t module,
                              const char* name) {
  if (!function || !name) return invalid("drift_module_get_function: no name");
  if (!module) {
    const KernelEntry* entry = find_kernel(name);
    if (!entry) return invalid("no kernel %s in libdrift_cuda", name);
    *function = new Function{entry->function, name};
    return 0;
  }
  cudaKernel_t kernel;
  DRIFT_CUDA(cudaLibraryGetKernel(&kernel, reinterpret_cast<cudaLibrary_t>(module), name));
  *function = new Function{reinterpret_cast<const void*>(kernel), name};
  return 0;
}

int drift_module_launch_kernel(drift_function_t function, unsigned grid_x, unsigned grid_y,
                               unsigned grid_z, unsigned block_x, unsigned block_y,
                               unsigned block_z, unsigned shared_bytes, drift_stream_t stream,
                               void** kernel_params, void** extra) {
  if (!function) return invalid("launch of no function");
  if (extra) return invalid("launch: `extra` must be NULL");
  const Function* f = static_cast<const Function*>(function);
  const cudaError_t status =
      cudaLaunchKernel(f->launchable, dim3(grid_x, grid_y, grid_z), dim3(block_x, block_y, block_z),
                       kernel_params, size_t(shared_bytes), cudaStream_t(stream));
  if (status != cudaSuccess) {
    set_error("launch of %s failed with CUDA error %d: %s", f->name.c_str(), int(status),
              cudaGetErrorString(status));
    return int(status);
  }
  return 0;
}

int drift_kernel_count(void) { return kernel_count(); }

const char* drift_kernel_name(int index) {
  const KernelEntry* e = kernel_at(index);
  return e ? e->name : nullptr;
}

}  // extern "C"
