// Shared definitions of libdrift_cuda: status codes, dtype codes, argument
// checks that report like the reference's `require`s, and launch helpers.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

#include <atomic>
#include <cstdarg>
#include <cstdio>
#include <string>

#include "../../include/drift_ops.h"
#include "../../include/drift_runtime.h"

namespace drift {

// The calling thread's last error message (what a HipException or a failed
// `require` would carry), kept until the next failing call.
void set_error(const char* format, ...);
const char* last_error();

// Returns DRIFT_ERROR_INVALID_ARGUMENT with the message set, as a failed
// `require` throws IllegalArgumentException.
int invalid(const char* format, ...);

// A CUDA status as a drift status: 0 stays 0, anything else is returned as is
// with a message naming the call.
int cuda_status(cudaError_t status, const char* call);

// Bytes of storage for `elements` values of `dtype`, or -1 if they are not
// whole blocks (DType.byteSize, runner/src/drift/runner/tensor/DType.scala:24-30).
int64_t byte_size(int dtype, int64_t elements);
int block_elements(int dtype);
int block_bytes(int dtype);
const char* dtype_name(int dtype);

// Streaming multiprocessors of the current device (cached per device).
int sm_count();

constexpr int WARP = 32;

// A kernel attribute set once per device: attributes such as the dynamic
// shared memory limit belong to a device's context, so a process that runs
// products on several GPUs sets them on each (devices 0-63; others are set on
// every call).
class PerDevice {
 public:
  bool done() const {
    const int d = current();
    return d >= 0 && d < 64 && ((bits_.load(std::memory_order_acquire) >> d) & 1u);
  }
  void mark() {
    const int d = current();
    if (d >= 0 && d < 64) bits_.fetch_or(uint64_t(1) << d, std::memory_order_release);
  }

 private:
  static int current() {
    int d = -1;
    return cudaGetDevice(&d) == cudaSuccess ? d : -1;
  }
  std::atomic<uint64_t> bits_{0};
};

// Raises `kernel`'s dynamic shared memory limit to `bytes` on the current
// device the first time it is asked there (and, with carveout >= 0, the
// shared-memory share of L1); 0 or a drift status.
template <typename Kernel>
int ensure_shared_memory(PerDevice& once, Kernel* kernel, int bytes, int carveout = -1) {
  if (once.done()) return 0;
  cudaError_t status =
      cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
  if (status == cudaSuccess && carveout >= 0)
    status = cudaFuncSetAttribute(kernel, cudaFuncAttributePreferredSharedMemoryCarveout, carveout);
  if (status != cudaSuccess) return cuda_status(status, "cudaFuncSetAttribute");
  once.mark();
  return 0;
}

}  // namespace drift

#define DRIFT_TRY(call)                                                      \
  do {                                                                       \
    const int drift_status_ = (call);                                        \
    if (drift_status_ != 0) return drift_status_;                            \
  } while (0)

#define DRIFT_CUDA(call) DRIFT_TRY(::drift::cuda_status((call), #call))

// ---- programmatic dependent launch ------------------------------------------
// The products launch with programmatic stream serialization: a kernel may
// start while the kernel before it in the stream finishes, and does what
// depends on nothing -- barrier set-up, the first weight copies (weights are
// never written by the kernels of this library) -- before pdl_wait(), which
// returns once the previous kernel has completed and its writes are visible.
// Every global read of data another kernel writes, and every global write,
// comes after pdl_wait(). pdl_trigger() lets the next such kernel start.
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_trigger() {
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}

template <typename... Params, typename... Args>
cudaError_t launch_pdl(void (*kernel)(Params...), dim3 grid, dim3 block, size_t smem,
                       cudaStream_t stream, Args... args) {
  cudaLaunchConfig_t config = {};
  config.gridDim = grid;
  config.blockDim = block;
  config.dynamicSmemBytes = smem;
  config.stream = stream;
  cudaLaunchAttribute attribute[1];
  attribute[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attribute[0].val.programmaticStreamSerializationAllowed = 1;
  config.attrs = attribute;
  config.numAttrs = 1;
  return cudaLaunchKernelEx(&config, kernel, static_cast<Params>(args)...);
}

// The launch just queued, checked (a bad configuration fails here, not later).
#define DRIFT_LAUNCHED(name) DRIFT_TRY(::drift::cuda_status(cudaGetLastError(), name))
