// drift_linear_static: the quantized product of 1 to 31 rows of x with no
// device allocation, for hosts that cannot allocate device memory on the call
// path: memory reserved up front, an FFM host's own allocator, a loop that must
// not let cudaMalloc/cudaFree synchronize the device (drift_ops.h). Its scratch -- the prepared x -- is a fixed array in
// this library's device image instead of the grow-only workspace that
// drift_linear uses; the kernels are drift_linear's.
#include <cuda_runtime.h>

#include <mutex>

#include "common.cuh"

namespace drift {

int check_linear(int x_dtype, const void* x, int weight_dtype, const void* weight,
                 const float* out, int64_t m, int64_t n, int64_t k);
size_t mma_workspace_bytes(int64_t m, int64_t k);
int prepare_x_mma(int x_dtype, const void* x, int64_t m, int64_t k, uint8_t* records,
                  cudaStream_t stream);
int matvec_prepared(int weight_dtype, const void* weight, const uint8_t* records, float* y,
                    int64_t rows, int64_t cols, int64_t vectors, cudaStream_t stream);
int matvec_f32_weights(int x_dtype, const void* x, const float* weight, float* y, int64_t m,
                       int64_t n, int64_t k, cudaStream_t stream);

// The prepared x of one call: 896 bytes per 32-column block and pass of 8
// rows of x, so 1 MiB holds 1,170 of them (8 rows of up to 37,440 columns; 31
// rows of up to 9,344). Every device that loads the library holds it until
// the process exits.
constexpr size_t LINEAR_STATIC_SCRATCH_BYTES = size_t(1) << 20;
static __device__ __align__(256) uint8_t linear_static_scratch[LINEAR_STATIC_SCRATCH_BYTES];

// The array's device address on the current device. In host code the name
// `linear_static_scratch` is a host-side stand-in, not an address a kernel
// can use; the runtime gives the real one, once per device.
static int static_scratch_address(uint8_t** address) {
  static std::mutex lock;
  static uint8_t* addresses[64] = {nullptr};
  int device = 0;
  DRIFT_CUDA(cudaGetDevice(&device));
  if (device < 0 || device >= 64) return invalid("device %d out of range", device);
  std::lock_guard<std::mutex> guard(lock);
  if (!addresses[device]) {
    void* p = nullptr;
    const cudaError_t status = cudaGetSymbolAddress(&p, linear_static_scratch);
    if (status != cudaSuccess)
      return cuda_status(status, "cudaGetSymbolAddress(linear_static_scratch)");
    addresses[device] = static_cast<uint8_t*>(p);
  }
  *address = addresses[device];
  return 0;
}

}  // namespace drift

using namespace drift;

extern "C" int drift_linear_static(int x_dtype, const void* x, int weight_dtype,
                                   const void* weight, float* out, int64_t m, int64_t n,
                                   int64_t k, drift_stream_t stream) {
  DRIFT_TRY(check_linear(x_dtype, x, weight_dtype, weight, out, m, n, k));
  if (m >= 32)
    return invalid(
        "drift_linear_static takes 1 to 31 rows of x (the products its fixed scratch "
        "serves), not %lld: use drift_linear",
        (long long)m);
  const cudaStream_t s = cudaStream_t(stream);
  if (m == 0 || n == 0) return 0;
  if (k == 0) return cuda_status(cudaMemsetAsync(out, 0, size_t(m * n) * 4, s), "cudaMemsetAsync");
  if (weight_dtype == DRIFT_F32)
    return matvec_f32_weights(x_dtype, x, static_cast<const float*>(weight), out, m, n, k, s);
  const size_t need = mma_workspace_bytes(m, k);
  if (need > LINEAR_STATIC_SCRATCH_BYTES)
    return invalid(
        "drift_linear_static: %lld rows of %lld columns need %zu bytes of scratch; its fixed "
        "scratch holds %zu (use drift_linear)",
        (long long)m, (long long)k, need, LINEAR_STATIC_SCRATCH_BYTES);
  uint8_t* scratch = nullptr;
  DRIFT_TRY(static_scratch_address(&scratch));
  // every byte the product reads is written first: nothing needs clearing
  DRIFT_TRY(prepare_x_mma(x_dtype, x, m, k, scratch, s));
  return matvec_prepared(weight_dtype, weight, scratch, out, n, k, m, s);
}
