// Ops.linear / Ops.linears behind the C ABI (include/drift_ops.h): the shape
// rules of Ops.checkLinear (runner/src/drift/runner/ops/LinearOps.scala:
// 227-249) and the dispatch of HipLinear.linears (ops/HipLinear.scala:104-276),
// re-decided for B200.
#include <cuda_runtime.h>

#include <vector>

#include "common.cuh"
#include "quant.cuh"
#include "registry.cuh"

namespace drift {

int workspace_reserve(size_t bytes, void** pointer);
int matvec_prepared(int weight_dtype, const void* weight, const uint8_t* records, float* y,
                    int64_t rows, int64_t cols, int64_t vectors, cudaStream_t stream);
size_t mma_workspace_bytes(int64_t m, int64_t k);
int prepare_x_mma(int x_dtype, const void* x, int64_t m, int64_t k, uint8_t* records,
                  cudaStream_t stream);
int matvec_f32_many(int x_dtype, const void* x, int count, const float* const* weights,
                    float* const* ys, const int64_t* ns, int64_t m, int64_t k,
                    cudaStream_t stream);
int matvec_f32_weights(int x_dtype, const void* x, const float* weight, float* y, int64_t m,
                       int64_t n, int64_t k, cudaStream_t stream);
bool tc_supports(int weight_dtype, const void* weight, int64_t k);
bool ring_many_fits(int weight_dtype, int count, const void* const* weights, const int64_t* rows,
                    int64_t cols);
int kquant_linear(int x_dtype, const void* x, int weight_dtype, const void* weight, float* y,
                  int64_t m, int64_t n, int64_t k, cudaStream_t stream);
int matvec_ring_many(int weight_dtype, int count, const void* const* weights,
                     const uint8_t* records, float* const* ys, const int64_t* rows, int64_t cols,
                     int64_t vectors, cudaStream_t stream);
size_t tc_workspace_bytes(int64_t m, int64_t k);
int linear_tc(int x_dtype, const void* x, int weight_dtype, const void* weight, float* y,
              int64_t m, int64_t n, int64_t k, uint8_t* workspace, cudaStream_t stream);

// From this many rows of x a product is a tensor-core product, as the
// runner's GemmMinimumRows (ops/HipLinear.scala:14-19); below, the weight is
// streamed once for all rows of x (up to 8 per pass in the reference).
constexpr int64_t GEMM_MINIMUM_ROWS = 32;

// Ops.checkLinear, plus what the kernels need of a stored weight.
int check_linear(int x_dtype, const void* x, int weight_dtype, const void* weight,
                        const float* out, int64_t m, int64_t n, int64_t k) {
  if (x_dtype != DRIFT_F32 && x_dtype != DRIFT_BF16)
    return invalid("linear takes F32 (or BF16) x, not %s", dtype_name(x_dtype));
  if (m < 0 || n < 0 || k < 0) return invalid("linear over [%lld, %lld] x [%lld, %lld]",
                                               (long long)m, (long long)k, (long long)n,
                                               (long long)k);
  if (weight_dtype != DRIFT_Q8_0 && weight_dtype != DRIFT_Q4_0 && weight_dtype != DRIFT_Q4_1 &&
      weight_dtype != DRIFT_Q4_K && weight_dtype != DRIFT_Q6_K && weight_dtype != DRIFT_F32)
    return invalid("no kernels for %s weights yet", dtype_name(weight_dtype));
  const int64_t row = byte_size(weight_dtype, k);
  if (row < 0)
    return invalid("%lld elements are not whole %s blocks of %d", (long long)k,
                   dtype_name(weight_dtype), block_elements(weight_dtype));
  if (weight_dtype != DRIFT_F32 && weight_dtype != DRIFT_Q6_K && row % 4 != 0)
    return invalid("%s rows of %lld are not whole words", dtype_name(weight_dtype), (long long)k);
  if (k > (1ll << 30) || m * k > 0x7fffffffll || n > 0x7fffffffll)
    return invalid("linear over [%lld, %lld]", (long long)m, (long long)k);
  if (m > 0 && n > 0 && k > 0 && (!x || !weight || !out))
    return invalid("linear: a null tensor");
  if ((reinterpret_cast<uintptr_t>(weight) & 3) != 0)
    return invalid("linear: the weight does not start on a 4-byte boundary");
  return 0;
}

}  // namespace drift

using namespace drift;

extern "C" {

// Scratch of one drift_linears call: the x records of the streamed products,
// then (from GEMM_MINIMUM_ROWS rows) the tensor-core products' own region, so
// a list that mixes the two never has one overwrite the other's x.
static size_t records_region(int64_t m, int64_t k) {
  return (mma_workspace_bytes(m, k) + 255) & ~size_t(255);
}

size_t drift_linear_workspace_bytes(int64_t m, int64_t k) {
  // (the experts' products use the records region alone)
  return records_region(m, k) + (m >= GEMM_MINIMUM_ROWS ? tc_workspace_bytes(m, k) : 0);
}

int drift_workspace_reserve(size_t bytes) { return workspace_reserve(bytes, nullptr); }

// drift_linears, with x's records already written (`prepared`, or null to
// write them here).
static int linears(int x_dtype, const void* x, const void* prepared, int count,
                   const int* weight_dtypes, const void* const* weights, float* const* outs,
                   const int64_t* ns, int64_t m, int64_t k, cudaStream_t s) {
  if (count < 0 || (count > 0 && (!weight_dtypes || !weights || !outs || !ns)))
    return invalid("linears: %d products without their weights", count);
  for (int i = 0; i < count; ++i)
    DRIFT_TRY(check_linear(x_dtype, x, weight_dtypes[i], weights[i], outs[i], m, ns[i], k));
  if (m == 0 || k == 0 || count == 0) {
    // an empty sum: zero rows of out, or rows of zeros
    for (int i = 0; i < count; ++i)
      if (m > 0 && ns[i] > 0)
        DRIFT_CUDA(cudaMemsetAsync(outs[i], 0, size_t(m * ns[i]) * 4, s));
    return 0;
  }
  // the K-quants: their own products, on x as it is (F32 or BF16)
  auto k_quant = [&](int i) {
    return weight_dtypes[i] == DRIFT_Q4_K || weight_dtypes[i] == DRIFT_Q6_K;
  };
  bool quantized = false, tensor_cores = false;
  for (int i = 0; i < count; ++i) {
    if (k_quant(i)) continue;
    const bool tc = weight_dtypes[i] != DRIFT_F32 && m >= GEMM_MINIMUM_ROWS &&
                    tc_supports(weight_dtypes[i], weights[i], k);
    tensor_cores |= tc;
    quantized |= weight_dtypes[i] != DRIFT_F32 && !tc;
  }
  for (int i = 0; i < count; ++i)
    if (k_quant(i) && ns[i] > 0)
      DRIFT_TRY(kquant_linear(x_dtype, x, weight_dtypes[i], weights[i], outs[i], m, ns[i], k, s));
  const size_t records_bytes = quantized && !prepared ? records_region(m, k) : 0;
  void* w = nullptr;
  if ((quantized && !prepared) || tensor_cores)
    DRIFT_TRY(workspace_reserve(records_bytes + (tensor_cores ? tc_workspace_bytes(m, k) : 0), &w));
  const uint8_t* records =
      prepared ? static_cast<const uint8_t*>(prepared) : static_cast<uint8_t*>(w);
  uint8_t* tc_region = static_cast<uint8_t*>(w) + records_bytes;
  if (quantized && !prepared)  // one preparation for all
    DRIFT_TRY(prepare_x_mma(x_dtype, x, m, k, static_cast<uint8_t*>(w), s));
  // Shared launches, each product's bits those of its own launch: streamed
  // products of one type that fit one balanced launch (up to 4) take it
  // together, and the F32 products one launch (up to 4).
  constexpr int SHARED = 4;
  auto streamed = [&](int i) {
    return weight_dtypes[i] != DRIFT_F32 && !k_quant(i) &&
           !(m >= GEMM_MINIMUM_ROWS && tc_supports(weight_dtypes[i], weights[i], k));
  };
  std::vector<char> done(size_t(count), 0);
  for (int i = 0; i < count; ++i) done[i] = k_quant(i);
  for (int i = 0; i < count; ++i) {
    if (done[i] || ns[i] == 0 || !streamed(i)) continue;
    int which[SHARED], c = 0;
    const void* w[SHARED];
    float* o[SHARED];
    int64_t n[SHARED];
    for (int j = i; j < count && c < SHARED; ++j)
      if (!done[j] && ns[j] > 0 && streamed(j) && weight_dtypes[j] == weight_dtypes[i]) {
        which[c] = j;
        w[c] = weights[j];
        o[c] = outs[j];
        n[c] = ns[j];
        ++c;
      }
    if (c < 2 || !ring_many_fits(weight_dtypes[i], c, w, n, k)) continue;
    DRIFT_TRY(matvec_ring_many(weight_dtypes[i], c, w, records, o, n, k, m, s));
    for (int j = 0; j < c; ++j) done[which[j]] = 1;
  }
  {
    int which[SHARED], c = 0;
    const float* w[SHARED];
    float* o[SHARED];
    int64_t n[SHARED];
    auto flush = [&]() -> int {
      if (c >= 2) {
        DRIFT_TRY(matvec_f32_many(x_dtype, x, c, w, o, n, m, k, s));
        for (int j = 0; j < c; ++j) done[which[j]] = 1;
      }
      c = 0;
      return 0;
    };
    for (int i = 0; i < count; ++i) {
      if (done[i] || ns[i] == 0 || weight_dtypes[i] != DRIFT_F32) continue;
      which[c] = i;
      w[c] = static_cast<const float*>(weights[i]);
      o[c] = outs[i];
      n[c] = ns[i];
      if (++c == SHARED) DRIFT_TRY(flush());
    }
    DRIFT_TRY(flush());
  }
  for (int i = 0; i < count; ++i) {
    if (done[i] || ns[i] == 0) continue;
    if (weight_dtypes[i] == DRIFT_F32)
      DRIFT_TRY(matvec_f32_weights(x_dtype, x, static_cast<const float*>(weights[i]), outs[i], m,
                                   ns[i], k, s));
    else if (m >= GEMM_MINIMUM_ROWS && tc_supports(weight_dtypes[i], weights[i], k))
      DRIFT_TRY(linear_tc(x_dtype, x, weight_dtypes[i], weights[i], outs[i], m, ns[i], k,
                          tc_region, s));
    else
      DRIFT_TRY(matvec_prepared(weight_dtypes[i], weights[i], records, outs[i], ns[i], k, m, s));
  }
  return 0;
}

int drift_linears(int x_dtype, const void* x, int count, const int* weight_dtypes,
                  const void* const* weights, float* const* outs, const int64_t* ns, int64_t m,
                  int64_t k, drift_stream_t stream) {
  return linears(x_dtype, x, nullptr, count, weight_dtypes, weights, outs, ns, m, k,
                 cudaStream_t(stream));
}

int drift_linears_prepared(int x_dtype, const void* x, const void* prepared, int count,
                           const int* weight_dtypes, const void* const* weights,
                           float* const* outs, const int64_t* ns, int64_t m, int64_t k,
                           drift_stream_t stream) {
  if (!prepared) return invalid("linears: no prepared x");
  if (x_dtype != DRIFT_F32) return invalid("linears: prepared x comes from F32 x");
  return linears(x_dtype, x, prepared, count, weight_dtypes, weights, outs, ns, m, k,
                 cudaStream_t(stream));
}

int drift_linear(int x_dtype, const void* x, int weight_dtype, const void* weight, float* out,
                 int64_t m, int64_t n, int64_t k, drift_stream_t stream) {
  const void* weights[1] = {weight};
  float* outs[1] = {out};
  const int64_t ns[1] = {n};
  const int dtypes[1] = {weight_dtype};
  return drift_linears(x_dtype, x, 1, dtypes, weights, outs, ns, m, k, stream);
}

}  // extern "C"
