// The layer operations around the products: the embedding gather, RMS norm
// (with the residual add fused), add, the gated activation (SwiGLU), rotary
// embedding, and products with F32 weights (routers).
//
// Reference kernels: gather_<t> (kernels/matvec.hip:830-839), gather_rows_f32
// (elementwise.hip:89-93), rms_norm_f32 (norm.hip:15-41), add_f32 /
// gated_f32 (elementwise.hip:14-65), rope_f32 (rope.hip:6-15, rope.h:20-51),
// matvec_rows_f32 (matvec.hip:1696-1734). Their CPU twins, which the results
// are checked against: ops/CpuLinear.scala:12-41, CpuNormalisation.scala:
// 11-71, CpuElementwise.scala:9-13, CpuAttention.scala:92-146.
#include <cuda_runtime.h>

#include "common.cuh"
#include "rowwise.cuh"
#include "x22.cuh"
#include "quant.cuh"
#include "registry.cuh"

namespace drift {

size_t mma_workspace_bytes(int64_t m, int64_t k);
int prepare_x_mma(int x_dtype, const void* x, int64_t m, int64_t k, uint8_t* records,
                  cudaStream_t stream);

// ---- the device error word -----------------------------------------------------------
// Set (first flag wins) by kernels that meet an input the reference refuses,
// instead of reading out of bounds; read and cleared by drift_device_error_take.
__device__ int error_word = 0;

int* device_error_word() {
  static int* words[64] = {nullptr};
  int device = 0;
  if (cudaGetDevice(&device) != cudaSuccess || device < 0 || device >= 64) return nullptr;
  if (!words[device]) {
    void* address = nullptr;
    if (cudaGetSymbolAddress(&address, error_word) != cudaSuccess) return nullptr;
    words[device] = static_cast<int*>(address);
  }
  return words[device];
}

__device__ __forceinline__ void flag_error(int* error, int code) {
  if (error) atomicCAS(error, 0, code);
}

// ---- embedding gather -----------------------------------------------------------------
// One warp per id; lane l decodes blocks l, l + 32, ... of row ids[i] into 32
// floats each, bit for bit the CPU decode (quant.cuh T::value).
template <typename T>
__global__ void __launch_bounds__(256) gather_kernel(const uint8_t* __restrict__ table,
                                                     const int* __restrict__ ids,
                                                     float* __restrict__ out, int count, int cols,
                                                     long long vocab, int* error) {
  pdl_trigger();  // the next kernel may launch and wait for this one
  pdl_wait();     // what the kernels before this one wrote is visible
  const int index = blockIdx.x * (blockDim.x / WARP) + threadIdx.x / WARP;
  if (index >= count) return;
  const int lane = threadIdx.x % WARP;
  const long long id = ids[index];
  float4* target = reinterpret_cast<float4*>(out + (long long)index * cols);
  const int blocks = cols / 32;
  if (id < 0 || id >= vocab) {
    const float nan = __int_as_float(0x7fc00000);
    for (int i = lane; i < cols / 4; i += WARP) target[i] = make_float4(nan, nan, nan, nan);
    if (lane == 0) flag_error(error, 1);
    return;
  }
  const uint8_t* row = table + id * (long long)blocks * T::BYTES;
  for (int c = lane; c < blocks; c += WARP) {
    uint32_t w[T::WORDS];
    load_block<T>(row, c, w);
    const Codes codes = T::decode(w, c);
#pragma unroll
    for (int i = 0; i < 8; ++i)
      target[c * 8 + i] = make_float4(T::value(codes, 4 * i), T::value(codes, 4 * i + 1),
                                      T::value(codes, 4 * i + 2), T::value(codes, 4 * i + 3));
  }
}

// F32 tables of any width: one thread per value.
__global__ void gather_rows_f32_kernel(const float* __restrict__ table, const int* __restrict__ ids,
                                       float* __restrict__ out, int count, int cols,
                                       long long vocab, int* error) {
  pdl_trigger();  // the next kernel may launch and wait for this one
  pdl_wait();     // what the kernels before this one wrote is visible
  const long long index = (long long)blockIdx.x * blockDim.x + threadIdx.x;
  if (index >= (long long)count * cols) return;
  const long long id = ids[index / cols];
  if (id < 0 || id >= vocab) {
    out[index] = __int_as_float(0x7fc00000);
    flag_error(error, 1);
    return;
  }
  out[index] = table[id * cols + index % cols];
}

DRIFT_REGISTER(gather_checked_q8_0, gather_kernel<Q8_0T>)
DRIFT_REGISTER(gather_checked_q4_0, gather_kernel<Q4_0T>)
DRIFT_REGISTER(gather_checked_q4_1, gather_kernel<Q4_1T>)
DRIFT_REGISTER(gather_rows_checked_f32, gather_rows_f32_kernel)

// ---- RMS norm ----------------------------------------------------------------------------
// One block of 256 threads per row (1024 for rows of more than 1024 values).
// With `y`, x += y first (written back: the residual stream). The sum of squares is float (each thread's values in
// order, then a fixed tree); 1 / sqrt(mean + eps) is rounded as IEEE division
// and square root round it, not rsqrtf's approximation. Rows of up to 256 PER
// values are held in registers, every load issued before the first use (a
// row is one round trip to memory, not PER of them).
template <int PER, int THREADS>
__global__ void __launch_bounds__(THREADS) rms_norm_kernel(float* __restrict__ x, const float* __restrict__ y,
                                                       const float* __restrict__ weight,
                                                       float* __restrict__ out, int cols,
                                                       float epsilon, float weight_offset,
                                                       uint8_t* __restrict__ records) {
  pdl_trigger();  // the next kernel may launch and wait for this one
  pdl_wait();     // what the kernels before this one wrote is visible
  __shared__ float partial[32];
  float* row = x + (long long)blockIdx.x * cols;
  const float* add = y ? y + (long long)blockIdx.x * cols : nullptr;
  float* target = out + (long long)blockIdx.x * cols;
  float value[PER], w[PER];
#pragma unroll
  for (int i = 0; i < PER; ++i) {
    const int c = threadIdx.x + i * THREADS;
    value[i] = c < cols ? row[c] : 0.0f;
    w[i] = c < cols ? weight[c] : 0.0f;
  }
  if (add) {
    float extra[PER];
#pragma unroll
    for (int i = 0; i < PER; ++i) {
      const int c = threadIdx.x + i * THREADS;
      extra[i] = c < cols ? add[c] : 0.0f;
    }
#pragma unroll
    for (int i = 0; i < PER; ++i) {
      const int c = threadIdx.x + i * THREADS;
      value[i] = value[i] + extra[i];
      if (c < cols) row[c] = value[i];
    }
  }
  float sum = 0.0f;
#pragma unroll
  for (int i = 0; i < PER; ++i) sum = fmaf(value[i], value[i], sum);
  const float total = block_sum(sum, partial);
  const float scale = 1.0f / sqrtf(total / float(cols) + epsilon);
#pragma unroll
  for (int i = 0; i < PER; ++i) {
    const int c = threadIdx.x + i * THREADS;
    const float normed = value[i] * scale * (w[i] + weight_offset);
    if (c < cols) target[c] = normed;
    // the next product's x records: warp w holds block 8 i + w of the row
    // (cols a multiple of 32, so the test is the same for the whole warp)
    if (records && c < cols) x22_record_block(normed, records, blockIdx.x, c / 32, cols / 32);
  }
}

// Rows longer than 4096: the same arithmetic, a pass over memory per 256.
__global__ void __launch_bounds__(256) rms_norm_long_kernel(float* __restrict__ x,
                                                            const float* __restrict__ y,
                                                            const float* __restrict__ weight,
                                                            float* __restrict__ out, int cols,
                                                            float epsilon, float weight_offset) {
  pdl_trigger();  // the next kernel may launch and wait for this one
  pdl_wait();     // what the kernels before this one wrote is visible
  __shared__ float partial[32];
  float* row = x + (long long)blockIdx.x * cols;
  const float* add = y ? y + (long long)blockIdx.x * cols : nullptr;
  float* target = out + (long long)blockIdx.x * cols;
  float sum = 0.0f;
  for (int c = threadIdx.x; c < cols; c += blockDim.x) {
    float value = row[c];
    if (add) {
      value = value + add[c];
      row[c] = value;
    }
    sum = fmaf(value, value, sum);
  }
  const float total = block_sum(sum, partial);
  const float scale = 1.0f / sqrtf(total / float(cols) + epsilon);
  for (int c = threadIdx.x; c < cols; c += blockDim.x)
    target[c] = row[c] * scale * (weight[c] + weight_offset);
}

int launch_rms_norm(float* x, const float* y, const float* weight, float* out, int64_t rows,
                    int64_t cols, float epsilon, float weight_offset, cudaStream_t stream,
                    uint8_t* records = nullptr) {
  const unsigned grid = unsigned(rows);
  const int c = int(cols);
#define DRIFT_NORM(PER, THREADS)                                                             \
  DRIFT_CUDA(launch_pdl(rms_norm_kernel<PER, THREADS>, grid, THREADS, 0, stream, x, y, weight, \
                        out, c, epsilon, weight_offset, records))
  if (cols <= 256) DRIFT_NORM(1, 256);
  else if (cols <= 512) DRIFT_NORM(2, 256);
  else if (cols <= 1024) DRIFT_NORM(4, 256);
  else if (cols <= 2048) DRIFT_NORM(2, 1024);
  else if (cols <= 4096) DRIFT_NORM(4, 1024);
  else if (cols <= 8192) DRIFT_NORM(8, 1024);
  else if (cols <= 16384) DRIFT_NORM(16, 1024);
  else
    DRIFT_CUDA(launch_pdl(rms_norm_long_kernel, grid, 256, 0, stream, x, y, weight, out, c, epsilon,
                          weight_offset));
#undef DRIFT_NORM
  DRIFT_LAUNCHED("rms_norm_f32");
  return 0;
}

DRIFT_REGISTER(rms_norm_records_f32, (rms_norm_kernel<4, 1024>))
DRIFT_REGISTER(rms_norm_long_f32, rms_norm_long_kernel)

// ---- elementwise ---------------------------------------------------------------------------
#define DRIFT_FOR_EACH(i, n)                                                     \
  for (long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x; i < (n); \
       i += (long long)gridDim.x * blockDim.x)

__global__ void add_kernel(const float* a, const float* b, float* out, long long n) {
  pdl_trigger();  // the next kernel may launch and wait for this one
  pdl_wait();     // what the kernels before this one wrote is visible
  DRIFT_FOR_EACH(i, n) out[i] = a[i] + b[i];
}

// With `records`, also the next product's x records of rows of `cols` values
// (cols and n multiples of 32: a warp's 32 consecutive values are one block,
// and the loop's test is the same for the whole warp).
__global__ void gated_kernel(const float* gate, const float* up, float* out, long long n, int kind,
                             int cols, uint8_t* records) {
  pdl_trigger();  // the next kernel may launch and wait for this one
  pdl_wait();     // what the kernels before this one wrote is visible
  DRIFT_FOR_EACH(i, n) {
    const float value = activate(gate[i], kind) * gated_up(up[i], kind);
    out[i] = value;
    if (records)  // n < 2^31 here
      x22_record_block(value, records, int(i) / cols, int(i) % cols / 32, cols / 32);
  }
}

DRIFT_REGISTER(add_f32, add_kernel)
DRIFT_REGISTER(gated_records_f32, gated_kernel)

// ---- rotary embedding ---------------------------------------------------------------------
// One thread per value of x [tokens, heads, head_dim]. The angle is the CPU
// reference's to the bit: the inverse frequency 1f / (float) pow(theta,
// 2 pair / rotary) (pow in double, then float), times float(position) in
// float; the turn is then in double, as CpuAttention.rope turns it, and
// rounded once. (The runner's own kernel uses powf/cosf/sinf and is held to
// 1e-2 against the CPU, SmallOpsTests.scala:450-500; this one lands within an
// ulp.)
__global__ void rope_kernel(const float* __restrict__ x, const int* __restrict__ positions,
                            float* __restrict__ out, int tokens, int heads, int head_dim,
                            int rotary, float theta, int layout) {
  pdl_trigger();  // the next kernel may launch and wait for this one
  pdl_wait();     // what the kernels before this one wrote is visible
  const long long index = (long long)blockIdx.x * blockDim.x + threadIdx.x;
  if (index >= (long long)tokens * heads * head_dim) return;
  const int d = int(index % head_dim);
  const int t = int(index / ((long long)heads * head_dim));
  out[index] = rope_turn(x + (index - d), d, positions[t], theta, rotary, layout);
}

DRIFT_REGISTER(rope_single_f32, rope_kernel)

// ---- products with F32 weights (routers) -----------------------------------------------------
// F32 weights (routers, DeltaNet's a and b): a CTA of 256 threads per (row,
// vector), the row summed by f32_row_dot (rowwise.cuh).
template <bool BF16>
__global__ void __launch_bounds__(256) matvec_f32_kernel(const void* __restrict__ x,
                                                         const float* __restrict__ weight,
                                                         float* __restrict__ y, int m, int n, int k) {
  pdl_trigger();  // the next kernel may launch and wait for this one
  pdl_wait();     // what the kernels before this one wrote is visible
  __shared__ float partial[32];
  const int row = blockIdx.x % n, vector = blockIdx.x / n;
  const float total = f32_row_dot<BF16>(x, weight, weight + (long long)row * k, vector, k, partial);
  if (threadIdx.x == 0) y[(long long)vector * n + row] = total;
}

// Up to four F32 products of the same x in one launch: CTA (vector, r) takes
// row r of the matrices' rows laid end to end.
constexpr int MAX_F32_MATRICES = 4;
struct F32Launch {
  const float* weight[MAX_F32_MATRICES];
  float* y[MAX_F32_MATRICES];
  int n[MAX_F32_MATRICES];
  int end[MAX_F32_MATRICES];  // matrix i holds rows [end[i - 1], end[i])
  int count;
};

template <bool BF16>
__global__ void __launch_bounds__(256) matvec_f32_many_kernel(const void* __restrict__ x,
                                                              const __grid_constant__ F32Launch L,
                                                              int k) {
  pdl_trigger();  // the next kernel may launch and wait for this one
  pdl_wait();     // what the kernels before this one wrote is visible
  __shared__ float partial[32];
  const int rows = L.end[L.count - 1];
  const int r = blockIdx.x % rows, vector = blockIdx.x / rows;
  int i = 0;
  while (i + 1 < L.count && r >= L.end[i]) ++i;
  const int row = r - (i > 0 ? L.end[i - 1] : 0);
  const float total =
      f32_row_dot<BF16>(x, L.weight[i], L.weight[i] + (long long)row * k, vector, k, partial);
  if (threadIdx.x == 0) L.y[i][(long long)vector * L.n[i] + row] = total;
}

DRIFT_REGISTER(matvec_f32_f32x, matvec_f32_kernel<false>)
DRIFT_REGISTER(matvec_f32_bf16x, matvec_f32_kernel<true>)
DRIFT_REGISTER(matvec_f32_many_f32x, matvec_f32_many_kernel<false>)
DRIFT_REGISTER(matvec_f32_many_bf16x, matvec_f32_many_kernel<true>)

int matvec_f32_weights(int x_dtype, const void* x, const float* weight, float* y, int64_t m,
                       int64_t n, int64_t k, cudaStream_t stream) {
  const long long ctas = m * n;
  if (ctas > 0x7fffffffll) return invalid("F32 product of %lld rows x %lld vectors", (long long)n,
                                          (long long)m);
  const unsigned grid = unsigned(ctas);
  if (x_dtype == DRIFT_BF16)
    DRIFT_CUDA(launch_pdl(matvec_f32_kernel<true>, grid, 256, 0, stream, x, weight, y, int(m),
                          int(n), int(k)));
  else
    DRIFT_CUDA(launch_pdl(matvec_f32_kernel<false>, grid, 256, 0, stream, x, weight, y, int(m),
                          int(n), int(k)));
  DRIFT_LAUNCHED("matvec_f32");
  return 0;
}

// F32 products of the same x (count <= 4, no empty matrix), one launch: each
// row the bits of matvec_f32_weights.
int matvec_f32_many(int x_dtype, const void* x, int count, const float* const* weights,
                    float* const* ys, const int64_t* ns, int64_t m, int64_t k,
                    cudaStream_t stream) {
  if (count < 1 || count > MAX_F32_MATRICES) return invalid("%d F32 products in one launch", count);
  F32Launch launch = {};
  long long rows = 0;
  for (int i = 0; i < count; ++i) {
    if (ns[i] <= 0) return invalid("an empty F32 product in a shared launch");
    rows += ns[i];
    launch.weight[i] = weights[i];
    launch.y[i] = ys[i];
    launch.n[i] = int(ns[i]);
    launch.end[i] = int(rows);
  }
  launch.count = count;
  const long long ctas = m * rows;
  if (rows > 0x7fffffffll || ctas > 0x7fffffffll)
    return invalid("F32 products of %lld rows x %lld vectors", rows, (long long)m);
  if (x_dtype == DRIFT_BF16)
    DRIFT_CUDA(launch_pdl(matvec_f32_many_kernel<true>, unsigned(ctas), 256, 0, stream, x, launch,
                          int(k)));
  else
    DRIFT_CUDA(launch_pdl(matvec_f32_many_kernel<false>, unsigned(ctas), 256, 0, stream, x,
                          launch, int(k)));
  DRIFT_LAUNCHED("matvec_f32_many");
  return 0;
}

static unsigned elementwise_grid(long long n) {
  long long blocks = (n + 255) / 256;
  const long long cap = (long long)sm_count() * 16;
  return unsigned(blocks < 1 ? 1 : (blocks > cap ? cap : blocks));
}

}  // namespace drift

using namespace drift;

extern "C" {

int drift_device_error_take(int* code) {
  if (!code) return invalid("drift_device_error_take: no slot for the code");
  int* word = device_error_word();
  if (!word) return invalid("the device error word is not reachable");
  DRIFT_CUDA(cudaDeviceSynchronize());
  DRIFT_CUDA(cudaMemcpy(code, word, sizeof(int), cudaMemcpyDeviceToHost));
  DRIFT_CUDA(cudaMemset(word, 0, sizeof(int)));
  return 0;
}

int drift_embedding(int table_dtype, const void* table, int64_t vocab, int64_t cols,
                    const int32_t* ids, int64_t count, float* out, drift_stream_t stream) {
  if (vocab < 0 || cols < 0 || count < 0)
    return invalid("an embedding table is [vocabulary, D], not [%lld, %lld]", (long long)vocab,
                   (long long)cols);
  if (table_dtype != DRIFT_Q8_0 && table_dtype != DRIFT_Q4_0 && table_dtype != DRIFT_Q4_1 &&
      table_dtype != DRIFT_F32)
    return invalid("no kernels for %s tables yet", dtype_name(table_dtype));
  const int64_t row = byte_size(table_dtype, cols);
  if (row < 0)
    return invalid("%lld elements are not whole %s blocks of %d", (long long)cols,
                   dtype_name(table_dtype), block_elements(table_dtype));
  if (table_dtype != DRIFT_F32 && row % 4 != 0)
    return invalid("%s rows of %lld are not whole words", dtype_name(table_dtype),
                   (long long)cols);
  if (count == 0 || cols == 0) return 0;
  if (!table || !ids || !out) return invalid("embedding: a null tensor");
  if (count > 0x7fffffffll || cols > 0x7fffffffll) return invalid("embedding too large");
  int* error = device_error_word();
  const cudaStream_t s = cudaStream_t(stream);
  const uint8_t* t = static_cast<const uint8_t*>(table);
  if (table_dtype == DRIFT_F32) {
    const long long values = count * cols;
    DRIFT_CUDA(launch_pdl(gather_rows_f32_kernel, unsigned((values + 255) / 256), 256, 0, s,
                          static_cast<const float*>(table), ids, out, int(count), int(cols), vocab,
                          error));
  } else {
    const unsigned grid = unsigned((count + 7) / 8);
    if (table_dtype == DRIFT_Q8_0)
      DRIFT_CUDA(launch_pdl(gather_kernel<Q8_0T>, grid, 256, 0, s, t, ids, out, int(count),
                            int(cols), vocab, error));
    else if (table_dtype == DRIFT_Q4_0)
      DRIFT_CUDA(launch_pdl(gather_kernel<Q4_0T>, grid, 256, 0, s, t, ids, out, int(count),
                            int(cols), vocab, error));
    else
      DRIFT_CUDA(launch_pdl(gather_kernel<Q4_1T>, grid, 256, 0, s, t, ids, out, int(count),
                            int(cols), vocab, error));
  }
  DRIFT_LAUNCHED("gather");
  return 0;
}

static int check_rows(const char* name, const void* x, const void* out, int64_t rows,
                      int64_t cols) {
  if (rows < 0 || cols < 0) return invalid("%s over [%lld, %lld]", name, (long long)rows,
                                           (long long)cols);
  if (rows > 0 && cols > 0 && (!x || !out)) return invalid("%s: a null tensor", name);
  if (rows > 0x7fffffffll || cols > 0x7fffffffll) return invalid("%s too large", name);
  return 0;
}

int drift_rms_norm(const float* x, const float* weight, float epsilon, float weight_offset,
                   float* out, int64_t rows, int64_t cols, drift_stream_t stream) {
  DRIFT_TRY(check_rows("rmsNorm", x, out, rows, cols));
  if (rows == 0 || cols == 0) return 0;
  if (!weight) return invalid("rmsNorm: no weight");
  return launch_rms_norm(const_cast<float*>(x), nullptr, weight, out, rows, cols, epsilon,
                         weight_offset, cudaStream_t(stream));
}

int drift_add_rms_norm(float* x, const float* y, const float* weight, float epsilon,
                       float weight_offset, float* out, int64_t rows, int64_t cols,
                       drift_stream_t stream) {
  DRIFT_TRY(check_rows("addRmsNorm", x, out, rows, cols));
  if (rows == 0 || cols == 0) return 0;
  if (!weight || !y) return invalid("addRmsNorm: no weight or no y");
  return launch_rms_norm(x, y, weight, out, rows, cols, epsilon, weight_offset,
                         cudaStream_t(stream));
}

size_t drift_prepared_x_bytes(int64_t m, int64_t k) {
  return m > 0 && k > 0 && k % 32 == 0 ? mma_workspace_bytes(m, k) : 0;
}

int drift_add_rms_norm_prepared(float* x, const float* y, const float* weight, float epsilon,
                                float weight_offset, float* out, int64_t rows, int64_t cols,
                                void* prepared, drift_stream_t stream) {
  DRIFT_TRY(check_rows(y ? "addRmsNorm" : "rmsNorm", x, out, rows, cols));
  if (rows == 0 || cols == 0) return 0;
  if (!weight) return invalid("rmsNorm: no weight");
  if (!prepared) return invalid("rmsNorm: no prepared x");
  if (cols % 32 != 0) return invalid("rmsNorm: prepared x needs rows of whole 32-value blocks");
  uint8_t* records = static_cast<uint8_t*>(prepared);
  const cudaStream_t s = cudaStream_t(stream);
  if (cols > 16384) {
    // the long rows' kernel leaves the records to the preparation kernel
    DRIFT_TRY(launch_rms_norm(x, y, weight, out, rows, cols, epsilon, weight_offset, s));
    return prepare_x_mma(DRIFT_F32, out, rows, cols, records, s);
  }
  return launch_rms_norm(x, y, weight, out, rows, cols, epsilon, weight_offset, s, records);
}

int drift_gated_prepared(int kind, const float* gate, const float* up, float* out, int64_t rows,
                         int64_t cols, void* prepared, drift_stream_t stream) {
  if (kind < 0 || kind > 4) return invalid("gated: activation code %d", kind);
  if (rows < 0 || cols < 0) return invalid("gated over [%lld, %lld]", (long long)rows,
                                           (long long)cols);
  if (rows == 0 || cols == 0) return 0;
  if (!gate || !up || !out || !prepared) return invalid("gated: a null tensor");
  if (cols % 32 != 0) return invalid("gated: prepared x needs rows of whole 32-value blocks");
  if (rows * cols > 0x7fffffffll) return invalid("gated: %lld values to prepare", rows * cols);
  const long long n = rows * cols;
  DRIFT_CUDA(launch_pdl(gated_kernel, elementwise_grid(n), 256, 0, cudaStream_t(stream), gate, up,
                        out, n, kind, int(cols), static_cast<uint8_t*>(prepared)));
  DRIFT_LAUNCHED("gated_f32");
  return 0;
}

int drift_add(const float* a, const float* b, float* out, int64_t n, drift_stream_t stream) {
  if (n < 0) return invalid("add over %lld values", (long long)n);
  if (n == 0) return 0;
  if (!a || !b || !out) return invalid("add: a null tensor");
  DRIFT_CUDA(launch_pdl(add_kernel, elementwise_grid(n), 256, 0, cudaStream_t(stream), a, b, out,
                        n));
  DRIFT_LAUNCHED("add_f32");
  return 0;
}

int drift_gated(int kind, const float* gate, const float* up, float* out, int64_t n,
                drift_stream_t stream) {
  if (kind < 0 || kind > 4) return invalid("gated: activation code %d", kind);
  if (n < 0) return invalid("gated over %lld values", (long long)n);
  if (n == 0) return 0;
  if (!gate || !up || !out) return invalid("gated: a null tensor");
  DRIFT_CUDA(launch_pdl(gated_kernel, elementwise_grid(n), 256, 0, cudaStream_t(stream), gate, up,
                        out, n, kind, 32, static_cast<uint8_t*>(nullptr)));
  DRIFT_LAUNCHED("gated_f32");
  return 0;
}

int drift_rope(const float* x, const int32_t* positions, float* out, int tokens, int heads,
               int head_dim, float theta, int rotary, int layout, drift_stream_t stream) {
  if (tokens < 0 || heads < 0 || head_dim < 0)
    return invalid("rope takes [tokens, heads, headDimension], got [%d, %d, %d]", tokens, heads,
                   head_dim);
  if (rotary <= 0 || rotary % 2 != 0 || rotary > head_dim)
    return invalid("rope: %d rotary values of a head of %d", rotary, head_dim);
  if (layout != DRIFT_ROPE_NEOX && layout != DRIFT_ROPE_INTERLEAVED)
    return invalid("rope: layout %d", layout);
  const long long values = (long long)tokens * heads * head_dim;
  if (values == 0) return 0;
  if (!x || !positions || !out) return invalid("rope: a null tensor");
  DRIFT_CUDA(launch_pdl(rope_kernel, unsigned((values + 255) / 256), 256, 0, cudaStream_t(stream), x,
                        positions, out, tokens, heads, head_dim, rotary, theta, layout));
  DRIFT_LAUNCHED("rope_f32");
  return 0;
}

}  // extern "C"
