// The runner's kernels by name: for a host that keeps HipOps' dispatch
// (runner/src/drift/runner/ops/Hip*.scala) and launches kernels through
// drift_module_get_function(&f, NULL, name) + drift_module_launch_kernel,
// these are registered under the runner's own kernel names with the runner's
// own argument lists (runner/kernels/*.hip), each working with the grid and
// block that dispatch computes. What each one computes is the operation the
// reference names; its arithmetic is this library's (results within the
// tests' bars of the CPU reference, gathers bit for bit).
//
// The `xq, xd, xs` outputs of rms_norm_f32, gated_f32, gated_rms_norm_f32 and
// moe_combine_norm are written in the runner's int8 format (kernels/
// quantize.h:6-25: per 32 values xd = max|x| / 127, xq = round(x / xd),
// xs = xd * sum(xq)) when non-null, as the runner's int8 products read them.
//
// The product kernels take float x, the runner's MatVecInputs.Float mode:
// matvec_float_x(_narrow)_<t>, matvec_float_x_multi(_narrow)_<t> and
// matvec_split_<t> for Q8_0, Q4_0 and (new) Q4_1, and matvec_rows_f32 for F32
// routers. Each (row, vector) sums in one fixed order whatever the number of
// vectors, so a verification's tokens get a decode step's bits.
#include <cuda_runtime.h>
#include <math.h>

#include "common.cuh"
#include "quant.cuh"
#include "registry.cuh"
#include "rowwise.cuh"

namespace drift {
namespace {

constexpr unsigned FULL = 0xffffffffu;

__device__ __forceinline__ long long global_warp() {
  const long long block = (long long)blockIdx.y * gridDim.x + blockIdx.x;
  return block * (blockDim.x / WARP) + threadIdx.x / WARP;
}
__device__ __forceinline__ long long total_warps() {
  return (long long)gridDim.x * gridDim.y * (blockDim.x / WARP);
}

// The runner's int8 x format for one 32-value block held by one warp (lane l
// value l): every lane of the warp calls.
__device__ __forceinline__ void quantize_int8_block(float value, long long block, int8_t* xq,
                                                    float* xd, float* xs) {
  const int lane = threadIdx.x % WARP;
  float amax = fabsf(value);
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(FULL, amax, o));
  const float d = amax / 127.0f;
  const int q = d == 0.0f ? 0 : int(roundf(value / d));
  xq[block * 32 + lane] = int8_t(q);
  int sum = q;
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) sum += __shfl_xor_sync(FULL, sum, o);
  if (lane == 0) {
    xd[block] = d;
    xs[block] = d * float(sum);
  }
}

// The words covering block c of a row, as T::decode reads them. Rows that
// start on a 4-byte boundary and are whole words (every row the runner's
// dispatch sends) take aligned loads; any other row is read byte by byte,
// never past the block's own bytes.
template <typename T>
__device__ __forceinline__ void block_words(const uint8_t* row, int c, bool aligned,
                                            uint32_t (&w)[T::WORDS]) {
  if (aligned) {
    load_block<T>(row, c, w);
    return;
  }
  const int off = (c * T::BYTES) & 3;
  const uint8_t* p = row + (long long)c * T::BYTES;
#pragma unroll
  for (int i = 0; i < T::WORDS; ++i) {
    uint32_t word = 0;
#pragma unroll
    for (int b = 0; b < 4; ++b) {
      const int source = 4 * i + b - off;
      if (source >= 0 && source < T::BYTES) word |= uint32_t(p[source]) << (8 * b);
    }
    w[i] = word;
  }
}

template <typename T>
__device__ __forceinline__ bool word_rows(const void* base, int cols) {
  return (reinterpret_cast<uintptr_t>(base) & 3) == 0 && (cols / 32 * T::BYTES) % 4 == 0;
}

// ---- gathers (matvec.hip:894-896, elementwise.hip:89-93) --------------------------------------
// gather_<t>(weight, ids, out, count, cols): a warp per id, grid (count + 7) / 8
// of 256. The runner checks ids on the host (there is no vocabulary here).
template <typename T>
__global__ void gather_by_name(const uint8_t* __restrict__ table, const int* __restrict__ ids,
                               float* __restrict__ out, int count, int cols) {
  const int lane = threadIdx.x % WARP, blocks = cols / 32;
  const bool aligned = word_rows<T>(table, cols);
  for (long long index = global_warp(); index < count; index += total_warps()) {
    const uint8_t* row = table + (long long)ids[index] * blocks * T::BYTES;
    float* target = out + index * cols;
    for (int c = lane; c < blocks; c += WARP) {
      uint32_t w[T::WORDS];
      block_words<T>(row, c, aligned, w);
      const Codes codes = T::decode(w, c);
#pragma unroll
      for (int j = 0; j < 32; ++j) target[c * 32 + j] = T::value(codes, j);
    }
  }
}

__global__ void gather_rows_by_name(const float* __restrict__ table, const int* __restrict__ ids,
                                    float* __restrict__ out, int count, int cols) {
  const long long n = (long long)count * cols;
  for (long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x; i < n;
       i += (long long)gridDim.x * blockDim.x)
    out[i] = table[(long long)ids[i / cols] * cols + i % cols];
}

// ---- rms_norm_f32 (norm.hip:34-35) ----------------------------------------------------------
// A block per row (256 or 1024 threads). x += y first when y is given;
// weight row r % weight_rows. The arithmetic of drift_rms_norm: each thread's
// squares in column order, then the block's fixed tree, 1 / sqrt in IEEE.
__global__ void rms_norm_by_name(float* __restrict__ x, const float* __restrict__ y,
                                 const float* __restrict__ weight, float* __restrict__ out,
                                 int cols, float epsilon, float offset, int weight_rows,
                                 int8_t* xq, float* xd, float* xs) {
  __shared__ float partial[32];
  const long long r = blockIdx.x;
  float* row = x + r * cols;
  const float* w = weight + (r % weight_rows) * cols;
  float sum = 0.0f;
  for (int c = threadIdx.x; c < cols; c += blockDim.x) {
    float value = row[c];
    if (y) {
      value = value + y[r * cols + c];
      row[c] = value;
    }
    sum = fmaf(value, value, sum);
  }
  const float scale = 1.0f / sqrtf(block_sum(sum, partial) / float(cols) + epsilon);
  // (whole warps of whole blocks only: a warp's 32 values are one block)
  const bool quantized = xq && cols % 32 == 0 && blockDim.x % 32 == 0;
  for (int c = threadIdx.x; c < cols; c += blockDim.x) {
    const float value = row[c] * scale * (w[c] + offset);
    out[r * cols + c] = value;
    if (quantized) quantize_int8_block(value, (r * cols + c) / 32, xq, xd, xs);
  }
}

// ---- gated_f32 (elementwise.hip:58-59) ---------------------------------------------------------
__global__ void gated_by_name(const float* __restrict__ gate, const float* __restrict__ up,
                              float* __restrict__ out, long long n, int kind, int8_t* xq,
                              float* xd, float* xs) {
  // (a warp's 32 consecutive values are one block: n whole blocks only)
  const bool quantized = xq && n % 32 == 0 && blockDim.x % 32 == 0;
  for (long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x; i < n;
       i += (long long)gridDim.x * blockDim.x) {
    const float value = activate(gate[i], kind) * gated_up(up[i], kind);
    out[i] = value;
    if (quantized) quantize_int8_block(value, i / 32, xq, xd, xs);
  }
}

// ---- rope_f32 (rope.hip:6-8) --------------------------------------------------------------------
__global__ void rope_by_name(const float* __restrict__ x, const int* __restrict__ positions,
                             float* __restrict__ out, int tokens, int heads, int head_dim,
                             int rotary, float theta, int layout, int sections, int s0, int s1,
                             int s2, int s3) {
  const long long n = (long long)tokens * heads * head_dim;
  for (long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x; i < n;
       i += (long long)gridDim.x * blockDim.x) {
    const int d = int(i % head_dim);
    const int t = int(i / ((long long)heads * head_dim));
    out[i] = rope_turn_sections(x + (i - d), d, positions, t, tokens, theta, rotary, layout,
                                sections, s0, s1, s2, s3);
  }
}

// ---- products over float x (matvec.hip:899-924; HipLinear.scala:246-273) ------------------
// One warp per weight row: lane l takes blocks l, l + 32, ... of the row, each
// value (decoded exactly, as the CPU decodes it) times x by a fused
// multiply-add in column order, then the warp's fixed tree. All vectors of a
// row in one pass over its bytes, eight at a time.
template <typename T>
__device__ void row_products(const uint8_t* __restrict__ weight, const float* __restrict__ x,
                             float* __restrict__ y, long long row, int rows, int cols,
                             int vectors) {
  const int lane = threadIdx.x % WARP, blocks = cols / 32;
  const uint8_t* bytes = weight + row * blocks * T::BYTES;
  const bool aligned = word_rows<T>(weight, cols);
  const bool x4 = (reinterpret_cast<uintptr_t>(x) & 15) == 0;
  for (int v0 = 0; v0 < vectors; v0 += 8) {
    float sum[8];
#pragma unroll
    for (int v = 0; v < 8; ++v) sum[v] = 0.0f;
    for (int c = lane; c < blocks; c += WARP) {
      uint32_t w[T::WORDS];
      block_words<T>(bytes, c, aligned, w);
      const Codes codes = T::decode(w, c);
#pragma unroll
      for (int j4 = 0; j4 < 8; ++j4) {
        const float a = T::value(codes, 4 * j4), b = T::value(codes, 4 * j4 + 1);
        const float e = T::value(codes, 4 * j4 + 2), f = T::value(codes, 4 * j4 + 3);
#pragma unroll
        for (int v = 0; v < 8; ++v) {
          if (v0 + v >= vectors) break;
          const float* at = x + (long long)(v0 + v) * cols + c * 32 + 4 * j4;
          const float4 xv = x4 ? *reinterpret_cast<const float4*>(at)
                               : make_float4(at[0], at[1], at[2], at[3]);
          sum[v] = fmaf(f, xv.w, fmaf(e, xv.z, fmaf(b, xv.y, fmaf(a, xv.x, sum[v]))));
        }
      }
    }
#pragma unroll
    for (int v = 0; v < 8; ++v) {
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) sum[v] += __shfl_xor_sync(FULL, sum[v], o);
      if (lane == 0 && v0 + v < vectors) y[(long long)(v0 + v) * rows + row] = sum[v];
    }
  }
}

// matvec_float_x_<t> / _narrow_<t>(weight, x, y, rows, cols, vectors): grid
// (rows + 7) / 8 of 256, a warp per row.
template <typename T>
__global__ void matvec_by_name(const uint8_t* __restrict__ weight, const float* __restrict__ x,
                               float* __restrict__ y, int rows, int cols, int vectors) {
  for (long long row = global_warp(); row < rows; row += total_warps())
    row_products<T>(weight, x, y, row, rows, cols, vectors);
}

// matvec_float_x_multi(_narrow)_<t>: up to four matrices of one type and width
// over the same x, their rows numbered one after the other.
template <typename T>
__global__ void matvec_multi_by_name(const uint8_t* w0, float* y0, int r0, const uint8_t* w1,
                                     float* y1, int r1, const uint8_t* w2, float* y2, int r2,
                                     const uint8_t* w3, float* y3, int r3, const float* x,
                                     int cols, int vectors) {
  const long long total = (long long)r0 + r1 + r2 + r3;
  for (long long g = global_warp(); g < total; g += total_warps()) {
    long long row = g;
    const uint8_t* weight = w0;
    float* y = y0;
    int rows = r0;
    if (row >= r0) {
      row -= r0, weight = w1, y = y1, rows = r1;
      if (row >= r1) {
        row -= r1, weight = w2, y = y2, rows = r2;
        if (row >= r2) row -= r2, weight = w3, y = y3, rows = r3;
      }
    }
    row_products<T>(weight, x, y, row, rows, cols, vectors);
  }
}

// matvec_split_<t>(weight, x, y, rows, cols): grid (rows, vectors) of 256, the
// block's threads sharing one (row, vector): thread i takes blocks i, i +
// 256, ..., then the block's fixed tree.
template <typename T>
__global__ void matvec_split_by_name(const uint8_t* __restrict__ weight,
                                     const float* __restrict__ x, float* __restrict__ y, int rows,
                                     int cols) {
  __shared__ float partial[32];
  const long long row = blockIdx.x, vector = blockIdx.y;
  if (row >= rows) return;
  const int blocks = cols / 32;
  const uint8_t* bytes = weight + row * blocks * T::BYTES;
  const float* xv = x + vector * cols;
  float sum = 0.0f;
  const bool aligned = word_rows<T>(weight, cols);
  for (int c = threadIdx.x; c < blocks; c += blockDim.x) {
    uint32_t w[T::WORDS];
    block_words<T>(bytes, c, aligned, w);
    const Codes codes = T::decode(w, c);
#pragma unroll
    for (int j = 0; j < 32; ++j) sum = fmaf(T::value(codes, j), xv[c * 32 + j], sum);
  }
  const float total = block_sum(sum, partial);
  if (threadIdx.x == 0) y[vector * rows + row] = total;
}

// matvec_rows_f32(weight, x, out, n, k, m): F32 weights (routers), grid
// (n + 3) / 4 of 256; a warp per row, every vector.
__global__ void matvec_rows_f32_by_name(const float* __restrict__ weight,
                                        const float* __restrict__ x, float* __restrict__ out,
                                        int n, int k, int m) {
  const int lane = threadIdx.x % WARP;
  for (long long row = global_warp(); row < n; row += total_warps()) {
    const float* w = weight + row * k;
    for (int v = 0; v < m; ++v) {
      float sum = 0.0f;
      for (int c = lane; c < k; c += WARP) sum = fmaf(w[c], x[(long long)v * k + c], sum);
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) sum += __shfl_xor_sync(FULL, sum, o);
      if (lane == 0) out[(long long)v * n + row] = sum;
    }
  }
}

// ---- mixture of experts (linear_attention.hip:286-297, norm.hip:46-59) ------------------------
// The shared expert's gate sigmoid(x . router), by the block's threads.
__device__ __forceinline__ float shared_gate(const float* x, const float* router, int hidden,
                                             float* partial) {
  float dot = 0.0f;
  for (int c = threadIdx.x; c < hidden; c += blockDim.x) dot = fmaf(x[c], router[c], dot);
  return 1.0f / (1.0f + expf(-block_sum(dot, partial)));
}

// Element c of token t: residual + sum_j w_j out_j (slot order) + gate shared.
__device__ __forceinline__ float combined(const float* expert_out, const float* weights,
                                          const float* shared, float gate, const float* residual,
                                          long long t, int c, int k, int hidden) {
  float routed = 0.0f;
  for (int j = 0; j < k; ++j)
    routed = fmaf(weights[t * k + j], expert_out[(t * k + j) * hidden + c], routed);
  float sum = (residual ? residual[t * hidden + c] : 0.0f) + routed;
  if (shared) sum = fmaf(gate, shared[t * hidden + c], sum);
  return sum;
}

// moe_combine(expert_out, weights, shared, x, shared_router, residual, out, k,
// hidden): grid tokens * 8 of 256, block b taking slice b % 8 of token b / 8.
constexpr int SLICES = 8;
__global__ void moe_combine_by_name(const float* __restrict__ expert_out,
                                    const float* __restrict__ weights, const float* shared,
                                    const float* x, const float* shared_router,
                                    const float* residual, float* out, int k, int hidden) {
  __shared__ float partial[32];
  const long long t = blockIdx.x / SLICES;
  const int slice = blockIdx.x % SLICES;
  const float gate = shared ? shared_gate(x + t * hidden, shared_router, hidden, partial) : 0.0f;
  const int begin = int((long long)hidden * slice / SLICES);
  const int end = int((long long)hidden * (slice + 1) / SLICES);
  for (int c = begin + threadIdx.x; c < end; c += blockDim.x)
    out[t * hidden + c] = combined(expert_out, weights, shared, gate, residual, t, c, k, hidden);
}

// moe_combine_norm(expert_out, weights, shared, x, shared_router, residual, k,
// hidden, norm_weight, normed, eps, offset, xq, xd, xs): a block of 1024 per
// token; residual becomes the combined row, normed its RMS norm.
__global__ void __launch_bounds__(1024)
    moe_combine_norm_by_name(const float* __restrict__ expert_out,
                             const float* __restrict__ weights, const float* shared,
                             const float* x, const float* shared_router, float* residual, int k,
                             int hidden, const float* __restrict__ norm_weight,
                             float* __restrict__ normed, float epsilon, float offset, int8_t* xq,
                             float* xd, float* xs) {
  __shared__ float partial[32];
  const long long t = blockIdx.x;
  const float gate = shared ? shared_gate(x + t * hidden, shared_router, hidden, partial) : 0.0f;
  float squares = 0.0f;
  for (int c = threadIdx.x; c < hidden; c += blockDim.x) {
    const float value = combined(expert_out, weights, shared, gate, residual, t, c, k, hidden);
    residual[t * hidden + c] = value;  // (each element read and written by one thread)
    squares = fmaf(value, value, squares);
  }
  const float scale = 1.0f / sqrtf(block_sum(squares, partial) / float(hidden) + epsilon);
  const bool quantized = xq && hidden % 32 == 0 && blockDim.x % 32 == 0;
  for (int c = threadIdx.x; c < hidden; c += blockDim.x) {
    const float value = residual[t * hidden + c] * scale * (norm_weight[c] + offset);
    normed[t * hidden + c] = value;
    if (quantized) quantize_int8_block(value, (t * hidden + c) / 32, xq, xd, xs);
  }
}

// ---- Gated DeltaNet's convolution and norm (linear_attention.hip:16-17, norm.hip:99-101) -----
// causal_conv_silu(x, weight, state, out, tokens, channels, taps, dilation,
// history): a thread per channel, grid (channels + 255) / 256; the window of
// the last (taps - 1) * dilation <= 16 inputs in registers, state (and
// history, when given) written back as drift_causal_conv writes them.
constexpr int MAX_SPAN = 16;
__global__ void causal_conv_by_name(const float* __restrict__ x, const float* __restrict__ weight,
                                    float* __restrict__ state, float* __restrict__ out,
                                    int tokens, int channels, int taps, int dilation,
                                    float* __restrict__ history) {
  const int c = blockIdx.x * blockDim.x + threadIdx.x;
  if (c >= channels) return;
  const int span = (taps - 1) * dilation;
  float window[MAX_SPAN];
#pragma unroll
  for (int i = 0; i < MAX_SPAN; ++i) window[i] = i < span ? state[(long long)i * channels + c] : 0.0f;
  const float* w = weight + (long long)c * taps;
  for (int t = 0; t < tokens; ++t) {
    const float current = x[(long long)t * channels + c];
    float sum = 0.0f;
    for (int i = 0; i < taps - 1; ++i) {
      const int at = span - (taps - 1 - i) * dilation;
      float seen = 0.0f;
#pragma unroll
      for (int s = 0; s < MAX_SPAN; ++s)
        if (s == at) seen = window[s];
      sum = fmaf(w[i], seen, sum);
    }
    sum = fmaf(w[taps - 1], current, sum);
    out[(long long)t * channels + c] = sum / (1.0f + expf(-sum));
#pragma unroll
    for (int s = 0; s + 1 < MAX_SPAN; ++s)
      if (s + 1 < span) window[s] = window[s + 1];
#pragma unroll
    for (int s = 0; s < MAX_SPAN; ++s)
      if (s == span - 1) window[s] = current;
    if (history)
#pragma unroll
      for (int s = 0; s < MAX_SPAN; ++s)
        if (s < span) history[((long long)t * span + s) * channels + c] = window[s];
  }
#pragma unroll
  for (int s = 0; s < MAX_SPAN; ++s)
    if (s < span) state[(long long)s * channels + c] = window[s];
}

// gated_rms_norm_f32(x, weight, gate, out, cols, eps, sigmoid_gate, xq, xd,
// xs): a block of 256 per row; out = rmsNorm(x) * weight * act(gate), act
// SiLU or sigmoid. out may be x.
__global__ void gated_rms_norm_by_name(const float* x, const float* __restrict__ weight,
                                       const float* __restrict__ gate, float* out, int cols,
                                       float epsilon, int sigmoid_gate, int8_t* xq, float* xd,
                                       float* xs) {
  __shared__ float partial[32];
  const long long base = (long long)blockIdx.x * cols;
  float squares = 0.0f;
  for (int c = threadIdx.x; c < cols; c += blockDim.x) squares = fmaf(x[base + c], x[base + c], squares);
  const float scale = 1.0f / sqrtf(block_sum(squares, partial) / float(cols) + epsilon);
  const bool quantized = xq && cols % 32 == 0 && blockDim.x % 32 == 0;
  for (int c = threadIdx.x; c < cols; c += blockDim.x) {
    const float g = gate[base + c];
    const float act = sigmoid_gate ? 1.0f / (1.0f + expf(-g)) : g / (1.0f + expf(-g));
    const float value = x[base + c] * scale * weight[c] * act;
    out[base + c] = value;
    if (quantized) quantize_int8_block(value, (base + c) / 32, xq, xd, xs);
  }
}

// ---- the read-only bandwidth probe (bandwidth.hip:5-20) ---------------------------------------
// read_sum_f32x4(x, n4, partials): n4 float4 values read once, one partial
// sum per block -- how fast HBM serves pure reads (the copy peak counts a
// write for every read). Four loads of a thread in flight at a time.
__global__ void __launch_bounds__(256)
    read_sum_by_name(const float4* __restrict__ x, long long n4, float* __restrict__ partials) {
  __shared__ float partial[32];
  const long long stride = (long long)gridDim.x * blockDim.x;
  long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x;
  float sum = 0.0f;
  for (; i + 3 * stride < n4; i += 4 * stride) {
    float4 v[4];
#pragma unroll
    for (int u = 0; u < 4; ++u) v[u] = __ldcs(x + i + u * stride);
#pragma unroll
    for (int u = 0; u < 4; ++u) sum += (v[u].x + v[u].y) + (v[u].z + v[u].w);
  }
  for (; i < n4; i += stride) {
    const float4 v = __ldcs(x + i);
    sum += (v.x + v.y) + (v.z + v.w);
  }
  const float total = block_sum(sum, partial);
  if (threadIdx.x == 0) partials[blockIdx.x] = total;
}

}  // namespace

DRIFT_REGISTER(read_sum_f32x4, read_sum_by_name)

#define DRIFT_BY_NAME_TYPE(name, T)                                               \
  DRIFT_REGISTER(gather_##name, gather_by_name<T>)                                  \
  DRIFT_REGISTER(matvec_float_x_##name, matvec_by_name<T>)                         \
  DRIFT_REGISTER(matvec_float_x_narrow_##name, matvec_by_name<T>)                  \
  DRIFT_REGISTER(matvec_float_x_multi_##name, matvec_multi_by_name<T>)             \
  DRIFT_REGISTER(matvec_float_x_multi_narrow_##name, matvec_multi_by_name<T>)      \
  DRIFT_REGISTER(matvec_split_##name, matvec_split_by_name<T>)
DRIFT_BY_NAME_TYPE(q8_0, Q8_0T)
DRIFT_BY_NAME_TYPE(q4_0, Q4_0T)
DRIFT_BY_NAME_TYPE(q4_1, Q4_1T)
DRIFT_REGISTER(gather_rows_f32, gather_rows_by_name)
DRIFT_REGISTER(rms_norm_f32, rms_norm_by_name)
DRIFT_REGISTER(gated_f32, gated_by_name)
DRIFT_REGISTER(rope_f32, rope_by_name)
DRIFT_REGISTER(matvec_rows_f32, matvec_rows_f32_by_name)
DRIFT_REGISTER(moe_combine, moe_combine_by_name)
DRIFT_REGISTER(moe_combine_norm, moe_combine_norm_by_name)
DRIFT_REGISTER(causal_conv_silu, causal_conv_by_name)
DRIFT_REGISTER(gated_rms_norm_f32, gated_rms_norm_by_name)

}  // namespace drift
