// Products over GGML's K-quants Q4_K and Q6_K (the runner's Q4_K / Q6_K
// matvec types, runner/kernels/matvec.hip:278-358; CPU decode
// tensor/KQuants.scala:99-134): super-blocks of 256 values, in sub-blocks of
// 32 (Q4_K: a 6-bit scale and min each) or 16 (Q6_K: an int8 scale each).
//
// A warp takes one row for a pass of up to 8 vectors of x; lane l walks the
// row's 32-value chunks l, l + 32, ... -- one chunk a step: its codes
// (32 bytes of nibbles, and for Q6_K 32 bytes of high bits; as words, or as
// halfwords for Q6_K, whose 210-byte super-blocks are only 2-byte aligned),
// its scales -- decodes each value exactly as KQuants.element
// does (d * sc then * q, minus dmin * m, in float, no contraction; for Q6_K
// d * sc then * (q - 32)), and adds value * x in F32 per vector. The lanes'
// sums meet by a shuffle tree. x is F32 or BF16, read through L1 (every warp
// of a CTA reads the same x). The reference's CPU product sums in Double;
// the F32 sums here hold to the 1e-4 + 1e-3 |e| bar. The weights stream at
// one pass per 8 vectors: a HBM-bound kernel at 1-8 vectors.
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include "common.cuh"
#include "registry.cuh"

namespace drift {

namespace {

constexpr int K_WARPS = 8, K_MAX_VECTORS = 8;

__device__ __forceinline__ float f16_at(const uint8_t* p) {
  return __half2float(__ushort_as_half(uint16_t(p[0] | (p[1] << 8))));
}

// 32 bytes of a field: as words where the field is 4-byte aligned (Q4_K:
// 144-byte super-blocks, rows of whole 16-byte units), as halfwords where it
// is only 2-byte aligned (Q6_K: 210-byte super-blocks).
template <int ALIGN>
__device__ __forceinline__ void load32(const uint8_t* p, uint8_t (&b)[32]) {
  if constexpr (ALIGN == 4) {
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const uint32_t w = __ldg(reinterpret_cast<const uint32_t*>(p) + i);
      b[4 * i] = uint8_t(w);
      b[4 * i + 1] = uint8_t(w >> 8);
      b[4 * i + 2] = uint8_t(w >> 16);
      b[4 * i + 3] = uint8_t(w >> 24);
    }
  } else {
#pragma unroll
    for (int i = 0; i < 16; ++i) {
      const uint16_t h = __ldg(reinterpret_cast<const unsigned short*>(p) + i);
      b[2 * i] = uint8_t(h);
      b[2 * i + 1] = uint8_t(h >> 8);
    }
  }
}

// Chunk c (0..7) of a Q4_K super-block: values 32c..32c+31.
__device__ __forceinline__ void q4k_chunk(const uint8_t* block, int c, float (&v)[32]) {
  const uint8_t* s = block + 4;
  int scale, min;
  if (c < 4) {
    scale = s[c] & 63;
    min = s[c + 4] & 63;
  } else {
    scale = (s[c + 4] & 0xf) | ((s[c - 4] >> 2) & 0x30);
    min = (s[c + 4] >> 4) | ((s[c] >> 2) & 0x30);
  }
  const float d = __fmul_rn(f16_at(block), float(scale));
  const float m = __fmul_rn(f16_at(block + 2), float(min));
  uint8_t q[32];
  load32<4>(block + 16 + (c / 2) * 32, q);
  const int shift = 4 * (c % 2);
#pragma unroll
  for (int j = 0; j < 32; ++j) v[j] = __fsub_rn(__fmul_rn(d, float((q[j] >> shift) & 0xf)), m);
}

// Chunk c (0..7) of a Q6_K super-block: values 32c..32c+31, two sub-blocks
// of 16 with their own scale.
__device__ __forceinline__ void q6k_chunk(const uint8_t* block, int c, float (&v)[32]) {
  const int half = c / 4, plane = c % 4;
  uint8_t low[32], high[32];
  load32<2>(block + half * 64 + (plane % 2) * 32, low);
  load32<2>(block + 128 + half * 32, high);
  const float d = f16_at(block + 208);
  const float d0 = __fmul_rn(d, float(int8_t(block[192 + 2 * c])));
  const float d1 = __fmul_rn(d, float(int8_t(block[193 + 2 * c])));
  const int low_shift = 4 * (plane / 2), high_shift = 2 * plane;
#pragma unroll
  for (int j = 0; j < 32; ++j) {
    const int q = (((low[j] >> low_shift) & 0xf) | (((high[j] >> high_shift) & 3) << 4)) - 32;
    v[j] = __fmul_rn(j < 16 ? d0 : d1, float(q));
  }
}

template <int DTYPE>
struct KType;
template <>
struct KType<DRIFT_Q4_K> {
  static constexpr int BYTES = 144;
  __device__ static void chunk(const uint8_t* block, int c, float (&v)[32]) { q4k_chunk(block, c, v); }
};
template <>
struct KType<DRIFT_Q6_K> {
  static constexpr int BYTES = 210;
  __device__ static void chunk(const uint8_t* block, int c, float (&v)[32]) { q6k_chunk(block, c, v); }
};

template <bool BF16>
__device__ __forceinline__ float x_at(const void* x, long long i) {
  if constexpr (BF16)
    return __bfloat162float(__ldg(static_cast<const __nv_bfloat16*>(x) + i));
  else
    return __ldg(static_cast<const float*>(x) + i);
}

// y[v][row] = sum_c value_c x[v][c] for vectors [0, vectors) of this pass.
template <int DTYPE, int V, bool BF16>
__global__ void __launch_bounds__(K_WARPS * 32) kquant_linear_kernel(
    const uint8_t* __restrict__ weight, const void* __restrict__ x, float* __restrict__ y,
    int rows, int cols, int vectors) {
  pdl_trigger();  // the next kernel may launch and wait for this one
  pdl_wait();     // what the kernels before this one wrote is visible
  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  const int row = blockIdx.x * K_WARPS + warp;
  if (row >= rows) return;
  const int chunks = cols / 32;
  const uint8_t* base = weight + (long long)row * (cols / 256) * KType<DTYPE>::BYTES;
  float acc[V];
#pragma unroll
  for (int v = 0; v < V; ++v) acc[v] = 0.0f;
  for (int c = lane; c < chunks; c += 32) {
    float value[32];
    KType<DTYPE>::chunk(base + (c / 8) * KType<DTYPE>::BYTES, c % 8, value);
#pragma unroll
    for (int v = 0; v < V; ++v) {
      if (v >= vectors) break;
      const long long at = (long long)v * cols + 32ll * c;
#pragma unroll
      for (int j = 0; j < 32; ++j) acc[v] = fmaf(value[j], x_at<BF16>(x, at + j), acc[v]);
    }
  }
#pragma unroll
  for (int v = 0; v < V; ++v) {
#pragma unroll
    for (int o = 16; o > 0; o /= 2) acc[v] += __shfl_xor_sync(0xffffffffu, acc[v], o);
  }
  if (lane == 0)
#pragma unroll
    for (int v = 0; v < V; ++v)
      if (v < vectors) y[(long long)v * rows + row] = acc[v];
}

#define DRIFT_KQ_REGISTER(D, name)                                                    \
  DRIFT_REGISTER(kquant_linear_##name##_f32, (kquant_linear_kernel<D, 8, false>))      \
  DRIFT_REGISTER(kquant_linear_##name##_bf16, (kquant_linear_kernel<D, 8, true>))
DRIFT_KQ_REGISTER(DRIFT_Q4_K, q4_k)
DRIFT_KQ_REGISTER(DRIFT_Q6_K, q6_k)

template <int DTYPE, bool BF16>
int launch_kquant(const uint8_t* w, const void* x, float* y, int64_t m, int64_t n, int64_t k,
                  cudaStream_t stream) {
  const unsigned grid = unsigned((n + K_WARPS - 1) / K_WARPS);
  const size_t x_bytes = BF16 ? 2 : 4;
  for (int64_t first = 0; first < m; first += K_MAX_VECTORS) {
    const int count = int(m - first < K_MAX_VECTORS ? m - first : K_MAX_VECTORS);
    const void* xs = static_cast<const uint8_t*>(x) + first * k * x_bytes;
    float* ys = y + first * n;
    if (count == 1)
      DRIFT_CUDA(launch_pdl(kquant_linear_kernel<DTYPE, 1, BF16>, grid, K_WARPS * 32, 0, stream,
                            w, xs, ys, int(n), int(k), count));
    else if (count <= 2)
      DRIFT_CUDA(launch_pdl(kquant_linear_kernel<DTYPE, 2, BF16>, grid, K_WARPS * 32, 0, stream,
                            w, xs, ys, int(n), int(k), count));
    else if (count <= 4)
      DRIFT_CUDA(launch_pdl(kquant_linear_kernel<DTYPE, 4, BF16>, grid, K_WARPS * 32, 0, stream,
                            w, xs, ys, int(n), int(k), count));
    else
      DRIFT_CUDA(launch_pdl(kquant_linear_kernel<DTYPE, 8, BF16>, grid, K_WARPS * 32, 0, stream,
                            w, xs, ys, int(n), int(k), count));
  }
  DRIFT_LAUNCHED("kquant_linear");
  return 0;
}

}  // namespace

// x [m, k] (F32 or BF16) . W^T for W [n, k] of Q4_K or Q6_K.
int kquant_linear(int x_dtype, const void* x, int weight_dtype, const void* weight, float* y,
                  int64_t m, int64_t n, int64_t k, cudaStream_t stream) {
  if (k % 256 != 0) return invalid("%s rows of %lld: not whole super-blocks of 256",
                                   dtype_name(weight_dtype), (long long)k);
  if ((reinterpret_cast<uintptr_t>(weight) & 3) != 0)
    return invalid("linear: the weight does not start on a 4-byte boundary");
  if (m > 0 && n > 0 && (!x || !weight || !y)) return invalid("linear: a null tensor");
  const uint8_t* w = static_cast<const uint8_t*>(weight);
  const bool bf16 = x_dtype == DRIFT_BF16;
  if (weight_dtype == DRIFT_Q4_K)
    return bf16 ? launch_kquant<DRIFT_Q4_K, true>(w, x, y, m, n, k, stream)
                : launch_kquant<DRIFT_Q4_K, false>(w, x, y, m, n, k, stream);
  return bf16 ? launch_kquant<DRIFT_Q6_K, true>(w, x, y, m, n, k, stream)
              : launch_kquant<DRIFT_Q6_K, false>(w, x, y, m, n, k, stream);
}

}  // namespace drift
