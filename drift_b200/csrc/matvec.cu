// Decode-shaped products over quantized weights: y[v, row] = sum_k W[row, k] *
// x[v, k] for up to 8 vectors v (the runner's matvec_float_x_<t>,
// kernels/matvec.hip:418-543, 915-924, and its dispatch
// ops/HipLinear.scala:104-276).
//
// B200 design (not the reference's): x is first prepared per 32-value block
// into exact integer byte planes (quantize_x22, quant.cuh), so a weight block
// meets x in dp4a -- 24 dp4a and a short float epilogue per 32 weights and
// vector, about 2.5 instructions per weight byte for Q4_1 at one vector -- and
// the streaming of weights, not the arithmetic, bounds the kernel at HBM rate.
//
// Work split: a warp takes a group of 8 rows and KS warps of a 256-thread CTA
// split those rows' blocks between them (lane l of k-split w takes blocks
// 32 w + l, 32 (w + KS) + l, ...), so small matrices still fill every SM.
// Each lane loads the aligned words of its block in 8 rows before decoding any
// (40-72 loads in flight per lane), meets them with the x records of up to V
// vectors (kept in registers across the 8 rows), and sums in float. The
// warp's sums reduce by shuffles, the k-splits' through shared memory.
#include <cuda_runtime.h>

#include "common.cuh"
#include "mma_i8.cuh"
#include "x22.cuh"
#include "quant.cuh"
#include "registry.cuh"

namespace drift {

// ---- x preparation ---------------------------------------------------------------
// One warp per 32-value block of x (m rows of k, blocks = m * k / 32), lane j
// holding value j; the record layout is quant.cuh's.
template <bool BF16>
__device__ __forceinline__ void quantize_x22_block(const void* x, uint32_t* records, long long block) {
  const int lane = threadIdx.x % WARP;
  float v;
  if (BF16) {
    const uint16_t bits = reinterpret_cast<const uint16_t*>(x)[block * 32 + lane];
    v = __uint_as_float(uint32_t(bits) << 16);
  } else {
    v = reinterpret_cast<const float*>(x)[block * 32 + lane];
  }
  float amax = fabsf(v);
  bool finite = isfinite(v);
#pragma unroll
  for (int o = 16; o > 0; o /= 2) {
    amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
    finite = __all_sync(0xffffffffu, finite);
  }
  int X = 0;
  float s = 0.0f;
  if (!finite) {
    s = __int_as_float(0x7fc00000);  // a NaN scale: the block's products come out NaN
  } else if (amax > 0.0f) {
    const int e = ilogbf(amax) + 1;  // 2^(e-1) <= amax < 2^e
    s = ldexpf(1.0f, e - X_BITS);
    X = __float2int_rn(ldexpf(v, X_BITS - e));  // exact scaling, then round to nearest even
  }
  uint32_t* record = records + block * X_RECORD_WORDS;
  uint8_t* bytes = reinterpret_cast<uint8_t*>(record);
  bytes[lane] = uint8_t(X & 0xff);
  bytes[32 + lane] = uint8_t((X >> 8) & 0xff);
  bytes[64 + lane] = uint8_t((X >> 16) & 0xff);
  int sum = X;
#pragma unroll
  for (int o = 16; o > 0; o /= 2) sum += __shfl_xor_sync(0xffffffffu, sum, o);
  if (lane == 0) {
    record[24] = __float_as_uint(s);
    record[25] = uint32_t(sum);
  }
}

template <bool BF16>
__global__ void __launch_bounds__(256) quantize_x22_kernel(const void* x, uint32_t* records,
                                                          long long blocks) {
  pdl_trigger();  // the next kernel may launch and wait for this one
  pdl_wait();     // what the kernels before this one wrote is visible
  const long long block = (long long)blockIdx.x * (blockDim.x / WARP) + threadIdx.x / WARP;
  if (block >= blocks) return;
  quantize_x22_block<BF16>(x, records, block);
}

extern "C" __global__ void __launch_bounds__(256)
    quantize_x22_f32(const float* x, uint32_t* records, long long blocks) {
  const long long block = (long long)blockIdx.x * (blockDim.x / WARP) + threadIdx.x / WARP;
  if (block >= blocks) return;
  quantize_x22_block<false>(x, records, block);
}

extern "C" __global__ void __launch_bounds__(256)
    quantize_x22_bf16(const uint16_t* x, uint32_t* records, long long blocks) {
  const long long block = (long long)blockIdx.x * (blockDim.x / WARP) + threadIdx.x / WARP;
  if (block >= blocks) return;
  quantize_x22_block<true>(x, records, block);
}

// The same preparation into the MMA layout (mma_i8.cuh): block `block` of
// vector v (pass v / 8, slot g = v % 8).
template <bool BF16>
__global__ void __launch_bounds__(256) quantize_x22_mma_kernel(const void* x, uint8_t* records,
                                                              int vectors, int blocks) {
  pdl_trigger();  // the product may launch and start on its weights
  pdl_wait();     // x, and the records the previous product reads, are ours now
  const long long index = (long long)blockIdx.x * (blockDim.x / WARP) + threadIdx.x / WARP;
  const int passes = (vectors + 7) / 8;
  if (index >= (long long)passes * 8 * blocks) return;
  const int lane = threadIdx.x % WARP;
  const int block = int(index % blocks);
  const int v = int(index / blocks);  // pass * 8 + slot
  float value = 0.0f;
  if (v < vectors) {
    const long long at = ((long long)v * blocks + block) * 32 + lane;
    value = BF16 ? __uint_as_float(uint32_t(reinterpret_cast<const uint16_t*>(x)[at]) << 16)
                 : reinterpret_cast<const float*>(x)[at];
  }
  x22_record_block(value, records, v, block, blocks);
}

// ---- the product -----------------------------------------------------------------
constexpr int ROWS_PER_GROUP = 8;
constexpr int MAX_V = 2;

// y[v * rows + row] for rows [row0, row0 + 8) of one warp's share of blocks;
// `sums` collects them per (row, vector).
template <typename T, int V, int KS>
__device__ __forceinline__ void matvec_x22_group(const uint8_t* __restrict__ weight,
                                                 const uint32_t* __restrict__ records, int rows,
                                                 int cols, int vectors, int row0, int kw,
                                                 float (&sums)[ROWS_PER_GROUP][V]) {
  const int lane = threadIdx.x % WARP;
  const int blocks = cols / 32;
  const long long row_bytes = (long long)blocks * T::BYTES;
#pragma unroll
  for (int r = 0; r < ROWS_PER_GROUP; ++r)
#pragma unroll
    for (int v = 0; v < V; ++v) sums[r][v] = 0.0f;

  for (int c = kw * WARP + lane; c < blocks; c += WARP * KS) {
    uint32_t w[ROWS_PER_GROUP][T::WORDS];
#pragma unroll
    for (int r = 0; r < ROWS_PER_GROUP; ++r) {
      if (row0 + r < rows) {
        load_block<T>(weight + (long long)(row0 + r) * row_bytes, c, w[r]);
      } else {
#pragma unroll
        for (int i = 0; i < T::WORDS; ++i) w[r][i] = 0;
      }
    }
    uint32_t planes[V][24];
    float s[V];
    int sum_x[V];
#pragma unroll
    for (int v = 0; v < V; ++v) {
      if (v < vectors) {
        const uint4* rec =
            reinterpret_cast<const uint4*>(records + ((long long)v * blocks + c) * X_RECORD_WORDS);
#pragma unroll
        for (int i = 0; i < 6; ++i) {
          const uint4 q = __ldg(rec + i);
          planes[v][4 * i] = q.x;
          planes[v][4 * i + 1] = q.y;
          planes[v][4 * i + 2] = q.z;
          planes[v][4 * i + 3] = q.w;
        }
        const uint4 tail = __ldg(rec + 6);
        s[v] = __uint_as_float(tail.x);
        sum_x[v] = int(tail.y);
      }
    }
#pragma unroll
    for (int r = 0; r < ROWS_PER_GROUP; ++r) {
      const Codes codes = T::decode(w[r], c);
#pragma unroll
      for (int v = 0; v < V; ++v) {
        if (v < vectors) {
          int a0, a1, a2;
          plane_sums<T>(codes, planes[v], a0, a1, a2);
          sums[r][v] += block_dot<T>(codes, a0, a1, a2, s[v], sum_x[v]);
        }
      }
    }
  }
}

// Grid: ceil(rows / (8 * 8 / KS)) CTAs of 256 threads; the x records of
// `vectors` <= V vectors at `records`.
template <typename T, int V, int KS>
__global__ void __launch_bounds__(256) matvec_x22_kernel(const uint8_t* __restrict__ weight,
                                                         const uint32_t* __restrict__ records,
                                                         float* __restrict__ y, int rows, int cols,
                                                         int vectors) {
  pdl_trigger();  // the next kernel may launch and wait for this one
  pdl_wait();     // what the kernels before this one wrote is visible
  constexpr int GROUPS = 8 / KS;  // row groups per CTA
  __shared__ float partial[8][ROWS_PER_GROUP][V];
  const int warp = threadIdx.x / WARP, lane = threadIdx.x % WARP;
  const int kw = warp % KS, group = warp / KS;
  const int row0 = (blockIdx.x * GROUPS + group) * ROWS_PER_GROUP;
  float sums[ROWS_PER_GROUP][V];
  if (row0 < rows) {
    matvec_x22_group<T, V, KS>(weight, records, rows, cols, vectors, row0, kw, sums);
  } else {
#pragma unroll
    for (int r = 0; r < ROWS_PER_GROUP; ++r)
#pragma unroll
      for (int v = 0; v < V; ++v) sums[r][v] = 0.0f;
  }
#pragma unroll
  for (int r = 0; r < ROWS_PER_GROUP; ++r)
#pragma unroll
    for (int v = 0; v < V; ++v) {
      float total = sums[r][v];
#pragma unroll
      for (int o = 16; o > 0; o /= 2) total += __shfl_xor_sync(0xffffffffu, total, o);
      sums[r][v] = total;
    }
  if (lane == 0) {
#pragma unroll
    for (int r = 0; r < ROWS_PER_GROUP; ++r)
#pragma unroll
      for (int v = 0; v < V; ++v) partial[warp][r][v] = sums[r][v];
  }
  __syncthreads();
  // thread (group, r, v): the k-splits' sums in a fixed order
  const int t = threadIdx.x;
  if (t < GROUPS * ROWS_PER_GROUP * V) {
    const int g = t / (ROWS_PER_GROUP * V), r = (t / V) % ROWS_PER_GROUP, v = t % V;
    const int row = (blockIdx.x * GROUPS + g) * ROWS_PER_GROUP + r;
    if (row < rows && v < vectors) {
      float total = 0.0f;
#pragma unroll
      for (int k = 0; k < KS; ++k) total += partial[g * KS + k][r][v];
      y[(long long)v * rows + row] = total;
    }
  }
}

// Grid: ceil(rows / (16 MT (8 / KS))) CTAs of 256 threads. Warp (group, kw)
// takes rows [16 MT group, +16 MT) of the CTA's and the kw-th contiguous
// share of the blocks; up to 8 vectors, x records in the MMA layout.
template <typename T, int MT, int KS>
__global__ void __launch_bounds__(256) matvec_mma_kernel(const uint8_t* __restrict__ weight,
                                                         const uint8_t* __restrict__ records,
                                                         float* __restrict__ y, int rows, int cols,
                                                         int vectors) {
  pdl_trigger();  // the next kernel may launch and wait for this one
  pdl_wait();     // what the kernels before this one wrote is visible
  constexpr int GROUPS = 8 / KS;
  constexpr int ROWS = 16 * MT;
  __shared__ float partial[KS][GROUPS][ROWS][8];
  const int warp = threadIdx.x / WARP, lane = threadIdx.x % WARP;
  const int kw = warp % KS, group = warp / KS;
  const int g = lane / 4, t = lane % 4;
  const int blocks = cols / 32;
  const long long row_bytes = (long long)blocks * T::BYTES;
  const int row0 = (blockIdx.x * GROUPS + group) * ROWS;
  const int first = int((long long)blocks * kw / KS), end = int((long long)blocks * (kw + 1) / KS);

  float acc[MT][4];
#pragma unroll
  for (int i = 0; i < MT; ++i)
#pragma unroll
    for (int j = 0; j < 4; ++j) acc[i][j] = 0.0f;

  const uint8_t* row_ptr[MT][2];
#pragma unroll
  for (int i = 0; i < MT; ++i)
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      int r = row0 + 16 * i + g + 8 * h;
      r = r < rows ? r : rows - 1;
      row_ptr[i][h] = weight + (long long)r * row_bytes;
    }
  const bool have_vector = g < vectors;

  if (row0 < rows) {
    for (int c = first; c < end; ++c) {
      const uint8_t* rec = records + (long long)c * MMA_RECORD_BYTES;
      XFragment xf;
      load_fragment<T>(rec, have_vector, xf);
      const uint2* planes = xf.planes;
      const float2 s = xf.s;
      const int2 sum = xf.sum;
      const float2 fsum = xf.fsum;
#pragma unroll
      for (int i = 0; i < MT; ++i) {
        uint32_t lo0, hi0, lo1, hi1;
        float d0, m0, d1, m1;
        fragment_row<T>(row_ptr[i][0], c, t, lo0, hi0, d0, m0);
        fragment_row<T>(row_ptr[i][1], c, t, lo1, hi1, d1, m1);
        const uint32_t a[4] = {lo0, lo1, hi0, hi1};
        int p0[4], p1[4], p2[4];
        mma_i8_zero<T::SIGNED, false>(p0, a, planes[0].x, planes[0].y);
        mma_i8_zero<T::SIGNED, false>(p1, a, planes[1].x, planes[1].y);
        mma_i8_zero<T::SIGNED, true>(p2, a, planes[2].x, planes[2].y);
        acc[i][0] = fmaf(s.x, mma_block_value<T>(p0[0], p1[0], p2[0], d0, m0, sum.x, fsum.x), acc[i][0]);
        acc[i][1] = fmaf(s.y, mma_block_value<T>(p0[1], p1[1], p2[1], d0, m0, sum.y, fsum.y), acc[i][1]);
        acc[i][2] = fmaf(s.x, mma_block_value<T>(p0[2], p1[2], p2[2], d1, m1, sum.x, fsum.x), acc[i][2]);
        acc[i][3] = fmaf(s.y, mma_block_value<T>(p0[3], p1[3], p2[3], d1, m1, sum.y, fsum.y), acc[i][3]);
      }
    }
  }
#pragma unroll
  for (int i = 0; i < MT; ++i) {
    partial[kw][group][16 * i + g][2 * t] = acc[i][0];
    partial[kw][group][16 * i + g][2 * t + 1] = acc[i][1];
    partial[kw][group][16 * i + g + 8][2 * t] = acc[i][2];
    partial[kw][group][16 * i + g + 8][2 * t + 1] = acc[i][3];
  }
  __syncthreads();
  for (int e = threadIdx.x; e < GROUPS * ROWS * 8; e += blockDim.x) {
    const int gi = e / (ROWS * 8), r = (e / 8) % ROWS, v = e % 8;
    const int row = (blockIdx.x * GROUPS + gi) * ROWS + r;
    if (row < rows && v < vectors) {
      float total = 0.0f;
#pragma unroll
      for (int k = 0; k < KS; ++k) total += partial[k][gi][r][v];
      y[(long long)v * rows + row] = total;
    }
  }
}

// ---- by-name kernels ------------------------------------------------------------------
// Every instantiation, for hosts that launch by name (drift_module_get_function
// with a NULL module): matvec_x22_<type>_v<V>_ks<KS>, 256 threads, grid
// ceil(rows / (64 / KS)), arguments (weight, records, y, rows, cols, vectors).
#define DRIFT_MATVEC_REGISTER(T, name)                                        \
  DRIFT_REGISTER(matvec_x22_##name##_v1_ks1, (matvec_x22_kernel<T, 1, 1>))    \
  DRIFT_REGISTER(matvec_x22_##name##_v1_ks2, (matvec_x22_kernel<T, 1, 2>))    \
  DRIFT_REGISTER(matvec_x22_##name##_v1_ks4, (matvec_x22_kernel<T, 1, 4>))    \
  DRIFT_REGISTER(matvec_x22_##name##_v2_ks1, (matvec_x22_kernel<T, 2, 1>))    \
  DRIFT_REGISTER(matvec_x22_##name##_v2_ks2, (matvec_x22_kernel<T, 2, 2>))    \
  DRIFT_REGISTER(matvec_x22_##name##_v2_ks4, (matvec_x22_kernel<T, 2, 4>))
#define DRIFT_MMA_REGISTER(T, name)                                               \
  DRIFT_REGISTER(matvec_mma_##name##_mt2_ks1, (matvec_mma_kernel<T, 2, 1>))       \
  DRIFT_REGISTER(matvec_mma_##name##_mt2_ks2, (matvec_mma_kernel<T, 2, 2>))       \
  DRIFT_REGISTER(matvec_mma_##name##_mt2_ks4, (matvec_mma_kernel<T, 2, 4>))       \
  DRIFT_REGISTER(matvec_mma_##name##_mt1_ks8, (matvec_mma_kernel<T, 1, 8>))
DRIFT_MMA_REGISTER(Q8_0T, q8_0)
DRIFT_MMA_REGISTER(Q4_0T, q4_0)
DRIFT_MMA_REGISTER(Q4_1T, q4_1)
DRIFT_MATVEC_REGISTER(Q8_0T, q8_0)
DRIFT_MATVEC_REGISTER(Q4_0T, q4_0)
DRIFT_MATVEC_REGISTER(Q4_1T, q4_1)
DRIFT_REGISTER(quantize_x22_f32, quantize_x22_f32)
DRIFT_REGISTER(quantize_x22_bf16, quantize_x22_bf16)

// ---- dispatch ----------------------------------------------------------------------------
struct Workspace {
  void* pointer = nullptr;
  size_t bytes = 0;
};

static Workspace workspaces[64];

int workspace_reserve(size_t bytes, void** pointer) {
  int device = 0;
  DRIFT_CUDA(cudaGetDevice(&device));
  if (device < 0 || device >= 64) return invalid("device %d out of range", device);
  Workspace& w = workspaces[device];
  if (w.bytes < bytes) {
    if (w.pointer) DRIFT_CUDA(cudaFree(w.pointer));
    w.pointer = nullptr;
    w.bytes = 0;
    const size_t rounded = (bytes + (1u << 20) - 1) & ~size_t((1u << 20) - 1);
    DRIFT_CUDA(cudaMalloc(&w.pointer, rounded));
    w.bytes = rounded;
  }
  if (pointer) *pointer = w.pointer;
  return 0;
}

size_t linear_workspace_bytes(int64_t m, int64_t k) {
  return size_t(m) * size_t(k / 32) * X_RECORD_BYTES;
}

size_t mma_workspace_bytes(int64_t m, int64_t k) {
  return size_t((m + 7) / 8) * size_t(k / 32) * MMA_RECORD_BYTES;
}

int prepare_x_mma(int x_dtype, const void* x, int64_t m, int64_t k, uint8_t* records,
                  cudaStream_t stream) {
  const long long blocks = k / 32;
  const long long warps = (m + 7) / 8 * 8 * blocks;
  if (warps == 0) return 0;
  const unsigned grid = unsigned((warps + 7) / 8);
  if (x_dtype == DRIFT_BF16)
    DRIFT_CUDA(launch_pdl(quantize_x22_mma_kernel<true>, grid, 256, 0, stream, x, records, int(m),
                          int(blocks)));
  else
    DRIFT_CUDA(launch_pdl(quantize_x22_mma_kernel<false>, grid, 256, 0, stream, x, records, int(m),
                          int(blocks)));
  return 0;
}

int prepare_x(int x_dtype, const void* x, int64_t m, int64_t k, uint32_t* records,
              cudaStream_t stream) {
  const long long blocks = m * (k / 32);
  if (blocks == 0) return 0;
  const unsigned grid = unsigned((blocks + 7) / 8);
  if (x_dtype == DRIFT_BF16)
    DRIFT_CUDA(launch_pdl(quantize_x22_kernel<true>, grid, 256, 0, stream, x, records, blocks));
  else
    DRIFT_CUDA(launch_pdl(quantize_x22_kernel<false>, grid, 256, 0, stream, x, records, blocks));
  DRIFT_LAUNCHED("quantize_x22");
  return 0;
}

template <typename T, int V>
static int launch_matvec_v(const uint8_t* weight, const uint32_t* records, float* y, int rows,
                           int cols, int vectors, cudaStream_t stream) {
  const int blocks = cols / 32;
  // k-splits: one block per lane at most in the first pass when the row is
  // short; up to 4 warps share a row group's blocks
  const int ks = blocks >= 128 ? 4 : (blocks >= 64 ? 2 : 1);
  const int rows_per_cta = ROWS_PER_GROUP * 8 / ks;
  const unsigned grid = unsigned((rows + rows_per_cta - 1) / rows_per_cta);
  if (ks == 4)
    DRIFT_CUDA(launch_pdl(matvec_x22_kernel<T, V, 4>, grid, 256, 0, stream, weight, records, y, rows,
                          cols, vectors));
  else if (ks == 2)
    DRIFT_CUDA(launch_pdl(matvec_x22_kernel<T, V, 2>, grid, 256, 0, stream, weight, records, y, rows,
                          cols, vectors));
  else
    DRIFT_CUDA(launch_pdl(matvec_x22_kernel<T, V, 1>, grid, 256, 0, stream, weight, records, y, rows,
                          cols, vectors));
  DRIFT_LAUNCHED("matvec_x22");
  return 0;
}

template <typename T>
static int launch_mma(const uint8_t* weight, const uint8_t* records, float* y, int rows, int cols,
                      int vectors, cudaStream_t stream) {
  const int blocks = cols / 32;
  // enough warps for every SM: split the blocks between more warps when the
  // matrix has few rows
  const long long groups32 = (rows + 31) / 32;
  int ks = 1;
  while (ks < 4 && groups32 * ks < 8LL * sm_count() && blocks / (ks * 2) >= 8) ks *= 2;
  if (rows <= 2048 && blocks >= 64) {
    const unsigned grid = unsigned((rows + 16 - 1) / 16);  // MT 1, 8 k-splits, 16 rows per CTA
    DRIFT_CUDA(launch_pdl(matvec_mma_kernel<T, 1, 8>, grid, 256, 0, stream, weight, records, y, rows,
                          cols, vectors));
  } else if (ks == 4) {
    const unsigned grid = unsigned((rows + 64 - 1) / 64);
    DRIFT_CUDA(launch_pdl(matvec_mma_kernel<T, 2, 4>, grid, 256, 0, stream, weight, records, y, rows,
                          cols, vectors));
  } else if (ks == 2) {
    const unsigned grid = unsigned((rows + 128 - 1) / 128);
    DRIFT_CUDA(launch_pdl(matvec_mma_kernel<T, 2, 2>, grid, 256, 0, stream, weight, records, y, rows,
                          cols, vectors));
  } else {
    const unsigned grid = unsigned((rows + 256 - 1) / 256);
    DRIFT_CUDA(launch_pdl(matvec_mma_kernel<T, 2, 1>, grid, 256, 0, stream, weight, records, y, rows,
                          cols, vectors));
  }
  DRIFT_LAUNCHED("matvec_mma");
  return 0;
}

// Passes of up to 8 vectors, each one launch of a single kernel whose block
// order depends on the matrix only: a row sums to the same bits alone or
// beside 7 others (the runner's guarantee that a verification's tokens get a
// decode step's logits, ops/HipLinear.scala:197-201).
template <typename T>
static int launch_matvec(const uint8_t* weight, const uint8_t* records, float* y, int rows,
                         int cols, int vectors, cudaStream_t stream) {
  const long long blocks = cols / 32;
  for (int first = 0; first < vectors; first += 8) {
    const int count = vectors - first < 8 ? vectors - first : 8;
    DRIFT_TRY(launch_mma<T>(weight, records + (first / 8) * blocks * MMA_RECORD_BYTES,
                            y + (long long)first * rows, rows, cols, count, stream));
  }
  return 0;
}

bool ring_supports(int weight_dtype, const void* weight, int64_t k);
int matvec_ring(int weight_dtype, const void* weight, const uint8_t* records, float* y,
                int64_t rows, int64_t cols, int64_t vectors, cudaStream_t stream);

// The quantized product of prepared x; `vectors` rows of x, y [vectors, rows].
// Weights whose rows are whole 16-byte units stream through shared memory
// (matvec_ring.cu); the rest are read straight from global memory.
int matvec_prepared(int weight_dtype, const void* weight, const uint8_t* records, float* y,
                    int64_t rows, int64_t cols, int64_t vectors, cudaStream_t stream) {
  if (ring_supports(weight_dtype, weight, cols)) {
    const int64_t blocks = cols / 32;
    for (int64_t first = 0; first < vectors; first += 8) {
      const int64_t count = vectors - first < 8 ? vectors - first : 8;
      DRIFT_TRY(matvec_ring(weight_dtype, weight, records + (first / 8) * blocks * MMA_RECORD_BYTES,
                            y + first * rows, rows, cols, count, stream));
    }
    return 0;
  }
  const uint8_t* w = static_cast<const uint8_t*>(weight);
  switch (weight_dtype) {
    case DRIFT_Q8_0: return launch_matvec<Q8_0T>(w, records, y, int(rows), int(cols), int(vectors), stream);
    case DRIFT_Q4_0: return launch_matvec<Q4_0T>(w, records, y, int(rows), int(cols), int(vectors), stream);
    case DRIFT_Q4_1: return launch_matvec<Q4_1T>(w, records, y, int(rows), int(cols), int(vectors), stream);
    default: return invalid("no kernels for %s weights yet", dtype_name(weight_dtype));
  }
}

}  // namespace drift
