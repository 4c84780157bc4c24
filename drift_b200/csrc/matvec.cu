// Decode-shaped products over quantized weights: y[v, row] = sum_k W[row, k] *
// x[v, k] for up to 8 vectors v at a pass (the runner's matvec_float_x_<t>,
// kernels/matvec.hip:418-543, 915-924, and its dispatch
// ops/HipLinear.scala:104-276).
//
// B200 design (not the reference's): x is first prepared per 32-value block
// into exact integer byte planes (quantize_x22_mma, quant.cuh / mma_i8.cuh),
// so a weight block meets x in integer dot products -- dp4a for one or two
// vectors, mma.sync m16n8k32 for more -- and a short float epilogue per 32
// weights and vector. Weights whose rows are whole 16-byte units stream
// through shared memory (matvec_ring.cu); this file holds the preparation,
// the same MMA arithmetic reading weights straight from global memory for
// the other rows, and the dispatch between them.
#include <cuda_runtime.h>

#include "common.cuh"
#include "mma_i8.cuh"
#include "x22.cuh"
#include "quant.cuh"
#include "registry.cuh"

namespace drift {

// ---- x preparation ---------------------------------------------------------------
// One warp per 32-value block of each vector (lane j holding value j), into
// the MMA record layout (mma_i8.cuh): block `block` of vector v (pass v / 8,
// slot g = v % 8); vectors past m in the last pass get zero slots.
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
// with a NULL module): matvec_mma_<type>_mt<MT>_ks<KS>, 256 threads, grid
// ceil(rows / (16 MT (8 / KS))), arguments (weight, records, y, rows, cols,
// vectors); quantize_x22_mma_<x type>, a warp per (vector, block), arguments
// (x, records, vectors, blocks).
#define DRIFT_MMA_REGISTER(T, name)                                               \
  DRIFT_REGISTER(matvec_mma_##name##_mt2_ks1, (matvec_mma_kernel<T, 2, 1>))       \
  DRIFT_REGISTER(matvec_mma_##name##_mt2_ks2, (matvec_mma_kernel<T, 2, 2>))       \
  DRIFT_REGISTER(matvec_mma_##name##_mt2_ks4, (matvec_mma_kernel<T, 2, 4>))       \
  DRIFT_REGISTER(matvec_mma_##name##_mt1_ks8, (matvec_mma_kernel<T, 1, 8>))
DRIFT_MMA_REGISTER(Q8_0T, q8_0)
DRIFT_MMA_REGISTER(Q4_0T, q4_0)
DRIFT_MMA_REGISTER(Q4_1T, q4_1)
DRIFT_REGISTER(quantize_x22_mma_f32, quantize_x22_mma_kernel<false>)
DRIFT_REGISTER(quantize_x22_mma_bf16, quantize_x22_mma_kernel<true>)

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
    // up to 16 vectors a launch (two passes' records met by each weight fragment)
    const int64_t blocks = cols / 32;
    for (int64_t first = 0; first < vectors; first += 16) {
      const int64_t count = vectors - first < 16 ? vectors - first : 16;
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
