// Batch-shaped products on the 5th-generation tensor cores: out[m, n] =
// x[m, k] . W[n, k]^T for m >= 32 (the runner's GEMM path: W dequantized to
// F16 and multiplied by hipBLAS with F32 compute, ops/HipLinear.scala:
// 389-469, kernels/matvec.hip:801-810), fused into one persistent kernel.
//
// One CTA per SM, 10 warps, a tile of 128 weight rows x 64 vectors at a time:
//  - warp 8 (TMA): streams each 256-column chunk of the tile's raw GGML blocks
//    (a 2-D tensor copy, 128 rows) and the matching four 64-column tiles of x
//    (F16, 128-byte swizzled, the UMMA canonical K-major layout) into a
//    3-stage shared-memory ring;
//  - warps 0-7 (dequant, two warpgroups taking alternate 64-column steps):
//    each thread turns its row's two blocks into 64 F16 weights -- d * q + m
//    rounded once, as the reference's dequantize_<t> does -- and stores them
//    straight into tensor memory (tcgen05.st), which is where the MMA reads
//    A from: the dequantized tile never touches shared memory;
//  - warp 9 (MMA): one thread issues tcgen05.mma kind::f16 with A in TMEM, B
//    in shared memory and the F32 accumulator in TMEM (128 x 64), committing
//    to mbarriers that free the A buffers and ring stages.
// After the last step of a tile, the dequant warps read the accumulator back
// (tcgen05.ld) and store F32 out. Every wait is bounded (tc_common.cuh).
//
// The weights' values within a 32-block come out of the unpacking in a
// permuted order (pairs of nibbles that one LOP3 makes into an F16x2), so x
// is staged in the same permuted order by tc_prepare_x; a product's sum is
// the same over any order of its terms.
#include <cuda.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include "common.cuh"
#include "quant.cuh"
#include "registry.cuh"
#include "tc_common.cuh"
#include "tma_host.cuh"

namespace drift {

int* device_error_word();
int workspace_reserve(size_t bytes, void** pointer);

namespace {

constexpr int TILE_ROWS = 128;
constexpr int TILE_VECTORS = 64;
constexpr int CHUNK = 256;  // columns per ring stage
constexpr int STEP = 64;    // columns per MMA step (one 128-byte swizzle atom of F16)
constexpr int STAGES = 3;
constexpr int THREADS = 320;
constexpr int B_STAGE_BYTES = 4 * TILE_VECTORS * 128;  // four [64 vectors x 64 F16] tiles

__device__ __forceinline__ uint32_t h2u(__half2 h) { return *reinterpret_cast<uint32_t*>(&h); }
__device__ __forceinline__ __half2 u2h(uint32_t u) { return *reinterpret_cast<__half2*>(&u); }

// ---- unpacking, per storage type -------------------------------------------------------
// step(): the 64 weights of one row's 64-column step (two blocks) as 32 F16x2
// words, from that row's raw words in the ring. perm(p): which value of a
// 32-block sits at position p of the unpacked order.
template <typename T>
struct Unpack;

// Q4_1 and Q4_0: a word of nibble bytes b0..b3 (values 4i..4i+3 low,
// 16+4i.. high) gives four F16x2 pairs, each from one LOP3 with the magic
// exponent of 1024: (v0, v2), (v1, v3) from the low nibbles (after >> 8 for
// the second), (v16, v18), (v17, v19) from the high nibbles in place, which
// read as 1024 + 16 q.
__device__ __forceinline__ void nibble_pairs(uint32_t w, __half2& lo0, __half2& lo1, __half2& hi0,
                                             __half2& hi1) {
  const uint32_t t = w >> 8;
  const __half2 k1024 = u2h(0x64006400u);
  lo0 = __hsub2(u2h((w & 0x000F000Fu) | 0x64006400u), k1024);
  lo1 = __hsub2(u2h((t & 0x000F000Fu) | 0x64006400u), k1024);
  const __half2 sixteenth = u2h(0x2C002C00u);  // 1/16
  const __half2 minus64 = u2h(0xD400D400u);    // -64
  hi0 = __hfma2(u2h((w & 0x00F000F0u) | 0x64006400u), sixteenth, minus64);
  hi1 = __hfma2(u2h((t & 0x00F000F0u) | 0x64006400u), sixteenth, minus64);
}

__host__ __device__ constexpr int perm_q4(int p) {
  // p = 8 i + 2 t + h
  return ((p % 8) / 2 >= 2 ? 16 : 0) + 4 * (p / 8) + ((p % 8) / 2 & 1) + 2 * (p % 2);
}

template <>
struct Unpack<Q4_1T> {
  static constexpr int RAW_WORDS = 40;  // 8 blocks of 20 bytes
  __device__ static void block(const uint32_t* w, uint32_t* out) {
    const __half2 d = u2h(__byte_perm(w[0], 0, 0x1010));
    const __half2 m = u2h(__byte_perm(w[0], 0, 0x3232));
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      __half2 lo0, lo1, hi0, hi1;
      nibble_pairs(w[1 + i], lo0, lo1, hi0, hi1);
      out[4 * i + 0] = h2u(__hfma2(lo0, d, m));
      out[4 * i + 1] = h2u(__hfma2(lo1, d, m));
      out[4 * i + 2] = h2u(__hfma2(hi0, d, m));
      out[4 * i + 3] = h2u(__hfma2(hi1, d, m));
    }
  }
  __device__ static void step(const uint32_t* row, int sub, uint32_t (&out)[32]) {
    const uint2* p = reinterpret_cast<const uint2*>(row + 10 * sub);  // 8-byte aligned
    uint32_t w[10];
#pragma unroll
    for (int i = 0; i < 5; ++i) {
      const uint2 v = p[i];
      w[2 * i] = v.x;
      w[2 * i + 1] = v.y;
    }
    block(w, out);
    block(w + 5, out + 16);
  }
  __host__ __device__ static constexpr int perm(int p) { return perm_q4(p); }
};

template <>
struct Unpack<Q4_0T> {
  static constexpr int RAW_WORDS = 36;  // 8 blocks of 18 bytes
  // d: the block's f16 scale bits; q: its four nibble words
  __device__ static void block(uint32_t d_bits, const uint32_t* q, uint32_t* out) {
    const __half2 d = u2h(__byte_perm(d_bits, 0, 0x1010));
    const __half2 eight = u2h(0x48004800u);  // 8
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      __half2 lo0, lo1, hi0, hi1;
      nibble_pairs(q[i], lo0, lo1, hi0, hi1);
      out[4 * i + 0] = h2u(__hmul2(__hsub2(lo0, eight), d));
      out[4 * i + 1] = h2u(__hmul2(__hsub2(lo1, eight), d));
      out[4 * i + 2] = h2u(__hmul2(__hsub2(hi0, eight), d));
      out[4 * i + 3] = h2u(__hmul2(__hsub2(hi1, eight), d));
    }
  }
  __device__ static void step(const uint32_t* row, int sub, uint32_t (&out)[32]) {
    const uint32_t* p = row + 9 * sub;  // 36 bytes: block 0 at byte 0, block 1 at byte 18
    uint32_t w[9];
#pragma unroll
    for (int i = 0; i < 9; ++i) w[i] = p[i];
    uint32_t q[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) q[i] = __funnelshift_r(w[i], w[i + 1], 16);
    block(w[0], q, out);
    block(w[4] >> 16, w + 5, out + 16);
  }
  __host__ __device__ static constexpr int perm(int p) { return perm_q4(p); }
};

template <>
struct Unpack<Q8_0T> {
  static constexpr int RAW_WORDS = 68;  // 8 blocks of 34 bytes
  // Signed codes c0..c3 of a word become (c0, c2), (c1, c3): bytes biased by
  // 128 under the magic exponent of 1024, less 1152.
  __device__ static void block(uint32_t d_bits, const uint32_t* q, uint32_t* out) {
    const __half2 d = u2h(__byte_perm(d_bits, 0, 0x1010));
    const __half2 k1152 = u2h(0x64806480u);
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const uint32_t u = q[i] ^ 0x80808080u;
      const __half2 p0 = __hsub2(u2h(__byte_perm(u, 0x64646464u, 0x4240)), k1152);
      const __half2 p1 = __hsub2(u2h(__byte_perm(u, 0x64646464u, 0x4341)), k1152);
      out[2 * i] = h2u(__hmul2(p0, d));
      out[2 * i + 1] = h2u(__hmul2(p1, d));
    }
  }
  __device__ static void step(const uint32_t* row, int sub, uint32_t (&out)[32]) {
    const uint32_t* p = row + 17 * sub;  // 68 bytes: block 0 at byte 0, block 1 at byte 34
    uint32_t w[17];
#pragma unroll
    for (int i = 0; i < 17; ++i) w[i] = p[i];
    uint32_t q[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) q[i] = __funnelshift_r(w[i], w[i + 1], 16);
    block(w[0], q, out);
    block(w[8] >> 16, w + 9, out + 16);
  }
  // p = 4 i + 2 t + h -> 4 i + t + 2 h
  __host__ __device__ static constexpr int perm(int p) {
    return 4 * (p / 4) + ((p % 4) / 2) + 2 * (p % 2);
  }
};

// ---- x, staged for the tensor cores -------------------------------------------------------
// out[v][k] (F16, [vectors_padded][k]): x[v][32 b + perm(p)] at k = 32 b + p,
// zero for v >= vectors. x is F32 or BF16 [vectors][k].
template <typename T, bool BF16>
__global__ void tc_prepare_x_kernel(const void* __restrict__ x, __half* __restrict__ out,
                                    int vectors, int padded, int cols) {
  const long long total = (long long)padded * cols;
  for (long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x; i < total;
       i += (long long)gridDim.x * blockDim.x) {
    const int v = int(i / cols), k = int(i % cols);
    float value = 0.0f;
    if (v < vectors) {
      const long long source = (long long)v * cols + (k & ~31) + Unpack<T>::perm(k & 31);
      if (BF16)
        value = __uint_as_float(uint32_t(reinterpret_cast<const uint16_t*>(x)[source]) << 16);
      else
        value = reinterpret_cast<const float*>(x)[source];
    }
    out[i] = __float2half_rn(value);
  }
}

// ---- the product ------------------------------------------------------------------------------
template <typename T>
struct TcLayout {
  static constexpr int RAW_BYTES = TILE_ROWS * Unpack<T>::RAW_WORDS * 4;
  static constexpr int RAW_PADDED = (RAW_BYTES + 1023) / 1024 * 1024;
  static constexpr int STAGE_BYTES = B_STAGE_BYTES + RAW_PADDED;
  static constexpr int BARRIER_OFFSET = STAGES * STAGE_BYTES;
  // + full[S], empty[S], a_full[2], a_empty[2], acc_full, acc_empty, tmem slot, abort
  static constexpr int SMEM_BYTES = BARRIER_OFFSET + 256 + 1024;  // + alignment slack
};

template <typename T>
__global__ void __launch_bounds__(THREADS, 1)
    linear_tc_kernel(const __grid_constant__ CUtensorMap wmap,
                     const __grid_constant__ CUtensorMap xmap, float* __restrict__ y, int rows,
                     int cols, int vectors, int row_tiles, int tiles, int* error) {
  using L = TcLayout<T>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~uintptr_t(1023));
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + L::BARRIER_OFFSET);
  uint64_t* full = bars;
  uint64_t* empty = bars + STAGES;
  uint64_t* a_full = bars + 2 * STAGES;
  uint64_t* a_empty = a_full + 2;
  uint64_t* acc_full = a_empty + 2;
  uint64_t* acc_empty = acc_full + 1;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(acc_empty + 1);
  volatile int* abort = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  const int chunks = (cols + CHUNK - 1) / CHUNK;

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      tc::mbar_init(&full[s], 1);
      tc::mbar_init(&empty[s], 9);  // 8 dequant warps + the MMA's commit
    }
    for (int b = 0; b < 2; ++b) {
      tc::mbar_init(&a_full[b], 4);  // the four warps of a warpgroup
      tc::mbar_init(&a_empty[b], 1);
    }
    tc::mbar_init(acc_full, 1);
    tc::mbar_init(acc_empty, 8);
    *abort = 0;
    tc::fence_barrier_init();
  }
  if (warp == 8 && lane == 0) {
    tc::prefetch_tensor_map(&wmap);
    tc::prefetch_tensor_map(&xmap);
  }
  if (warp == 0) tc::tmem_alloc(tmem_slot, 128);
  __syncthreads();
  tc::fence_after_sync();
  const uint32_t tmem = *tmem_slot;  // columns 0..63: accumulator; 64..127: two A buffers

  if (warp == 8) {
    // ---- TMA producer ----
    if (lane == 0) {
      int gc = 0;
      bool ok = true;
      for (int tile = blockIdx.x; ok && tile < tiles; tile += gridDim.x) {
        const int rt = tile % row_tiles, pass = tile / row_tiles;
        for (int c = 0; c < chunks; ++c, ++gc) {
          const int s = gc % STAGES;
          if (gc >= STAGES && !(ok = tc::mbar_wait(&empty[s], ((gc / STAGES) - 1) & 1, abort, error)))
            break;
          uint8_t* stage = smem + s * L::STAGE_BYTES;
          tc::mbar_expect_tx(&full[s], B_STAGE_BYTES + L::RAW_BYTES);
          tc::tma_load_2d(stage + B_STAGE_BYTES, &wmap, &full[s], c * Unpack<T>::RAW_WORDS,
                          rt * TILE_ROWS);
#pragma unroll
          for (int sub = 0; sub < 4; ++sub)
            tc::tma_load_2d(stage + sub * TILE_VECTORS * 128, &xmap, &full[s],
                            (c * 4 + sub) * STEP, pass * TILE_VECTORS);
        }
      }
      if (!ok) {
        // let the copies already issued land before the CTA leaves
        for (int j = gc - STAGES < 0 ? 0 : gc - STAGES; j < gc; ++j) {
          volatile int never = 0;
          tc::mbar_wait(&full[j % STAGES], (j / STAGES) & 1, &never, nullptr);
        }
      }
    }
  } else if (warp == 9) {
    // ---- MMA issuer ----
    if (lane == 0) {
      const uint32_t idesc = tc::instr_desc_f16(TILE_ROWS, TILE_VECTORS);
      int gs = 0, gc = 0, local = 0;
      bool ok = true;
      for (int tile = blockIdx.x; ok && tile < tiles; tile += gridDim.x, ++local) {
        if (local > 0 && !(ok = tc::mbar_wait(acc_empty, (local - 1) & 1, abort, error))) break;
        for (int c = 0; ok && c < chunks; ++c, ++gc) {
          const int s = gc % STAGES;
          if (!(ok = tc::mbar_wait(&full[s], (gc / STAGES) & 1, abort, error))) break;
          const uint32_t b_base = tc::smem_u32(smem + s * L::STAGE_BYTES);
          for (int sub = 0; sub < 4; ++sub, ++gs) {
            const int buf = gs & 1;
            if (!(ok = tc::mbar_wait(&a_full[buf], (gs >> 1) & 1, abort, error))) break;
            tc::fence_after_sync();
#pragma unroll
            for (int j = 0; j < 4; ++j) {
              const uint64_t b_desc =
                  tc::smem_desc_sw128(b_base + sub * TILE_VECTORS * 128 + j * 32);
              tc::mma_f16_ts(tmem, tmem + 64 + buf * 32 + j * 8, b_desc, idesc,
                             (c | sub | j) != 0);
            }
            tc::mma_commit(&a_empty[buf]);
            if (sub == 3) tc::mma_commit(&empty[s]);
          }
        }
        if (ok) tc::mma_commit(acc_full);
      }
    }
  } else {
    // ---- dequant warpgroups, then the epilogue ----
    const int group = warp / 4, quarter = warp % 4;
    const int row_in_tile = quarter * 32 + lane;
    const uint32_t lane_base = uint32_t(quarter * 32) << 16;
    int gs = 0, gc = 0, local = 0;
    bool ok = true;
    for (int tile = blockIdx.x; ok && tile < tiles; tile += gridDim.x, ++local) {
      const int rt = tile % row_tiles, pass = tile / row_tiles;
      for (int c = 0; ok && c < chunks; ++c, ++gc) {
        const int s = gc % STAGES;
        if (!(ok = tc::mbar_wait_warp(&full[s], (gc / STAGES) & 1, abort, error))) break;
        const uint32_t* raw_row = reinterpret_cast<const uint32_t*>(
            smem + s * L::STAGE_BYTES + B_STAGE_BYTES + row_in_tile * Unpack<T>::RAW_WORDS * 4);
        for (int sub = 0; sub < 4; ++sub, ++gs) {
          if ((gs & 1) != group) continue;
          if (gs >= 2 && !(ok = tc::mbar_wait_warp(&a_empty[group], ((gs >> 1) - 1) & 1, abort, error)))
            break;
          tc::fence_after_sync();
          uint32_t a[32];
          Unpack<T>::step(raw_row, sub, a);
          tc::tmem_store_32(tmem + lane_base + 64 + group * 32, a);
          tc::tmem_store_wait();
          tc::fence_before_sync();
          __syncwarp();
          if (lane == 0) tc::mbar_arrive(&a_full[group]);
        }
        __syncwarp();
        if (ok && lane == 0) tc::mbar_arrive(&empty[s]);
      }
      if (!ok) break;
      // epilogue: this warp's 32 rows x 32 of the tile's 64 vectors
      if (!(ok = tc::mbar_wait_warp(acc_full, local & 1, abort, error))) break;
      tc::fence_after_sync();
      uint32_t acc[32];
      tc::tmem_load_32(tmem + lane_base + group * 32, acc);
      const int row = rt * TILE_ROWS + row_in_tile;
      if (row < rows) {
#pragma unroll
        for (int i = 0; i < 32; ++i) {
          const int v = pass * TILE_VECTORS + group * 32 + i;
          if (v < vectors) y[(long long)v * rows + row] = __uint_as_float(acc[i]);
        }
      }
      tc::fence_before_sync();
      __syncwarp();
      if (lane == 0) tc::mbar_arrive(acc_empty);
    }
  }
  __syncthreads();
  if (warp == 0) {
    tc::fence_after_sync();
    tc::tmem_dealloc(tmem, 128);
  }
}

DRIFT_REGISTER(linear_tc_q8_0, linear_tc_kernel<Q8_0T>)
DRIFT_REGISTER(linear_tc_q4_0, linear_tc_kernel<Q4_0T>)
DRIFT_REGISTER(linear_tc_q4_1, linear_tc_kernel<Q4_1T>)

// ---- host ---------------------------------------------------------------------------------------
template <typename T>
static int launch_tc(int x_dtype, const void* x, const void* weight, float* y, int64_t m,
                     int64_t n, int64_t k, cudaStream_t stream) {
  using L = TcLayout<T>;
  const int64_t padded = (m + TILE_VECTORS - 1) / TILE_VECTORS * TILE_VECTORS;
  void* ws = nullptr;
  DRIFT_TRY(workspace_reserve(size_t(padded * k * 2), &ws));
  __half* xh = static_cast<__half*>(ws);
  {
    const long long total = padded * k;
    long long blocks = (total + 255) / 256;
    if (blocks > (long long)sm_count() * 32) blocks = (long long)sm_count() * 32;
    if (x_dtype == DRIFT_BF16)
      tc_prepare_x_kernel<T, true><<<unsigned(blocks), 256, 0, stream>>>(x, xh, int(m),
                                                                           int(padded), int(k));
    else
      tc_prepare_x_kernel<T, false><<<unsigned(blocks), 256, 0, stream>>>(x, xh, int(m),
                                                                            int(padded), int(k));
    DRIFT_LAUNCHED("tc_prepare_x");
  }
  const int64_t row_bytes = k / 32 * T::BYTES;
  CUtensorMap wmap, xmap;
  DRIFT_TRY(encode_word_rows(&wmap, weight, row_bytes / 4, n, Unpack<T>::RAW_WORDS, TILE_ROWS));
  DRIFT_TRY(encode_f16_sw128(&xmap, xh, k, padded, TILE_VECTORS));
  static bool configured[3] = {false, false, false};
  const int which = T::DTYPE == DRIFT_Q8_0 ? 0 : (T::DTYPE == DRIFT_Q4_0 ? 1 : 2);
  if (!configured[which]) {
    DRIFT_CUDA(cudaFuncSetAttribute(linear_tc_kernel<T>,
                                    cudaFuncAttributeMaxDynamicSharedMemorySize, L::SMEM_BYTES));
    configured[which] = true;
  }
  const int row_tiles = int((n + TILE_ROWS - 1) / TILE_ROWS);
  const int tiles = row_tiles * int(padded / TILE_VECTORS);
  const int grid = tiles < sm_count() ? tiles : sm_count();
  linear_tc_kernel<T><<<grid, THREADS, L::SMEM_BYTES, stream>>>(
      wmap, xmap, y, int(n), int(k), int(m), row_tiles, tiles, device_error_word());
  DRIFT_LAUNCHED("linear_tc");
  return 0;
}

}  // namespace

// Whether the tensor-core path takes a product: rows in whole 16-byte units
// and a 16-byte aligned weight (what the tensor copies need).
bool tc_supports(int weight_dtype, const void* weight, int64_t k) {
  if (weight_dtype != DRIFT_Q8_0 && weight_dtype != DRIFT_Q4_0 && weight_dtype != DRIFT_Q4_1)
    return false;
  const int64_t row = byte_size(weight_dtype, k);
  return row > 0 && row % 16 == 0 && (reinterpret_cast<uintptr_t>(weight) & 15) == 0 &&
         tensor_maps_available();
}

int linear_tc(int x_dtype, const void* x, int weight_dtype, const void* weight, float* y,
              int64_t m, int64_t n, int64_t k, cudaStream_t stream) {
  switch (weight_dtype) {
    case DRIFT_Q8_0: return launch_tc<Q8_0T>(x_dtype, x, weight, y, m, n, k, stream);
    case DRIFT_Q4_0: return launch_tc<Q4_0T>(x_dtype, x, weight, y, m, n, k, stream);
    default: return launch_tc<Q4_1T>(x_dtype, x, weight, y, m, n, k, stream);
  }
}

}  // namespace drift
