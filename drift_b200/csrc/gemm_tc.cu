// Batch-shaped products on the 5th-generation tensor cores: out[m, n] =
// x[m, k] . W[n, k]^T for m >= 32 (the runner's GEMM path: W dequantized to
// F16 and multiplied by hipBLAS with F32 compute, ops/HipLinear.scala:
// 389-469, kernels/matvec.hip:801-810), fused into one persistent kernel.
//
// One CTA per SM, 19 warps, units of 128 weight rows x 64 vectors (x a
// K-range of the columns, when a matrix has too few rows to fill the SMs):
//  - warp 16 (weights): streams each 256-column chunk of the unit's raw GGML
//    blocks (a 2-D tensor copy, 128 rows) into a 5-stage ring (3 for Q8_0),
//    freed as soon as the dequant warps hold a stage in registers;
//  - warp 18 (x): one bulk copy per chunk of the four 64-column x tiles (F16,
//    pre-swizzled by tc_prepare_x into the UMMA canonical K-major layout)
//    into a 3-stage ring, freed by the MMA's commit;
//  - warps 0-15 (dequant, four warpgroups, warpgroup g taking 64-column step g
//    of every chunk): each thread turns its row's two blocks into 64 F16
//    weights -- d * q + m rounded once, as the reference's dequantize_<t>
//    does -- and stores them straight into tensor memory (tcgen05.st), into
//    one of three sets of A buffers, which is where the MMA reads A from: the
//    dequantized tile never touches shared memory;
//  - warp 17 (MMA): the whole warp waits, one elected lane issues the chunk's
//    16 tcgen05.mma kind::f16 back to back (A in TMEM, B in shared memory,
//    the F32 accumulator in TMEM: 128 x 64, two of them so a unit's epilogue
//    overlaps the next unit's products) and commits once per ring.
// One chunk into the next unit, the dequant warps read the last unit's
// accumulator back (tcgen05.ld) and store F32 out -- or, for a unit that
// holds a K-range, store it as a partial sum; the last of a tile's K-ranges
// to finish adds the partials in K order, so the result does not depend on
// which CTA finishes first. Every wait is bounded (tc_common.cuh). The kernel
// is launched as a programmatic dependent of the x preparation: it sets up
// and starts the weight copies while that kernel finishes.
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

namespace {

constexpr int TILE_ROWS = 128;
constexpr int TILE_VECTORS = 64;
constexpr int CHUNK = 256;  // columns per ring stage
constexpr int STEP = 64;    // columns per MMA step (one 128-byte swizzle atom of F16)

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
  // a chunk's row as copied: 16 bytes past the chunk, so rows sit 44 words
  // apart and 16-byte reads of one column of 8 rows hit 8 distinct bank groups
  static constexpr int PITCH_WORDS = 44;
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
  // step SUB: bytes [40 SUB, 40 SUB + 40) of the row's chunk
  template <int SUB>
  __device__ static void step(const uint8_t* row, uint32_t (&out)[32]) {
    constexpr int A = 40 * SUB, C0 = A & ~15, C1 = (A + 40 + 15) & ~15;
    uint32_t w[(C1 - C0) / 4];
    lds_span<C0, C1>(row, w);
    block(w + (A - C0) / 4, out);
    block(w + (A - C0) / 4 + 5, out + 16);
  }
  __host__ __device__ static constexpr int perm(int p) { return perm_q4(p); }
};

template <>
struct Unpack<Q4_0T> {
  static constexpr int RAW_WORDS = 36;  // 8 blocks of 18 bytes
  static constexpr int PITCH_WORDS = 36;  // 36 words apart: 16-byte reads are conflict-free
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
  // step SUB: bytes [36 SUB, 36 SUB + 36): block 0 at byte 0, block 1 at 18
  template <int SUB>
  __device__ static void step(const uint8_t* row, uint32_t (&out)[32]) {
    constexpr int A = 36 * SUB, C0 = A & ~15, C1 = (A + 36 + 15) & ~15;
    uint32_t w[(C1 - C0) / 4];
    lds_span<C0, C1>(row, w);
    const uint32_t* p = w + (A - C0) / 4;
    uint32_t q[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) q[i] = __funnelshift_r(p[i], p[i + 1], 16);
    block(p[0], q, out);
    block(p[4] >> 16, p + 5, out + 16);
  }
  __host__ __device__ static constexpr int perm(int p) { return perm_q4(p); }
};

template <>
struct Unpack<Q8_0T> {
  static constexpr int RAW_WORDS = 68;  // 8 blocks of 34 bytes
  static constexpr int PITCH_WORDS = 68;
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
  // step SUB: bytes [68 SUB, 68 SUB + 68): block 0 at byte 0, block 1 at 34
  template <int SUB>
  __device__ static void step(const uint8_t* row, uint32_t (&out)[32]) {
    constexpr int A = 68 * SUB, C0 = A & ~15, C1 = (A + 68 + 15) & ~15;
    uint32_t w[(C1 - C0) / 4];
    lds_span<C0, C1>(row, w);
    const uint32_t* p = w + (A - C0) / 4;
    uint32_t q[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) q[i] = __funnelshift_r(p[i], p[i + 1], 16);
    block(p[0], q, out);
    block(p[8] >> 16, p + 9, out + 16);
  }
  // p = 4 i + 2 t + h -> 4 i + t + 2 h
  __host__ __device__ static constexpr int perm(int p) {
    return 4 * (p / 4) + ((p % 4) / 2) + 2 * (p % 2);
  }
};

// ---- x, staged for the tensor cores -------------------------------------------------------
// The F16 x as the MMA reads it, laid out so that ONE contiguous bulk copy
// brings a chunk's four [64 vectors x 64 columns] tiles: tile (pass, chunk,
// step) is 8 KB at ((pass * chunks + chunk) * 4 + step) * 8 KB, each in the
// 128-byte swizzled K-major layout (the 16-byte unit u of row r at u ^ (r % 8))
// that a swizzled tensor copy would have made. Column 32 b + p of a tile row
// holds x[v][32 b + perm(p)]; vectors past m and columns past k are zeros.
constexpr int X_TILE_BYTES = TILE_VECTORS * 128;
constexpr int X_CHUNK_BYTES = 4 * X_TILE_BYTES;

template <typename T, bool BF16>
__global__ void tc_prepare_x_kernel(const void* __restrict__ x, __half* __restrict__ out,
                                    int vectors, int cols, int chunks, long long total,
                                    int* counters, int count) {
  pdl_trigger();  // the product may launch and start on its weights
  pdl_wait();
  // the split product's arrival counters start at zero
  for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < count; i += gridDim.x * blockDim.x)
    counters[i] = 0;
  for (long long e = (long long)blockIdx.x * blockDim.x + threadIdx.x; e < total;
       e += (long long)gridDim.x * blockDim.x) {
    const long long tile = e / (X_TILE_BYTES / 2);
    const int swizzled = int(e % (X_TILE_BYTES / 2)) * 2;  // byte offset in the tile
    const int plain = swizzled ^ (((swizzled >> 7) & 7) << 4);
    const int row = plain / 128, column = (plain % 128) / 2;
    const int step = int(tile % 4), chunk = int((tile / 4) % chunks), pass = int(tile / (4LL * chunks));
    const int v = pass * TILE_VECTORS + row;
    const int k = chunk * CHUNK + step * STEP + column;
    float value = 0.0f;
    if (v < vectors && k < cols) {
      const long long source = (long long)v * cols + (k & ~31) + Unpack<T>::perm(k & 31);
      if (BF16)
        value = __uint_as_float(uint32_t(reinterpret_cast<const uint16_t*>(x)[source]) << 16);
      else
        value = reinterpret_cast<const float*>(x)[source];
    }
    out[e] = __float2half_rn(value);
  }
}

// ---- the product ------------------------------------------------------------------------------
// Dequant warps: GROUPS warpgroups (one warp per TMEM lane quarter each),
// warpgroup g taking the STEPS 64-column steps g * STEPS.. of every chunk.
constexpr int DEQUANT_WARPS = 16;
constexpr int GROUPS = DEQUANT_WARPS / 4, STEPS = 4 / GROUPS;
constexpr int VCOLS = TILE_VECTORS / GROUPS;  // accumulator columns a dequant warp reads back
constexpr int W_WARP = DEQUANT_WARPS, MMA_WARP = DEQUANT_WARPS + 1, X_WARP = DEQUANT_WARPS + 2;
constexpr int TC_THREADS = 32 * (DEQUANT_WARPS + 3);
// TMEM columns: accumulators 0-63 and 64-127; three sets of A buffers (chunk
// number mod 3), warpgroup g's at 128 + 128 set + 32 g: the dequant warps
// fill one set while the MMA reads another
constexpr uint32_t TMEM_COLUMNS = 512;

// Two rings: raw weights (freed by the dequant warps, so they run ahead of
// the MMA) and x (freed by the MMA's commit).
template <typename T>
struct TcLayout {
  static constexpr int W_STAGES = T::DTYPE == DRIFT_Q8_0 ? 3 : 5;
  static constexpr int X_STAGES = 3;
  static constexpr int RAW_BYTES = TILE_ROWS * Unpack<T>::PITCH_WORDS * 4;
  static constexpr int RAW_PADDED = (RAW_BYTES + 1023) / 1024 * 1024;
  static constexpr int X_OFFSET = W_STAGES * RAW_PADDED;
  static constexpr int BARRIER_OFFSET = X_OFFSET + X_STAGES * X_CHUNK_BYTES;
  // w_full, w_empty [W], x_full, x_empty [X], a_full, a_empty, acc_full,
  // acc_empty [2], tmem slot, abort
  static constexpr int SMEM_BYTES = BARRIER_OFFSET + 512 + 1024;  // + alignment slack
  static_assert((2 * W_STAGES + 2 * X_STAGES + 10) * 8 + 8 <= 512, "barrier area");
  static_assert(SMEM_BYTES <= 232448, "shared memory");
};

// What a CTA's units are: unit u is K-range u % splits of tile u / splits,
// tile = pass * row_tiles + row tile.
struct TcPlan {
  int row_tiles, tiles, splits, chunks;
  __device__ int units() const { return tiles * splits; }
  __device__ int chunk_begin(int u) const { return int((long long)chunks * (u % splits) / splits); }
  __device__ int chunk_end(int u) const { return int((long long)chunks * (u % splits + 1) / splits); }
};

// Scratch of the split products: partial sums [tile][split][64 vectors][128
// rows] and one arrival counter per (tile, dequant warp), zeroed by
// tc_prepare_x.
struct TcScratch {
  float* partial;
  int* arrivals;
};

// 16 consecutive 32-bit columns of this thread's lane, to registers.
__device__ __forceinline__ void tmem_load_16(uint32_t address, uint32_t (&v)[16]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, "
      "%12, %13, %14, %15}, [%16];"
      : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]),
        "=r"(v[7]), "=r"(v[8]), "=r"(v[9]), "=r"(v[10]), "=r"(v[11]), "=r"(v[12]), "=r"(v[13]),
        "=r"(v[14]), "=r"(v[15])
      : "r"(address)
      : "memory");
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}

__device__ __forceinline__ void tmem_load_cols(uint32_t address, uint32_t (&v)[16]) {
  tmem_load_16(address, v);
}
__device__ __forceinline__ void tmem_load_cols(uint32_t address, uint32_t (&v)[32]) {
  tc::tmem_load_32(address, v);
}

template <typename T>
__device__ __forceinline__ void dequant_step(int group, const uint8_t* row, uint32_t (&a)[32]) {
  switch (group) {
    case 0: Unpack<T>::template step<0>(row, a); break;
    case 1: Unpack<T>::template step<1>(row, a); break;
    case 2: Unpack<T>::template step<2>(row, a); break;
    default: Unpack<T>::template step<3>(row, a); break;
  }
}

template <typename T>
__global__ void __launch_bounds__(TC_THREADS, 1)
    linear_tc_kernel(const __grid_constant__ CUtensorMap wmap, const uint8_t* __restrict__ xs,
                     float* __restrict__ y, int rows, int vectors, TcPlan plan,
                     TcScratch scratch, int* error) {
  using L = TcLayout<T>;
  constexpr int WS = L::W_STAGES, XS = L::X_STAGES;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~uintptr_t(1023));
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + L::BARRIER_OFFSET);
  uint64_t* w_full = bars;
  uint64_t* w_empty = w_full + WS;
  uint64_t* x_full = w_empty + WS;
  uint64_t* x_empty = x_full + XS;
  uint64_t* a_full = x_empty + XS;  // [3]: chunk number mod 3
  uint64_t* a_empty = a_full + 3;
  uint64_t* acc_full = a_empty + 3;
  uint64_t* acc_empty = acc_full + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(acc_empty + 2);
  volatile int* abort = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  const int units = plan.units();

  if (threadIdx.x == 0) {
    for (int s = 0; s < WS; ++s) {
      tc::mbar_init(&w_full[s], 1);
      tc::mbar_init(&w_empty[s], DEQUANT_WARPS);
    }
    for (int s = 0; s < XS; ++s) {
      tc::mbar_init(&x_full[s], 1);
      tc::mbar_init(&x_empty[s], 1);  // the MMA's commit
    }
    for (int i = 0; i < 3; ++i) {
      tc::mbar_init(&a_full[i], DEQUANT_WARPS);  // a chunk's A, all four steps
      tc::mbar_init(&a_empty[i], 1);             // the MMA's commit
    }
    for (int b = 0; b < 2; ++b) {
      tc::mbar_init(&acc_full[b], 1);
      tc::mbar_init(&acc_empty[b], DEQUANT_WARPS);
    }
    *abort = 0;
    tc::fence_barrier_init();
  }
  if (warp == W_WARP && lane == 0) tc::prefetch_tensor_map(&wmap);
  if (warp == 0) tc::tmem_alloc(tmem_slot, TMEM_COLUMNS);
  __syncthreads();
  tc::fence_after_sync();
  const uint32_t tmem = *tmem_slot;
  pdl_trigger();
  // Only the weight producer may run ahead of the previous kernel: everything
  // else reads x or writes out, scratch and counters.
  if (warp != W_WARP) pdl_wait();

  if (warp == W_WARP || warp == X_WARP) {
    // ---- producers: raw weights (2-D tensor copy of 128 rows), x (one bulk copy) ----
    if (lane == 0) {
      const bool weights = warp == W_WARP;
      const int S = weights ? WS : XS;
      uint64_t* full = weights ? w_full : x_full;
      uint64_t* empty = weights ? w_empty : x_empty;
      int gc = 0;
      bool ok = true;
      for (int u = blockIdx.x; ok && u < units; u += gridDim.x) {
        const int tile = u / plan.splits;
        const int rt = tile % plan.row_tiles, pass = tile / plan.row_tiles;
        for (int c = plan.chunk_begin(u); c < plan.chunk_end(u); ++c, ++gc) {
          const int s = gc % S;
          if (gc >= S && !(ok = tc::mbar_wait(&empty[s], ((gc / S) - 1) & 1, abort, error))) break;
          if (weights) {
            tc::mbar_expect_tx(&full[s], L::RAW_BYTES);
            tc::tma_load_2d(smem + s * L::RAW_PADDED, &wmap, &full[s], c * Unpack<T>::RAW_WORDS,
                            rt * TILE_ROWS);
          } else {
            tc::mbar_expect_tx(&full[s], X_CHUNK_BYTES);
            tc::bulk_load(smem + L::X_OFFSET + s * X_CHUNK_BYTES,
                          xs + ((long long)pass * plan.chunks + c) * X_CHUNK_BYTES, X_CHUNK_BYTES,
                          &full[s]);
          }
        }
      }
      if (!ok) {
        // let the copies already issued land before the CTA leaves
        for (int j = gc - S < 0 ? 0 : gc - S; j < gc; ++j) {
          volatile int never = 0;
          tc::mbar_wait(&full[j % S], (j / S) & 1, &never, nullptr);
        }
      }
    }
  } else if (warp == MMA_WARP) {
    // ---- MMA issuer: the whole warp, one elected lane issuing ----
    {
      const uint32_t idesc = tc::instr_desc_f16(TILE_ROWS, TILE_VECTORS);
      int gc = 0, local = 0;
      bool ok = true;
      for (int u = blockIdx.x; ok && u < units; u += gridDim.x, ++local) {
        const int b = local & 1;
        if (local >= 2 &&
            !(ok = tc::mbar_wait_warp(&acc_empty[b], ((local >> 1) - 1) & 1, abort, error)))
          break;
        tc::fence_after_sync();
        const uint32_t acc = tmem + 64 * b;
        const int c0 = plan.chunk_begin(u);
        for (int c = c0; ok && c < plan.chunk_end(u); ++c, ++gc) {
          const int s = gc % XS;
          if (!(ok = tc::mbar_wait_warp(&x_full[s], (gc / XS) & 1, abort, error))) break;
          if (!(ok = tc::mbar_wait_warp(&a_full[gc % 3], (gc / 3) & 1, abort, error))) break;
          tc::fence_after_sync();
          // one chunk: 16 MMAs back to back (the tensor core's queue stays full
          // while the warp waits for the next chunk), then one commit per ring
          const uint64_t b_desc =
              tc::smem_desc_sw128(tc::smem_u32(smem + L::X_OFFSET + s * X_CHUNK_BYTES));
          const uint32_t a_base = tmem + 128 + 128 * (gc % 3);
          const uint32_t first = c != c0;
#pragma unroll
          for (int g = 0; g < 4; ++g) {
#pragma unroll
            for (int j = 0; j < 4; ++j)
              tc::mma_f16_ts_warp(acc, a_base + 32 * g + 8 * j,
                                  b_desc + uint64_t((g * X_TILE_BYTES + j * 32) >> 4), idesc,
                                  (g | j) ? 1u : first);
          }
          tc::mma_commit_warp(&a_empty[gc % 3]);
          tc::mma_commit_warp(&x_empty[s]);
        }
        if (ok) tc::mma_commit_warp(&acc_full[b]);
      }
    }
  } else {
    // ---- dequant warpgroups, and the epilogues ----
    const int group = warp / 4, quarter = warp % 4;
    const int row_in_tile = quarter * 32 + lane;
    const uint32_t lane_base = uint32_t(quarter * 32) << 16;
    int gc = 0, local = 0;
    bool ok = true;
    // the epilogue of the CTA's unit number `l` (its u), one chunk into the next
    auto epilogue = [&](int u, int l) -> bool {
      const int b = l & 1;
      if (!tc::mbar_wait_warp(&acc_full[b], (l >> 1) & 1, abort, error)) return false;
      tc::fence_after_sync();
      uint32_t acc[VCOLS];
      tmem_load_cols(tmem + lane_base + 64 * b + VCOLS * group, acc);
      tc::fence_before_sync();
      __syncwarp();
      if (lane == 0) tc::mbar_arrive(&acc_empty[b]);
      const int tile = u / plan.splits;
      const int rt = tile % plan.row_tiles, pass = tile / plan.row_tiles;
      const int row = rt * TILE_ROWS + row_in_tile;
      const int v0 = pass * TILE_VECTORS + VCOLS * group;
      if (plan.splits == 1) {
        if (row < rows) {
#pragma unroll
          for (int i = 0; i < VCOLS; ++i)
            if (v0 + i < vectors) y[(long long)(v0 + i) * rows + row] = __uint_as_float(acc[i]);
        }
        return true;
      }
      // A K-range: leave this warp's slice of the partial sum (32 rows x VCOLS
      // vectors); the warp that brings a slice's last range adds the ranges
      // in K order. Slices are counted apart, so no warp waits for another.
      const int split = u % plan.splits;
      float* mine = scratch.partial + ((long long)tile * plan.splits + split) * TILE_VECTORS * TILE_ROWS;
#pragma unroll
      for (int i = 0; i < VCOLS; ++i) mine[(VCOLS * group + i) * TILE_ROWS + row_in_tile] = __uint_as_float(acc[i]);
      __threadfence();
      __syncwarp();
      int arrived = 0;
      if (lane == 0) arrived = atomicAdd(&scratch.arrivals[tile * DEQUANT_WARPS + warp], 1);
      arrived = __shfl_sync(0xffffffffu, arrived, 0);
      if (arrived == plan.splits - 1) {
        __threadfence();
        if (row < rows) {
#pragma unroll
          for (int i = 0; i < VCOLS; ++i) {
            float total = 0.0f;
            for (int k = 0; k < plan.splits; ++k) {
              const float* part = scratch.partial +
                                  ((long long)tile * plan.splits + k) * TILE_VECTORS * TILE_ROWS;
              total += k == split ? __uint_as_float(acc[i])
                                  : __ldcg(part + (VCOLS * group + i) * TILE_ROWS + row_in_tile);
            }
            if (v0 + i < vectors) y[(long long)(v0 + i) * rows + row] = total;
          }
        }
      }
      return true;
    };
    int pending = -1, pending_local = 0;
    for (int u = blockIdx.x; ok && u < units; u += gridDim.x, ++local) {
      for (int c = plan.chunk_begin(u); ok && c < plan.chunk_end(u); ++c, ++gc) {
        const int s = gc % WS;
        if (!(ok = tc::mbar_wait_warp(&w_full[s], (gc / WS) & 1, abort, error))) break;
        if (gc >= 3 && !(ok = tc::mbar_wait_warp(&a_empty[gc % 3], ((gc / 3) - 1) & 1, abort, error)))
          break;
        tc::fence_after_sync();
        const uint8_t* raw_row = smem + s * L::RAW_PADDED + row_in_tile * Unpack<T>::PITCH_WORDS * 4;
        uint32_t a[STEPS][32];
#pragma unroll
        for (int st = 0; st < STEPS; ++st) {
          dequant_step<T>(group * STEPS + st, raw_row, a[st]);
          if (st == STEPS - 1) {
            __syncwarp();
            if (lane == 0) tc::mbar_arrive(&w_empty[s]);  // the raw weights are in registers
          }
          tc::tmem_store_32(tmem + lane_base + 128 + 128 * (gc % 3) + 32 * (group * STEPS + st), a[st]);
        }
        tc::tmem_store_wait();
        tc::fence_before_sync();
        __syncwarp();
        if (lane == 0) tc::mbar_arrive(&a_full[gc % 3]);
        if (pending >= 0) {
          ok = epilogue(pending, pending_local);
          pending = -1;
        }
      }
      pending = u;
      pending_local = local;
    }
    if (ok && pending >= 0) ok = epilogue(pending, pending_local);
  }
  __syncthreads();
  if (warp == 0) {
    tc::fence_after_sync();
    tc::tmem_dealloc(tmem, TMEM_COLUMNS);
  }
}

DRIFT_REGISTER(linear_tc_q8_0, linear_tc_kernel<Q8_0T>)
DRIFT_REGISTER(linear_tc_q4_0, linear_tc_kernel<Q4_0T>)
DRIFT_REGISTER(linear_tc_q4_1, linear_tc_kernel<Q4_1T>)

// ---- host ---------------------------------------------------------------------------------------
// How many K-ranges a tile splits into: the fewest chunk-times per SM, a
// split unit paying about two chunks for its partial sums, and at most
// 4 units per SM in all when split (the scratch is sized for that).
static int choose_splits(long long tiles, int chunks, int sms) {
  int best = 1;
  long long best_cost = ((tiles + sms - 1) / sms) * chunks;
  for (int splits = 2; splits <= 8 && splits <= chunks; ++splits) {
    const long long units = tiles * splits;
    if (units > 4LL * sms) break;
    const long long cost = ((units + sms - 1) / sms) * ((chunks + splits - 1) / splits + 2);
    if (cost < best_cost) {
      best_cost = cost;
      best = splits;
    }
  }
  return best;
}

template <typename T>
static int launch_tc(int x_dtype, const void* x, const void* weight, float* y, int64_t m,
                     int64_t n, int64_t k, uint8_t* workspace, cudaStream_t stream) {
  using L = TcLayout<T>;
  const int sms = sm_count();
  const int64_t padded = (m + TILE_VECTORS - 1) / TILE_VECTORS * TILE_VECTORS;
  TcPlan plan;
  plan.row_tiles = int((n + TILE_ROWS - 1) / TILE_ROWS);
  plan.tiles = plan.row_tiles * int(padded / TILE_VECTORS);
  plan.chunks = int((k + CHUNK - 1) / CHUNK);
  plan.splits = choose_splits(plan.tiles, plan.chunks, sms);
  const size_t x_bytes = size_t(padded / TILE_VECTORS) * plan.chunks * X_CHUNK_BYTES;
  __half* xs = reinterpret_cast<__half*>(workspace);
  TcScratch scratch;
  scratch.partial = reinterpret_cast<float*>(workspace + x_bytes);
  scratch.arrivals = reinterpret_cast<int*>(
      reinterpret_cast<uint8_t*>(scratch.partial) +
      (plan.splits > 1 ? size_t(plan.tiles) * plan.splits * TILE_VECTORS * TILE_ROWS * 4 : 0));
  {
    const long long total = (long long)(x_bytes / 2);
    long long blocks = (total + 255) / 256;
    if (blocks > (long long)sms * 32) blocks = (long long)sms * 32;
    const int counters = plan.splits > 1 ? plan.tiles * DEQUANT_WARPS : 0;
    if (x_dtype == DRIFT_BF16)
      DRIFT_CUDA(launch_pdl(tc_prepare_x_kernel<T, true>, unsigned(blocks), 256, 0, stream, x, xs,
                            int(m), int(k), plan.chunks, total, scratch.arrivals, counters));
    else
      DRIFT_CUDA(launch_pdl(tc_prepare_x_kernel<T, false>, unsigned(blocks), 256, 0, stream, x, xs,
                            int(m), int(k), plan.chunks, total, scratch.arrivals, counters));
  }
  const int64_t row_bytes = k / 32 * T::BYTES;
  CUtensorMap wmap;
  DRIFT_TRY(encode_word_rows(&wmap, weight, row_bytes / 4, n, Unpack<T>::PITCH_WORDS, TILE_ROWS));
  static bool configured[3] = {false, false, false};
  const int which = T::DTYPE == DRIFT_Q8_0 ? 0 : (T::DTYPE == DRIFT_Q4_0 ? 1 : 2);
  if (!configured[which]) {
    DRIFT_CUDA(cudaFuncSetAttribute(linear_tc_kernel<T>,
                                    cudaFuncAttributeMaxDynamicSharedMemorySize, L::SMEM_BYTES));
    configured[which] = true;
  }
  const long long units = (long long)plan.tiles * plan.splits;
  const int grid = units < sms ? int(units) : sms;
  DRIFT_CUDA(launch_pdl(linear_tc_kernel<T>, grid, TC_THREADS, L::SMEM_BYTES, stream, wmap,
                        reinterpret_cast<const uint8_t*>(xs), y, int(n), int(m), plan, scratch,
                        device_error_word()));
  return 0;
}

}  // namespace

// Bytes of scratch a tensor-core product of m rows of k (new) needs at most:
// the F16 x (whole chunks), and for split products the partial sums (at most 4 units per SM)
// and the counters.
size_t tc_workspace_bytes(int64_t m, int64_t k) {
  const size_t passes = size_t((m + TILE_VECTORS - 1) / TILE_VECTORS);
  const size_t chunks = size_t((k + CHUNK - 1) / CHUNK);
  const size_t units = size_t(4) * size_t(sm_count());  // split tiles are at most half that
  return passes * chunks * X_CHUNK_BYTES + units * TILE_VECTORS * TILE_ROWS * 4 +
         units * DEQUANT_WARPS * 4 + 256;
}

// Whether the tensor-core path takes a product: rows in whole 16-byte units
// and a 16-byte aligned weight (what the tensor copies need).
bool tc_supports(int weight_dtype, const void* weight, int64_t k) {
  if (weight_dtype != DRIFT_Q8_0 && weight_dtype != DRIFT_Q4_0 && weight_dtype != DRIFT_Q4_1)
    return false;
  const int64_t row = byte_size(weight_dtype, k);
  return row > 0 && row % 16 == 0 && (reinterpret_cast<uintptr_t>(weight) & 15) == 0 &&
         tensor_maps_available();
}

// `workspace`: tc_workspace_bytes(m, k) bytes of device scratch.
int linear_tc(int x_dtype, const void* x, int weight_dtype, const void* weight, float* y,
              int64_t m, int64_t n, int64_t k, uint8_t* workspace, cudaStream_t stream) {
  switch (weight_dtype) {
    case DRIFT_Q8_0: return launch_tc<Q8_0T>(x_dtype, x, weight, y, m, n, k, workspace, stream);
    case DRIFT_Q4_0: return launch_tc<Q4_0T>(x_dtype, x, weight, y, m, n, k, workspace, stream);
    default: return launch_tc<Q4_1T>(x_dtype, x, weight, y, m, n, k, workspace, stream);
  }
}

}  // namespace drift
