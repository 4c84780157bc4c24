// Batch-shaped products on the 5th-generation tensor cores: out[m, n] =
// x[m, k] . W[n, k]^T for m >= 32 (the runner's GEMM path, ops/HipLinear.scala:
// 389-469, kernels/matvec.hip:801-810, which dequantizes W to F16 and calls
// hipBLAS), fused into one persistent kernel that keeps F32 accuracy: results
// are held to the CPU reference (CpuLinear.linear, Double sums) within
// 1e-4 + 1e-3 |y|, not to an F16 GEMM's bound.
//
// Exact operands. tcgen05.mma kind::f16 multiplies F16 values exactly and
// sums in F32, so each operand enters as F16 terms whose sum is its value:
//  - weights: a block's value is d * q (+ m for Q4_1), with q a small integer.
//    d * q needs up to 18 significant bits; HMUL2 gives its F16 rounding hi
//    and HFMA2(q, d, -hi) the exact remainder lo (TwoProduct through a fused
//    multiply-add), so hi + lo = d * q. Q4_1's m enters apart: sum_k m_b x_k
//    = sum_b m_b S_b, with S_b the block sums of x, one more K=16 MMA a chunk
//    against an [m_0..m_7, m_0..m_7] x [S_hi; S_lo] pair of tiles;
//  - x: each vector is scaled by a power of two 2^-e (max |x| to [2^9, 2^10),
//    undone exactly in the epilogue), so BF16 x is exact in one F16 term and
//    F32 x takes two (hi + lo, 22 bits). The block sums S_b stay below 2^15.
// Per k-step the MMAs are hi*x and lo*x (and hi*x_lo for F32 x): the
// product's error is F32 summation alone.
//
// One CTA per SM, 19 warps, units of 128 weight rows x 64 vectors (x a
// K-range of the columns, when a matrix has too few rows to fill the SMs):
//  - warp 16 (weights): streams each 256-column chunk of the unit's raw GGML
//    blocks (a 2-D tensor copy, 128 rows) into a ring of stages, freed as
//    soon as the dequant warps have used a stage;
//  - warp 18 (x): one bulk copy per chunk of its staged x (the four 64-column
//    F16 tiles, pre-swizzled by tc_prepare_x into the UMMA canonical K-major
//    layout; their low terms for F32 x; the block-sum tile for Q4_1) into a
//    ring, freed by the MMA's commit;
//  - warps 0-15 (dequant, four warpgroups, warpgroup g taking 64-column step
//    g of every chunk): each thread turns its row's two blocks into 64
//    weights as hi and lo F16 terms and stores them straight into tensor
//    memory (tcgen05.st) -- a chunk's two 128-column halves go to two of three
//    A sets, which the dequant warps fill while the MMA reads another -- and,
//    for Q4_1, the row's block mins into a small shared-memory tile;
//  - warp 17 (MMA): the whole warp waits, one elected lane issues each half's
//    MMAs back to back (A in TMEM, B in shared memory) into an F32
//    accumulator in TMEM (128 x 64), a fresh one for each chunk -- two
//    alternate -- and commits once per ring.
// The tensor core's F32 sums drop low bits as a chain of accumulating MMAs
// grows (an error that grows with the chain's length, not as a random walk),
// so no chain spans more than a chunk: one chunk late, the dequant warps read
// each chunk's accumulator back (tcgen05.ld) and add it to the unit's running
// sums in F32 registers, rounding to nearest. At a unit's end they scale the
// sums by 2^e per vector and store F32 out -- or, for a unit that holds a
// K-range, store them as a partial sum; the last of a tile's K-ranges to
// finish adds the partials in K order, so the result does not depend on which
// CTA finishes first. Every wait is bounded (tc_common.cuh). The kernel is
// launched as a programmatic dependent of the x preparation: it sets up and
// starts the weight copies while that kernel finishes.
//
// The weights' values within a 32-block come out of the unpacking in a
// permuted order (pairs of nibbles that one LOP3 makes into an F16x2), so x
// is staged in the same permuted order by tc_prepare_x; a product's sum is
// the same over any order of its terms.
//
// Range: d * q, m and d * q's F16 remainder must be finite F16 values, as
// the reference's F16 dequantization requires of the same weights.
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

__device__ __forceinline__ uint32_t h2u(__half2 h) { return *reinterpret_cast<uint32_t*>(&h); }
__device__ __forceinline__ __half2 u2h(uint32_t u) { return *reinterpret_cast<__half2*>(&u); }


// ---- unpacking, per storage type -------------------------------------------------------
// half<H>(row, store, mins): the 128 weights of one row's half chunk H (steps
// 2H and 2H + 1, four blocks) as hi and lo F16x2 words -- store(sub, hi, lo)
// takes step 2H + sub's 32 of each -- from that row's raw words in the ring,
// and the four blocks' F16 min terms (Q4 types; block 0 lowest). perm(p):
// which value of a 32-block sits at position p of the unpacked order.
template <typename T>
struct Unpack;

__host__ __device__ constexpr int perm_q4(int p) {
  // p = 8 i + 2 t + h
  return ((p % 8) / 2 >= 2 ? 16 : 0) + 4 * (p / 8) + ((p % 8) / 2 & 1) + 2 * (p % 2);
}

// A block's d, split exactly into dh (its 7 leading significant bits) and
// dl (the other 4), with the offsets that take a magic-exponent code to q:
// for a code read as 1024 + q or 64 + q (below), HFMA2(code, dh, -1024 dh)
// is q dh exactly -- the fused product is exact and q dh has at most
// 4 + 7 = 11 significant bits -- and likewise q dl (4 + 4 bits). So
// hi + lo = q d with no rounding, in two instructions a pair of values.
struct Q4Scale {
  __half2 dh, dl, h1024, l1024, h64, l64;
  __device__ __forceinline__ explicit Q4Scale(uint32_t d_bits) {
    const uint32_t dd = __byte_perm(d_bits, 0, 0x1010);
    dh = u2h(dd & 0xFFF0FFF0u);
    dl = __hsub2(u2h(dd), dh);  // exact
    h1024 = __hmul2(dh, u2h(0xE400E400u));  // * -1024, exact
    l1024 = __hmul2(dl, u2h(0xE400E400u));
    h64 = __hmul2(dh, u2h(0xD400D400u));  // * -64, exact
    l64 = __hmul2(dl, u2h(0xD400D400u));
  }
};

// One word of Q4 nibbles (bytes b0..b3: values 4i..4i+3 low, 16+4i.. high)
// as four pairs (v0, v2), (v1, v3) from the low nibbles under the magic
// exponent of 1024 (0x6400: 1024 + q), (v16, v18), (v17, v19) from the high
// nibbles in place under that of 64 (0x5400: the nibble lands 4 bits up the
// mantissa, 64 + q) -- one LOP3 each -- then hi and lo of each.
__device__ __forceinline__ void q4_word(uint32_t w, const Q4Scale& k, uint32_t* hi, uint32_t* lo) {
  const uint32_t t = w >> 8;
  const __half2 p0 = u2h((w & 0x000F000Fu) | 0x64006400u);
  const __half2 p1 = u2h((t & 0x000F000Fu) | 0x64006400u);
  const __half2 p2 = u2h((w & 0x00F000F0u) | 0x54005400u);
  const __half2 p3 = u2h((t & 0x00F000F0u) | 0x54005400u);
  hi[0] = h2u(__hfma2(p0, k.dh, k.h1024));
  lo[0] = h2u(__hfma2(p0, k.dl, k.l1024));
  hi[1] = h2u(__hfma2(p1, k.dh, k.h1024));
  lo[1] = h2u(__hfma2(p1, k.dl, k.l1024));
  hi[2] = h2u(__hfma2(p2, k.dh, k.h64));
  lo[2] = h2u(__hfma2(p2, k.dl, k.l64));
  hi[3] = h2u(__hfma2(p3, k.dh, k.h64));
  lo[3] = h2u(__hfma2(p3, k.dl, k.l64));
}

// Field access at a constant byte offset O of the loaded words (blocks start
// on 2-byte boundaries): the f16 d at O, and N code words from byte C on.
template <int O>
__device__ __forceinline__ uint32_t half_at(const uint32_t* w) {
  return O % 4 == 0 ? (w[O / 4] & 0xffffu) : (w[O / 4] >> 16);
}
template <int C, int N>
__device__ __forceinline__ void words_at(const uint32_t* w, uint32_t (&q)[N]) {
#pragma unroll
  for (int i = 0; i < N; ++i)
    q[i] = C % 4 == 0 ? w[C / 4 + i] : __funnelshift_r(w[C / 4 + i], w[C / 4 + i + 1], 16);
}

// The span of a half chunk's bytes as loaded: [C0, C0 + 4 WORDS) of the row's
// chunk, 16-byte aligned, and block b's offset in it.
template <typename T, int H>
struct HalfSpan {
  static constexpr int BEGIN = 4 * T::BYTES * H;
  static constexpr int C0 = BEGIN & ~15;
  static constexpr int WORDS = ((BEGIN + 4 * T::BYTES + 15) / 16 * 16 - C0) / 4;
  static constexpr int at(int b) { return BEGIN - C0 + b * T::BYTES; }
};

// Q4_0 and Q4_1 share the product part d q (q the unsigned code); value =
// d q + m with m the block's min (Q4_1) or -8 d (Q4_0), which enters through
// the block sums of x.
template <typename T>
struct UnpackQ4 {
  template <int H, int B>
  __device__ static void block(const uint32_t* w, uint32_t* hi, uint32_t* lo, uint32_t& min) {
    constexpr int O = HalfSpan<T, H>::at(B);
    const uint32_t d_bits = half_at<O>(w);
    const Q4Scale k(d_bits);
    if constexpr (T::DTYPE == DRIFT_Q4_1)
      min = half_at<O + 2>(w);
    else
      min = h2u(__hmul2(u2h(d_bits), u2h(0xC800C800u))) & 0xffffu;  // -8 d, exact
    uint32_t q[4];
    words_at<O + T::BYTES - 16, 4>(w, q);
#pragma unroll
    for (int i = 0; i < 4; ++i) q4_word(q[i], k, hi + 4 * i, lo + 4 * i);
  }
  template <int H, typename Store>
  __device__ static void half(const uint8_t* row, Store store, uint32_t (&mins)[2]) {
    using S = HalfSpan<T, H>;
    uint32_t w[S::WORDS];
    lds_span<S::C0, S::C0 + 4 * S::WORDS>(row, w);
    uint32_t m[4];
    {
      uint32_t hi[32], lo[32];
      block<H, 0>(w, hi, lo, m[0]);
      block<H, 1>(w, hi + 16, lo + 16, m[1]);
      store(0, hi, lo);
    }
    {
      uint32_t hi[32], lo[32];
      block<H, 2>(w, hi, lo, m[2]);
      block<H, 3>(w, hi + 16, lo + 16, m[3]);
      store(1, hi, lo);
    }
    mins[0] = m[0] | (m[1] << 16);
    mins[1] = m[2] | (m[3] << 16);
  }
  __host__ __device__ static constexpr int perm(int p) { return perm_q4(p); }
};

template <>
struct Unpack<Q4_1T> : UnpackQ4<Q4_1T> {
  static constexpr int RAW_WORDS = 40;  // 8 blocks of 20 bytes
  // a chunk's row as copied: 16 bytes past the chunk, so rows sit 44 words
  // apart and 16-byte reads of one column of 8 rows hit 8 distinct bank groups
  static constexpr int PITCH_WORDS = 44;
};

template <>
struct Unpack<Q4_0T> : UnpackQ4<Q4_0T> {
  static constexpr int RAW_WORDS = 36;    // 8 blocks of 18 bytes
  static constexpr int PITCH_WORDS = 36;  // 36 words apart: 16-byte reads are conflict-free
};

// q * d as two F16 terms whose sum is exact: hi its rounding, lo the rest
// (a fused multiply-add gives the remainder exactly).
__device__ __forceinline__ void two_product(__half2 q, __half2 d, uint32_t& hi, uint32_t& lo) {
  const __half2 h = __hmul2(q, d);
  hi = h2u(h);
  lo = h2u(__hfma2(q, d, __hneg2(h)));
}

template <>
struct Unpack<Q8_0T> {
  static constexpr int RAW_WORDS = 68;  // 8 blocks of 34 bytes
  static constexpr int PITCH_WORDS = 68;
  // Signed codes c0..c3 of a word become (c0, c2), (c1, c3): bytes biased by
  // 128 under the magic exponent of 1024, less 1152 (exact); then d c, up to
  // 18 significant bits, as hi and lo by two_product.
  template <int H, int B>
  __device__ static void block(const uint32_t* w, uint32_t* hi, uint32_t* lo) {
    constexpr int O = HalfSpan<Q8_0T, H>::at(B);
    const __half2 d = u2h(__byte_perm(half_at<O>(w), 0, 0x1010));
    const __half2 k1152 = u2h(0x64806480u);
    uint32_t q[8];
    words_at<O + 2, 8>(w, q);
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const uint32_t u = q[i] ^ 0x80808080u;
      const __half2 p0 = __hsub2(u2h(__byte_perm(u, 0x64646464u, 0x4240)), k1152);
      const __half2 p1 = __hsub2(u2h(__byte_perm(u, 0x64646464u, 0x4341)), k1152);
      two_product(p0, d, hi[2 * i], lo[2 * i]);
      two_product(p1, d, hi[2 * i + 1], lo[2 * i + 1]);
    }
  }
  template <int H, typename Store>
  __device__ static void half(const uint8_t* row, Store store, uint32_t (&mins)[2]) {
    using S = HalfSpan<Q8_0T, H>;
    uint32_t w[S::WORDS];
    lds_span<S::C0, S::C0 + 4 * S::WORDS>(row, w);
    {
      uint32_t hi[32], lo[32];
      block<H, 0>(w, hi, lo);
      block<H, 1>(w, hi + 16, lo + 16);
      store(0, hi, lo);
    }
    {
      uint32_t hi[32], lo[32];
      block<H, 2>(w, hi, lo);
      block<H, 3>(w, hi + 16, lo + 16);
      store(1, hi, lo);
    }
    mins[0] = mins[1] = 0;
  }
  // p = 4 i + 2 t + h -> 4 i + t + 2 h
  __host__ __device__ static constexpr int perm(int p) {
    return 4 * (p / 4) + ((p % 4) / 2) + 2 * (p % 2);
  }
};

// ---- x, staged for the tensor cores -------------------------------------------------------
// The F16 x terms as the MMA reads them, laid out so that ONE contiguous bulk
// copy brings a chunk: at ((pass * chunks + chunk) * BYTES)
//  - hi: four [64 vectors x 64 columns] tiles of 8 KB, one per step, each in
//    the 128-byte swizzled K-major layout (the 16-byte unit u of row r at
//    u ^ (r % 8)) that a swizzled tensor copy would have made; column 32 b + p
//    of a tile row holds x'[v][32 b + perm(p)], x' = x 2^-e(v);
//  - lo (F32 x): the same four tiles of x' - hi;
//  - S (Q4 types): [64 vectors x 16] in the no-swizzle K-major layout: column
//    b < 8 the F16 rounding of block b's sum of x', column 8 + b its remainder.
// Vectors past m and columns past k are zeros.
constexpr int X_TILE_BYTES = TILE_VECTORS * 128;
constexpr int X_TERM_BYTES = 4 * X_TILE_BYTES;
constexpr int S_TILE_BYTES = TILE_VECTORS * 32;
constexpr int M_TILE_BYTES = TILE_ROWS * 32;  // [128 rows x 16] mins, no swizzle
constexpr size_t X_CHUNK_MAX = 2 * X_TERM_BYTES + S_TILE_BYTES;

template <typename T, bool XSPLIT>
struct XChunk {
  static constexpr bool SUMS = T::DTYPE != DRIFT_Q8_0;  // the Q4 types' min terms
  static constexpr int LO_OFFSET = X_TERM_BYTES;
  static constexpr int S_OFFSET = X_TERM_BYTES * (XSPLIT ? 2 : 1);
  static constexpr int BYTES = S_OFFSET + (SUMS ? S_TILE_BYTES : 0);
};

// Byte offset of element (r, k), k < 16, of an F16 tile in the no-swizzle
// K-major canonical layout: 8-row core matrices of 16 bytes a row, the two
// K halves 128 bytes apart (LBO), 8-row groups 256 bytes apart (SBO).
__host__ __device__ constexpr int interleave_offset(int r, int k) {
  return (r / 8) * 256 + (k / 8) * 128 + (r % 8) * 16 + (k % 8) * 2;
}

__device__ __forceinline__ uint64_t smem_desc_interleave(uint32_t address) {
  return uint64_t((address >> 4) & 0x3fff) | (uint64_t(128 >> 4) << 16) |
         (uint64_t(256 >> 4) << 32) | (uint64_t(1) << 46);
}

// D[tmem] (+)= A[smem] x B[smem]^T, issued by one elected lane of the warp.
__device__ __forceinline__ void mma_f16_ss_warp(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc,
                                                uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p, e;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "elect.sync _|e, 0xffffffff;\n\t"
      "@e tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}

constexpr int PREP_THREADS = 256;
constexpr int PREP_CHUNKS = 8;  // chunks of x one preparation CTA stages

// Grid (padded vectors, chunk groups): each CTA finds its vector's largest
// |x| (every CTA of the vector reads the whole row, so no other launch is
// needed), sets e, then stages PREP_CHUNKS chunks of it, a warp per block.
template <typename T, bool BF16, bool XSPLIT>
__global__ void __launch_bounds__(PREP_THREADS)
    tc_prepare_x_kernel(const void* __restrict__ x, uint8_t* __restrict__ staged,
                        float* __restrict__ scales, int vectors, int cols, int chunks,
                        int* counters, int count) {
  using XC = XChunk<T, XSPLIT>;
  pdl_trigger();  // the product may launch and start on its weights
  pdl_wait();
  {
    // the split product's arrival counters start at zero
    const int threads = gridDim.x * gridDim.y * PREP_THREADS;
    for (int i = (blockIdx.y * gridDim.x + blockIdx.x) * PREP_THREADS + threadIdx.x; i < count;
         i += threads)
      counters[i] = 0;
  }
  const int v = blockIdx.x, warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  auto load = [&](long long k) -> float {
    const long long at = (long long)v * cols + k;
    return BF16 ? __uint_as_float(uint32_t(reinterpret_cast<const uint16_t*>(x)[at]) << 16)
                : reinterpret_cast<const float*>(x)[at];
  };
  __shared__ float largest[PREP_THREADS / 32];
  float mx = 0.0f;
  if (v < vectors)
    for (int k = threadIdx.x; k < cols; k += PREP_THREADS) mx = fmaxf(mx, fabsf(load(k)));
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
  if (lane == 0) largest[warp] = mx;
  __syncthreads();
  mx = 0.0f;
#pragma unroll
  for (int w = 0; w < PREP_THREADS / 32; ++w) mx = fmaxf(mx, largest[w]);
  // 2^-e takes max |x| to [2^9, 2^10): block sums of 32 stay below 2^15
  int e = 0;
  if (mx > 0.0f && mx <= 3.4028235e38f) e = min(max(ilogbf(mx) - 9, -100), 100);
  const float down = __int_as_float((127 - e) << 23);
  if (blockIdx.y == 0 && threadIdx.x == 0) scales[v] = __int_as_float((127 + e) << 23);

  const int pass = v / TILE_VECTORS, row = v % TILE_VECTORS;
  const int first = blockIdx.y * PREP_CHUNKS * 8;
  for (int bi = warp; bi < PREP_CHUNKS * 8; bi += PREP_THREADS / 32) {
    const int b = first + bi, chunk = b / 8;
    if (chunk >= chunks) break;
    const int k = b * 32 + lane;
    const float value = v < vectors && k < cols ? load(k) : 0.0f;
    const float scaled = __fmul_rn(value, down);  // exact: a power of two
    const __half hi = __float2half_rn(scaled);
    const __half lo = __float2half_rn(__fsub_rn(scaled, __half2float(hi)));
    // position p of the staged block holds value perm(p)
    const int source = Unpack<T>::perm(lane);
    const uint32_t hi_bits = __shfl_sync(0xffffffffu, uint32_t(__half_as_ushort(hi)), source);
    const uint32_t lo_bits = __shfl_sync(0xffffffffu, uint32_t(__half_as_ushort(lo)), source);
    uint8_t* base = staged + ((long long)pass * chunks + chunk) * XC::BYTES;
    const int col = 32 * (b % 2) + lane;  // column in the step's tile
    const int at = ((b % 8) / 2) * X_TILE_BYTES + row * 128 + (((col / 8) ^ (row % 8)) * 16) +
                   (col % 8) * 2;
    *reinterpret_cast<uint16_t*>(base + at) = uint16_t(hi_bits);
    if (XSPLIT) *reinterpret_cast<uint16_t*>(base + XC::LO_OFFSET + at) = uint16_t(lo_bits);
    if (XC::SUMS) {
      // the block's sum in one fixed order (every lane ends with the same bits)
      float sum = scaled;
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) sum = __fadd_rn(sum, __shfl_xor_sync(0xffffffffu, sum, o));
      if (lane < 2) {
        const __half s_hi = __float2half_rn(sum);
        const __half term = lane == 0 ? s_hi : __float2half_rn(__fsub_rn(sum, __half2float(s_hi)));
        *reinterpret_cast<__half*>(base + XC::S_OFFSET + interleave_offset(row, b % 8 + 8 * lane)) =
            term;
      }
    }
  }
}

// ---- the product ------------------------------------------------------------------------------
// Warps 0-7 dequantize (warp w: TMEM lane quarter w % 4, half chunk w / 4 of
// every chunk), warps 8-11 read the accumulators back and write out (lane
// quarter w % 4), warp 12 streams weights, 13 issues the MMAs, 14 streams x.
constexpr int DEQUANT_WARPS = 8;
constexpr int EPILOGUE_WARPS = 4;
constexpr int FIRST_EPILOGUE = DEQUANT_WARPS;
constexpr int W_WARP = DEQUANT_WARPS + EPILOGUE_WARPS, MMA_WARP = W_WARP + 1, X_WARP = W_WARP + 2;
constexpr int TC_THREADS = 32 * (X_WARP + 1);
// TMEM columns: accumulators 0-63 and 64-127 (chunks alternate); three A
// sets at 128 + 128 s, each a 128-column half chunk: hi terms at +0 (32
// columns a step), lo at +64
constexpr uint32_t TMEM_COLUMNS = 512;

// Rings: raw weights (freed by the dequant warps, so they run ahead of the
// MMA), staged x (freed by the MMA's commit), and for the Q4 types the min
// tiles.
template <typename T, bool XSPLIT>
struct TcLayout {
  using XC = XChunk<T, XSPLIT>;
  static constexpr int X_STAGES = XSPLIT ? 2 : 3;
  static constexpr int M_SLOTS = XC::SUMS ? 3 : 0;
  static constexpr int RAW_BYTES = TILE_ROWS * Unpack<T>::PITCH_WORDS * 4;
  static constexpr int RAW_PADDED = (RAW_BYTES + 1023) / 1024 * 1024;
  static constexpr int FIXED = X_STAGES * XC::BYTES + M_SLOTS * M_TILE_BYTES + 512 + 1024;
  static constexpr int W_FIT = (232448 - FIXED) / RAW_PADDED;
  static constexpr int W_STAGES = W_FIT > 5 ? 5 : W_FIT;
  static constexpr int X_OFFSET = W_STAGES * RAW_PADDED;
  static constexpr int M_OFFSET = X_OFFSET + X_STAGES * XC::BYTES;
  static constexpr int BARRIER_OFFSET = M_OFFSET + M_SLOTS * M_TILE_BYTES;
  // w_full, w_empty [W], ready, half1, a_empty, done [3], tmem slot, abort
  static constexpr int SMEM_BYTES = BARRIER_OFFSET + 512 + 1024;  // + alignment slack
  static_assert(W_STAGES >= 2, "raw weight ring");
  static_assert(XC::BYTES % 1024 == 0, "x chunks keep the swizzle atoms aligned");
  static_assert((2 * W_STAGES + 12) * 8 + 8 <= 512, "barrier area");
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
// rows] and one arrival counter per (tile, epilogue warp), zeroed by
// tc_prepare_x.
struct TcScratch {
  float* partial;
  int* arrivals;
};

// A ring position: slot and phase parity, advanced without division.
template <int N>
struct Ring {
  int slot = 0;
  uint32_t phase = 0;
  __device__ __forceinline__ void advance(int by = 1) {
    slot += by;
    if (slot >= N) {
      slot -= N;
      phase ^= 1u;
    }
  }
};

// The bounded wait of a whole warp, the common case (already complete) kept
// short and the sleeping loop out of line.
__device__ __noinline__ bool wait_slow(uint64_t* bar, uint32_t parity, volatile int* abort,
                                       int* error) {
  return tc::mbar_wait(bar, parity, abort, error);
}
__device__ __forceinline__ bool wait_warp(uint64_t* bar, uint32_t parity, volatile int* abort,
                                          int* error) {
  const bool ok = tc::mbar_try_wait(bar, parity) || wait_slow(bar, parity, abort, error);
  return __all_sync(0xffffffffu, ok);
}

__device__ __forceinline__ void tmem_load_32_nowait(uint32_t address, uint32_t (&v)[32]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, "
      "%12, %13, %14, %15, %16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, "
      "%30, %31}, [%32];"
      : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]),
        "=r"(v[7]), "=r"(v[8]), "=r"(v[9]), "=r"(v[10]), "=r"(v[11]), "=r"(v[12]), "=r"(v[13]),
        "=r"(v[14]), "=r"(v[15]), "=r"(v[16]), "=r"(v[17]), "=r"(v[18]), "=r"(v[19]),
        "=r"(v[20]), "=r"(v[21]), "=r"(v[22]), "=r"(v[23]), "=r"(v[24]), "=r"(v[25]),
        "=r"(v[26]), "=r"(v[27]), "=r"(v[28]), "=r"(v[29]), "=r"(v[30]), "=r"(v[31])
      : "r"(address)
      : "memory");
}

// One dequant warp's half chunk: its 32 rows' four blocks into the A set at
// column `set` (step sub's hi at + 32 sub, lo 64 columns on); the blocks'
// min terms come back in `mins`.
template <typename T>
__device__ __forceinline__ void dequant_half(int half, const uint8_t* row, uint32_t set,
                                             uint32_t (&mins)[2]) {
  auto store = [&](int sub, const uint32_t (&hi)[32], const uint32_t (&lo)[32]) {
    tc::tmem_store_32(set + 32 * sub, hi);
    tc::tmem_store_32(set + 64 + 32 * sub, lo);
  };
  if (half == 0)
    Unpack<T>::template half<0>(row, store, mins);
  else
    Unpack<T>::template half<1>(row, store, mins);
}

template <typename T, bool XSPLIT>
__global__ void __launch_bounds__(TC_THREADS, 1)
    linear_tc_kernel(const __grid_constant__ CUtensorMap wmap, const uint8_t* __restrict__ xs,
                     const float* __restrict__ scales, float* __restrict__ y, int rows,
                     int vectors, TcPlan plan, TcScratch scratch, int* error) {
  using L = TcLayout<T, XSPLIT>;
  using XC = typename L::XC;
  constexpr int WS = L::W_STAGES, XS = L::X_STAGES;
  constexpr bool SUMS = XC::SUMS;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~uintptr_t(1023));
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + L::BARRIER_OFFSET);
  // Chunk c's hand-offs, so the MMA warp waits twice a chunk and commits
  // three times:
  //  - ready[c % 3]: the MMA may start chunk c -- its x landed (the x
  //    producer's expected bytes), its first half's A is in TMEM (four dequant
  //    warps) and its accumulator (c % 2) was read back (four epilogue warps,
  //    after chunk c - 2);
  //  - half1[c % 3]: its second half's A is in TMEM (four dequant warps);
  //  - a_empty[q % 3]: half chunk q's A set may be refilled (MMA commit);
  //  - done[c % 3]: chunk c's MMAs completed (MMA commit): its accumulator
  //    may be read, its x slot and min tile reused.
  uint64_t* w_full = bars;
  uint64_t* w_empty = w_full + WS;
  uint64_t* ready = w_empty + WS;
  uint64_t* half1 = ready + 3;
  uint64_t* a_empty = half1 + 3;
  uint64_t* done = a_empty + 3;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(done + 3);
  volatile int* abort = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  const int units = plan.units();

  if (threadIdx.x == 0) {
    for (int s = 0; s < WS; ++s) {
      tc::mbar_init(&w_full[s], 1);
      tc::mbar_init(&w_empty[s], DEQUANT_WARPS);
    }
    for (int i = 0; i < 3; ++i) {
      tc::mbar_init(&ready[i], DEQUANT_WARPS / 2 + EPILOGUE_WARPS + 1);
      tc::mbar_init(&half1[i], DEQUANT_WARPS / 2);
      tc::mbar_init(&a_empty[i], 1);
      tc::mbar_init(&done[i], 1);
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

  if (warp == W_WARP) {
    // ---- weight producer: a 2-D tensor copy of 128 rows' chunk into the ring ----
    if (lane == 0) {
      int gc = 0;
      bool ok = true;
      for (int u = blockIdx.x; ok && u < units; u += gridDim.x) {
        const int rt = (u / plan.splits) % plan.row_tiles;
        const int c1 = plan.chunk_end(u);
        for (int c = plan.chunk_begin(u); c < c1; ++c, ++gc) {
          const int s = gc % WS;
          if (gc >= WS && !(ok = tc::mbar_wait(&w_empty[s], ((gc / WS) - 1) & 1, abort, error)))
            break;
          tc::mbar_expect_tx(&w_full[s], L::RAW_BYTES);
          tc::tma_load_2d(smem + s * L::RAW_PADDED, &wmap, &w_full[s], c * Unpack<T>::RAW_WORDS,
                          rt * TILE_ROWS);
        }
      }
      if (!ok) {
        // let the copies already issued land before the CTA leaves
        for (int j = gc - WS < 0 ? 0 : gc - WS; j < gc; ++j) {
          volatile int never = 0;
          tc::mbar_wait(&w_full[j % WS], (j / WS) & 1, &never, nullptr);
        }
      }
    }
  } else if (warp == X_WARP) {
    // ---- x producer: one bulk copy per chunk, completing on the chunk's ready ----
    if (lane == 0) {
      int gc = 0;
      bool ok = true;
      for (int u = blockIdx.x; ok && u < units; u += gridDim.x) {
        const int pass = (u / plan.splits) / plan.row_tiles;
        const int c1 = plan.chunk_end(u);
        for (int c = plan.chunk_begin(u); c < c1; ++c, ++gc) {
          // the slot's last chunk, gc - XS, is done
          if (gc >= XS &&
              !(ok = tc::mbar_wait(&done[(gc - XS) % 3], ((gc - XS) / 3) & 1, abort, error)))
            break;
          tc::mbar_expect_tx(&ready[gc % 3], XC::BYTES);
          tc::bulk_load(smem + L::X_OFFSET + (gc % XS) * XC::BYTES,
                        xs + ((long long)pass * plan.chunks + c) * XC::BYTES, XC::BYTES,
                        &ready[gc % 3]);
        }
      }
      if (!ok) {
        for (int j = gc - XS < 0 ? 0 : gc - XS; j < gc; ++j) {
          volatile int never = 0;
          tc::mbar_wait(&ready[j % 3], (j / 3) & 1, &never, nullptr);
        }
      }
    }
  } else if (warp == MMA_WARP) {
    // ---- MMA issuer: the whole warp, one elected lane issuing ----
    // Each chunk sums into a fresh accumulator (the two alternate by chunk),
    // which the epilogue warps read back and add in F32 registers: the tensor
    // core's own F32 sums, which drop low bits as a chain of MMAs grows, span
    // one chunk only.
    const uint32_t idesc = tc::instr_desc_f16(TILE_ROWS, TILE_VECTORS);
    Ring<3> cr;  // chunk gc: ready, half1 and done slot, and their phase
    Ring<3> ar;  // half chunk 2 gc + h: A set
    int gc = 0;
    bool ok = true;
    for (int u = blockIdx.x; ok && u < units; u += gridDim.x) {
      const int c1 = plan.chunk_end(u);  // (a 64-bit division: once a unit)
      for (int c = plan.chunk_begin(u); ok && c < c1; ++c, ++gc) {
        const uint32_t acc = tmem + 64 * (gc & 1);
        const uint32_t x_address = tc::smem_u32(smem + L::X_OFFSET + (gc % XS) * XC::BYTES);
        const uint64_t x_desc = tc::smem_desc_sw128(x_address);
#pragma unroll
        for (int h = 0; h < 2; ++h) {
          uint64_t* gate = h == 0 ? &ready[cr.slot] : &half1[cr.slot];
          if (!(ok = wait_warp(gate, cr.phase, abort, error))) break;
          tc::fence_after_sync();
          const uint32_t a = tmem + 128 + 128 * ar.slot;
          // one half: its 8 K-steps, each hi * x and lo * x (and hi * x_lo),
          // back to back; the tensor core's queue stays full meanwhile
#pragma unroll
          for (int j = 0; j < 8; ++j) {
            const uint64_t bd =
                x_desc + uint64_t(((2 * h + j / 4) * X_TILE_BYTES + (j % 4) * 32) >> 4);
            tc::mma_f16_ts_warp(acc, a + 8 * j, bd, idesc, (h || j) ? 1u : 0u);
            tc::mma_f16_ts_warp(acc, a + 64 + 8 * j, bd, idesc, 1u);
            if (XSPLIT)
              tc::mma_f16_ts_warp(acc, a + 8 * j, bd + uint64_t(XC::LO_OFFSET >> 4), idesc, 1u);
          }
          if (SUMS && h == 1)
            mma_f16_ss_warp(acc,
                            smem_desc_interleave(
                                tc::smem_u32(smem + L::M_OFFSET + cr.slot * M_TILE_BYTES)),
                            smem_desc_interleave(x_address + XC::S_OFFSET), idesc, 1u);
          tc::mma_commit_warp(&a_empty[ar.slot]);
          ar.advance();
        }
        if (!ok) break;
        tc::mma_commit_warp(&done[cr.slot]);
        cr.advance();
      }
    }
  } else if (warp < DEQUANT_WARPS) {
    // ---- dequant warps: lane quarter warp % 4, half chunk warp / 4 ----
    const int quarter = warp % 4, half = warp / 4;
    const int row_in_tile = quarter * 32 + lane;
    const uint32_t lane_base = uint32_t(quarter * 32) << 16;
    Ring<WS> wr;
    Ring<3> ar;  // this warp's half chunks are every other one
    Ring<3> cr;  // the chunk: its ready / half1 slot and min tile
    ar.advance(half);
    int gc = 0;
    bool ok = true;
    for (int u = blockIdx.x; ok && u < units; u += gridDim.x) {
      const int c1 = plan.chunk_end(u);
      for (int c = plan.chunk_begin(u); ok && c < c1; ++c, ++gc) {
        if (!(ok = wait_warp(&w_full[wr.slot], wr.phase, abort, error))) break;
        if (2 * gc + half >= 3 &&
            !(ok = wait_warp(&a_empty[ar.slot], ar.phase ^ 1u, abort, error)))
          break;
        // the min tile's last chunk, gc - 3, is done
        if (SUMS && gc >= 3 && !(ok = wait_warp(&done[cr.slot], cr.phase ^ 1u, abort, error)))
          break;
        tc::fence_after_sync();
        const uint8_t* raw_row =
            smem + wr.slot * L::RAW_PADDED + row_in_tile * Unpack<T>::PITCH_WORDS * 4;
        uint32_t mins[2];
        dequant_half<T>(half, raw_row, tmem + lane_base + 128 + 128 * ar.slot, mins);
        __syncwarp();
        if (lane == 0) tc::mbar_arrive(&w_empty[wr.slot]);  // the raw weights are used
        wr.advance();
        if (SUMS) {
          // the four blocks' min terms at K 4h.. and 8 + 4h.. of the chunk's
          // min tile row
          uint8_t* tile = smem + L::M_OFFSET + cr.slot * M_TILE_BYTES;
          const uint2 pair = make_uint2(mins[0], mins[1]);
          *reinterpret_cast<uint2*>(tile + interleave_offset(row_in_tile, 4 * half)) = pair;
          *reinterpret_cast<uint2*>(tile + interleave_offset(row_in_tile, 8 + 4 * half)) = pair;
          asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
        }
        tc::tmem_store_wait();
        tc::fence_before_sync();
        __syncwarp();
        if (lane == 0) tc::mbar_arrive(half == 0 ? &ready[cr.slot] : &half1[cr.slot]);
        ar.advance(2);
        cr.advance();
      }
    }
  } else if (warp < FIRST_EPILOGUE + EPILOGUE_WARPS) {
    // ---- epilogue warps: each chunk's accumulator (lane quarter warp % 4,
    // all 64 vectors) into the unit's running sums, then the unit's output ----
    const int quarter = warp % 4;
    const int row_in_tile = quarter * 32 + lane;
    const uint32_t lane_base = uint32_t(quarter * 32) << 16;
    float sum[TILE_VECTORS];
#pragma unroll
    for (int i = 0; i < TILE_VECTORS; ++i) sum[i] = 0.0f;
    // both accumulators start empty: chunks 0 and 1 may start
    if (lane == 0) {
      tc::mbar_arrive(&ready[0]);
      tc::mbar_arrive(&ready[1]);
    }
    Ring<3> cr;
    int gc = 0;
    bool ok = true;
    for (int u = blockIdx.x; ok && u < units; u += gridDim.x) {
      const int c0 = plan.chunk_begin(u), c1 = plan.chunk_end(u);
      for (int c = c0; ok && c < c1; ++c, ++gc) {
        if (!(ok = wait_warp(&done[cr.slot], cr.phase, abort, error))) break;
        tc::fence_after_sync();
        const uint32_t at = tmem + lane_base + 64 * (gc & 1);
#pragma unroll
        for (int part = 0; part < 2; ++part) {
          uint32_t v[32];
          tmem_load_32_nowait(at + 32 * part, v);
          asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
          if (part == 1) {
            // the accumulator is free for chunk gc + 2
            tc::fence_before_sync();
            __syncwarp();
            if (lane == 0) tc::mbar_arrive(&ready[(cr.slot + 2) % 3]);
          }
          if (c == c0) {
#pragma unroll
            for (int i = 0; i < 32; ++i) sum[32 * part + i] = __uint_as_float(v[i]);
          } else {
#pragma unroll
            for (int i = 0; i < 32; ++i)
              sum[32 * part + i] = __fadd_rn(sum[32 * part + i], __uint_as_float(v[i]));
          }
        }
        cr.advance();
      }
      if (!ok) break;
      // the unit's output: this thread's row, all 64 vectors of the pass
      const int tile = u / plan.splits;
      const int rt = tile % plan.row_tiles, pass = tile / plan.row_tiles;
      const int row = rt * TILE_ROWS + row_in_tile;
      const int v0 = pass * TILE_VECTORS;
      if (plan.splits == 1) {
        if (row < rows) {
#pragma unroll
          for (int i = 0; i < TILE_VECTORS; ++i)
            if (v0 + i < vectors)
              y[(long long)(v0 + i) * rows + row] = __fmul_rn(sum[i], __ldg(scales + v0 + i));
        }
        continue;
      }
      // A K-range: leave this warp's slice of the partial sum (32 rows x 64
      // vectors); the warp that brings a slice's last range adds the ranges
      // in K order. Slices are counted apart, so no warp waits for another.
      const int split = u % plan.splits;
      float* mine =
          scratch.partial + ((long long)tile * plan.splits + split) * TILE_VECTORS * TILE_ROWS;
#pragma unroll
      for (int i = 0; i < TILE_VECTORS; ++i) mine[i * TILE_ROWS + row_in_tile] = sum[i];
      __threadfence();
      __syncwarp();
      int arrived = 0;
      if (lane == 0) arrived = atomicAdd(&scratch.arrivals[tile * EPILOGUE_WARPS + quarter], 1);
      arrived = __shfl_sync(0xffffffffu, arrived, 0);
      if (arrived == plan.splits - 1) {
        // every range's slice, this one's included, read back in K order: a
        // whole range's 64 loads in flight at a time
        __threadfence();
#pragma unroll
        for (int i = 0; i < TILE_VECTORS; ++i) sum[i] = 0.0f;
        for (int k = 0; k < plan.splits; ++k) {
          const float* part =
              scratch.partial + ((long long)tile * plan.splits + k) * TILE_VECTORS * TILE_ROWS;
#pragma unroll
          for (int i = 0; i < TILE_VECTORS; ++i)
            sum[i] = __fadd_rn(sum[i], __ldcg(part + i * TILE_ROWS + row_in_tile));
        }
        if (row < rows) {
#pragma unroll
          for (int i = 0; i < TILE_VECTORS; ++i)
            if (v0 + i < vectors)
              y[(long long)(v0 + i) * rows + row] = __fmul_rn(sum[i], __ldg(scales + v0 + i));
        }
      }
    }
  }
  __syncthreads();
  if (warp == 0) {
    tc::fence_after_sync();
    tc::tmem_dealloc(tmem, TMEM_COLUMNS);
  }
}

// (BF16 x: one x term; F32 x: two)
#define DRIFT_TC_REGISTER(name, T)                                \
  DRIFT_REGISTER(linear_tc_##name, (linear_tc_kernel<T, false>)) \
  DRIFT_REGISTER(linear_tc_split_x_##name, (linear_tc_kernel<T, true>))
DRIFT_TC_REGISTER(q8_0, Q8_0T)
DRIFT_TC_REGISTER(q4_0, Q4_0T)
DRIFT_TC_REGISTER(q4_1, Q4_1T)

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

template <typename T, bool XSPLIT>
static int launch_tc(int x_dtype, const void* x, const void* weight, float* y, int64_t m,
                     int64_t n, int64_t k, uint8_t* workspace, cudaStream_t stream) {
  using L = TcLayout<T, XSPLIT>;
  using XC = typename L::XC;
  const int sms = sm_count();
  const int64_t padded = (m + TILE_VECTORS - 1) / TILE_VECTORS * TILE_VECTORS;
  TcPlan plan;
  plan.row_tiles = int((n + TILE_ROWS - 1) / TILE_ROWS);
  plan.tiles = plan.row_tiles * int(padded / TILE_VECTORS);
  plan.chunks = int((k + CHUNK - 1) / CHUNK);
  plan.splits = choose_splits(plan.tiles, plan.chunks, sms);
  // [staged x][scales: a float a padded vector][partial sums][arrival counters]
  const size_t x_bytes = size_t(padded / TILE_VECTORS) * plan.chunks * XC::BYTES;
  float* scales = reinterpret_cast<float*>(workspace + x_bytes);
  TcScratch scratch;
  scratch.partial = scales + padded;
  scratch.arrivals = reinterpret_cast<int*>(
      reinterpret_cast<uint8_t*>(scratch.partial) +
      (plan.splits > 1 ? size_t(plan.tiles) * plan.splits * TILE_VECTORS * TILE_ROWS * 4 : 0));
  {
    const dim3 grid(unsigned(padded), unsigned((plan.chunks + PREP_CHUNKS - 1) / PREP_CHUNKS));
    const int counters = plan.splits > 1 ? plan.tiles * EPILOGUE_WARPS : 0;
    if (x_dtype == DRIFT_BF16)
      DRIFT_CUDA(launch_pdl(tc_prepare_x_kernel<T, true, XSPLIT>, grid, PREP_THREADS, 0, stream,
                            x, workspace, scales, int(m), int(k), plan.chunks, scratch.arrivals,
                            counters));
    else
      DRIFT_CUDA(launch_pdl(tc_prepare_x_kernel<T, false, XSPLIT>, grid, PREP_THREADS, 0, stream,
                            x, workspace, scales, int(m), int(k), plan.chunks, scratch.arrivals,
                            counters));
  }
  const int64_t row_bytes = k / 32 * T::BYTES;
  CUtensorMap wmap;
  DRIFT_TRY(encode_word_rows(&wmap, weight, row_bytes / 4, n, Unpack<T>::PITCH_WORDS, TILE_ROWS));
  static PerDevice configured;
  DRIFT_TRY(ensure_shared_memory(configured, linear_tc_kernel<T, XSPLIT>, L::SMEM_BYTES));
  const long long units = (long long)plan.tiles * plan.splits;
  const int grid = units < sms ? int(units) : sms;
  DRIFT_CUDA(launch_pdl(linear_tc_kernel<T, XSPLIT>, grid, TC_THREADS, L::SMEM_BYTES, stream, wmap,
                        reinterpret_cast<const uint8_t*>(workspace), scales, y, int(n), int(m),
                        plan, scratch, device_error_word()));
  return 0;
}

// BF16 x is exact in one F16 term; F32 x takes two.
template <typename T>
static int launch_tc_x(int x_dtype, const void* x, const void* weight, float* y, int64_t m,
                       int64_t n, int64_t k, uint8_t* workspace, cudaStream_t stream) {
  if (x_dtype == DRIFT_BF16)
    return launch_tc<T, false>(x_dtype, x, weight, y, m, n, k, workspace, stream);
  return launch_tc<T, true>(x_dtype, x, weight, y, m, n, k, workspace, stream);
}

}  // namespace

// Bytes of scratch a tensor-core product of m rows of k (new) needs at most:
// the staged x (whole chunks, both terms and the block sums), a scale per
// vector, and for split products the partial sums (at most 4 units per SM)
// and the counters.
size_t tc_workspace_bytes(int64_t m, int64_t k) {
  const size_t passes = size_t((m + TILE_VECTORS - 1) / TILE_VECTORS);
  const size_t chunks = size_t((k + CHUNK - 1) / CHUNK);
  const size_t units = size_t(4) * size_t(sm_count());  // split tiles are at most half that
  return passes * chunks * X_CHUNK_MAX + passes * TILE_VECTORS * 4 +
         units * TILE_VECTORS * TILE_ROWS * 4 + units * EPILOGUE_WARPS * 4 + 256;
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

// `workspace`: tc_workspace_bytes(m, k) bytes of device scratch, 256-byte aligned.
int linear_tc(int x_dtype, const void* x, int weight_dtype, const void* weight, float* y,
              int64_t m, int64_t n, int64_t k, uint8_t* workspace, cudaStream_t stream) {
  switch (weight_dtype) {
    case DRIFT_Q8_0: return launch_tc_x<Q8_0T>(x_dtype, x, weight, y, m, n, k, workspace, stream);
    case DRIFT_Q4_0: return launch_tc_x<Q4_0T>(x_dtype, x, weight, y, m, n, k, workspace, stream);
    default: return launch_tc_x<Q4_1T>(x_dtype, x, weight, y, m, n, k, workspace, stream);
  }
}

}  // namespace drift
