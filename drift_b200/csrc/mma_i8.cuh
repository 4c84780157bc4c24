// The integer tensor-core pieces of the 1-8 vector products, shared by the
// kernels that stream weights straight from global memory (matvec.cu) and
// those that stage them through shared memory (matvec_ring.cu).
#pragma once

#include <stdint.h>

#include "quant.cuh"

namespace drift {

// ---- 3 to 8 vectors: the same exact sums on the integer tensor cores -------------------------
// mma.sync m16n8k32 (8-bit in, 32-bit integer accumulate) meets a 16-row x
// 32-column tile of codes with the byte planes of 8 vectors: three MMAs per
// 32-block (planes 0, 1 unsigned, plane 2 signed), then the same float
// epilogue per block and output as block_dot. The fragment layouts line up
// with GGML's blocks: thread (g = lane / 4, t = lane % 4) holds columns
// 4t..4t+3 and 16+4t..16+4t+3 of rows g and g+8 -- word t of a Q4 block's
// nibbles, masked low and high -- and the same columns of vector g's planes.
template <bool SIGNED_A, bool SIGNED_B>
__device__ __forceinline__ void mma_i8(int (&d)[4], const uint32_t (&a)[4], uint32_t b0,
                                       uint32_t b1) {
  if (SIGNED_A && SIGNED_B)
    asm volatile(
        "mma.sync.aligned.m16n8k32.row.col.s32.s8.s8.s32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
        "{%0,%1,%2,%3};"
        : "+r"(d[0]), "+r"(d[1]), "+r"(d[2]), "+r"(d[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
  else if (SIGNED_A)
    asm volatile(
        "mma.sync.aligned.m16n8k32.row.col.s32.s8.u8.s32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
        "{%0,%1,%2,%3};"
        : "+r"(d[0]), "+r"(d[1]), "+r"(d[2]), "+r"(d[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
  else if (SIGNED_B)
    asm volatile(
        "mma.sync.aligned.m16n8k32.row.col.s32.u8.s8.s32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
        "{%0,%1,%2,%3};"
        : "+r"(d[0]), "+r"(d[1]), "+r"(d[2]), "+r"(d[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
  else
    asm volatile(
        "mma.sync.aligned.m16n8k32.row.col.s32.u8.u8.s32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
        "{%0,%1,%2,%3};"
        : "+r"(d[0]), "+r"(d[1]), "+r"(d[2]), "+r"(d[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

// ---- x for the integer tensor cores --------------------------------------------------
// The prepared x of up to 8 vectors (a pass), one 896-byte record per block:
// eight 112-byte slots, slot v holding vector v's part of the block (zeros for
// vectors past the pass), so one vector's x for a block is one 128-byte line
// -- what the one- and two-vector products read, for every block of a row:
//   slot bytes  0..95   plane p (0..2) at 32 p: its 8 words in the order
//                       0, 4, 1, 5, 2, 6, 3, 7, so the m16n8k32 B fragment of
//                       lane (g, t) -- words t and 4 + t, values 4t..4t+3 and
//                       16+4t..16+4t+3 -- is the 8 bytes at 8 t
//   slot bytes 96..107  s (float), sum_j X_j (int), the same sum as float
constexpr int MMA_SLOT_BYTES = 112;
constexpr int MMA_RECORD_BYTES = 8 * MMA_SLOT_BYTES;
// byte of plane p, word w (0..7) of vector v's slot
__host__ __device__ constexpr int mma_plane_byte(int v, int p, int w) {
  return MMA_SLOT_BYTES * v + 32 * p + 8 * (w % 4) + 4 * (w / 4);
}
__host__ __device__ constexpr int mma_scale_byte(int v) { return MMA_SLOT_BYTES * v + 96; }
constexpr int MMA_RECORD_WORDS = MMA_RECORD_BYTES / 4;

// The same product with a zero accumulator (no registers to clear first).
template <bool SIGNED_A, bool SIGNED_B>
__device__ __forceinline__ void mma_i8_zero(int (&d)[4], const uint32_t (&a)[4], uint32_t b0,
                                            uint32_t b1) {
  const int zero = 0;
  if (SIGNED_A && SIGNED_B)
    asm volatile(
        "mma.sync.aligned.m16n8k32.row.col.s32.s8.s8.s32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
        "{%10,%10,%10,%10};"
        : "=r"(d[0]), "=r"(d[1]), "=r"(d[2]), "=r"(d[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1), "r"(zero));
  else if (SIGNED_A)
    asm volatile(
        "mma.sync.aligned.m16n8k32.row.col.s32.s8.u8.s32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
        "{%10,%10,%10,%10};"
        : "=r"(d[0]), "=r"(d[1]), "=r"(d[2]), "=r"(d[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1), "r"(zero));
  else if (SIGNED_B)
    asm volatile(
        "mma.sync.aligned.m16n8k32.row.col.s32.u8.s8.s32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
        "{%10,%10,%10,%10};"
        : "=r"(d[0]), "=r"(d[1]), "=r"(d[2]), "=r"(d[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1), "r"(zero));
  else
    asm volatile(
        "mma.sync.aligned.m16n8k32.row.col.s32.u8.u8.s32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
        "{%10,%10,%10,%10};"
        : "=r"(d[0]), "=r"(d[1]), "=r"(d[2]), "=r"(d[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1), "r"(zero));
}

// A row's part of block `c` as this thread's fragment needs it: the codes of
// values 4t..4t+3 (lo) and 16+4t..16+4t+3 (hi), and the block's d and m.
// LOAD reads a word: __ldg for global memory, a plain load for shared.
struct GlobalWords {
  __device__ static uint32_t at(const uint32_t* p) { return __ldg(p); }
};
struct SharedWords {
  __device__ static uint32_t at(const uint32_t* p) { return *p; }
};

template <typename T, typename LOAD = GlobalWords>
__device__ __forceinline__ void fragment_row(const uint8_t* __restrict__ row, int c, int t,
                                             uint32_t& lo, uint32_t& hi, float& d, float& m) {
  const int start = c * T::BYTES;
  const uint32_t* words = reinterpret_cast<const uint32_t*>(row + (start & ~3));
  const int off = start & 3;  // 0, or 2 for the 2-byte aligned Q8_0 / Q4_0 blocks
  if (T::DTYPE == DRIFT_Q4_1) {
    const uint32_t head = LOAD::at(words);
    const uint32_t w = LOAD::at(words + 1 + t);
    d = half_bits_to_float(head);
    m = half_bits_to_float(head >> 16);
    lo = w & 0x0F0F0F0Fu;
    hi = (w >> 4) & 0x0F0F0F0Fu;
  } else if (T::DTYPE == DRIFT_Q4_0) {
    // nibbles start 2 bytes in: word t of them spans aligned words t, t+1
    // (off 0, shift 16) or is aligned word t+1 (off 2)
    const uint32_t head = LOAD::at(words);
    const uint32_t w0 = LOAD::at(words + t + (off >> 1)), w1 = LOAD::at(words + t + 1);
    const uint32_t w = off ? w1 : __funnelshift_r(w0, w1, 16);
    d = half_bits_to_float(off ? (head >> 16) : head);
    m = 0.0f;
    lo = w & 0x0F0F0F0Fu;
    hi = (w >> 4) & 0x0F0F0F0Fu;
  } else {
    const uint32_t head = LOAD::at(words);
    const uint32_t a0 = LOAD::at(words + t + (off >> 1)), a1 = LOAD::at(words + t + 1);
    const uint32_t b0 = LOAD::at(words + t + 4 + (off >> 1)), b1 = LOAD::at(words + t + 5);
    lo = off ? a1 : __funnelshift_r(a0, a1, 16);
    hi = off ? b1 : __funnelshift_r(b0, b1, 16);
    d = half_bits_to_float(off ? (head >> 16) : head);
    m = 0.0f;
  }
}

// x's fragment of one block for the m16n8k32 products: lane (g, t) holds
// vector g's plane words (t, t + 4) and s, sum for vectors 2t, 2t + 1.
struct XFragment {
  uint2 planes[3];
  float2 s, fsum;
  int2 sum;
};

template <typename T>
__device__ __forceinline__ void load_fragment(const uint8_t* rec, bool have_vector, XFragment& x) {
  const int lane = threadIdx.x % 32, g = lane / 4, t = lane % 4;
#pragma unroll
  for (int p = 0; p < 3; ++p)
    x.planes[p] = have_vector
                      ? __ldg(reinterpret_cast<const uint2*>(rec + mma_plane_byte(g, p, t)))
                      : make_uint2(0, 0);
  const uint8_t* s0 = rec + mma_scale_byte(2 * t);
  const uint8_t* s1 = rec + mma_scale_byte(2 * t + 1);
  x.s = make_float2(__ldg(reinterpret_cast<const float*>(s0)), __ldg(reinterpret_cast<const float*>(s1)));
  x.sum = T::DTYPE == DRIFT_Q4_0
              ? make_int2(__ldg(reinterpret_cast<const int*>(s0) + 1), __ldg(reinterpret_cast<const int*>(s1) + 1))
              : make_int2(0, 0);
  x.fsum = T::DTYPE == DRIFT_Q4_1 ? make_float2(__ldg(reinterpret_cast<const float*>(s0) + 2),
                                                __ldg(reinterpret_cast<const float*>(s1) + 2))
                                  : make_float2(0.0f, 0.0f);
}

// One output's share of a block before the x scale s: the three plane sums
// joined (exactly for the Q4 types, |sum| < 2^31; in float for Q8_0) and
// scaled by the block's d (and m). The caller adds s times it.
template <typename T>
__device__ __forceinline__ float mma_block_value(int p0, int p1, int p2, float d, float m,
                                                 int sum_x, float sum_x_float) {
  if (T::DTYPE == DRIFT_Q8_0) {
    return d * fmaf(256.0f, float(p1 + (p2 << 8)), float(p0));
  } else if (T::DTYPE == DRIFT_Q4_0) {
    return d * float(p0 + (p1 << 8) + (p2 << 16) - 8 * sum_x);
  } else {
    return fmaf(d, float(p0 + (p1 << 8) + (p2 << 16)), m * sum_x_float);
  }
}


}  // namespace drift
