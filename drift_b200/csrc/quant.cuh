// Device-side GGML block access for Q8_0, Q4_0 and Q4_1, and the prepared-x
// record the products meet them with.
//
// Block layouts (runner/src/drift/runner/tensor/GgmlQuants.scala:11-118):
//   Q8_0  34 bytes: f16 d, 32 int8 codes; value j = code_j * d
//   Q4_0  18 bytes: f16 d, 16 bytes of nibbles; value j = d * (q_j - 8)
//   Q4_1  20 bytes: f16 d, f16 m, 16 bytes of nibbles; value j = d * q_j + m
// where q_j is the low nibble of byte j for j < 16 and the high nibble of
// byte j - 16 after.
//
// A row of [N, K] is K/32 blocks, rows one after the other. Rows are whole
// 4-byte words (the runner refuses others: ops/HipLinear.scala:126-131), so
// every block's bytes lie in the 4-byte aligned words that cover it, and those
// words never reach past the row: Q8_0 and Q4_0 blocks alternate between
// 4-byte and 2-byte alignment, and with an even block count the last one is
// the 2-byte aligned kind, which ends on a word boundary.
#pragma once

#include <cuda_fp16.h>
#include <stdint.h>

#include "../../include/drift_ops.h"

namespace drift {

// ---- prepared x ---------------------------------------------------------------
// The products take x as exact integers per 32-value block: X_j =
// rint(x_j * 2^(21 - e)) with 2^e > max|x| over the block, so |X_j| <= 2^21
// and x_j = s * X_j up to s/2, s = 2^(e - 21): 21 bits below the block's
// largest value, some 10^4 times finer than the runner's own int8 x path
// (kernels/quantize.h:6-25, max|x|/127). X is split into three byte planes
// X = P0 + 256 P1 + 65536 P2 (P0, P1 unsigned, P2 signed) that dp4a meets
// four at a time with the weights' integer codes; the code-times-plane sums
// are exact, so the only rounding is of x to s and the float epilogue. The
// records' layout (eight vectors to a 896-byte record per block, one slot
// each) is mma_i8.cuh's; s is NaN when the block holds a NaN or infinity.
constexpr int X_BITS = 21;

// ---- dp4a in the four signednesses ----------------------------------------------
__device__ __forceinline__ int dp4a_uu(uint32_t a, uint32_t b, int c) {
  uint32_t d;
  asm("dp4a.u32.u32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(c));
  return int(d);
}
__device__ __forceinline__ int dp4a_us(uint32_t a, uint32_t b, int c) {
  int d;
  asm("dp4a.u32.s32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(c));
  return d;
}
__device__ __forceinline__ int dp4a_su(uint32_t a, uint32_t b, int c) {
  int d;
  asm("dp4a.s32.u32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(c));
  return d;
}
__device__ __forceinline__ int dp4a_ss(uint32_t a, uint32_t b, int c) {
  int d;
  asm("dp4a.s32.s32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(c));
  return d;
}

__device__ __forceinline__ float half_bits_to_float(uint32_t bits) {
  return __half2float(__ushort_as_half((unsigned short)(bits & 0xffffu)));
}

// A read-only 4-byte load that does not keep the line in L1 for long: each
// weight byte is read once.
__device__ __forceinline__ uint32_t load_stream(const uint32_t* p) {
  uint32_t v;
  asm volatile("ld.global.nc.L1::no_allocate.b32 %0, [%1];" : "=r"(v) : "l"(p));
  return v;
}

// A decoded block as the products use it: eight words of codes, word i holding
// the codes of values 4i..4i+3 in its bytes (unsigned nibbles for the Q4
// types, signed bytes for Q8_0), and the block's d and m.
struct Codes {
  uint32_t q[8];
  float d, m;
};

struct Q8_0T {
  static constexpr int DTYPE = DRIFT_Q8_0;
  static constexpr int BYTES = 34;
  static constexpr int WORDS = 9;  // the aligned words that cover a block
  static constexpr bool SIGNED = true;
  static constexpr const char* NAME = "q8_0";

  __device__ static Codes decode(const uint32_t (&w)[WORDS], int block) {
    Codes c;
    const int off = (block * BYTES) & 3;  // 0 or 2
    c.d = half_bits_to_float(__funnelshift_r(w[0], w[1], off * 8));
    c.m = 0.0f;
    const int shift = (off + 2) * 8;  // the codes start 2 bytes in: 16 or 32 bits
#pragma unroll
    for (int i = 0; i < 8; ++i) c.q[i] = __funnelshift_rc(w[i], w[i + 1], shift);
    return c;
  }
  // Value j of a block, exactly as the CPU decode computes it (int8 * d is
  // exact in float).
  __device__ static float value(const Codes& c, int j) {
    return float(int8_t(c.q[j >> 2] >> (8 * (j & 3)))) * c.d;
  }
};

struct Q4_0T {
  static constexpr int DTYPE = DRIFT_Q4_0;
  static constexpr int BYTES = 18;
  static constexpr int WORDS = 5;
  static constexpr bool SIGNED = false;
  static constexpr const char* NAME = "q4_0";

  __device__ static Codes decode(const uint32_t (&w)[WORDS], int block) {
    Codes c;
    const int off = (block * BYTES) & 3;
    c.d = half_bits_to_float(__funnelshift_r(w[0], w[1], off * 8));
    c.m = 0.0f;
    const int shift = (off + 2) * 8;
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const uint32_t raw = __funnelshift_rc(w[i], w[i + 1], shift);
      c.q[i] = raw & 0x0F0F0F0Fu;
      c.q[i + 4] = (raw >> 4) & 0x0F0F0F0Fu;
    }
    return c;
  }
  // d * (q - 8): one float product, exact.
  __device__ static float value(const Codes& c, int j) {
    return c.d * float(int((c.q[j >> 2] >> (8 * (j & 3))) & 0xffu) - 8);
  }
};

struct Q4_1T {
  static constexpr int DTYPE = DRIFT_Q4_1;
  static constexpr int BYTES = 20;
  static constexpr int WORDS = 5;
  static constexpr bool SIGNED = false;
  static constexpr const char* NAME = "q4_1";

  __device__ static Codes decode(const uint32_t (&w)[WORDS], int) {
    Codes c;
    c.d = half_bits_to_float(w[0]);
    c.m = half_bits_to_float(w[0] >> 16);
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      c.q[i] = w[i + 1] & 0x0F0F0F0Fu;
      c.q[i + 4] = (w[i + 1] >> 4) & 0x0F0F0F0Fu;
    }
    return c;
  }
  // d * q + m as the CPU decode does it: the product rounded, then the sum
  // rounded (no fused multiply-add), so gathers are bit for bit the CPU's.
  __device__ static float value(const Codes& c, int j) {
    const float q = float((c.q[j >> 2] >> (8 * (j & 3))) & 0xffu);
    return __fadd_rn(__fmul_rn(c.d, q), c.m);
  }
};

// Bytes [OFF, END) of a 16-byte aligned row in shared memory, as words, by the
// widest aligned loads (OFF and END multiples of 8).
template <int OFF, int END>
__device__ __forceinline__ void lds_span(const uint8_t* row, uint32_t* w) {
  if constexpr (OFF < END) {
    if constexpr (OFF % 16 == 0 && OFF + 16 <= END) {
      const uint4 q = *reinterpret_cast<const uint4*>(row + OFF);
      w[0] = q.x;
      w[1] = q.y;
      w[2] = q.z;
      w[3] = q.w;
      lds_span<OFF + 16, END>(row, w + 4);
    } else {
      const uint2 q = *reinterpret_cast<const uint2*>(row + OFF);
      w[0] = q.x;
      w[1] = q.y;
      lds_span<OFF + 8, END>(row, w + 2);
    }
  }
}

// The aligned words covering block `block` of a row that starts at `row`
// (4-byte aligned).
template <typename T>
__device__ __forceinline__ void load_block(const uint8_t* row, int block, uint32_t (&w)[T::WORDS]) {
  const uint32_t* p = reinterpret_cast<const uint32_t*>(row + ((block * T::BYTES) & ~3));
#pragma unroll
  for (int i = 0; i < T::WORDS; ++i) w[i] = load_stream(p + i);
}

// The three plane sums of one block's codes against one x record:
// a0 = sum q * P0, a1 = sum q * P1, a2 = sum q * P2, each exact.
template <typename T>
__device__ __forceinline__ void plane_sums(const Codes& c, const uint32_t* planes, int& a0, int& a1,
                                           int& a2) {
  a0 = a1 = a2 = 0;
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    if (T::SIGNED) {
      a0 = dp4a_su(c.q[i], planes[i], a0);
      a1 = dp4a_su(c.q[i], planes[8 + i], a1);
      a2 = dp4a_ss(c.q[i], planes[16 + i], a2);
    } else {
      a0 = dp4a_uu(c.q[i], planes[i], a0);
      a1 = dp4a_uu(c.q[i], planes[8 + i], a1);
      a2 = dp4a_us(c.q[i], planes[16 + i], a2);
    }
  }
}

// One block's contribution to a row's sum for one vector: sum_j w_j * x_j with
// x_j = s * X_j. `sum_x` is sum_j X_j.
template <typename T>
__device__ __forceinline__ float block_dot(const Codes& c, int a0, int a1, int a2, float s,
                                           int sum_x) {
  if (T::DTYPE == DRIFT_Q8_0) {
    // |sum q X| can pass 2^31 for int8 codes: the planes join in float
    // (a0 < 2^24 exactly; a1 + 256 a2 < 2^26, rounded once).
    const float total = fmaf(256.0f, float(a1 + (a2 << 8)), float(a0));
    return s * c.d * total;
  } else if (T::DTYPE == DRIFT_Q4_0) {
    // sum (q - 8) X, |.| <= 736 * 2^21 < 2^31
    const int total = a0 + (a1 << 8) + (a2 << 16) - 8 * sum_x;
    return s * c.d * float(total);
  } else {
    // sum (d q + m) X = d sum q X + m sum X, |sum q X| <= 480 * 2^21 < 2^31
    const int total = a0 + (a1 << 8) + (a2 << 16);
    return s * fmaf(c.d, float(total), c.m * float(sum_x));
  }
}

}  // namespace drift
