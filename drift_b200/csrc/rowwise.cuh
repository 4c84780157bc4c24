// Row-wise device helpers shared by the layer kernels (layers.cu) and the
// fused attention inputs (attention.cu): the same arithmetic in both, so a
// fused kernel gives the bits of the kernels it replaces.
#pragma once

#include "common.cuh"

namespace drift {

// ---- block reductions -------------------------------------------------------------------
// The sum over a block of `blockDim.x` threads (a multiple of 32): warps by
// shuffles, then the warps' sums in warp order. Every thread gets it.
__device__ __forceinline__ float block_sum(float value, float* partial) {
#pragma unroll
  for (int o = 16; o > 0; o /= 2) value += __shfl_xor_sync(0xffffffffu, value, o);
  const int warp = threadIdx.x / WARP, warps = blockDim.x / WARP;
  if (threadIdx.x % WARP == 0) partial[warp] = value;
  __syncthreads();
  float total = 0.0f;
  for (int w = 0; w < warps; ++w) total += partial[w];
  __syncthreads();  // partial is reused by the next reduction
  return total;
}

// ---- rotary embedding ---------------------------------------------------------------------
// Value d of a head after the turn: the angle is the CPU reference's to the
// bit -- the inverse frequency 1f / (float) pow(theta, 2 pair / rotary) (pow
// in double, then float), times float(position) in float -- and the turn is in
// double, as CpuAttention.rope turns it, rounded once. Values past `rotary`
// pass through.
__device__ __forceinline__ float rope_turn(const float* head, int d, int position, float theta,
                                           int rotary, int layout) {
  if (d >= rotary) return head[d];
  const int half = rotary / 2;
  int pair, partner;
  bool first;
  if (layout == DRIFT_ROPE_NEOX) {
    pair = d % half;
    first = d < half;
    partner = first ? d + half : d - half;
  } else {
    pair = d / 2;
    first = d % 2 == 0;
    partner = first ? d + 1 : d - 1;
  }
  const float power = float(pow(double(theta), __ddiv_rn(2.0 * pair, double(rotary))));
  const float inverse = __fdiv_rn(1.0f, power);
  const float angle = __fmul_rn(float(position), inverse);
  double s, c;
  sincos(double(angle), &s, &c);
  const double a = first ? double(head[d]) : double(head[partner]);
  const double b = first ? double(head[partner]) : double(head[d]);
  const double value = first ? __dsub_rn(__dmul_rn(a, c), __dmul_rn(b, s))
                             : __dadd_rn(__dmul_rn(a, s), __dmul_rn(b, c));
  return float(value);
}

}  // namespace drift
