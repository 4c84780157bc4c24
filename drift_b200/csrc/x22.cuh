// Writing x's records (the x22 planes of mma_i8.cuh) from the kernel that
// produces x: the step the reference's own norm and gated kernels take for
// the product that follows them (their xq/xd/xs outputs, runner/kernels/
// norm.hip:34-35, elementwise.hip:58-59), so that the product launches on
// prepared records with no preparation launch of its own.
#pragma once

#include <cuda_runtime.h>

#include "mma_i8.cuh"
#include "quant.cuh"

namespace drift {

// A warp's 32 values of one block (lane j holding value j) into one vector's
// 112-byte slot of a record (mma_i8.cuh): the same bytes the preparation
// kernel (matvec.cu) writes for the same values. All 32 lanes take part.
__device__ __forceinline__ void x22_record_slot(float value, uint8_t* slot) {
  const int lane = threadIdx.x % 32;
  // the largest magnitude by its bits (one warp reduction): an Inf or NaN
  // anywhere shows as bits of 0x7f800000 or more
  const unsigned top = __reduce_max_sync(0xffffffffu, __float_as_uint(fabsf(value)));
  int X = 0;
  float s = 0.0f;
  if (top >= 0x7f800000u) {
    s = __int_as_float(0x7fc00000);
  } else if (top >= (21u << 23)) {
    // top = 1.f x 2^(E - 127), E its biased exponent, so e = ilogb(top) + 1
    // = E - 126; s = 2^(e - 21) and the scaling by 2^(21 - e) are powers of
    // two made from their exponent bits (both normal for E >= 21): the same
    // values as ldexpf's, with no call
    static_assert(X_BITS == 21, "the exponent arithmetic below assumes 21 bits");
    const int E = int(top >> 23);
    s = __int_as_float((E - 20) << 23);
    X = __float2int_rn(value * __int_as_float((274 - E) << 23));
  } else if (top > 0) {
    const int e = ilogbf(__uint_as_float(top)) + 1;
    s = ldexpf(1.0f, e - X_BITS);
    X = __float2int_rn(ldexpf(value, X_BITS - e));
  }
  // value j = lane sits in byte j % 4 of word j / 4 of each plane
  const int w = lane / 4;
  slot[mma_plane_byte(0, 0, w) + lane % 4] = uint8_t(X & 0xff);
  slot[mma_plane_byte(0, 1, w) + lane % 4] = uint8_t((X >> 8) & 0xff);
  slot[mma_plane_byte(0, 2, w) + lane % 4] = uint8_t((X >> 16) & 0xff);
  const int sum = __reduce_add_sync(0xffffffffu, X);
  if (lane == 0) {
    uint8_t* scales = slot + mma_scale_byte(0);
    reinterpret_cast<float*>(scales)[0] = s;
    reinterpret_cast<int*>(scales)[1] = sum;
    reinterpret_cast<float*>(scales)[2] = float(sum);
  }
}

// The same for block `block` of vector v of `blocks`-block vectors, in the
// records' own layout (pass v / 8, slot v % 8).
__device__ __forceinline__ void x22_record_block(float value, uint8_t* records, int v, int block,
                                                 int blocks) {
  const int pass = v / 8, g = v % 8;
  x22_record_slot(value, records + ((long long)pass * blocks + block) * MMA_RECORD_BYTES +
                             MMA_SLOT_BYTES * g);
}

}  // namespace drift
