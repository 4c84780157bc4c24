// Row-wise device helpers shared by the layer kernels (layers.cu), the
// attention inputs (attention.cu) and the whole-mixture launch (experts.cu):
// the same arithmetic everywhere, so a fused kernel gives the bits of the
// kernels it replaces.
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

// ---- thread-block clusters ------------------------------------------------------------
// Every CTA of the cluster past this point sees the others' shared memory
// writes from before it.
__device__ __forceinline__ void cluster_sync() {
  asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;"
               ::: "memory");
}
// `local`'s float in the shared memory of the cluster's CTA `rank`.
__device__ __forceinline__ float cluster_load(const float* local, unsigned rank) {
  uint32_t address = static_cast<uint32_t>(__cvta_generic_to_shared(local)), remote;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(remote) : "r"(address), "r"(rank));
  float value;
  asm volatile("ld.shared::cluster.f32 %0, [%1];" : "=f"(value) : "r"(remote) : "memory");
  return value;
}
__device__ __forceinline__ unsigned cluster_rank() {
  unsigned rank;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(rank));
  return rank;
}

// ---- products with F32 weights -------------------------------------------------------------
// (routers, DeltaNet's a and b; matvec_f32_kernel in layers.cu, and the
// whole-mixture launch in experts.cu): a CTA of 256 threads per (row,
// vector), the row in 16-byte loads, every load of a thread issued before
// its first use (a 4096-value row is one round trip), summed per thread in
// column order, then the block's fixed tree. `weight` is the matrix's first
// row (whose alignment picks the path, so a row sums the same way in either
// kernel), w the row's.
template <bool BF16>
__device__ __forceinline__ float f32_row_dot(const void* __restrict__ x,
                                             const float* __restrict__ weight,
                                             const float* __restrict__ w, int vector, int k,
                                             float* partial) {
  float sum = 0.0f;
  if (!BF16 && k % 4 == 0 && (reinterpret_cast<uintptr_t>(weight) & 15) == 0 &&
      (reinterpret_cast<uintptr_t>(x) & 15) == 0) {
    const float4* w4 = reinterpret_cast<const float4*>(w);
    const float4* x4 = reinterpret_cast<const float4*>(reinterpret_cast<const float*>(x) +
                                                       (long long)vector * k);
    const int quads = k / 4;
    for (int base = 0; base < quads; base += 4 * 256) {
      float4 wv[4], xv[4];
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        const int q = base + u * 256 + threadIdx.x;
        wv[u] = q < quads ? __ldg(w4 + q) : make_float4(0.f, 0.f, 0.f, 0.f);
        xv[u] = q < quads ? x4[q] : make_float4(0.f, 0.f, 0.f, 0.f);
      }
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        sum = fmaf(wv[u].x, xv[u].x, sum);
        sum = fmaf(wv[u].y, xv[u].y, sum);
        sum = fmaf(wv[u].z, xv[u].z, sum);
        sum = fmaf(wv[u].w, xv[u].w, sum);
      }
    }
  } else {
    for (int c = threadIdx.x; c < k; c += 256) {
      const float xv =
          BF16 ? __uint_as_float(uint32_t(reinterpret_cast<const uint16_t*>(x)[(long long)vector * k + c]) << 16)
               : reinterpret_cast<const float*>(x)[(long long)vector * k + c];
      sum = fmaf(w[c], xv, sum);
    }
  }
  return block_sum(sum, partial);
}

// ---- activations ----------------------------------------------------------------------------
// Activation codes of ops/Activation.scala:5-19 (expf and tanhf called, as the
// runner's own kernels call them, elementwise.hip:31-42).
__device__ __forceinline__ float activate(float v, int kind) {
  switch (kind) {
    case DRIFT_SILU: return v / (1.0f + expf(-v));
    case DRIFT_GELU_TANH: {
      const float inner = 0.7978845608028654f * (v + 0.044715f * v * v * v);
      return 0.5f * v * (1.0f + tanhf(inner));
    }
    case DRIFT_GELU_ERF: return 0.5f * v * (1.0f + erff(v * 0.7071067811865476f));
    case DRIFT_SIGMOID: return 1.0f / (1.0f + expf(-v));
    default: return 4.0f * tanhf(v * 0.25f) / (1.0f + expf(-v));
  }
}

// The up half of a gated activation: SiTU-GLU bounds it, 25 tanh(up / 25).
__device__ __forceinline__ float gated_up(float up, int kind) {
  return kind == DRIFT_SITU ? 25.0f * tanhf(up * 0.04f) : up;
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

// The same turn with mRoPE sections (ops/Rope.scala:12-35, CpuAttention.rope:
// ops/CpuAttention.scala:92-146): pair i takes positions[section * tokens + t]
// where `sections` is 0 (one position a token), 1 (contiguous: s0 temporal,
// s1 height pairs, the rest width), 2 (interleaved: height when i % 3 == 1
// and i < 3 s1, width when i % 3 == 2 and i < 3 s2, else temporal) or 3
// (axes: s0..s3 pairs in turn, axis a's pair j of n turning by theta^(-j/n)).
__device__ __forceinline__ float rope_turn_sections(const float* head, int d,
                                                    const int* positions, int t, int tokens,
                                                    float theta, int rotary, int layout,
                                                    int sections, int s0, int s1, int s2,
                                                    int s3) {
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
  int section = 0;
  double exponent = __ddiv_rn(2.0 * pair, double(rotary));
  if (sections == 1) {
    section = pair < s0 ? 0 : (pair < s0 + s1 ? 1 : 2);
  } else if (sections == 2) {
    section = (pair % 3 == 1 && pair < 3 * s1) ? 1 : ((pair % 3 == 2 && pair < 3 * s2) ? 2 : 0);
  } else if (sections == 3) {
    const int sizes[4] = {s0, s1, s2, s3};
    int start = 0;
    section = 3;
    for (int a = 0; a < 4; ++a) {
      if (pair < start + sizes[a]) {
        section = a;
        break;
      }
      start += sizes[a];
    }
    if (section == 3 && pair >= start + s3) start -= s3;  // past every axis: the last one's
    exponent = __ddiv_rn(double(pair - start), double(sizes[section]));
  }
  const float power = float(pow(double(theta), exponent));
  const float inverse = __fdiv_rn(1.0f, power);
  const float angle = __fmul_rn(float(positions[(long long)section * tokens + t]), inverse);
  double s, c;
  sincos(double(angle), &s, &c);
  const double a = first ? double(head[d]) : double(head[partner]);
  const double b = first ? double(head[partner]) : double(head[d]);
  const double value = first ? __dsub_rn(__dmul_rn(a, c), __dmul_rn(b, s))
                             : __dadd_rn(__dmul_rn(a, s), __dmul_rn(b, c));
  return float(value);
}

}  // namespace drift
