// Mixtures of experts: top-k routing, the experts' products (plain and gated
// SwiGLU), and their weighted sum with the shared expert and the residual,
// optionally followed by the next RMS norm.
//
// Reference kernels: route_topk / route.h (kernels/linear_attention.hip:
// 274-281, route.h:9-41), matvec_experts[_gated]_<t> (matvec.hip:579-656),
// moe_combine (linear_attention.hip:286-297), moe_combine_norm (norm.hip:
// 43-59, combine.h:10-32); dispatch ops/HipExperts.scala. CPU twins:
// ops/CpuExperts.scala:11-106.
#include <cuda_runtime.h>

#include "common.cuh"
#include "mma_i8.cuh"
#include "quant.cuh"
#include "registry.cuh"
#include "rowwise.cuh"
#include "tc_common.cuh"
#include "x22.cuh"

namespace drift {

int* device_error_word();
int workspace_reserve(size_t bytes, void** pointer);
size_t mma_workspace_bytes(int64_t m, int64_t k);
int prepare_x_mma(int x_dtype, const void* x, int64_t m, int64_t k, uint8_t* records,
                  cudaStream_t stream);

// ---- routing ----------------------------------------------------------------------------
// One warp per token: the k largest of `experts` <= 512 logits, the lower
// expert first among equals, then their softmax among themselves in double
// (as CpuExperts.route computes it), rounded once. The logits are read
// through L2: in the whole-mixture launch other CTAs of the same launch
// wrote them.
__device__ __forceinline__ void route_token(const float* logits, int* __restrict__ ids,
                                            float* __restrict__ weights, int t, int experts,
                                            int k) {
  const int lane = threadIdx.x % WARP;
  const float* row = logits + (long long)t * experts;
  float v[16];
#pragma unroll
  for (int i = 0; i < 16; ++i) {
    const int e = lane + 32 * i;
    v[i] = e < experts ? __ldcg(row + e) : -INFINITY;
  }
  float chosen[16];
  int chosen_id[16];
  unsigned taken = 0;  // bit i: expert lane + 32 i is chosen already
  for (int j = 0; j < k; ++j) {
    float best = -INFINITY;
    int best_expert = 1 << 30;
#pragma unroll
    for (int i = 0; i < 16; ++i) {
      const int e = lane + 32 * i;
      if (e < experts && !((taken >> i) & 1u) &&
          (v[i] > best || (v[i] == best && e < best_expert))) {
        best = v[i];
        best_expert = e;
      }
    }
    // the warp's largest (value, then lowest expert) in two reductions: the
    // largest value by an order-keeping key (-0 folded into +0, which
    // compare equal; 0 for a lane with no candidate), then the lowest expert
    // among the lanes holding it; its value from its own lane
    unsigned key = 0;
    if (best_expert != (1 << 30)) {
      unsigned bits = __float_as_uint(best);
      if ((bits << 1) == 0) bits = 0;
      key = (bits & 0x80000000u) ? ~bits : (bits | 0x80000000u);
    }
    const unsigned top = __reduce_max_sync(0xffffffffu, key);
    best_expert = int(__reduce_min_sync(0xffffffffu, key == top ? unsigned(best_expert)
                                                                : unsigned(1 << 30)));
    best = top == 0 ? -INFINITY : __shfl_sync(0xffffffffu, best, best_expert & 31);
    chosen[j] = best;
    chosen_id[j] = best_expert;
    if ((best_expert & 31) == lane && best_expert < experts) taken |= 1u << (best_expert >> 5);
  }
  // the softmax over the chosen: lane j's exponential (every lane holds the
  // same chosen values), summed in slot order
  double mine = 0.0;
#pragma unroll
  for (int j = 0; j < 16; ++j)
    if (j == lane && j < k) mine = exp(double(chosen[j]) - double(chosen[0]));
  double e[16];
  double sum = 0.0;
#pragma unroll
  for (int j = 0; j < 16; ++j) {
    e[j] = __shfl_sync(0xffffffffu, mine, j);
    if (j < k) sum += e[j];
  }
  if (lane < k) {
    double ej = 0.0;
    int id = 0;
#pragma unroll
    for (int j = 0; j < 16; ++j)
      if (j == lane) {
        ej = e[j];
        id = chosen_id[j];
      }
    ids[(long long)t * k + lane] = id;
    weights[(long long)t * k + lane] = float(ej / sum);
  }
}

__global__ void __launch_bounds__(256) route_kernel(const float* __restrict__ logits,
                                                    int* __restrict__ ids,
                                                    float* __restrict__ weights, int tokens,
                                                    int experts, int k) {
  pdl_trigger();  // the next kernel may launch and wait for this one
  pdl_wait();     // what the kernels before this one wrote is visible
  const int t = blockIdx.x * (blockDim.x / WARP) + threadIdx.x / WARP;
  if (t >= tokens) return;
  route_token(logits, ids, weights, t, experts, k);
}

DRIFT_REGISTER(route_topk, route_kernel)

// ---- experts' products ---------------------------------------------------------------------
// Slot s (blockIdx.y) multiplies expert ids[s] of a [experts][rows][cols]
// weight with x row s / divisor -- or, past `routed_slots` (a shared expert's
// slots, one per x row), x row s - routed_slots -- prepared as for the plain
// product (the
// tensor-core layout: row v's part of block c is the 112-byte slot v % 8 of
// record (v / 8, c), its plane words in the order 0, 4, 1, 5, 2, 6, 3, 7).
// GATED: a gate and an up weight of the same shape, out = silu(gate . x) *
// (up . x). XQ (plain products, one x row a slot): each CTA prepares its
// slot's F32 x row itself, into shared memory (x22_record_slot: the bytes
// of the preparation launch it replaces), rather than read records. The 8
// warps of a CTA are 8 / KS row groups of KS k-splits: warp
// (group, kw) takes 4 rows of its group and, lane l, blocks 32 kw + l,
// 32 (kw + KS) + l, ...; the k-splits' sums meet in shared memory in a fixed
// order.
// One CTA's unit of the experts' products: row tile `tile` of slot `slot`
// (the kernel's blockIdx.x, blockIdx.y). `x_slots`: XQ's x in shared memory.
template <typename T, int KS, bool GATED, bool XQ>
__device__ __forceinline__ void experts_unit(
    const uint8_t* __restrict__ gate, const uint8_t* __restrict__ up, long long expert_bytes,
    const int* __restrict__ ids, const uint8_t* __restrict__ records, int divisor,
    int routed_slots, float* __restrict__ y, int rows, int cols, long long experts,
    long long first_expert, int others_zero, int* error, const float* __restrict__ x,
    int tile, int slot, uint8_t* x_slots) {
  constexpr int GROUPS = 8 / KS;
  constexpr int ROWS = 4;  // rows per warp
  __shared__ float partial[8][ROWS][2];
  const int warp = threadIdx.x / WARP, lane = threadIdx.x % WARP;
  const int kw = warp % KS, group = warp / KS;
  // the slot's expert in this weight (which holds experts [first_expert,
  // first_expert + experts)); with others_zero, a slot of another rank's
  // expert is zeros, not an error
  const long long expert = ids[slot] - first_expert;
  const int row0 = (tile * GROUPS + group) * ROWS;
  const int blocks = cols / 32;
  const int v = slot < routed_slots ? slot / divisor : slot - routed_slots;
  const uint8_t* record =
      XQ ? x_slots
         : records + (long long)(v / 8) * blocks * MMA_RECORD_BYTES + MMA_SLOT_BYTES * (v % 8);
  constexpr int STRIDE = XQ ? MMA_SLOT_BYTES : MMA_RECORD_BYTES;  // from one block to the next
  if (expert < 0 || expert >= experts) {
    if (!others_zero && threadIdx.x == 0 && blockIdx.x == 0 && error) atomicCAS(error, 0, 1);
    for (int r = threadIdx.x; r < GROUPS * ROWS; r += blockDim.x) {
      const int row = tile * GROUPS * ROWS + r;
      if (row < rows) y[(long long)slot * rows + row] = others_zero ? 0.0f : __int_as_float(0x7fc00000);
    }
    return;
  }
  // the warp's rows side by side: each block of x is read once for all of
  // them, and every row's weights of the block are in flight together; a
  // row's sum is its lane's blocks in order, then the warp's lanes. A
  // lane's first block's weights are asked for before x is prepared (XQ),
  // so the two waits overlap.
  const long long row_bytes = (long long)blocks * T::BYTES;
  const uint8_t* gate_base = gate + expert * expert_bytes;
  const uint8_t* up_base = up + expert * expert_bytes;
  uint32_t wg[ROWS][T::WORDS], wu[ROWS][T::WORDS];
  auto fetch = [&](int c) {
#pragma unroll
    for (int r = 0; r < ROWS; ++r) {
      const long long row = row0 + r < rows ? row0 + r : row0;
      load_block<T>(gate_base + row * row_bytes, c, wg[r]);
      if (GATED) load_block<T>(up_base + row * row_bytes, c, wu[r]);
    }
  };
  const int c0 = kw * WARP + lane;
  if (c0 < blocks) fetch(c0);
  if constexpr (XQ) {
    for (int c = warp; c < blocks; c += 8)
      x22_record_slot(x[(long long)v * cols + 32 * c + lane], x_slots + c * MMA_SLOT_BYTES);
    __syncthreads();
  }
  auto load = [](const uint4* a) {
    if constexpr (XQ) return *a;
    else return __ldg(a);
  };
  float g[ROWS], u[ROWS];
#pragma unroll
  for (int r = 0; r < ROWS; ++r) g[r] = u[r] = 0.0f;
  for (int c = c0; c < blocks; c += WARP * KS) {
    if (c != c0) fetch(c);
    const uint4* rec = reinterpret_cast<const uint4*>(record + (long long)c * STRIDE);
    // stored words 0..7 of a plane hold words 0, 4, 1, 5, 2, 6, 3, 7
    uint32_t planes[24];
#pragma unroll
    for (int p = 0; p < 3; ++p) {
      const uint4 q0 = load(rec + 2 * p), q1 = load(rec + 2 * p + 1);
      planes[8 * p + 0] = q0.x;
      planes[8 * p + 4] = q0.y;
      planes[8 * p + 1] = q0.z;
      planes[8 * p + 5] = q0.w;
      planes[8 * p + 2] = q1.x;
      planes[8 * p + 6] = q1.y;
      planes[8 * p + 3] = q1.z;
      planes[8 * p + 7] = q1.w;
    }
    const uint4 tail = load(rec + 6);  // s, sum X at bytes 96, 100
#pragma unroll
    for (int r = 0; r < ROWS; ++r) {
      int a0, a1, a2;
      const Codes cg = T::decode(wg[r], c);
      plane_sums<T>(cg, planes, a0, a1, a2);
      g[r] += block_dot<T>(cg, a0, a1, a2, __uint_as_float(tail.x), int(tail.y));
      if (GATED) {
        const Codes cu = T::decode(wu[r], c);
        plane_sums<T>(cu, planes, a0, a1, a2);
        u[r] += block_dot<T>(cu, a0, a1, a2, __uint_as_float(tail.x), int(tail.y));
      }
    }
  }
#pragma unroll
  for (int r = 0; r < ROWS; ++r) {
#pragma unroll
    for (int o = 16; o > 0; o /= 2) {
      g[r] += __shfl_xor_sync(0xffffffffu, g[r], o);
      if (GATED) u[r] += __shfl_xor_sync(0xffffffffu, u[r], o);
    }
  }
  if (lane == 0) {
#pragma unroll
    for (int r = 0; r < ROWS; ++r) {
      partial[warp][r][0] = g[r];
      partial[warp][r][1] = u[r];
    }
  }
  __syncthreads();
  const int t = threadIdx.x;
  if (t < GROUPS * ROWS) {
    const int gi = t / ROWS, r = t % ROWS;
    const int row = (tile * GROUPS + gi) * ROWS + r;
    if (row < rows) {
      float gs = 0.0f, us = 0.0f;
#pragma unroll
      for (int kk = 0; kk < KS; ++kk) {
        gs += partial[gi * KS + kk][r][0];
        us += partial[gi * KS + kk][r][1];
      }
      y[(long long)slot * rows + row] = GATED ? gs / (1.0f + expf(-gs)) * us : gs;
    }
  }
}

template <typename T, int KS, bool GATED, bool XQ = false>
__global__ void __launch_bounds__(256) experts_x22_kernel(
    const uint8_t* __restrict__ gate, const uint8_t* __restrict__ up, long long expert_bytes,
    const int* __restrict__ ids, const uint8_t* __restrict__ records, int divisor,
    int routed_slots, float* __restrict__ y, int rows, int cols, long long experts,
    long long first_expert, int others_zero, int* error, const float* __restrict__ x) {
  pdl_trigger();  // the next kernel may launch and wait for this one
  pdl_wait();     // what the kernels before this one wrote is visible
  extern __shared__ __align__(16) uint8_t x_slots[];  // XQ: [blocks][112 bytes]
  experts_unit<T, KS, GATED, XQ>(gate, up, expert_bytes, ids, records, divisor, routed_slots, y,
                                 rows, cols, experts, first_expert, others_zero, error, x,
                                 blockIdx.x, blockIdx.y, x_slots);
}

#define DRIFT_EXPERTS_REGISTER(T, name)                                                   \
  DRIFT_REGISTER(experts_x22_##name##_ks1, (experts_x22_kernel<T, 1, false>))             \
  DRIFT_REGISTER(experts_x22_##name##_ks2, (experts_x22_kernel<T, 2, false>))             \
  DRIFT_REGISTER(experts_x22_##name##_ks4, (experts_x22_kernel<T, 4, false>))             \
  DRIFT_REGISTER(experts_gated_x22_##name##_ks1, (experts_x22_kernel<T, 1, true>))        \
  DRIFT_REGISTER(experts_gated_x22_##name##_ks2, (experts_x22_kernel<T, 2, true>))        \
  DRIFT_REGISTER(experts_gated_x22_##name##_ks4, (experts_x22_kernel<T, 4, true>))
DRIFT_EXPERTS_REGISTER(Q8_0T, q8_0)
DRIFT_EXPERTS_REGISTER(Q4_0T, q4_0)
DRIFT_EXPERTS_REGISTER(Q4_1T, q4_1)

// ---- the experts' products, streamed through shared memory ----------------------------------
// The same products as experts_x22_kernel, bit for bit, for weights whose
// rows are whole 16-byte units. A launch's units are (slot, tile of 64 / KS
// rows), slot-major, a contiguous run of them a CTA (one CTA of 16 warps an
// SM). Thread 0 brings each unit's rows of the slot's expert -- and, gated,
// of its up weight -- into one of the stages by bulk copies (an expert's
// rows are contiguous), as many units ahead as there are stages, refilling a
// stage as soon as the CTA has left it. The 16 warps are 16 / KS row groups
// of KS k-splits, as experts_unit's 8: warp (group, kw) takes 4 rows and,
// lane l, blocks 32 kw + l, 32 (kw + KS) + l, ... (each block of x read once
// for the 4 rows); a row's k-splits meet in shared memory in order -- the
// arithmetic of experts_unit, so the bits are its. The slot's x records sit
// in shared memory too (copied, or made from the F32 row, once a slot). The
// copies keep bytes in flight while the warps compute; experts_x22_kernel is
// one round trip of 4-byte loads a CTA, then its sums.
constexpr int ES_WARPS = 16;
struct ExpertsStream {
  const uint8_t* gate;
  const uint8_t* up;
  long long expert_bytes;
  const int* ids;
  const uint8_t* records;
  int divisor, routed_slots;
  float* y;
  int rows, cols;
  long long experts, first_expert;
  int others_zero;
  int* error;
  const float* x;        // XQ: the slots' F32 x rows
  int tiles;             // units a slot
  int units, stage_bytes, stages;
};

__host__ __device__ constexpr int es_x_bytes(int blocks) { return (blocks * MMA_SLOT_BYTES + 127) / 128 * 128; }

// HALF (plain products of at most 16 blocks a row, KS = 1): a warp's two
// half-warps take a row each, 8 rows a warp in four passes, and a row's
// lanes meet by the tree of its half-warp -- the bits of the full warp's
// tree, in which the other half's lanes hold zeros (a lane's sum, 0 plus its
// block's, is never -0, so adding those zeros changes nothing).
template <typename T, int KS, bool GATED, bool XQ, bool HALF = false>
__global__ void __launch_bounds__(ES_WARPS * 32, 1) experts_stream_kernel(const __grid_constant__ ExpertsStream L) {
  static_assert(!HALF || (KS == 1 && !GATED), "half-warp rows: plain products, one k-split");
  constexpr int GROUPS = ES_WARPS / KS, ROWS = HALF ? 8 : 4, TILE = GROUPS * ROWS, MAX_STAGES = 4;
  pdl_trigger();  // the next kernel may launch and wait for this one
  pdl_wait();     // the ids and x are written (which weights to copy follows from the ids)
  extern __shared__ __align__(16) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 127) &
                                             ~uintptr_t(127));
  __shared__ float partial[2][ES_WARPS][ROWS][2];
  const int warp = threadIdx.x / WARP, lane = threadIdx.x % WARP;
  const int kw = warp % KS, group = warp / KS;
  const int blocks = L.cols / 32, S = L.stages;
  const long long row_bytes = (long long)blocks * T::BYTES;
  uint8_t* x_slot = smem + S * L.stage_bytes;  // the slot's x records
  uint64_t* full = reinterpret_cast<uint64_t*>(x_slot + es_x_bytes(blocks));
  volatile int* abort = reinterpret_cast<volatile int*>(full + MAX_STAGES);
  const int u0 = int((long long)L.units * blockIdx.x / gridDim.x);
  const int count = int((long long)L.units * (blockIdx.x + 1) / gridDim.x) - u0;
  if (threadIdx.x == 0) *abort = 0;
  if (threadIdx.x < S) tc::mbar_init(&full[threadIdx.x], 1);
  tc::fence_barrier_init();
  __syncthreads();

  auto expert_of = [&](int slot) { return (long long)L.ids[slot] - L.first_expert; };
  // unit j's rows into stage j mod S (thread 0); a slot of no expert here
  // copies nothing
  auto issue = [&](int j) {
    const int u = u0 + j, slot = u / L.tiles, tile = u % L.tiles, st = j % S;
    const long long e = expert_of(slot);
    if (e < 0 || e >= L.experts) {
      tc::mbar_arrive(&full[st]);
      return;
    }
    const int row0 = tile * TILE;
    const int n = L.rows - row0 < TILE ? L.rows - row0 : TILE;
    const uint32_t bytes = uint32_t(n * row_bytes);
    const long long at = e * L.expert_bytes + row0 * row_bytes;
    uint8_t* stage = smem + st * L.stage_bytes;
    tc::mbar_expect_tx(&full[st], GATED ? 2 * bytes : bytes);
    tc::bulk_load(stage, L.gate + at, bytes, &full[st]);
    if (GATED) tc::bulk_load(stage + TILE * row_bytes, L.up + at, bytes, &full[st]);
  };
  bool ok = true;
  int issued = 0;  // (thread 0's count)
  if (threadIdx.x == 0)
    for (; issued < S && issued < count; ++issued) issue(issued);
  int x_of = -1;  // the x row in x_slot
  for (int j = 0; j < count; ++j) {
    const int u = u0 + j, slot = u / L.tiles, tile = u % L.tiles;
    const int v = slot < L.routed_slots ? slot / L.divisor : slot - L.routed_slots;
    if (v != x_of) {
      // the slot's x records into shared memory, where every warp reads
      // them (read from global memory by every k-split's warps, they kept
      // the load queue full): XQ makes them from the F32 row
      // (x22_record_slot: the preparation launch's bytes), else they are
      // copied from the prepared records. Every warp has left the last
      // unit's x (the barrier at the end of each unit).
      if constexpr (XQ) {
        for (int c = warp; c < blocks; c += ES_WARPS)
          x22_record_slot(L.x[(long long)v * L.cols + 32 * c + lane], x_slot + c * MMA_SLOT_BYTES);
      } else {
        const uint8_t* from =
            L.records + (long long)(v / 8) * blocks * MMA_RECORD_BYTES + MMA_SLOT_BYTES * (v % 8);
        for (int i = threadIdx.x; i < blocks * (MMA_SLOT_BYTES / 16); i += blockDim.x) {
          const int c = i / (MMA_SLOT_BYTES / 16), part = i % (MMA_SLOT_BYTES / 16);
          *reinterpret_cast<uint4*>(x_slot + c * MMA_SLOT_BYTES + 16 * part) = __ldg(
              reinterpret_cast<const uint4*>(from + (long long)c * MMA_RECORD_BYTES + 16 * part));
        }
      }
      __syncthreads();
      x_of = v;
    }
    const long long e = expert_of(slot);
    const int row0 = tile * TILE;
    if (ok) ok = tc::mbar_wait_warp(&full[j % S], (j / S) & 1, abort, L.error);
    const bool valid = e >= 0 && e < L.experts;
    if (ok && valid) {
      const uint8_t* stage = smem + (j % S) * L.stage_bytes;
      const uint8_t* record = x_slot;
      constexpr int STRIDE = MMA_SLOT_BYTES;
      const uint8_t* wg = stage + group * ROWS * row_bytes;
      const uint8_t* wu = stage + (TILE + group * ROWS) * row_bytes;
      float g[ROWS], up[ROWS];
#pragma unroll
      for (int r = 0; r < ROWS; ++r) g[r] = up[r] = 0.0f;
      if constexpr (HALF) {
        // pass p: half-warp h takes row 2 p + h, lane its block lane % 16
        const int h = lane / 16, c = lane % 16;
        if (c < blocks) {
          const uint4* rec = reinterpret_cast<const uint4*>(record + (long long)c * STRIDE);
          uint32_t planes[24];
#pragma unroll
          for (int p = 0; p < 3; ++p) {
            const uint4 q0 = rec[2 * p];
            const uint4 q1 = rec[2 * p + 1];
            planes[8 * p + 0] = q0.x;
            planes[8 * p + 4] = q0.y;
            planes[8 * p + 1] = q0.z;
            planes[8 * p + 5] = q0.w;
            planes[8 * p + 2] = q1.x;
            planes[8 * p + 6] = q1.y;
            planes[8 * p + 3] = q1.z;
            planes[8 * p + 7] = q1.w;
          }
          const uint4 tail = rec[6];
          const int word0 = (c * T::BYTES) & ~3;
#pragma unroll
          for (int p = 0; p < ROWS / 2; ++p) {
            uint32_t w[T::WORDS];
            const uint32_t* pg =
                reinterpret_cast<const uint32_t*>(wg + (2 * p + h) * row_bytes + word0);
#pragma unroll
            for (int i = 0; i < T::WORDS; ++i) w[i] = pg[i];
            int a0, a1, a2;
            const Codes cg = T::decode(w, c);
            plane_sums<T>(cg, planes, a0, a1, a2);
            g[p] += block_dot<T>(cg, a0, a1, a2, __uint_as_float(tail.x), int(tail.y));
          }
        }
#pragma unroll
        for (int p = 0; p < ROWS / 2; ++p) {
#pragma unroll
          for (int o = 8; o > 0; o /= 2) g[p] += __shfl_xor_sync(0xffffffffu, g[p], o);
        }
        if (lane % 16 == 0) {
#pragma unroll
          for (int p = 0; p < ROWS / 2; ++p) {
            partial[j & 1][warp][2 * p + h][0] = g[p];
            partial[j & 1][warp][2 * p + h][1] = 0.0f;
          }
        }
      } else {
      for (int c = kw * WARP + lane; c < blocks; c += WARP * KS) {
        const uint4* rec = reinterpret_cast<const uint4*>(record + (long long)c * STRIDE);
        // stored words 0..7 of a plane hold words 0, 4, 1, 5, 2, 6, 3, 7
        uint32_t planes[24];
#pragma unroll
        for (int p = 0; p < 3; ++p) {
          const uint4 q0 = rec[2 * p];
          const uint4 q1 = rec[2 * p + 1];
          planes[8 * p + 0] = q0.x;
          planes[8 * p + 4] = q0.y;
          planes[8 * p + 1] = q0.z;
          planes[8 * p + 5] = q0.w;
          planes[8 * p + 2] = q1.x;
          planes[8 * p + 6] = q1.y;
          planes[8 * p + 3] = q1.z;
          planes[8 * p + 7] = q1.w;
        }
        const uint4 tail = rec[6];  // s, sum X at bytes 96, 100
        const int word0 = (c * T::BYTES) & ~3;
#pragma unroll
        for (int r = 0; r < ROWS; ++r) {
          uint32_t w[T::WORDS];
          const uint32_t* pg = reinterpret_cast<const uint32_t*>(wg + r * row_bytes + word0);
#pragma unroll
          for (int i = 0; i < T::WORDS; ++i) w[i] = pg[i];
          int a0, a1, a2;
          const Codes cg = T::decode(w, c);
          plane_sums<T>(cg, planes, a0, a1, a2);
          g[r] += block_dot<T>(cg, a0, a1, a2, __uint_as_float(tail.x), int(tail.y));
          if (GATED) {
            const uint32_t* pu = reinterpret_cast<const uint32_t*>(wu + r * row_bytes + word0);
#pragma unroll
            for (int i = 0; i < T::WORDS; ++i) w[i] = pu[i];
            const Codes cu = T::decode(w, c);
            plane_sums<T>(cu, planes, a0, a1, a2);
            up[r] += block_dot<T>(cu, a0, a1, a2, __uint_as_float(tail.x), int(tail.y));
          }
        }
      }
#pragma unroll
      for (int r = 0; r < ROWS; ++r) {
#pragma unroll
        for (int o = 16; o > 0; o /= 2) {
          g[r] += __shfl_xor_sync(0xffffffffu, g[r], o);
          if (GATED) up[r] += __shfl_xor_sync(0xffffffffu, up[r], o);
        }
      }
      if (lane == 0) {
#pragma unroll
        for (int r = 0; r < ROWS; ++r) {
          partial[j & 1][warp][r][0] = g[r];
          partial[j & 1][warp][r][1] = up[r];
        }
      }
      }
    }
    __syncthreads();  // the stage is free; the partial sums are in
    if (threadIdx.x == 0 && ok && issued < count) {
      issue(issued);
      ++issued;
    }
    const int t = threadIdx.x;
    if (t < TILE && row0 + t < L.rows) {
      const int gi = t / ROWS, r = t % ROWS;
      float* out = L.y + (long long)slot * L.rows + row0 + t;
      if (!valid) {
        // another rank's expert (zeros), or an id outside the table
        if (!L.others_zero && t == 0 && L.error) atomicCAS(L.error, 0, 1);
        *out = L.others_zero ? 0.0f : __int_as_float(0x7fc00000);
      } else if (ok) {
        float gs = 0.0f, us = 0.0f;
#pragma unroll
        for (int kk = 0; kk < KS; ++kk) {
          gs += partial[j & 1][gi * KS + kk][r][0];
          us += partial[j & 1][gi * KS + kk][r][1];
        }
        *out = GATED ? gs / (1.0f + expf(-gs)) * us : gs;
      }
    }
  }
  if (threadIdx.x == 0) {
    // the copies issued land before the CTA leaves (all of them, when every
    // wait came through; the last of each stage otherwise)
    volatile int never = 0;
    for (int q = issued - S > 0 ? issued - S : 0; q < issued; ++q)
      tc::mbar_wait(&full[q % S], (q / S) & 1, &never, nullptr);
  }
}

// The stages of a launch: a stage holds a unit's rows (both weights when
// gated), as many stages (up to 4) as fit.
struct EsShape {
  int tile_rows, stage_bytes, stages, smem;
};
inline EsShape es_shape(int ks, long long row_bytes, bool gated, int blocks, bool half) {
  EsShape s;
  s.tile_rows = (ES_WARPS / ks) * (half ? 8 : 4);
  s.stage_bytes = int((row_bytes * s.tile_rows * (gated ? 2 : 1) + 16 + 127) / 128 * 128);
  const int fixed = es_x_bytes(blocks) + 4 * 8 + 16 + 128;  // + the slot's x records
  s.stages = (232448 - 2048 - fixed) / s.stage_bytes;
  if (s.stages > 4) s.stages = 4;
  s.smem = s.stages * s.stage_bytes + fixed;
  return s;
}

template <typename T, int KS, bool GATED, bool XQ, bool HALF = false>
static int launch_stream(const ExpertsStream& L, const EsShape& shape, cudaStream_t stream) {
  static PerDevice configured;
  DRIFT_TRY(ensure_shared_memory(configured, experts_stream_kernel<T, KS, GATED, XQ, HALF>,
                                 232448 - 2048));
  const int grid = L.units < sm_count() ? L.units : sm_count();
  DRIFT_CUDA(launch_pdl(experts_stream_kernel<T, KS, GATED, XQ, HALF>, unsigned(grid),
                        ES_WARPS * 32, shape.smem, stream, L));
  DRIFT_LAUNCHED("experts_stream");
  return 0;
}

template <typename T, bool GATED>
static int launch_experts(const uint8_t* gate, const uint8_t* up, long long expert_bytes,
                          const int* ids, const uint8_t* records, int divisor, int routed_slots,
                          float* y, int rows,
                          int cols, int slots, long long experts, long long first_expert,
                          int others_zero, cudaStream_t stream, const float* xq = nullptr) {
  const int blocks = cols / 32;
  const int ks = blocks >= 128 ? 4 : (blocks >= 64 ? 2 : 1);
  const long long row_bytes = (long long)blocks * T::BYTES;
  const bool with_xq = !GATED && xq != nullptr;
  const bool half = !GATED && blocks <= 16;  // plain products of short rows: HALF
  const EsShape shape = es_shape(ks, row_bytes, GATED, blocks, half);
  if (row_bytes % 16 == 0 && (reinterpret_cast<uintptr_t>(gate) & 15) == 0 &&
      (reinterpret_cast<uintptr_t>(up) & 15) == 0 && expert_bytes % 16 == 0 && rows > 0 &&
      slots > 0 && shape.stages >= 2 && (GATED || half) &&
      (long long)slots * ((rows + shape.tile_rows - 1) / shape.tile_rows) >= sm_count()) {
    // rows of whole 16-byte units, gated or (plain) of at most 16 blocks, two
    // units' rows in shared memory at once, and a unit or more an SM:
    // streamed (C5's step 2.6 % shorter at batch 1 and 28 % at batch 16 than
    // with experts_x22 alone). Plain products of longer rows, a row a warp,
    // were slower streamed than direct.
    ExpertsStream L = {};
    L.gate = gate;
    L.up = up;
    L.expert_bytes = expert_bytes;
    L.ids = ids;
    L.records = records;
    L.divisor = divisor;
    L.routed_slots = routed_slots;
    L.y = y;
    L.rows = rows;
    L.cols = cols;
    L.experts = experts;
    L.first_expert = first_expert;
    L.others_zero = others_zero;
    L.error = device_error_word();
    L.x = xq;
    L.tiles = (rows + shape.tile_rows - 1) / shape.tile_rows;
    L.stage_bytes = shape.stage_bytes;
    L.stages = shape.stages;
    const long long units = (long long)slots * L.tiles;
    if (units > 0x7fffffffll) return invalid("%lld expert units", units);
    L.units = int(units);
    if constexpr (!GATED) {
      // (half: blocks <= 16, so ks is 1)
      if (with_xq) return launch_stream<T, 1, false, true, true>(L, shape, stream);
      return launch_stream<T, 1, false, false, true>(L, shape, stream);
    } else {
      if (ks == 4) return launch_stream<T, 4, true, false>(L, shape, stream);
      if (ks == 2) return launch_stream<T, 2, true, false>(L, shape, stream);
      return launch_stream<T, 1, true, false>(L, shape, stream);
    }
  }
  const int rows_per_cta = 4 * (8 / ks);
  const dim3 grid(unsigned((rows + rows_per_cta - 1) / rows_per_cta), unsigned(slots));
  int* error = device_error_word();
  if constexpr (!GATED) {
    if (xq) {
      // x prepared in the kernel: one x row a slot, blocks x 112 bytes of it
      const int smem = blocks * MMA_SLOT_BYTES;
#define DRIFT_EXPERTS_XQ(KS)                                                                     \
  DRIFT_CUDA(launch_pdl(experts_x22_kernel<T, KS, false, true>, grid, 256, smem, stream, gate, up, \
                        expert_bytes, ids, records, divisor, routed_slots, y, rows, cols, experts,  \
                        first_expert, others_zero, error, xq))
      if (ks == 4) DRIFT_EXPERTS_XQ(4);
      else if (ks == 2) DRIFT_EXPERTS_XQ(2);
      else DRIFT_EXPERTS_XQ(1);
#undef DRIFT_EXPERTS_XQ
      DRIFT_LAUNCHED("experts_x22");
      return 0;
    }
  }
  if (ks == 4)
    DRIFT_CUDA(launch_pdl(experts_x22_kernel<T, 4, GATED>, grid, 256, 0, stream, gate, up,
                          expert_bytes, ids, records, divisor, routed_slots, y, rows, cols, experts,
                          first_expert, others_zero, error, nullptr));
  else if (ks == 2)
    DRIFT_CUDA(launch_pdl(experts_x22_kernel<T, 2, GATED>, grid, 256, 0, stream, gate, up,
                          expert_bytes, ids, records, divisor, routed_slots, y, rows, cols, experts,
                          first_expert, others_zero, error, nullptr));
  else
    DRIFT_CUDA(launch_pdl(experts_x22_kernel<T, 1, GATED>, grid, 256, 0, stream, gate, up,
                          expert_bytes, ids, records, divisor, routed_slots, y, rows, cols, experts,
                          first_expert, others_zero, error, nullptr));
  DRIFT_LAUNCHED("experts_x22");
  return 0;
}

static int experts_common(bool gated, int x_dtype, const void* x, int64_t x_rows,
                          int weight_dtype, const void* gate, const void* up, int64_t experts,
                          int64_t n, int64_t k, const int32_t* ids, int64_t slots, float* out,
                          int64_t first_expert, int others_zero, const void* prepared,
                          cudaStream_t stream, int shared_tail = 0) {
  const char* name = gated ? "expertsGatedLinear" : "expertsLinear";
  if (x_dtype != DRIFT_F32 && x_dtype != DRIFT_BF16)
    return invalid("%s takes F32 (or BF16) x, not %s", name, dtype_name(x_dtype));
  if (weight_dtype != DRIFT_Q8_0 && weight_dtype != DRIFT_Q4_0 && weight_dtype != DRIFT_Q4_1)
    return invalid("no kernels for %s experts yet", dtype_name(weight_dtype));
  if (x_rows <= 0 || slots < 0 || slots % x_rows != 0 || (shared_tail && slots < 2 * x_rows))
    return invalid("%s: x [%lld, %lld] for %lld slots of %lld", name, (long long)x_rows,
                   (long long)k, (long long)slots, (long long)k);
  const int64_t row = byte_size(weight_dtype, k);
  if (row < 0 || row % 4 != 0)
    return invalid("%s rows of %lld are not whole words", dtype_name(weight_dtype), (long long)k);
  if (n <= 0 || experts <= 0 || k <= 0) return invalid("%s: weight [%lld, %lld, %lld]", name,
                                                       (long long)experts, (long long)n,
                                                       (long long)k);
  if (slots == 0) return 0;
  if (!x || !gate || (gated && !up) || !ids || !out) return invalid("%s: a null tensor", name);
  if (slots > 65535) return invalid("%s: %lld slots in one launch", name, (long long)slots);
  const uint8_t* records = static_cast<const uint8_t*>(prepared);
  // one F32 x row a slot (a down product): each CTA prepares its row itself,
  // the launch that would prepare x is left out (up to 128 blocks: 14 KB of
  // shared memory)
  const float* xq = !records && !gated && !shared_tail && x_dtype == DRIFT_F32 &&
                            x_rows == slots && k / 32 <= 128
                        ? static_cast<const float*>(x)
                        : nullptr;
  if (!records && !xq) {
    void* w = nullptr;
    DRIFT_TRY(workspace_reserve(mma_workspace_bytes(x_rows, k), &w));
    DRIFT_TRY(prepare_x_mma(x_dtype, x, x_rows, k, static_cast<uint8_t*>(w), stream));
    records = static_cast<const uint8_t*>(w);
  }
  const long long expert_bytes = n * row;
  // with a shared tail, the last x_rows slots are one per x row
  const int64_t routed = shared_tail ? slots - x_rows : slots;
  const int divisor = int(routed / x_rows);
  const int routed_slots = int(routed);
  const uint8_t* g = static_cast<const uint8_t*>(gate);
  const uint8_t* u = static_cast<const uint8_t*>(up);
#define DRIFT_EXPERTS_CASE(T)                                                                   \
  return gated ? launch_experts<T, true>(g, u, expert_bytes, ids, records, divisor,         \
                                         routed_slots, out, int(n),                            \
                                         int(k), int(slots), experts, first_expert, others_zero, \
                                         stream)                                                \
               : launch_experts<T, false>(g, g, expert_bytes, ids, records, divisor,       \
                                          routed_slots, out, int(n),                           \
                                          int(k), int(slots), experts, first_expert,             \
                                          others_zero, stream, xq);
  switch (weight_dtype) {
    case DRIFT_Q8_0: DRIFT_EXPERTS_CASE(Q8_0T)
    case DRIFT_Q4_0: DRIFT_EXPERTS_CASE(Q4_0T)
    default: DRIFT_EXPERTS_CASE(Q4_1T)
  }
#undef DRIFT_EXPERTS_CASE
}

// ---- combine ---------------------------------------------------------------------------------
// The shared expert's gate: sigmoid(x . router), reduced by the block in a
// fixed order.
__device__ __forceinline__ float shared_gate(const float* x, const float* router, int hidden,
                                             float* partial) {
  float dot = 0.0f;
  for (int c = threadIdx.x; c < hidden; c += blockDim.x) dot = fmaf(x[c], router[c], dot);
#pragma unroll
  for (int o = 16; o > 0; o /= 2) dot += __shfl_xor_sync(0xffffffffu, dot, o);
  if (threadIdx.x % WARP == 0) partial[threadIdx.x / WARP] = dot;
  __syncthreads();
  float total = 0.0f;
  for (int w = 0; w < int(blockDim.x / WARP); ++w) total += partial[w];
  __syncthreads();
  return 1.0f / (1.0f + expf(-total));
}

// One block of 1024 threads per token, PER values of the row a thread, every
// load issued before the first use. NORM: the combined row is also the
// residual stream (written back) and its RMS norm goes to `normed`.
constexpr int COMBINE_THREADS = 1024, MAX_COMBINE_K = 16;
template <bool NORM, int PER>
__global__ void __launch_bounds__(COMBINE_THREADS) combine_kernel(
    const float* __restrict__ expert_out, const float* __restrict__ weights,
    const float* __restrict__ shared_out, const float* __restrict__ shared_input,
    const float* __restrict__ shared_router, const float* residual, float* out, int k, int hidden,
    const float* __restrict__ norm_weight, float* __restrict__ normed, float epsilon,
    float weight_offset, uint8_t* records) {
  pdl_trigger();  // the next kernel may launch and wait for this one
  pdl_wait();     // what the kernels before this one wrote is visible
  __shared__ float partial[32];
  const long long t = blockIdx.x;
  float routed[PER], res[PER], shared[PER], dot = 0.0f;
#pragma unroll
  for (int i = 0; i < PER; ++i) {
    const int c = threadIdx.x + i * COMBINE_THREADS;
    const bool in = c < hidden;
    res[i] = residual && in ? residual[t * hidden + c] : 0.0f;
    shared[i] = shared_out && in ? shared_out[t * hidden + c] : 0.0f;
    if (shared_out && in) dot = fmaf(shared_input[t * hidden + c], shared_router[c], dot);
    routed[i] = 0.0f;
  }
  // the routed experts' outputs, weighted, in slot order: GROUP slots'
  // loads in flight at a time (32 values a thread)
  constexpr int GROUP = 32 / PER < MAX_COMBINE_K ? 32 / PER : MAX_COMBINE_K;
  for (int j0 = 0; j0 < k; j0 += GROUP) {
    float part[GROUP][PER];
#pragma unroll
    for (int j = 0; j < GROUP; ++j)
#pragma unroll
      for (int i = 0; i < PER; ++i) {
        const int c = threadIdx.x + i * COMBINE_THREADS;
        part[j][i] = j0 + j < k && c < hidden ? expert_out[(t * k + j0 + j) * hidden + c] : 0.0f;
      }
#pragma unroll
    for (int j = 0; j < GROUP; ++j) {
      if (j0 + j >= k) break;
      const float wj = weights[t * k + j0 + j];
#pragma unroll
      for (int i = 0; i < PER; ++i) routed[i] = fmaf(wj, part[j][i], routed[i]);
    }
  }
  // the shared expert's gate: sigmoid(x . router)
  float gate = 0.0f;
  if (shared_out) gate = 1.0f / (1.0f + expf(-block_sum(dot, partial)));
  float squares = 0.0f, sum[PER];
#pragma unroll
  for (int i = 0; i < PER; ++i) {
    const int c = threadIdx.x + i * COMBINE_THREADS;
    sum[i] = res[i] + routed[i];
    if (shared_out) sum[i] = fmaf(gate, shared[i], sum[i]);
    if (c < hidden) out[t * hidden + c] = sum[i];
    squares = fmaf(sum[i], sum[i], squares);
  }
  if (!NORM) return;
  const float total = block_sum(squares, partial);
  const float scale = 1.0f / sqrtf(total / float(hidden) + epsilon);
#pragma unroll
  for (int i = 0; i < PER; ++i) {
    const int c = threadIdx.x + i * COMBINE_THREADS;
    if (c >= hidden) continue;  // (whole warps when hidden is a multiple of 32)
    const float value = sum[i] * scale * (norm_weight[c] + weight_offset);
    normed[t * hidden + c] = value;
    // warp w holds columns 1024 i + 32 w .. + 31: block 32 i + w of the row
    if (records) x22_record_block(value, records, int(t), c / 32, hidden / 32);
  }
}

DRIFT_REGISTER(moe_combine_rows, (combine_kernel<false, 2>))
DRIFT_REGISTER(moe_combine_norm_records, (combine_kernel<true, 2>))

// ---- the whole mixture of a decode step in one launch ---------------------------------------
// The router product, the top-k, the routed and shared experts' gate/up and
// down products and the combine with the residual and the next norm -- five
// launches' work -- in one cooperative launch: each phase is its launch's
// work split into the same units (a (vector, row) of the router, a token's
// top-k, a (row tile, slot) of the experts' products, a token's combine),
// taken by the grid's CTAs in turn and computed by the same device code, so
// the bits are the separate launches'; a grid barrier between phases. The
// combine's 1024-thread block is stood in for by 256 threads, each holding
// four of its threads' values, so its two reductions keep their order.
constexpr int MOE_THREADS = 256;

// A grid barrier: every CTA's writes before it are visible to every CTA
// after it. Thread 0 of each CTA arrives on a count; the last to arrive
// resets it and advances the generation the others wait on (at most about a
// second, then device error 2 and false: the caller returns, its results
// void).
__device__ unsigned moe_arrivals, moe_generation;

__device__ bool moe_grid_barrier(unsigned ctas, int* error) {
  __shared__ int passed;
  __syncthreads();
  if (threadIdx.x == 0) {
    const unsigned generation = *reinterpret_cast<volatile unsigned*>(&moe_generation);
    __threadfence();
    passed = 1;
    if (atomicAdd(&moe_arrivals, 1u) == ctas - 1) {
      atomicExch(&moe_arrivals, 0u);
      __threadfence();
      atomicAdd(&moe_generation, 1u);
    } else {
      const uint64_t start = tc::global_ns();
      while (*reinterpret_cast<volatile unsigned*>(&moe_generation) == generation) {
        if (tc::global_ns() - start > 1000000000ull) {
          atomicCAS(error, 0, 2);
          passed = 0;
          break;
        }
        __nanosleep(32);
      }
      __threadfence();
    }
  }
  __syncthreads();
  return passed != 0;
}

// combine_kernel<true, 2> for token t with 256 threads: thread (w, l) holds
// the 1024-thread kernel's threads 32 (4 w + i) + l, i = 0..3, each with its
// two columns c and c + 1024.
__device__ void moe_combine_norm_token(
    const float* __restrict__ expert_out, const float* __restrict__ weights,
    const float* __restrict__ shared_out, const float* __restrict__ shared_input,
    const float* __restrict__ shared_router, float* residual, int k, int hidden,
    const float* __restrict__ norm_weight, float* __restrict__ normed, float epsilon,
    float weight_offset, uint8_t* records, long long t) {
  constexpr int V = 4, PER = 2, BIG = COMBINE_THREADS;
  __shared__ float partial[32];
  const int warp = threadIdx.x / WARP, lane = threadIdx.x % WARP;
  // block_sum's order over the big block's 32 warps: virtual warp 4 w + i
  // reduced by the same shuffle tree, then the 32 sums in order
  auto big_sum = [&](float (&values)[V]) {
#pragma unroll
    for (int i = 0; i < V; ++i) {
#pragma unroll
      for (int o = 16; o > 0; o /= 2) values[i] += __shfl_xor_sync(0xffffffffu, values[i], o);
      if (lane == 0) partial[4 * warp + i] = values[i];
    }
    __syncthreads();
    float total = 0.0f;
    for (int w = 0; w < BIG / WARP; ++w) total += partial[w];
    __syncthreads();
    return total;
  };
  float sum[V][PER], shared[V][PER], dot[V];
#pragma unroll
  for (int i = 0; i < V; ++i) {
    const int vt = WARP * (4 * warp + i) + lane;  // the big block's thread
    float routed[PER];
    dot[i] = 0.0f;
#pragma unroll
    for (int p = 0; p < PER; ++p) {
      const int c = vt + p * BIG;
      const bool in = c < hidden;
      sum[i][p] = in ? residual[t * hidden + c] : 0.0f;
      shared[i][p] = shared_out && in ? shared_out[t * hidden + c] : 0.0f;
      if (shared_out && in) dot[i] = fmaf(shared_input[t * hidden + c], shared_router[c], dot[i]);
      routed[p] = 0.0f;
    }
    // the routed experts' outputs, weighted, in slot order
    for (int j = 0; j < k; ++j) {
      const float wj = weights[t * k + j];
#pragma unroll
      for (int p = 0; p < PER; ++p) {
        const int c = vt + p * BIG;
        routed[p] = fmaf(wj, c < hidden ? expert_out[(t * k + j) * hidden + c] : 0.0f, routed[p]);
      }
    }
#pragma unroll
    for (int p = 0; p < PER; ++p) sum[i][p] = sum[i][p] + routed[p];  // residual + routed
  }
  // the shared expert's gate: sigmoid(x . router)
  float gate = 0.0f;
  if (shared_out) gate = 1.0f / (1.0f + expf(-big_sum(dot)));
  float squares[V];
#pragma unroll
  for (int i = 0; i < V; ++i) {
    const int vt = WARP * (4 * warp + i) + lane;
    squares[i] = 0.0f;
#pragma unroll
    for (int p = 0; p < PER; ++p) {
      const int c = vt + p * BIG;
      if (shared_out) sum[i][p] = fmaf(gate, shared[i][p], sum[i][p]);
      if (c < hidden) residual[t * hidden + c] = sum[i][p];
      squares[i] = fmaf(sum[i][p], sum[i][p], squares[i]);
    }
  }
  const float total = big_sum(squares);
  const float scale = 1.0f / sqrtf(total / float(hidden) + epsilon);
#pragma unroll
  for (int i = 0; i < V; ++i) {
    const int vt = WARP * (4 * warp + i) + lane;
#pragma unroll
    for (int p = 0; p < PER; ++p) {
      const int c = vt + p * BIG;
      if (c >= hidden) continue;  // whole warps: hidden is a multiple of 32
      const float value = sum[i][p] * scale * (norm_weight[c] + weight_offset);
      normed[t * hidden + c] = value;
      if (records) x22_record_block(value, records, int(t), c / 32, hidden / 32);
    }
  }
}

struct MoeArgs {
  // router: logits [tokens][experts] = x . router^T
  const float* x;            // [tokens][hidden], the post norm's output (also the shared gate's input)
  const uint8_t* x_records;  // its records, for the gate/up products
  const float* router;       // [experts][hidden] F32
  float* logits;
  int* ids;                  // [tokens k + tokens]: routed slots, then one shared slot a token
  float* route_weights;      // [tokens][k]
  // experts: the shared expert is expert `experts` of the weights
  const uint8_t* gate;
  const uint8_t* up;
  const uint8_t* down;
  long long gate_bytes, down_bytes;  // one expert's bytes
  float* gated;              // [slots][ffn]
  float* out;                // [slots][hidden]
  const float* shared_router;
  float* residual;           // [tokens][hidden], updated
  const float* norm_weight;
  float* normed;             // the next norm's output (may be x)
  uint8_t* records;          // its records (may be x_records)
  float epsilon, weight_offset;
  int tokens, experts, k, hidden, ffn;
  int* error;
};

template <typename T>
__global__ void __launch_bounds__(MOE_THREADS) moe_decode_kernel(const __grid_constant__ MoeArgs a) {
  pdl_trigger();  // the next kernel may launch and wait for this one
  pdl_wait();     // what the kernels before this one wrote is visible
  extern __shared__ __align__(16) uint8_t x_slots[];  // the down products' x
  __shared__ float partial[32];
  const unsigned G = gridDim.x;
  const int slots = a.tokens * a.k + a.tokens;
  // 1. the router's logits (matvec_f32_kernel: a (vector, row) a unit)
  for (int u = blockIdx.x; u < a.tokens * a.experts; u += G) {
    const int row = u % a.experts, vector = u / a.experts;
    const float total = f32_row_dot<false>(a.x, a.router, a.router + (long long)row * a.hidden,
                                           vector, a.hidden, partial);
    if (threadIdx.x == 0) a.logits[(long long)vector * a.experts + row] = total;
  }
  if (!moe_grid_barrier(G, a.error)) return;
  // 2. the top-k of each token (route_kernel: a warp a token)
  {
    const int t = blockIdx.x * (MOE_THREADS / WARP) + threadIdx.x / WARP;
    if (t < a.tokens) {
      route_token(a.logits, a.ids, a.route_weights, t, a.experts, a.k);
      // the token's shared slot: the shared expert, expert `experts`
      if (threadIdx.x % WARP == 0) a.ids[a.tokens * a.k + t] = a.experts;
    }
  }
  if (!moe_grid_barrier(G, a.error)) return;
  // 3. gate/up of every slot, the shared ones last (experts_x22_kernel, gated)
  {
    const int blocks = a.hidden / 32;
    const int ks = blocks >= 128 ? 4 : (blocks >= 64 ? 2 : 1);
    const int per_cta = 4 * (8 / ks);
    const int tiles = (a.ffn + per_cta - 1) / per_cta;
    for (int u = blockIdx.x; u < tiles * slots; u += G) {
      const int tile = u % tiles, slot = u / tiles;
#define DRIFT_MOE_GATE(KS)                                                                          experts_unit<T, KS, true, false>(a.gate, a.up, a.gate_bytes, a.ids, a.x_records, a.k,                                           a.tokens * a.k, a.gated, a.ffn, a.hidden, a.experts + 1, 0,                                     0, a.error, nullptr, tile, slot, x_slots)
      if (ks == 4) DRIFT_MOE_GATE(4);
      else if (ks == 2) DRIFT_MOE_GATE(2);
      else DRIFT_MOE_GATE(1);
#undef DRIFT_MOE_GATE
      __syncthreads();  // the unit's shared memory is the next unit's
    }
  }
  if (!moe_grid_barrier(G, a.error)) return;
  // 4. down of every slot (experts_x22_kernel, x prepared in the CTA)
  {
    const int blocks = a.ffn / 32;
    const int ks = blocks >= 128 ? 4 : (blocks >= 64 ? 2 : 1);
    const int per_cta = 4 * (8 / ks);
    const int tiles = (a.hidden + per_cta - 1) / per_cta;
    for (int u = blockIdx.x; u < tiles * slots; u += G) {
      const int tile = u % tiles, slot = u / tiles;
#define DRIFT_MOE_DOWN(KS)                                                                            experts_unit<T, KS, false, true>(a.down, a.down, a.down_bytes, a.ids, nullptr, 1, slots, a.out,                                    a.hidden, a.ffn, a.experts + 1, 0, 0, a.error, a.gated, tile,                                     slot, x_slots)
      if (ks == 4) DRIFT_MOE_DOWN(4);
      else if (ks == 2) DRIFT_MOE_DOWN(2);
      else DRIFT_MOE_DOWN(1);
#undef DRIFT_MOE_DOWN
      __syncthreads();
    }
  }
  if (!moe_grid_barrier(G, a.error)) return;
  // 5. the combine with the residual and the next norm (combine_kernel)
  for (int t = blockIdx.x; t < a.tokens; t += G) {
    moe_combine_norm_token(a.out, a.route_weights, a.out + (long long)a.tokens * a.k * a.hidden,
                           a.x, a.shared_router, a.residual, a.k, a.hidden, a.norm_weight,
                           a.normed, a.epsilon, a.weight_offset, a.records, t);
    __syncthreads();
  }
}

DRIFT_REGISTER(moe_decode_q8_0, moe_decode_kernel<Q8_0T>)
DRIFT_REGISTER(moe_decode_q4_0, moe_decode_kernel<Q4_0T>)
DRIFT_REGISTER(moe_decode_q4_1, moe_decode_kernel<Q4_1T>)

template <bool NORM>
static int launch_combine(const float* expert_out, const float* weights, int64_t tokens, int64_t k,
                          int64_t hidden, const float* shared_out, const float* shared_input,
                          const float* shared_router, const float* residual, float* out,
                          const float* norm_weight, float* normed, float epsilon,
                          float weight_offset, cudaStream_t stream, uint8_t* records = nullptr) {
  const unsigned grid = unsigned(tokens);
#define DRIFT_COMBINE(PER)                                                                        \
  DRIFT_CUDA(launch_pdl(combine_kernel<NORM, PER>, grid, COMBINE_THREADS, 0, stream, expert_out,  \
                        weights, shared_out, shared_input, shared_router, residual, out, int(k), \
                        int(hidden), norm_weight, normed, epsilon, weight_offset, records))
  if (hidden <= 1024) DRIFT_COMBINE(1);
  else if (hidden <= 2048) DRIFT_COMBINE(2);
  else if (hidden <= 4096) DRIFT_COMBINE(4);
  else DRIFT_COMBINE(8);
#undef DRIFT_COMBINE
  DRIFT_LAUNCHED(NORM ? "moe_combine_norm" : "moe_combine");
  return 0;
}

static int check_combine(const float* expert_out, const float* weights, int64_t tokens, int64_t k,
                         int64_t hidden, const float* shared_out, const float* shared_input,
                         const float* shared_router, const void* out) {
  if (tokens < 0 || k < 0 || hidden < 0 || tokens > 0x7fffffffll || hidden > 8192 ||
      k > MAX_COMBINE_K)
    return invalid("moeCombine over [%lld, %lld] with k %lld (at most 8192 wide, k 16)",
                   (long long)tokens, (long long)hidden, (long long)k);
  if (tokens > 0 && hidden > 0 && (!out || (k > 0 && (!expert_out || !weights))))
    return invalid("moeCombine: a null tensor");
  if (shared_out && (!shared_input || !shared_router))
    return invalid("moeCombine: a shared expert without its input and router");
  return 0;
}

}  // namespace drift

using namespace drift;

extern "C" {

int drift_route(const float* logits, int32_t* ids, float* weights, int tokens, int experts, int k,
                drift_stream_t stream) {
  if (tokens < 0 || experts <= 0 || k <= 0 || k > 16 || experts > 512 || k > experts)
    return invalid("route: top-%d of %d", k, experts);
  if (tokens == 0) return 0;
  if (!logits || !ids || !weights) return invalid("route: a null tensor");
  DRIFT_CUDA(launch_pdl(route_kernel, unsigned((tokens + 7) / 8), 256, 0, cudaStream_t(stream),
                        logits, ids, weights, tokens, experts, k));
  DRIFT_LAUNCHED("route_topk");
  return 0;
}

int drift_experts_linear(int x_dtype, const void* x, int64_t x_rows, int weight_dtype,
                         const void* weight, int64_t experts, int64_t n, int64_t k,
                         const int32_t* ids, int64_t slots, float* out, drift_stream_t stream) {
  return experts_common(false, x_dtype, x, x_rows, weight_dtype, weight, nullptr, experts, n, k,
                        ids, slots, out, 0, 0, nullptr, cudaStream_t(stream));
}

int drift_experts_linear_local(int x_dtype, const void* x, int64_t x_rows, int weight_dtype,
                               const void* weight, int64_t experts, int64_t first_expert,
                               int64_t n, int64_t k, const int32_t* ids, int64_t slots,
                               float* out, const void* prepared, drift_stream_t stream) {
  if (first_expert < -1) return invalid("expertsLinear: experts from %lld", (long long)first_expert);
  return experts_common(false, x_dtype, x, x_rows, weight_dtype, weight, nullptr, experts, n, k,
                        ids, slots, out, first_expert, 1, prepared, cudaStream_t(stream));
}

int drift_experts_gated_linear(int x_dtype, const void* x, int64_t x_rows, int weight_dtype,
                               const void* gate, const void* up, int64_t experts, int64_t n,
                               int64_t k, const int32_t* ids, int64_t slots, float* out,
                               drift_stream_t stream) {
  return experts_common(true, x_dtype, x, x_rows, weight_dtype, gate, up, experts, n, k, ids,
                        slots, out, 0, 0, nullptr, cudaStream_t(stream));
}

int drift_experts_gated_linear_local(int x_dtype, const void* x, int64_t x_rows, int weight_dtype,
                                     const void* gate, const void* up, int64_t experts,
                                     int64_t first_expert, int64_t n, int64_t k,
                                     const int32_t* ids, int64_t slots, float* out,
                                     const void* prepared, int shared_tail,
                                     drift_stream_t stream) {
  if (first_expert < -1)
    return invalid("expertsGatedLinear: experts from %lld", (long long)first_expert);
  return experts_common(true, x_dtype, x, x_rows, weight_dtype, gate, up, experts, n, k, ids,
                        slots, out, first_expert, 1, prepared, cudaStream_t(stream),
                        shared_tail != 0);
}

int drift_moe_combine(const float* expert_out, const float* weights, int64_t tokens, int64_t k,
                      int64_t hidden, const float* shared_out, const float* shared_input,
                      const float* shared_router, const float* residual, float* out,
                      drift_stream_t stream) {
  DRIFT_TRY(check_combine(expert_out, weights, tokens, k, hidden, shared_out, shared_input,
                          shared_router, out));
  if (tokens == 0 || hidden == 0) return 0;
  return launch_combine<false>(expert_out, weights, tokens, k, hidden, shared_out, shared_input,
                               shared_router, residual, out, nullptr, nullptr, 0.0f, 0.0f,
                               cudaStream_t(stream));
}

int drift_moe_combine_norm(const float* expert_out, const float* weights, int64_t tokens,
                           int64_t k, int64_t hidden, const float* shared_out,
                           const float* shared_input, const float* shared_router, float* residual,
                           const float* norm_weight, float epsilon, float weight_offset,
                           float* normed, drift_stream_t stream) {
  DRIFT_TRY(check_combine(expert_out, weights, tokens, k, hidden, shared_out, shared_input,
                          shared_router, residual));
  if (tokens == 0 || hidden == 0) return 0;
  if (!norm_weight || !normed) return invalid("moeCombineNorm: no norm weight or output");
  return launch_combine<true>(expert_out, weights, tokens, k, hidden, shared_out, shared_input,
                              shared_router, residual, residual, norm_weight, normed, epsilon,
                              weight_offset, cudaStream_t(stream));
}

int drift_moe_decode(int weight_dtype, const float* x, const void* x_prepared, const float* router,
                     float* logits, int32_t* ids, float* route_weights, const void* gate,
                     const void* up, const void* down, float* gated, float* out,
                     const float* shared_router, float* residual, const float* norm_weight,
                     float epsilon, float weight_offset, float* normed, void* prepared,
                     int64_t tokens, int64_t experts, int64_t k, int64_t hidden, int64_t ffn,
                     drift_stream_t stream) {
  if (weight_dtype != DRIFT_Q8_0 && weight_dtype != DRIFT_Q4_0 && weight_dtype != DRIFT_Q4_1)
    return invalid("no kernels for %s experts yet", dtype_name(weight_dtype));
  if (tokens < 0 || experts < 1 || experts > 512 || k < 1 || k > 16 || k > experts)
    return invalid("moe: top-%lld of %lld experts", (long long)k, (long long)experts);
  if (hidden <= 0 || hidden > 2 * COMBINE_THREADS || hidden % 32 != 0 || ffn <= 0 ||
      ffn % 32 != 0 || ffn / 32 > 128)
    return invalid("moe: hidden %lld (whole blocks, at most %d), expert rows of %lld (at most 4096)",
                   (long long)hidden, 2 * COMBINE_THREADS, (long long)ffn);
  const int64_t gate_row = byte_size(weight_dtype, hidden), down_row = byte_size(weight_dtype, ffn);
  if (gate_row % 4 != 0 || down_row % 4 != 0)
    return invalid("%s rows are not whole words", dtype_name(weight_dtype));
  if (tokens == 0) return 0;
  if (tokens * (k + 1) > 65535) return invalid("moe: %lld slots", (long long)(tokens * (k + 1)));
  if (!x || !x_prepared || !router || !logits || !ids || !route_weights || !gate || !up ||
      !down || !gated || !out || !shared_router || !residual || !norm_weight || !normed)
    return invalid("moe: a null tensor");
  MoeArgs a = {};
  a.x = x;
  a.x_records = static_cast<const uint8_t*>(x_prepared);
  a.router = router;
  a.logits = logits;
  a.ids = ids;
  a.route_weights = route_weights;
  a.gate = static_cast<const uint8_t*>(gate);
  a.up = static_cast<const uint8_t*>(up);
  a.down = static_cast<const uint8_t*>(down);
  a.gate_bytes = ffn * gate_row;
  a.down_bytes = hidden * down_row;
  a.gated = gated;
  a.out = out;
  a.shared_router = shared_router;
  a.residual = residual;
  a.norm_weight = norm_weight;
  a.normed = normed;
  a.records = static_cast<uint8_t*>(prepared);
  a.epsilon = epsilon;
  a.weight_offset = weight_offset;
  a.tokens = int(tokens);
  a.experts = int(experts);
  a.k = int(k);
  a.hidden = int(hidden);
  a.ffn = int(ffn);
  a.error = device_error_word();
  const size_t smem = size_t(ffn / 32) * MMA_SLOT_BYTES;  // the down products' x
  // every CTA resident at once (the grid barriers wait on all of them): the
  // occupancy's count, launched cooperatively
  auto launch = [&](auto kernel) -> int {
    int per_sm = 0;
    DRIFT_CUDA(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kernel, MOE_THREADS, smem));
    if (per_sm < 1) return invalid("moe: the launch does not fit an SM");
    cudaLaunchConfig_t config = {};
    config.gridDim = dim3(unsigned(per_sm * sm_count()));
    config.blockDim = dim3(MOE_THREADS);
    config.dynamicSmemBytes = smem;
    config.stream = cudaStream_t(stream);
    cudaLaunchAttribute attribute[1];
    attribute[0].id = cudaLaunchAttributeCooperative;
    attribute[0].val.cooperative = 1;
    config.attrs = attribute;
    config.numAttrs = 1;
    DRIFT_CUDA(cudaLaunchKernelEx(&config, kernel, a));
    DRIFT_LAUNCHED("moe_decode");
    return 0;
  };
  switch (weight_dtype) {
    case DRIFT_Q8_0: return launch(moe_decode_kernel<Q8_0T>);
    case DRIFT_Q4_0: return launch(moe_decode_kernel<Q4_0T>);
    default: return launch(moe_decode_kernel<Q4_1T>);
  }
}

int drift_moe_combine_norm_prepared(const float* expert_out, const float* weights, int64_t tokens,
                                    int64_t k, int64_t hidden, const float* shared_out,
                                    const float* shared_input, const float* shared_router,
                                    float* residual, const float* norm_weight, float epsilon,
                                    float weight_offset, float* normed, void* prepared,
                                    drift_stream_t stream) {
  if (!prepared)
    return drift_moe_combine_norm(expert_out, weights, tokens, k, hidden, shared_out, shared_input,
                                  shared_router, residual, norm_weight, epsilon, weight_offset,
                                  normed, stream);
  DRIFT_TRY(check_combine(expert_out, weights, tokens, k, hidden, shared_out, shared_input,
                          shared_router, residual));
  if (hidden % 32 != 0) return invalid("moeCombineNorm: records of %lld columns", (long long)hidden);
  if (tokens == 0 || hidden == 0) return 0;
  if (!norm_weight || !normed) return invalid("moeCombineNorm: no norm weight or output");
  return launch_combine<true>(expert_out, weights, tokens, k, hidden, shared_out, shared_input,
                              shared_router, residual, residual, norm_weight, normed, epsilon,
                              weight_offset, cudaStream_t(stream), static_cast<uint8_t*>(prepared));
}

}  // extern "C"
