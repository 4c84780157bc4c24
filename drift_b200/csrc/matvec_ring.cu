// The 1-8 vector products with weights staged through shared memory by bulk
// copies: what the products run as when rows are whole 16-byte units and the
// weight is 16-byte aligned (matvec.cu's direct-load kernel takes the rest).
//
// Each warp owns a ring of S stages in shared memory, one mbarrier each. A
// stage holds one 8-block (256-column) segment of 16 MT rows -- 160 (Q4_1),
// 144 (Q4_0) or 272 (Q8_0) bytes each -- brought by one 2-D tensor copy
// (one small copy per row would leave the copy engine, not DRAM, setting the
// pace). The warp keeps up to S segments in flight, consumes one
// (mma.sync m16n8k32 on the x byte planes, mma_i8.cuh), and refills the
// stage it freed -- with the next segment of the same rows or of the next
// tile it claims, so the pipeline does not drain between tiles.
//
// Two schedules:
//  - tiles (KS = 1): each warp sums whole rows. A CTA owns a contiguous range
//    of tiles and its warps claim them one at a time from a shared counter, so
//    the SMs finish within a tile of each other whatever the row count.
//  - split (KS > 1), for matrices with few rows: a CTA's 8 warps take 8/KS
//    tiles and split each tile's segments KS ways; the partial sums meet in
//    shared memory in a fixed order.
// Either way an output sums its blocks in an order fixed by the matrix's
// shape alone (KS is chosen from rows and columns), never by the number of
// vectors.
#include <cuda_runtime.h>

#include <type_traits>

#include "common.cuh"
#include "mma_i8.cuh"
#include "quant.cuh"
#include "registry.cuh"
#include "tc_common.cuh"
#include "tma_host.cuh"

namespace drift {

int* device_error_word();

namespace {

constexpr int SEG_BLOCKS = 8;
// Every tile is 64 rows: two rows per lane in the dp4a modes, four 16-row MMA
// tiles in the MMA modes, so all modes share one schedule -- and one order of
// summation -- per matrix.
constexpr int ROWS = 64;
// 1 or 2 vectors (dp4a), 3-8 vectors (MMA, one pass of x records) and 9-16
// vectors (MMA16: two passes' records met by each weight fragment, so the
// weights stream once for 16 vectors)
constexpr int MODE_DP4A_1 = 1, MODE_DP4A_2 = 2, MODE_MMA = 8, MODE_MMA16 = 16;
__host__ __device__ constexpr bool mma_mode(int mode) { return mode >= MODE_MMA; }
// 8-vector passes of x records a mode reads at once
__host__ __device__ constexpr int mode_passes(int mode) { return mode == MODE_MMA16 ? 2 : 1; }
// output slots per row of a tile (a pass's 8 in the MMA modes)
__host__ __device__ constexpr int mode_slots(int mode) { return mma_mode(mode) ? 8 * mode_passes(mode) : mode; }

template <typename T>
struct Ring {
  static constexpr int SEG = SEG_BLOCKS * T::BYTES;  // 160 (Q4_1), 144 (Q4_0), 272 (Q8_0)
  // The width each copy brings per row. Q4_1 takes 16 bytes past its segment
  // (the next segment's first bytes, or zeros past the row) so a row sits 176
  // bytes -- 44 words -- from the next: lanes reading one column of eight
  // consecutive rows then hit eight distinct 4-bank groups, where a 160-byte
  // pitch would put rows r and r + 4 on the same banks.
  static constexpr int PITCH = T::DTYPE == DRIFT_Q4_1 ? 176 : SEG;
  static constexpr int STAGE = ROWS * PITCH;
};

constexpr int MAX_SMEM = 232448;

// Warps per CTA and stages per warp, by type: about 180-210 KB of ring.
template <typename T>
struct RingShape {
  static constexpr int WARPS = T::DTYPE == DRIFT_Q8_0 ? 6 : 8;
  static constexpr int S = 2;
  static constexpr int BARS = WARPS * S * Ring<T>::STAGE;
  static constexpr int X_OFFSET = BARS + WARPS * S * 8 + 16;  // x staged for the dp4a modes
  static constexpr int BYTES = X_OFFSET + 1024;  // + room to align to 1024; + x when staged
  // the MMA modes keep a tile's chain of group sums here, not in registers
  // (16 floats a lane a pass)
  static constexpr int chain_bytes(int mode) {
    return mma_mode(mode) ? WARPS * 16 * mode_passes(mode) * WARP * 4 : 0;
  }
  // whether the MMA16 chain fits beside the ring (Q4_0, Q4_1; Q8_0's larger
  // ring leaves it two 8-vector passes)
  static constexpr bool MMA16 = BYTES + chain_bytes(MODE_MMA16) <= MAX_SMEM;
  // The tile schedule's MMA mode shares each segment's x records among the
  // CTA's warps: X_SLOTS slots of a segment's records (8 x 896 bytes) after
  // the chain, filled by bulk copies, then a full and an empty barrier per
  // slot. Up to 4 slots where they fit (Q4_0, Q4_1), else none (Q8_0: the
  // warps read x from global memory, as the other modes do).
  static constexpr int X_SLOT = SEG_BLOCKS * MMA_RECORD_BYTES;
  static constexpr int XS_OFFSET = (X_OFFSET + chain_bytes(MODE_MMA) + 127) / 128 * 128;
  static constexpr int X_ROOM = (MAX_SMEM - 1024 - XS_OFFSET) / (X_SLOT + 16);
  static constexpr int X_SLOTS = X_ROOM >= 4 ? 4 : X_ROOM >= 2 ? X_ROOM : 0;
  static constexpr int XBAR_OFFSET = XS_OFFSET + X_SLOTS * X_SLOT;
  // dynamic shared memory of the tile schedule's MMA modes (`slots`: with
  // the shared x slots)
  static constexpr int mma_bytes(int mode, bool slots) {
    return mode == MODE_MMA && slots && X_SLOTS ? XBAR_OFFSET + 16 * X_SLOTS + 1024
                                                : BYTES + chain_bytes(mode);
  }
};

// One vector's x for one block, as the dp4a modes use it.
struct XBlock {
  uint32_t planes[24];
  float s, fsum;
  int sum;
};

// Where the dp4a modes read x from: the records in global memory (896 bytes
// apart, read through L1) or their slots copied into shared memory.
struct XGlobal {
  static constexpr bool SHARED = false;
  __device__ static uint4 at(const uint8_t* p) { return __ldg(reinterpret_cast<const uint4*>(p)); }
};
struct XShared {
  static constexpr bool SHARED = true;
  __device__ static uint4 at(const uint8_t* p) { return *reinterpret_cast<const uint4*>(p); }
};

template <typename T, typename SRC>
__device__ __forceinline__ void load_x(const uint8_t* rec, int v, XBlock& x) {
  // vector v's slot: 96 bytes of planes, then s, sum, fsum -- one 128-byte line
  const uint8_t* slot = rec + MMA_SLOT_BYTES * v;
#pragma unroll
  for (int p = 0; p < 3; ++p) {
    // plane p: words (0, 4, 1, 5) then (2, 6, 3, 7)
    const uint4 q0 = SRC::at(slot + 32 * p), q1 = SRC::at(slot + 32 * p + 16);
    x.planes[8 * p + 0] = q0.x;
    x.planes[8 * p + 4] = q0.y;
    x.planes[8 * p + 1] = q0.z;
    x.planes[8 * p + 5] = q0.w;
    x.planes[8 * p + 2] = q1.x;
    x.planes[8 * p + 6] = q1.y;
    x.planes[8 * p + 3] = q1.z;
    x.planes[8 * p + 7] = q1.w;
  }
  const uint4 scales = SRC::at(slot + 96);
  x.s = __uint_as_float(scales.x);
  x.sum = T::DTYPE == DRIFT_Q4_0 ? int(scales.y) : 0;
  x.fsum = T::DTYPE == DRIFT_Q4_1 ? __uint_as_float(scales.z) : 0.0f;
}

// ---- dp4a modes: 1 or 2 vectors --------------------------------------------------------------
// Lane l takes rows l and l + 32 of the tile. A half segment (4 blocks) of
// each row comes out of shared memory in 16-byte reads; each block's codes
// meet x's planes -- the same for every lane, broadcast loads shared by the
// two rows, fetched one block ahead -- in 24 dp4a, and acc = fmaf(s, value,
// acc) with the same value and order as the MMA mode: the plane sums are
// exact integers either way, so a row's result does not depend on the mode.
template <typename T, int V, typename SRC, int STRIDE, bool FULL>
__device__ __forceinline__ void segment_dp4a_blocks(const uint8_t* row0, const uint8_t* row1,
                                                    const uint8_t* rec0, int count,
                                                    float (&acc)[2][4]) {
  constexpr int HALF = 4 * T::BYTES;  // bytes of 4 blocks: 80, 72 or 136
  uint32_t w0[HALF / 4], w1[HALF / 4];
  XBlock x[2][V];
#pragma unroll
  for (int v = 0; v < V; ++v) load_x<T, SRC>(rec0, v, x[0][v]);
#pragma unroll
  for (int b = 0; b < SEG_BLOCKS; ++b) {
    if (FULL || b < count) {
      if (b == 0) {
        lds_span<0, HALF>(row0, w0);
        lds_span<0, HALF>(row1, w1);
      } else if (b == 4) {
        lds_span<HALF, 2 * HALF>(row0, w0);
        lds_span<HALF, 2 * HALF>(row1, w1);
      }
      if (b + 1 < SEG_BLOCKS && (FULL || b + 1 < count)) {
#pragma unroll
        for (int v = 0; v < V; ++v) load_x<T, SRC>(rec0 + (b + 1) * STRIDE, v, x[(b + 1) & 1][v]);
      }
      const int word = (b * T::BYTES) / 4 - (b >= 4 ? HALF / 4 : 0);
      uint32_t a[T::WORDS], c[T::WORDS];
#pragma unroll
      for (int j = 0; j < T::WORDS; ++j) {
        a[j] = w0[word + j];
        c[j] = w1[word + j];
      }
      const Codes r0 = T::decode(a, b), r1 = T::decode(c, b);
#pragma unroll
      for (int v = 0; v < V; ++v) {
        const XBlock& xv = x[b & 1][v];
        int p0, p1, p2;
        plane_sums<T>(r0, xv.planes, p0, p1, p2);
        acc[0][v] = fmaf(xv.s, mma_block_value<T>(p0, p1, p2, r0.d, r0.m, xv.sum, xv.fsum), acc[0][v]);
        plane_sums<T>(r1, xv.planes, p0, p1, p2);
        acc[1][v] = fmaf(xv.s, mma_block_value<T>(p0, p1, p2, r1.d, r1.m, xv.sum, xv.fsum), acc[1][v]);
      }
    }
  }
}

// `x`: the records in global memory, or (XSMEM) their first V slots copied
// to shared memory, 112 V bytes a block.
template <typename T, int V, bool XSMEM>
__device__ __forceinline__ void segment_dp4a(const uint8_t* stage, int first_block, int count,
                                             const uint8_t* x, float (&acc)[2][4]) {
  const int lane = threadIdx.x % WARP;
  const uint8_t* row0 = stage + lane * Ring<T>::PITCH;
  const uint8_t* row1 = row0 + 32 * Ring<T>::PITCH;
  using SRC = typename std::conditional<XSMEM, XShared, XGlobal>::type;
  constexpr int STRIDE = XSMEM ? MMA_SLOT_BYTES * V : MMA_RECORD_BYTES;
  const uint8_t* rec0 = x + (long long)first_block * STRIDE;
  if (count == SEG_BLOCKS)
    segment_dp4a_blocks<T, V, SRC, STRIDE, true>(row0, row1, rec0, SEG_BLOCKS, acc);
  else
    segment_dp4a_blocks<T, V, SRC, STRIDE, false>(row0, row1, rec0, count, acc);
}

// ---- MMA modes: 3-16 vectors ----------------------------------------------------------------
// load_fragment's x fragment from records copied to shared memory.
template <typename T>
__device__ __forceinline__ void load_fragment_shared(const uint8_t* rec, bool have_vector,
                                                     XFragment& x) {
  const int lane = threadIdx.x % 32, g = lane / 4, t = lane % 4;
#pragma unroll
  for (int p = 0; p < 3; ++p)
    x.planes[p] = have_vector ? *reinterpret_cast<const uint2*>(rec + mma_plane_byte(g, p, t))
                              : make_uint2(0, 0);
  const float* s0 = reinterpret_cast<const float*>(rec + mma_scale_byte(2 * t));
  const float* s1 = reinterpret_cast<const float*>(rec + mma_scale_byte(2 * t + 1));
  x.s = make_float2(s0[0], s1[0]);
  x.sum = T::DTYPE == DRIFT_Q4_0 ? make_int2(reinterpret_cast<const int*>(s0)[1],
                                             reinterpret_cast<const int*>(s1)[1])
                                 : make_int2(0, 0);
  x.fsum = T::DTYPE == DRIFT_Q4_1 ? make_float2(s0[2], s1[2]) : make_float2(0.0f, 0.0f);
}

// acc[i][4 p + .] gains the segment's blocks for rows (16 i + g, 16 i + g + 8)
// and vectors (8 p + 2t, 8 p + 2t + 1) of pass p (P passes, their records
// `pass_bytes` apart), each as acc = fmaf(s, value, acc); a row's weight
// fragment is unpacked once for every pass, and x is fetched one block ahead.
// A vector's arithmetic is the same in either mode, so 16 vectors give the
// bits of two 8-vector passes.
// XS: rec0 is the segment's records in shared memory, not global.
template <typename T, int P, bool FULL, bool XS>
__device__ __forceinline__ void segment_mma_blocks(const uint8_t* row_g, const uint8_t* rec0,
                                                   long long pass_bytes, int count, int vectors,
                                                   float (&acc)[4][4 * P]) {
  const int lane = threadIdx.x % WARP, g = lane / 4, t = lane % 4;
  auto fetch = [&](const uint8_t* rec, bool have, XFragment& x) {
    if constexpr (XS)
      load_fragment_shared<T>(rec, have, x);
    else
      load_fragment<T>(rec, have, x);
  };
  XFragment x[2][P];
#pragma unroll
  for (int p = 0; p < P; ++p) fetch(rec0 + p * pass_bytes, g + 8 * p < vectors, x[0][p]);
#pragma unroll
  for (int b = 0; b < SEG_BLOCKS; ++b) {
    if (FULL || b < count) {
      if (b + 1 < SEG_BLOCKS && (FULL || b + 1 < count))
#pragma unroll
        for (int p = 0; p < P; ++p)
          fetch(rec0 + (b + 1) * MMA_RECORD_BYTES + p * pass_bytes, g + 8 * p < vectors,
                x[(b + 1) & 1][p]);
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        uint32_t lo0, hi0, lo1, hi1;
        float d0, m0, d1, m1;
        fragment_row<T, SharedWords>(row_g + 16 * i * Ring<T>::PITCH, b, t, lo0, hi0, d0, m0);
        fragment_row<T, SharedWords>(row_g + (16 * i + 8) * Ring<T>::PITCH, b, t, lo1, hi1, d1, m1);
        const uint32_t a[4] = {lo0, lo1, hi0, hi1};
#pragma unroll
        for (int p = 0; p < P; ++p) {
          const XFragment& xb = x[b & 1][p];
          float* out = acc[i] + 4 * p;
          int p0[4], p1[4], p2[4];
          mma_i8_zero<T::SIGNED, false>(p0, a, xb.planes[0].x, xb.planes[0].y);
          mma_i8_zero<T::SIGNED, false>(p1, a, xb.planes[1].x, xb.planes[1].y);
          mma_i8_zero<T::SIGNED, true>(p2, a, xb.planes[2].x, xb.planes[2].y);
          out[0] = fmaf(xb.s.x, mma_block_value<T>(p0[0], p1[0], p2[0], d0, m0, xb.sum.x, xb.fsum.x), out[0]);
          out[1] = fmaf(xb.s.y, mma_block_value<T>(p0[1], p1[1], p2[1], d0, m0, xb.sum.y, xb.fsum.y), out[1]);
          out[2] = fmaf(xb.s.x, mma_block_value<T>(p0[2], p1[2], p2[2], d1, m1, xb.sum.x, xb.fsum.x), out[2]);
          out[3] = fmaf(xb.s.y, mma_block_value<T>(p0[3], p1[3], p2[3], d1, m1, xb.sum.y, xb.fsum.y), out[3]);
        }
      }
    }
  }
}

template <typename T, int P>
__device__ __forceinline__ void segment_mma(const uint8_t* stage, int first_block, int count,
                                            const uint8_t* __restrict__ records, int blocks,
                                            int vectors, float (&acc)[4][4 * P]) {
  const int lane = threadIdx.x % WARP, g = lane / 4;
  const uint8_t* rec0 = records + (long long)first_block * MMA_RECORD_BYTES;
  const uint8_t* row_g = stage + g * Ring<T>::PITCH;
  const long long pass_bytes = (long long)blocks * MMA_RECORD_BYTES;
  if (count == SEG_BLOCKS)
    segment_mma_blocks<T, P, true, false>(row_g, rec0, pass_bytes, SEG_BLOCKS, vectors, acc);
  else
    segment_mma_blocks<T, P, false, false>(row_g, rec0, pass_bytes, count, vectors, acc);
}

// The same with the segment's records (one pass) in a shared-memory slot.
template <typename T>
__device__ __forceinline__ void segment_mma_staged(const uint8_t* stage, int count,
                                                   const uint8_t* slot, int vectors,
                                                   float (&acc)[4][4]) {
  const int lane = threadIdx.x % WARP, g = lane / 4;
  const uint8_t* row_g = stage + g * Ring<T>::PITCH;
  if (count == SEG_BLOCKS)
    segment_mma_blocks<T, 1, true, true>(row_g, slot, 0, SEG_BLOCKS, vectors, acc);
  else
    segment_mma_blocks<T, 1, false, true>(row_g, slot, 0, count, vectors, acc);
}

// The accumulators of a warp: dp4a modes acc[r][v] for rows lane + 32 r;
// MMA modes acc[i][4 p + e] for the fragment of rows 16 i + g (+8), vectors
// 8 p + 2t (+1) of pass p.
template <int MODE>
struct Acc {
  static constexpr int I = mma_mode(MODE) ? 4 : 2, E = mma_mode(MODE) ? 4 * mode_passes(MODE) : 4;
  float a[I][E];
  __device__ void zero() {
#pragma unroll
    for (int i = 0; i < I; ++i)
#pragma unroll
      for (int e = 0; e < E; ++e) a[i][e] = 0.0f;
  }
  // the chain in shared memory (MMA modes), lane-major: slot (i, e) of lane l
  // at chain[(E i + e) 32 + l]. first: the tile's first group (the chain
  // starts as it); returns nothing -- the last group is added by `finish`.
  __device__ void chain_into(float* chain, bool first) const {
    const int lane = threadIdx.x % WARP;
#pragma unroll
    for (int i = 0; i < I; ++i)
#pragma unroll
      for (int e = 0; e < E; ++e) {
        float* c = chain + (E * i + e) * WARP + lane;
        *c = first ? a[i][e] : *c + a[i][e];
      }
  }
  // this (the last group's sums) after the chain so far
  __device__ void finish(const float* chain, bool first) {
    const int lane = threadIdx.x % WARP;
#pragma unroll
    for (int i = 0; i < I; ++i)
#pragma unroll
      for (int e = 0; e < E; ++e) a[i][e] = first ? a[i][e] : chain[(E * i + e) * WARP + lane] + a[i][e];
  }
  __device__ void add(const Acc& o) {
#pragma unroll
    for (int i = 0; i < I; ++i)
#pragma unroll
      for (int e = 0; e < E; ++e) a[i][e] += o.a[i][e];
  }
  // call f(row within the tile, vector, value) for each output this lane holds
  template <typename F>
  __device__ void each(F f) const {
    const int lane = threadIdx.x % WARP, g = lane / 4, t = lane % 4;
    if constexpr (mma_mode(MODE)) {
#pragma unroll
      for (int i = 0; i < 4; ++i)
#pragma unroll
        for (int p = 0; p < mode_passes(MODE); ++p) {
          f(16 * i + g, 8 * p + 2 * t, a[i][4 * p]);
          f(16 * i + g, 8 * p + 2 * t + 1, a[i][4 * p + 1]);
          f(16 * i + g + 8, 8 * p + 2 * t, a[i][4 * p + 2]);
          f(16 * i + g + 8, 8 * p + 2 * t + 1, a[i][4 * p + 3]);
        }
    } else {
#pragma unroll
      for (int r = 0; r < 2; ++r)
#pragma unroll
        for (int v = 0; v < MODE; ++v) f(lane + 32 * r, v, a[r][v]);
    }
  }
};

// A row's sum is a chain over fixed groups of its segments -- G of them:
// min(16, segments) for rows of 32 segments (8192 columns) or more, else
// min(8, segments) -- group g holding segments [segments g / G,
// segments (g + 1) / G);
// a group is summed block by block from zero and the row is
// ((group_0 + group_1) + group_2) + ... Whichever warps take which groups,
// the bits are the same -- so the schedule (tiles per warp, splits between
// warps and CTAs, other matrices sharing a launch, the number of vectors)
// never shows in the result.
// (Long rows need 16 units a tile to spread a few tiles over the SMs; on
// 4096-column rows the extra partial sums cost more than they give back.)
constexpr int MAX_GROUPS = 16, LONG_SEGMENTS = 32;
__host__ __device__ constexpr int group_count(long long segments) {
  const long long most = segments >= LONG_SEGMENTS ? MAX_GROUPS : 8;
  return int(segments < most ? segments : most);
}
struct Groups {
  int segments, count, first_end;
  unsigned long long ends;  // bit s: segment s ends a group (segments below 64)
  __device__ explicit Groups(int s) : segments(s), count(group_count(s)), ends(0) {
    for (int g = 1; g <= count; ++g)
      if (begin(g) - 1 < 64) ends |= 1ull << (begin(g) - 1);
    first_end = begin(1);
  }
  __device__ int begin(int g) const { return segments * g / count; }
  __device__ int of(int s) const { return ((s + 1) * count - 1) / segments; }
  __device__ bool last(int s) const {
    return s < 64 ? (ends >> s) & 1 : s + 1 == begin(of(s) + 1);
  }
  __device__ bool in_first(int s) const { return s < first_end; }
};

// Group sums of tiles split between warps: [slot][group][ROWS][slots], the
// slot a tile's index in a balanced launch, or a CTA's leftover tile in the
// tile schedule.
// (the tile schedule's most: 148 CTAs x 8 warps x 16 groups x 64 rows x 8
// slots, 9.7 M; a balanced launch's: 8192 units x 64 rows x 8 slots, 4.2 M)
constexpr long long PARTIAL_FLOATS = 10ll << 20;
__device__ __align__(16) float group_partials[PARTIAL_FLOATS];

// The chain of a tile's group sums (each ROWS x VSLOTS floats, `stride`
// floats apart from the next group's), N outputs a lane at a time (4 for
// the MMA mode, 2 for the dp4a modes) with eight groups' loads in flight;
// out(e, sum) takes output e of the tile. The order is ((0 + g0) + g1) + ...
// whatever the schedule.
template <int N>
struct Lanes;
template <>
struct Lanes<4> {
  using type = float4;
  __device__ static float get(const float4& v, int i) {
    return i == 0 ? v.x : i == 1 ? v.y : i == 2 ? v.z : v.w;
  }
  __device__ static void add(float4& s, const float4& v) {
    s.x += v.x;
    s.y += v.y;
    s.z += v.z;
    s.w += v.w;
  }
};
template <>
struct Lanes<2> {
  using type = float2;
  __device__ static float get(const float2& v, int i) { return i == 0 ? v.x : v.y; }
  __device__ static void add(float2& s, const float2& v) {
    s.x += v.x;
    s.y += v.y;
  }
};

template <int VSLOTS, typename OUT>
__device__ __forceinline__ void chain_groups(const float* sums, long long stride, int count,
                                             int first, int step, OUT out) {
  constexpr int N = VSLOTS >= 8 ? 4 : 2, E = ROWS * VSLOTS, BATCH = VSLOTS == 2 ? 4 : 8;
  using V = typename Lanes<N>::type;
  for (int en = first; en < E / N; en += step) {
    V sum = {};
    for (int g0 = 0; g0 < count; g0 += BATCH) {
      V p[BATCH];
#pragma unroll
      for (int g = 0; g < BATCH; ++g)
        if (g0 + g < count) p[g] = __ldcg(reinterpret_cast<const V*>(sums + (g0 + g) * stride) + en);
#pragma unroll
      for (int g = 0; g < BATCH; ++g)
        if (g0 + g < count) Lanes<N>::add(sum, p[g]);
    }
#pragma unroll
    for (int i = 0; i < N; ++i) out(N * en + i, Lanes<N>::get(sum, i));
  }
}

// The CTA's schedule. CTA c owns tiles [t0, t0 + count), an even share of the
// matrix's. Its W warps take them in rounds -- warp w sums tile t0 + f W + w
// whole in round f -- and the (count mod W) tiles left over are split by
// groups, P warps to a tile (a power of two, at most W / left and the group
// count), whose group sums meet in global memory and are chained in group
// order. All of it follows from rows, cols and the grid, never from the
// number of vectors.
struct Schedule {
  int t0, rounds, left, parts, segments, warps;
  Groups groups;
  __device__ Schedule(int tiles, int segs, int w) : segments(segs), warps(w), groups(segs) {
    t0 = int((long long)tiles * blockIdx.x / gridDim.x);
    const int t1 = int((long long)tiles * (blockIdx.x + 1) / gridDim.x);
    rounds = (t1 - t0) / w;
    left = (t1 - t0) % w;
    const int most = left ? (w / left < groups.count ? w / left : groups.count) : 1;
    parts = 1;
    while (parts * 2 <= most) parts *= 2;
  }
  __device__ bool shares(int w) const { return w < left * parts; }
  __device__ int share_tile(int w) const { return t0 + rounds * warps + w / parts; }
  __device__ int share_begin(int w) const {
    return groups.begin(groups.count * (w % parts) / parts);
  }
  __device__ int share_end(int w) const {
    return groups.begin(groups.count * (w % parts + 1) / parts);
  }
  // job j of warp w: (tile, segment)
  __device__ void job(int w, int j, int& tile, int& segment) const {
    const int whole = rounds * segments;
    if (j < whole) {
      tile = t0 + (j / segments) * warps + w;
      segment = j % segments;
    } else {
      tile = share_tile(w);
      segment = share_begin(w) + (j - whole);
    }
  }
  __device__ int jobs(int w) const {
    return rounds * segments + (shares(w) ? share_end(w) - share_begin(w) : 0);
  }
};

template <typename T, int MODE, bool XSMEM>
__global__ void __launch_bounds__(RingShape<T>::WARPS * 32, 1)
    matvec_ring_kernel(const __grid_constant__ CUtensorMap wmap,
                       const uint8_t* __restrict__ records, float* __restrict__ y, int rows,
                       int cols, int vectors, int* error) {
  using Shape = RingShape<T>;
  constexpr int W = Shape::WARPS, S = Shape::S, STAGE = Ring<T>::STAGE;
  constexpr int VSLOTS = mode_slots(MODE);
  extern __shared__ __align__(16) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~uintptr_t(1023));
  const int warp = threadIdx.x / WARP, lane = threadIdx.x % WARP;
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + Shape::BARS) + warp * S;
  volatile int* abort = reinterpret_cast<int*>(smem + Shape::BARS + W * S * 8);
  uint8_t* ring = smem + warp * S * STAGE;
  // The MMA mode's shared x: the warps' whole tiles walk the row's segments
  // in step (job j of every warp is segment j mod segments), so one copy of
  // a segment's records serves all W warps. Slot j mod NX holds job j's;
  // x_full[slot] completes when they land, x_empty[slot] when all W warps
  // are done with them. Thread 0 fills the slots NX - 1 jobs ahead of its
  // own warp, each after every warp has left the job it held before.
  // (XSMEM in the MMA mode: the launch takes the slots; a CTA of fewer
  // tiles than warps has no whole tiles and launches without them)
  constexpr int NX = MODE == MODE_MMA && XSMEM ? Shape::X_SLOTS : 0;
  uint8_t* x_slots = smem + Shape::XS_OFFSET;
  uint64_t* x_full = reinterpret_cast<uint64_t*>(smem + Shape::XBAR_OFFSET);
  uint64_t* x_empty = x_full + NX;

  const int blocks = cols / 32;
  const int segments = (blocks + SEG_BLOCKS - 1) / SEG_BLOCKS;
  const Schedule plan((rows + ROWS - 1) / ROWS, segments, W);
  const int jobs = plan.jobs(warp);
  const int whole = plan.rounds * segments;  // jobs of whole tiles (every warp the same)

  if (threadIdx.x == 0) *abort = 0;
  if (lane < S) tc::mbar_init(&bars[lane], 1);
  if (NX > 0 && threadIdx.x < NX) {
    tc::mbar_init(&x_full[threadIdx.x], 1);
    tc::mbar_init(&x_empty[threadIdx.x], W);
  }
  tc::fence_barrier_init();
  __syncthreads();
  // job q's records (q < whole) into its slot, by thread 0
  auto issue_x = [&](int q) {
    const int first = (q % segments) * SEG_BLOCKS;
    const int count = blocks - first < SEG_BLOCKS ? blocks - first : SEG_BLOCKS;
    const uint32_t bytes = uint32_t(count * MMA_RECORD_BYTES);
    tc::mbar_expect_tx(&x_full[q % NX], bytes);
    tc::bulk_load(x_slots + (q % NX) * Shape::X_SLOT, records + (long long)first * MMA_RECORD_BYTES,
                  bytes, &x_full[q % NX]);
  };
  int x_issued = 0;  // (thread 0's count)

  // With the shared slots, the MMA mode's other jobs (a leftover tile's
  // groups) bring their segment's x records (7 lines a block) into L1
  // ahead of use -- only once x is written, after pdl_wait, so that no line
  // of the kernel before lands in L1 first. (Without the slots, CTAs of a
  // tile or two, the prefetch costs more than it saves.)
  bool x_ready = false;
  auto prefetch_x = [&](int j) {
    if constexpr (NX > 0) {
      if (!x_ready || (NX > 0 && j < whole)) return;
      int tile, segment;
      plan.job(warp, j, tile, segment);
      constexpr int LINES = MMA_RECORD_BYTES / 128;
      for (int i = lane; i < SEG_BLOCKS * LINES; i += WARP) {
        const int b = segment * SEG_BLOCKS + i / LINES;
        if (b < blocks)
          asm volatile("prefetch.global.L1 [%0];" ::"l"(records + (long long)b * MMA_RECORD_BYTES +
                                                        128 * (i % LINES)));
      }
    }
  };
  // job j: one 2-D tensor copy of 64 rows x PITCH bytes (rows past the
  // matrix, and columns past a row, arrive as zeros)
  auto issue = [&](int j) {
    int tile, segment;
    plan.job(warp, j, tile, segment);
    if (lane == 0) {
      tc::mbar_expect_tx(&bars[j % S], uint32_t(STAGE));
      tc::tma_load_2d(ring + (j % S) * STAGE, &wmap, &bars[j % S], segment * (Ring<T>::SEG / 4),
                      tile * ROWS);
    }
    prefetch_x(j);
    __syncwarp();
  };

  int issued = 0, consumed = 0;
  bool ok = true;
  while (issued < jobs && issued < S) issue(issued++);
  pdl_trigger();
  pdl_wait();  // the weights' first copies are in flight; x is now ready
  x_ready = true;
  for (int j = 0; j < issued; ++j) prefetch_x(j);
  const uint8_t* x = records;
  if (NX > 0 && threadIdx.x == 0)
    for (; x_issued < NX - 1 && x_issued < whole; ++x_issued) issue_x(x_issued);
  if constexpr (XSMEM && !mma_mode(MODE)) {
    // While the first copies fly: the vectors' slots of every block's record,
    // 112 V bytes a block, into shared memory, where every row of every tile
    // reads them.
    constexpr int SLOT = MMA_SLOT_BYTES * MODE;
    uint8_t* xs = smem + Shape::X_OFFSET;
    for (int i = threadIdx.x; i < blocks * (SLOT / 16); i += blockDim.x) {
      const int block = i / (SLOT / 16), part = i % (SLOT / 16);
      *reinterpret_cast<uint4*>(xs + block * SLOT + 16 * part) = __ldg(
          reinterpret_cast<const uint4*>(records + (long long)block * MMA_RECORD_BYTES + 16 * part));
    }
    __syncthreads();
    x = xs;
  } else if constexpr (!mma_mode(MODE)) {
    // x stays in global memory: bring the line or two of each record that the
    // vectors' slots occupy into L1 before the first rows need them.
    constexpr int LINES = MODE == MODE_DP4A_1 ? 1 : 2;
    for (int i = threadIdx.x; i < blocks * LINES; i += blockDim.x)
      asm volatile("prefetch.global.L1 [%0];" ::"l"(records + (long long)(i / LINES) * MMA_RECORD_BYTES +
                                                    128 * (i % LINES)));
  }
  Acc<MODE> part, total;  // the group being summed; the chain of the tile's groups
  part.zero();
  total.zero();
  const Groups& groups = plan.groups;
  float* chain = reinterpret_cast<float*>(smem + Shape::X_OFFSET) + warp * 16 * mode_passes(MODE) * WARP;
  float* shared_sums = group_partials + (long long)blockIdx.x * W * groups.count * ROWS * VSLOTS;
  while (consumed < issued) {
    const int j = consumed;
    int tile, segment;
    plan.job(warp, j, tile, segment);
    const bool staged = NX > 0 && j < whole;
    if (ok) ok = tc::mbar_wait_warp(&bars[j % S], (j / S) & 1, abort, error);
    if (ok && staged) ok = tc::mbar_wait_warp(&x_full[j % NX], (j / NX) & 1, abort, error);
    if (ok) {
      const int first = segment * SEG_BLOCKS;
      const int count = blocks - first < SEG_BLOCKS ? blocks - first : SEG_BLOCKS;
      if constexpr (NX > 0) {
        if (staged)
          segment_mma_staged<T>(ring + (j % S) * STAGE, count, x_slots + (j % NX) * Shape::X_SLOT,
                                vectors, part.a);
        else
          segment_mma<T, 1>(ring + (j % S) * STAGE, first, count, records, blocks, vectors, part.a);
      } else if constexpr (mma_mode(MODE)) {
        segment_mma<T, mode_passes(MODE)>(ring + (j % S) * STAGE, first, count, records, blocks,
                                          vectors, part.a);
      } else {
        segment_dp4a<T, MODE, XSMEM>(ring + (j % S) * STAGE, first, count, x, part.a);
      }
    }
    __syncwarp();
    ++consumed;
    if (ok && issued < jobs) issue(issued++);  // refill the freed stage
    if (NX > 0 && staged) {
      if (ok && lane == 0) tc::mbar_arrive(&x_empty[j % NX]);
      // thread 0: job j + NX - 1's records, into the slot of job j - 1 once
      // every warp has left it
      const int q = j + NX - 1;
      if (warp == 0 && ok && q < whole) {
        bool free = true;
        if (lane == 0) {
          if (q >= NX) free = tc::mbar_wait(&x_empty[q % NX], ((q / NX) - 1) & 1, abort, error);
          if (free) {
            issue_x(q);
            x_issued = q + 1;
          }
        }
        ok = __shfl_sync(0xffffffffu, free, 0);
      }
    }
    if (!groups.last(segment)) continue;
    if (j < whole) {
      const bool first_group = groups.in_first(segment);
      if constexpr (mma_mode(MODE)) {
        if (segment != segments - 1) {
          part.chain_into(chain, first_group);
        } else {
          part.finish(chain, first_group);
          part.each([&](int r, int v, float value) {
            const int row = tile * ROWS + r;
            if (row < rows && v < vectors) y[(long long)v * rows + row] = value;
          });
        }
      } else {
        total.add(part);
        if (segment == segments - 1) {
          // a whole tile: write its rows, start the next
          total.each([&](int r, int v, float value) {
            const int row = tile * ROWS + r;
            if (row < rows && v < vectors) y[(long long)v * rows + row] = value;
          });
          total.zero();
        }
      }
    } else {
      // a group of a leftover tile: its sums to memory, chained below
      float* sums = shared_sums + ((long long)(tile - plan.t0 - plan.rounds * W) * groups.count +
                                   groups.of(segment)) * ROWS * VSLOTS;
      part.each([&](int r, int v, float value) {
        if (v < VSLOTS) sums[r * VSLOTS + v] = value;
      });
    }
    part.zero();
  }
  if (!ok) {
    // let the copies already issued land before the ring is reused or left
    volatile int never = 0;
    for (int j = consumed; j < issued; ++j) tc::mbar_wait(&bars[j % S], (j / S) & 1, &never, nullptr);
  }
  if (NX > 0 && threadIdx.x == 0) {
    // the x copies in flight (at most one a slot) land before the CTA is left
    volatile int never = 0;
    for (int q = x_issued - NX > 0 ? x_issued - NX : 0; q < x_issued; ++q)
      tc::mbar_wait(&x_full[q % NX], (q / NX) & 1, &never, nullptr);
  }
  if (plan.left > 0) {
    // the leftover tiles: their group sums chained in group order, warp w
    // taking tiles w, w + W, ...
    __syncthreads();
    for (int l = warp; l < plan.left; l += W) {
      const int tile = plan.t0 + plan.rounds * W + l;
      chain_groups<VSLOTS>(shared_sums + (long long)l * groups.count * ROWS * VSLOTS,
                           ROWS * VSLOTS, groups.count, lane, WARP, [&](int e, float sum) {
                             const int r = e / VSLOTS, v = e % VSLOTS, row = tile * ROWS + r;
                             if (row < rows && v < vectors) y[(long long)v * rows + row] = sum;
                           });
    }
  }
}

// ---- the balanced schedule: small launches, one or several matrices ----------------------
// A launch's units are its (tile, group) pairs, tile-major across the
// matrices of the launch, and warp w of the grid's G takes units [U w / G,
// U (w + 1) / G) -- a contiguous run of segments -- so every warp of every SM
// gets the same share, whatever the row counts. A warp that holds a whole
// tile chains its groups in registers; a tile split between warps leaves its
// group sums in global memory and the warp whose arrival completes the tile
// (a count per tile) chains them. The bits are the tile schedule's.
constexpr int MAX_MATRICES = 4;
constexpr int SPLIT_UNITS = 8192;  // the most units a balanced launch takes

struct SplitLaunch {
  CUtensorMap maps[MAX_MATRICES];
  float* y[MAX_MATRICES];
  int rows[MAX_MATRICES];
  int tile_end[MAX_MATRICES];  // matrix m holds the launch's tiles [tile_end[m - 1], tile_end[m])
  int count, cols, vectors;
  const uint8_t* records;
  int* error;
};

// Groups arrived per tile of a balanced launch, zero between launches (the
// completing warp clears its tile's).
__device__ int split_arrivals[SPLIT_UNITS];

template <typename T, int MODE>
__global__ void __launch_bounds__(RingShape<T>::WARPS * 32, 1)
    matvec_split_kernel(const __grid_constant__ SplitLaunch L) {
  using Shape = RingShape<T>;
  constexpr int W = Shape::WARPS, S = Shape::S, STAGE = Ring<T>::STAGE;
  constexpr int VSLOTS = mode_slots(MODE);
  extern __shared__ __align__(16) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~uintptr_t(1023));
  const int warp = threadIdx.x / WARP, lane = threadIdx.x % WARP;
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + Shape::BARS) + warp * S;
  volatile int* abort = reinterpret_cast<int*>(smem + Shape::BARS + W * S * 8);
  uint8_t* ring = smem + warp * S * STAGE;

  const int blocks = L.cols / 32;
  const int segments = (blocks + SEG_BLOCKS - 1) / SEG_BLOCKS;
  const Groups groups(segments);
  const long long U = (long long)L.tile_end[L.count - 1] * groups.count;
  const long long G = (long long)gridDim.x * W, gw = (long long)blockIdx.x * W + warp;
  // unit u starts at segment job (u / groups) segments + begin(u mod groups)
  auto start = [&](long long u) {
    return int(u / groups.count) * segments + groups.begin(int(u % groups.count));
  };
  const int j0 = start(U * gw / G), jobs = start(U * (gw + 1) / G) - j0;
  if (threadIdx.x == 0) *abort = 0;
  if (lane < S) tc::mbar_init(&bars[lane], 1);
  tc::fence_barrier_init();
  __syncthreads();

  // the matrix of a launch tile, and the tile within it
  auto locate = [&](int tile, int& m, int& local) {
    m = 0;
    while (m + 1 < L.count && tile >= L.tile_end[m]) ++m;
    local = tile - (m > 0 ? L.tile_end[m - 1] : 0);
  };
  // job j's x records' lines (the vectors' slots) into L1 ahead of use --
  // only once x is written, after pdl_wait, so that no line of the kernel
  // before lands in L1 first
  bool x_ready = false;
  auto prefetch_x = [&](int j) {
    if (!x_ready) return;
    const int segment = (j0 + j) % segments;
    constexpr int LINES = MODE == MODE_DP4A_1 ? 1 : MODE == MODE_DP4A_2 ? 2 : 7;
    for (int i = lane; i < SEG_BLOCKS * LINES * mode_passes(MODE); i += WARP) {
      const int pass = i / (SEG_BLOCKS * LINES), at = i % (SEG_BLOCKS * LINES);
      const int b = segment * SEG_BLOCKS + at / LINES;
      if (b < blocks)
        asm volatile("prefetch.global.L1 [%0];" ::"l"(L.records +
                                                      ((long long)pass * blocks + b) * MMA_RECORD_BYTES +
                                                      128 * (at % LINES)));
    }
  };
  // job j: its weights by one 2-D tensor copy, and its x lines
  auto issue = [&](int j) {
    const int job = j0 + j, tile = job / segments, segment = job % segments;
    int m, local;
    locate(tile, m, local);
    if (lane == 0) {
      tc::mbar_expect_tx(&bars[j % S], uint32_t(STAGE));
      tc::tma_load_2d(ring + (j % S) * STAGE, &L.maps[m], &bars[j % S],
                      segment * (Ring<T>::SEG / 4), local * ROWS);
    }
    prefetch_x(j);
    __syncwarp();
  };

  int issued = 0, landed = 0;
  bool ok = true;
  while (issued < jobs && issued < S) issue(issued++);
  pdl_trigger();
  pdl_wait();  // the weights' first copies are in flight; x is now ready
  x_ready = true;
  for (int j = 0; j < issued; ++j) prefetch_x(j);
  Acc<MODE> part, total;
  part.zero();
  total.zero();
  float* chain = reinterpret_cast<float*>(smem + Shape::X_OFFSET) + warp * 16 * mode_passes(MODE) * WARP;
  bool whole = false;  // this warp holds the current tile whole
  int first_group = 0;
  // every job is walked, even after a failed wait (as zeros), so that the
  // arrival counts stay whole for the next launch; the error word voids the
  // results
  for (int j = 0; j < jobs; ++j) {
    const int job = j0 + j, tile = job / segments, segment = job % segments;
    if (j == 0 || segment == 0) {
      // a tile starts: whole if all its segments are in this warp's share
      first_group = groups.of(segment);
      whole = segment == 0 && j + segments <= jobs;
    }
    if (ok && j < issued) {
      ok = tc::mbar_wait_warp(&bars[j % S], (j / S) & 1, abort, L.error);
      if (ok) landed = j + 1;
    }
    if (ok && j < issued) {
      const int first = segment * SEG_BLOCKS;
      const int count = blocks - first < SEG_BLOCKS ? blocks - first : SEG_BLOCKS;
      if constexpr (mma_mode(MODE))
        segment_mma<T, mode_passes(MODE)>(ring + (j % S) * STAGE, first, count, L.records, blocks,
                                          L.vectors, part.a);
      else
        segment_dp4a<T, MODE, false>(ring + (j % S) * STAGE, first, count, L.records, part.a);
    }
    __syncwarp();
    if (ok && issued < jobs) issue(issued++);  // refill the freed stage
    if (!groups.last(segment)) continue;  // a warp's share ends on a group's end
    const int group = groups.of(segment);
    int m, local;
    locate(tile, m, local);
    if (whole) {
      const bool first_group = group == 0;
      if constexpr (mma_mode(MODE)) {
        if (segment != segments - 1) {
          part.chain_into(chain, first_group);
        } else {
          part.finish(chain, first_group);
          part.each([&](int r, int v, float value) {
            const int row = local * ROWS + r;
            if (row < L.rows[m] && v < L.vectors) L.y[m][(long long)v * L.rows[m] + row] = value;
          });
        }
      } else {
        total.add(part);
        if (segment == segments - 1) {
          total.each([&](int r, int v, float value) {
            const int row = local * ROWS + r;
            if (row < L.rows[m] && v < L.vectors) L.y[m][(long long)v * L.rows[m] + row] = value;
          });
          total.zero();
        }
      }
      part.zero();
      continue;
    }
    float* tile_sums = group_partials + (long long)tile * groups.count * ROWS * VSLOTS;
    part.each([&](int r, int v, float value) {
      if (v < VSLOTS) tile_sums[(group * ROWS + r) * VSLOTS + v] = value;
    });
    part.zero();
    if (segment != segments - 1 && j != jobs - 1) continue;
    // this warp's groups of the tile are in memory: count them in; the warp
    // that completes the tile chains its groups
    __threadfence();
    __syncwarp();
    int done = 0;
    if (lane == 0) {
      const int mine = group - first_group + 1;
      done = atomicAdd(&split_arrivals[tile], mine) + mine == groups.count;
    }
    if (!__shfl_sync(0xffffffffu, done, 0)) continue;
    __threadfence();
    chain_groups<VSLOTS>(tile_sums, ROWS * VSLOTS, groups.count, lane, WARP, [&](int e, float sum) {
      const int r = e / VSLOTS, v = e % VSLOTS, row = local * ROWS + r;
      if (row < L.rows[m] && v < L.vectors) L.y[m][(long long)v * L.rows[m] + row] = sum;
    });
    if (lane == 0) split_arrivals[tile] = 0;
  }
  if (!ok) {
    // let the copies already issued land before the ring is left
    volatile int never = 0;
    for (int j = landed; j < issued; ++j) tc::mbar_wait(&bars[j % S], (j / S) & 1, &never, nullptr);
  }
}

// Whether the tile schedule's leftover group sums fit group_partials: a CTA
// per SM (or per tile), W warps' tiles of G groups, ROWS x slots floats each.
template <typename T>
bool ring_partials_fit(int rows, int cols, int mode) {
  const long long tiles = (rows + ROWS - 1) / ROWS;
  const long long grid = tiles < sm_count() ? tiles : sm_count();
  const long long segments = (cols / 32 + SEG_BLOCKS - 1) / SEG_BLOCKS;
  return grid * RingShape<T>::WARPS * group_count(segments) * ROWS * mode_slots(mode) <=
         PARTIAL_FLOATS;
}

template <typename T, int MODE, bool XSMEM>
int launch_mode(const CUtensorMap& wmap, const uint8_t* records, float* y, int rows, int cols,
                int vectors, int smem, cudaStream_t stream) {
  using Shape = RingShape<T>;
  static PerDevice configured;
  DRIFT_TRY(ensure_shared_memory(configured, matvec_ring_kernel<T, MODE, XSMEM>, MAX_SMEM));
  const int tiles = (rows + ROWS - 1) / ROWS;
  const unsigned grid = unsigned(tiles < sm_count() ? tiles : sm_count());
  // each CTA's leftover tiles keep their group sums in group_partials
  if (!ring_partials_fit<T>(rows, cols, MODE))
    return invalid("%u CTAs of leftover sums (at most %lld)", grid,
                   PARTIAL_FLOATS / (Shape::WARPS * MAX_GROUPS * ROWS * mode_slots(MODE)));
  DRIFT_CUDA(launch_pdl(matvec_ring_kernel<T, MODE, XSMEM>, grid, Shape::WARPS * 32, smem, stream,
                        wmap, records, y, rows, cols, vectors, device_error_word()));
  return 0;
}

// The 1-2 vector products stage x in shared memory when it fits beside the
// ring (112 bytes a block a vector: up to 14,500 columns for one Q4 vector)
// and every CTA has tiles enough to repay the copy (a small matrix is over
// before the staged x would pay for itself).
template <typename T, int MODE>
int launch_dp4a(const CUtensorMap& wmap, const uint8_t* records, float* y, int rows, int cols,
                int vectors, cudaStream_t stream) {
  const long long staged = RingShape<T>::BYTES + (long long)(cols / 32) * MMA_SLOT_BYTES * MODE;
  const long long tiles = (rows + ROWS - 1) / ROWS;
  if (staged <= MAX_SMEM && tiles >= 4LL * sm_count())
    return launch_mode<T, MODE, true>(wmap, records, y, rows, cols, vectors, int(staged), stream);
  return launch_mode<T, MODE, false>(wmap, records, y, rows, cols, vectors, RingShape<T>::BYTES,
                                     stream);
}

template <typename T, int MODE>
int launch_split_mode(const SplitLaunch& launch, long long units, cudaStream_t stream) {
  using Shape = RingShape<T>;
  static PerDevice configured;
  DRIFT_TRY(ensure_shared_memory(configured, matvec_split_kernel<T, MODE>, MAX_SMEM));
  // 1-2 vectors: a CTA per unit up to the SM count, so a few-unit product
  // streams through every SM (8 units to a CTA left SMs idle: the C4 step at
  // batch 1 1.2 % slower); the MMA mode keeps 8 units to a CTA, faster there
  long long grid = mma_mode(MODE) ? (units + Shape::WARPS - 1) / Shape::WARPS : units;
  if (grid > sm_count()) grid = sm_count();
  DRIFT_CUDA(launch_pdl(matvec_split_kernel<T, MODE>, unsigned(grid), Shape::WARPS * 32,
                        Shape::BYTES + Shape::chain_bytes(MODE), stream, launch));
  return 0;
}

// The units of a product in the balanced schedule: tiles x groups.
long long split_units(int64_t rows, int64_t cols) {
  const int64_t segments = (cols / 32 + SEG_BLOCKS - 1) / SEG_BLOCKS;
  return ((rows + ROWS - 1) / ROWS) * group_count(segments);
}

// One balanced launch over `count` matrices of one type sharing x (at most
// 16 vectors, SPLIT_UNITS units together).
template <typename T>
int split_dispatch(int count, const uint8_t* const* weights, float* const* ys, const int64_t* rows,
                   int cols, const uint8_t* records, int vectors, cudaStream_t stream) {
  SplitLaunch launch = {};
  int n = 0, tiles = 0;
  for (int i = 0; i < count; ++i) {
    if (rows[i] == 0) continue;
    DRIFT_TRY(encode_word_rows(&launch.maps[n], weights[i], int64_t(cols / 32) * T::BYTES / 4,
                               rows[i], Ring<T>::PITCH / 4, ROWS));
    tiles += int((rows[i] + ROWS - 1) / ROWS);
    launch.tile_end[n] = tiles;
    launch.y[n] = ys[i];
    launch.rows[n] = int(rows[i]);
    ++n;
  }
  if (n == 0) return 0;
  launch.count = n;
  launch.cols = cols;
  launch.vectors = vectors;
  launch.records = records;
  launch.error = device_error_word();
  const long long segments = (cols / 32 + SEG_BLOCKS - 1) / SEG_BLOCKS;
  const long long units = (long long)tiles * group_count(segments);
  if (units > SPLIT_UNITS) return invalid("a balanced launch of %lld units", units);
  if (vectors == 1) return launch_split_mode<T, MODE_DP4A_1>(launch, units, stream);
  if (vectors == 2) return launch_split_mode<T, MODE_DP4A_2>(launch, units, stream);
  if (vectors <= 8) return launch_split_mode<T, MODE_MMA>(launch, units, stream);
  if constexpr (RingShape<T>::MMA16) {
    return launch_split_mode<T, MODE_MMA16>(launch, units, stream);
  } else {
    // two 8-vector passes, the second on the next pass's records
    DRIFT_TRY((launch_split_mode<T, MODE_MMA>(launch, units, stream)));
    launch.records = records + (long long)(cols / 32) * MMA_RECORD_BYTES;
    launch.vectors = vectors - 8;
    for (int i = 0; i < n; ++i) launch.y[i] += 8ll * launch.rows[i];
    if (launch.vectors == 1) return launch_split_mode<T, MODE_DP4A_1>(launch, units, stream);
    if (launch.vectors == 2) return launch_split_mode<T, MODE_DP4A_2>(launch, units, stream);
    return launch_split_mode<T, MODE_MMA>(launch, units, stream);
  }
}

// One configuration per matrix type, whatever the number of vectors (and the
// group chain makes a row's bits the same in any schedule). A matrix of
// fewer tiles than SMs takes the balanced schedule, whose (tile, group)
// units reach every SM, for 1-2 vectors, 9-16 vectors (C4's step at batch 16
// 2.7 % faster than with the tile schedule) and for long rows; the MMA mode's
// products of shorter rows keep the tile schedule, which leaves SMs free for
// the next launch's early weight copies. 9-16 vectors take one MMA16 launch
// (two 8-vector passes where its leftover sums would not fit).
template <typename T>
int ring_dispatch(const uint8_t* weight, const uint8_t* records, float* y, int rows, int cols,
                  int vectors, cudaStream_t stream) {
  const int64_t rows64 = rows;
  if (vectors > 8 && (!RingShape<T>::MMA16 || !ring_partials_fit<T>(rows, cols, MODE_MMA16))) {
    DRIFT_TRY(ring_dispatch<T>(weight, records, y, rows, cols, 8, stream));
    return ring_dispatch<T>(weight, records + (long long)(cols / 32) * MMA_RECORD_BYTES,
                            y + 8ll * rows, rows, cols, vectors - 8, stream);
  }
  const bool few_tiles = (rows + ROWS - 1) / ROWS < sm_count();
  const bool long_rows = (cols / 32 + SEG_BLOCKS - 1) / SEG_BLOCKS >= LONG_SEGMENTS;
  if (few_tiles && (vectors <= 2 || vectors > 8 || long_rows) && split_units(rows64, cols) <= SPLIT_UNITS)
    return split_dispatch<T>(1, &weight, &y, &rows64, cols, records, vectors, stream);
  CUtensorMap wmap;
  DRIFT_TRY(encode_word_rows(&wmap, weight, int64_t(cols / 32) * T::BYTES / 4, rows,
                             Ring<T>::PITCH / 4, ROWS));
  if (vectors == 1) return launch_dp4a<T, MODE_DP4A_1>(wmap, records, y, rows, cols, vectors, stream);
  if (vectors == 2) return launch_dp4a<T, MODE_DP4A_2>(wmap, records, y, rows, cols, vectors, stream);
  if (vectors <= 8) {
    // the shared x slots where every CTA holds whole tiles (as many as its warps)
    const long long tiles = (rows + ROWS - 1) / ROWS;
    if (RingShape<T>::X_SLOTS && tiles >= (long long)RingShape<T>::WARPS * sm_count())
      return launch_mode<T, MODE_MMA, true>(wmap, records, y, rows, cols, vectors,
                                            RingShape<T>::mma_bytes(MODE_MMA, true), stream);
    return launch_mode<T, MODE_MMA, false>(wmap, records, y, rows, cols, vectors,
                                           RingShape<T>::mma_bytes(MODE_MMA, false), stream);
  }
  if constexpr (RingShape<T>::MMA16)
    return launch_mode<T, MODE_MMA16, false>(wmap, records, y, rows, cols, vectors,
                                             RingShape<T>::mma_bytes(MODE_MMA16, false), stream);
  return invalid("%d vectors in one pass", vectors);  // (taken as two passes above)
}

#define DRIFT_RING_REGISTER(T, name)                                                        \
  DRIFT_REGISTER(matvec_split_##name##_dp4a1, (matvec_split_kernel<T, MODE_DP4A_1>))          \
  DRIFT_REGISTER(matvec_split_##name##_dp4a2, (matvec_split_kernel<T, MODE_DP4A_2>))          \
  DRIFT_REGISTER(matvec_split_##name##_mma, (matvec_split_kernel<T, MODE_MMA>))               \
  DRIFT_REGISTER(matvec_ring_##name##_dp4a1, (matvec_ring_kernel<T, MODE_DP4A_1, false>))    \
  DRIFT_REGISTER(matvec_ring_##name##_dp4a1_xs, (matvec_ring_kernel<T, MODE_DP4A_1, true>))  \
  DRIFT_REGISTER(matvec_ring_##name##_dp4a2, (matvec_ring_kernel<T, MODE_DP4A_2, false>))    \
  DRIFT_REGISTER(matvec_ring_##name##_dp4a2_xs, (matvec_ring_kernel<T, MODE_DP4A_2, true>))  \
  DRIFT_REGISTER(matvec_ring_##name##_mma, (matvec_ring_kernel<T, MODE_MMA, false>))          \
  DRIFT_REGISTER(matvec_ring_##name##_mma_xs, (matvec_ring_kernel<T, MODE_MMA, true>))
// the 16-vector kernels of the types whose chain fits beside the ring
#define DRIFT_RING16_REGISTER(T, name)                                                      \
  DRIFT_REGISTER(matvec_split_##name##_mma16, (matvec_split_kernel<T, MODE_MMA16>))           \
  DRIFT_REGISTER(matvec_ring_##name##_mma16, (matvec_ring_kernel<T, MODE_MMA16, false>))
DRIFT_RING_REGISTER(Q8_0T, q8_0)
DRIFT_RING_REGISTER(Q4_0T, q4_0)
DRIFT_RING_REGISTER(Q4_1T, q4_1)
DRIFT_RING16_REGISTER(Q4_0T, q4_0)
DRIFT_RING16_REGISTER(Q4_1T, q4_1)
static_assert(RingShape<Q4_0T>::MMA16 && RingShape<Q4_1T>::MMA16, "the 16-vector chain fits");

}  // namespace

// Whether the staged kernel takes a product: 16-byte rows, 16-byte aligned
// weight, and a whole number of 16 bytes in the last segment of a row.
bool ring_supports(int weight_dtype, const void* weight, int64_t k) {
  const int64_t row = byte_size(weight_dtype, k);
  if (weight_dtype != DRIFT_Q8_0 && weight_dtype != DRIFT_Q4_0 && weight_dtype != DRIFT_Q4_1)
    return false;
  return row > 0 && row % 16 == 0 && (reinterpret_cast<uintptr_t>(weight) & 15) == 0 &&
         tensor_maps_available();
}

// Whether one balanced launch takes these products together (rows of one
// type, the same columns): each alone would take the balanced schedule too,
// so the results are the bits of separate products.
bool ring_many_fits(int weight_dtype, int count, const void* const* weights, const int64_t* rows,
                    int64_t cols) {
  if (count < 2 || count > MAX_MATRICES) return false;
  long long units = 0;
  for (int i = 0; i < count; ++i) {
    if (!ring_supports(weight_dtype, weights[i], cols)) return false;
    units += split_units(rows[i], cols);
  }
  return units <= SPLIT_UNITS;
}

// Products sharing x's records in balanced launches, 16 vectors at a time.
int matvec_ring_many(int weight_dtype, int count, const void* const* weights,
                     const uint8_t* records, float* const* ys, const int64_t* rows, int64_t cols,
                     int64_t vectors, cudaStream_t stream) {
  if (count > MAX_MATRICES) return invalid("%d products in one launch", count);
  const int64_t blocks = cols / 32;
  for (int64_t first = 0; first < vectors; first += 16) {
    const int n = int(vectors - first < 16 ? vectors - first : 16);
    const uint8_t* w[MAX_MATRICES];
    float* y[MAX_MATRICES];
    for (int i = 0; i < count; ++i) {
      w[i] = static_cast<const uint8_t*>(weights[i]);
      y[i] = ys[i] + first * rows[i];
    }
    const uint8_t* r = records + (first / 8) * blocks * MMA_RECORD_BYTES;
    switch (weight_dtype) {
      case DRIFT_Q8_0:
        DRIFT_TRY(split_dispatch<Q8_0T>(count, w, y, rows, int(cols), r, n, stream));
        break;
      case DRIFT_Q4_0:
        DRIFT_TRY(split_dispatch<Q4_0T>(count, w, y, rows, int(cols), r, n, stream));
        break;
      default:
        DRIFT_TRY(split_dispatch<Q4_1T>(count, w, y, rows, int(cols), r, n, stream));
    }
  }
  return 0;
}

int matvec_ring(int weight_dtype, const void* weight, const uint8_t* records, float* y,
                int64_t rows, int64_t cols, int64_t vectors, cudaStream_t stream) {
  const uint8_t* w = static_cast<const uint8_t*>(weight);
  switch (weight_dtype) {
    case DRIFT_Q8_0: return ring_dispatch<Q8_0T>(w, records, y, int(rows), int(cols), int(vectors), stream);
    case DRIFT_Q4_0: return ring_dispatch<Q4_0T>(w, records, y, int(rows), int(cols), int(vectors), stream);
    default: return ring_dispatch<Q4_1T>(w, records, y, int(rows), int(cols), int(vectors), stream);
  }
}

}  // namespace drift
