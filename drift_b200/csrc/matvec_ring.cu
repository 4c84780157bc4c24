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

template <typename T>
struct Ring {
  static constexpr int SEG = SEG_BLOCKS * T::BYTES;
  // rows sit densely in a stage, as one 2-D tensor copy lays them out
  static constexpr int PITCH = SEG;
};

// Every tile is 32 rows: one row per lane in the dp4a modes, two 16-row MMA
// tiles in the MMA mode, so all modes share one schedule -- and one order of
// summation -- per matrix.
constexpr int ROWS = 32;
constexpr int MODE_DP4A_1 = 1, MODE_DP4A_2 = 2, MODE_MMA = 8;

template <typename T, int KS, int S, int WARPS>
struct RingLayout {
  static constexpr int STAGE = ROWS * Ring<T>::PITCH;
  static constexpr int RING = WARPS * S * STAGE;
  static constexpr int BARS = RING;                            // WARPS x S mbarriers
  static constexpr int PARTIAL = BARS + WARPS * S * 8;         // [KS][WARPS/KS][ROWS][8] floats
  static constexpr int COUNTER = PARTIAL + (KS > 1 ? WARPS * ROWS * 8 * 4 : 0);
  static constexpr int BYTES = COUNTER + 16 + 1024;  // + room to align the base to 1024
};

// ---- MMA mode: 3-8 vectors ---------------------------------------------------------------
// acc[i][.] gains the segment's blocks for rows (16 i + g, 16 i + g + 8) and
// vectors (2t, 2t + 1), each as acc = fmaf(s, value, acc).
template <typename T>
__device__ __forceinline__ void segment_mma(const uint8_t* stage, int first_block, int count,
                                            const uint8_t* __restrict__ records, int vectors,
                                            float (&acc)[2][4]) {
  const int lane = threadIdx.x % WARP, g = lane / 4, t = lane % 4;
  const bool have_vector = g < vectors;
  const uint8_t* rec0 = records + (long long)first_block * MMA_RECORD_BYTES;
  const uint8_t* rows_lo[2] = {stage + g * Ring<T>::PITCH, stage + (16 + g) * Ring<T>::PITCH};
#pragma unroll
  for (int b = 0; b < SEG_BLOCKS; ++b) {
    if (b < count) {
      const uint8_t* rec = rec0 + b * MMA_RECORD_BYTES;
      uint2 planes[3] = {make_uint2(0, 0), make_uint2(0, 0), make_uint2(0, 0)};
      if (have_vector) {
#pragma unroll
        for (int p = 0; p < 3; ++p) planes[p] = __ldg(reinterpret_cast<const uint2*>(rec) + p * 32 + lane);
      }
      const float2 s = __ldg(reinterpret_cast<const float2*>(rec + 768) + t);
      int2 sum = make_int2(0, 0);
      float2 fsum = make_float2(0.0f, 0.0f);
      if (T::DTYPE == DRIFT_Q4_0) sum = __ldg(reinterpret_cast<const int2*>(rec + 800) + t);
      if (T::DTYPE == DRIFT_Q4_1) fsum = __ldg(reinterpret_cast<const float2*>(rec + 832) + t);
#pragma unroll
      for (int i = 0; i < 2; ++i) {
        uint32_t lo0, hi0, lo1, hi1;
        float d0, m0, d1, m1;
        fragment_row<T, SharedWords>(rows_lo[i], b, t, lo0, hi0, d0, m0);
        fragment_row<T, SharedWords>(rows_lo[i] + 8 * Ring<T>::PITCH, b, t, lo1, hi1, d1, m1);
        const uint32_t a[4] = {lo0, lo1, hi0, hi1};
        int p0[4], p1[4], p2[4];
        mma_i8_zero<T::SIGNED, false>(p0, a, planes[0].x, planes[0].y);
        mma_i8_zero<T::SIGNED, false>(p1, a, planes[1].x, planes[1].y);
        mma_i8_zero<T::SIGNED, true>(p2, a, planes[2].x, planes[2].y);
        acc[i][0] = fmaf(s.x, mma_block_value<T>(p0[0], p1[0], p2[0], d0, m0, sum.x, fsum.x), acc[i][0]);
        acc[i][1] = fmaf(s.y, mma_block_value<T>(p0[1], p1[1], p2[1], d0, m0, sum.y, fsum.y), acc[i][1]);
        acc[i][2] = fmaf(s.x, mma_block_value<T>(p0[2], p1[2], p2[2], d1, m1, sum.x, fsum.x), acc[i][2]);
        acc[i][3] = fmaf(s.y, mma_block_value<T>(p0[3], p1[3], p2[3], d1, m1, sum.y, fsum.y), acc[i][3]);
      }
    }
  }
}

// ---- dp4a modes: 1 or 2 vectors ------------------------------------------------------------
// Lane r takes row r of the tile: its 8 blocks come out of shared memory in
// 16-byte reads, each block's codes meet x's planes (the same for every lane:
// broadcast loads) in 24 dp4a, and acc[v] = fmaf(s, value, acc[v]) with the
// same value and the same order as the MMA mode -- the plane sums are exact
// integers either way -- so a row's result does not depend on the mode.
template <typename T, int V>
__device__ __forceinline__ void segment_dp4a(const uint8_t* stage, int first_block, int count,
                                             const uint8_t* __restrict__ records, float (&acc)[4]) {
  constexpr int SEG = Ring<T>::SEG;
  constexpr int WORDS = SEG / 4;
  const int lane = threadIdx.x % WARP;
  uint32_t row[WORDS];
  const uint4* src = reinterpret_cast<const uint4*>(stage + lane * Ring<T>::PITCH);
#pragma unroll
  for (int i = 0; i < SEG / 16; ++i) {
    const uint4 q = src[i];
    row[4 * i] = q.x;
    row[4 * i + 1] = q.y;
    row[4 * i + 2] = q.z;
    row[4 * i + 3] = q.w;
  }
  const uint8_t* rec0 = records + (long long)first_block * MMA_RECORD_BYTES;
#pragma unroll
  for (int b = 0; b < SEG_BLOCKS; ++b) {
    if (b < count) {
      const int word = (b * T::BYTES) / 4;
      uint32_t w[T::WORDS];
#pragma unroll
      for (int i = 0; i < T::WORDS; ++i) w[i] = (word + i < WORDS) ? row[word + i] : 0u;
      const Codes codes = T::decode(w, b);
      const uint8_t* rec = rec0 + b * MMA_RECORD_BYTES;
#pragma unroll
      for (int v = 0; v < V; ++v) {
        uint32_t planes[24];
#pragma unroll
        for (int p = 0; p < 3; ++p) {
          const uint4* q = reinterpret_cast<const uint4*>(rec + 256 * p + 32 * v);
          const uint4 q0 = __ldg(q), q1 = __ldg(q + 1);
          planes[8 * p + 0] = q0.x;
          planes[8 * p + 4] = q0.y;
          planes[8 * p + 1] = q0.z;
          planes[8 * p + 5] = q0.w;
          planes[8 * p + 2] = q1.x;
          planes[8 * p + 6] = q1.y;
          planes[8 * p + 3] = q1.z;
          planes[8 * p + 7] = q1.w;
        }
        const float s = __ldg(reinterpret_cast<const float*>(rec + 768) + v);
        int sum = 0;
        float fsum = 0.0f;
        if (T::DTYPE == DRIFT_Q4_0) sum = __ldg(reinterpret_cast<const int*>(rec + 800) + v);
        if (T::DTYPE == DRIFT_Q4_1) fsum = __ldg(reinterpret_cast<const float*>(rec + 832) + v);
        int a0, a1, a2;
        plane_sums<T>(codes, planes, a0, a1, a2);
        acc[v] = fmaf(s, mma_block_value<T>(a0, a1, a2, codes.d, codes.m, sum, fsum), acc[v]);
      }
    }
  }
}

// Grid (tiles schedule, KS = 1): at most one CTA per SM.
// Grid (split schedule): ceil(tiles / (WARPS / KS)) CTAs, one unit each.
template <typename T, int KS, int S, int WARPS, int MODE>
__global__ void __launch_bounds__(WARPS * 32, 1)
    matvec_ring_kernel(const __grid_constant__ CUtensorMap wmap,
                       const uint8_t* __restrict__ records, float* __restrict__ y, int rows,
                       int cols, int vectors, int* error) {
  using L = RingLayout<T, KS, S, WARPS>;
  constexpr int GROUPS = WARPS / KS;
  extern __shared__ __align__(16) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~uintptr_t(1023));
  const int warp = threadIdx.x / WARP, lane = threadIdx.x % WARP;
  const int g = lane / 4, t = lane % 4;
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + L::BARS) + warp * S;
  uint8_t* ring = smem + warp * S * L::STAGE;
  int* counter = reinterpret_cast<int*>(smem + L::COUNTER);
  volatile int* abort = counter + 1;

  const int blocks = cols / 32;
  const int segments = (blocks + SEG_BLOCKS - 1) / SEG_BLOCKS;
  const int tiles = (rows + ROWS - 1) / ROWS;
  const int kw = warp % KS, slot = warp / KS;
  const int seg0 = int((long long)segments * kw / KS), seg1 = int((long long)segments * (kw + 1) / KS);
  const int nseg = seg1 - seg0;  // segments per tile for this warp

  // the CTA's tiles: a contiguous range (tiles schedule) or its unit's
  const int range0 = KS == 1 ? int((long long)tiles * blockIdx.x / gridDim.x) : 0;
  const int range1 = KS == 1 ? int((long long)tiles * (blockIdx.x + 1) / gridDim.x) : 0;
  if (threadIdx.x == 0) {
    *counter = range0;
    *abort = 0;
  }
  if (lane < S) tc::mbar_init(&bars[lane], 1);
  tc::fence_barrier_init();
  __syncthreads();

  // this warp's claimed tiles, in order (a short queue: at most S segments ahead)
  int claimed[8];
  int claimed_count = 0;
  bool more = nseg > 0;
  auto claim = [&]() -> bool {
    int tile;
    if (KS == 1) {
      int next = 0;
      if (lane == 0) next = atomicAdd(counter, 1);
      tile = __shfl_sync(0xffffffffu, next, 0);
      if (tile >= range1) return false;
    } else {
      if (claimed_count > 0) return false;  // one unit per CTA
      tile = blockIdx.x * GROUPS + slot;
      if (tile >= tiles) return false;
    }
    claimed[claimed_count % 8] = tile;
    ++claimed_count;
    return true;
  };
  // job j: segment seg0 + j % nseg of tile claimed[j / nseg], one 2-D tensor
  // copy of 32 rows x SEG bytes (rows past the matrix, and columns past a row,
  // arrive as zeros)
  auto issue = [&](int j) {
    const int tile = claimed[(j / nseg) % 8];
    const int segment = seg0 + j % nseg;
    uint64_t* bar = &bars[j % S];
    if (lane == 0) {
      tc::mbar_expect_tx(bar, uint32_t(L::STAGE));
      tc::tma_load_2d(ring + (j % S) * L::STAGE, &wmap, bar, segment * (Ring<T>::SEG / 4),
                      tile * ROWS);
    }
    __syncwarp();
  };

  int issued = 0, consumed = 0;
  bool ok = true;
  while (more && issued < S) {
    if (issued / nseg == claimed_count && !claim()) {
      more = false;
      break;
    }
    issue(issued++);
  }
  float acc[2][4];
#pragma unroll
  for (int i = 0; i < 2; ++i) acc[i][0] = acc[i][1] = acc[i][2] = acc[i][3] = 0.0f;
  while (consumed < issued) {
    const int j = consumed;
    const int segment = seg0 + j % nseg;
    if (j % nseg == 0) {
#pragma unroll
      for (int i = 0; i < 2; ++i) acc[i][0] = acc[i][1] = acc[i][2] = acc[i][3] = 0.0f;
    }
    if (ok) ok = tc::mbar_wait_warp(&bars[j % S], (j / S) & 1, abort, error);
    if (ok) {
      const int first = segment * SEG_BLOCKS;
      const int count = blocks - first < SEG_BLOCKS ? blocks - first : SEG_BLOCKS;
      if constexpr (MODE == MODE_MMA)
        segment_mma<T>(ring + (j % S) * L::STAGE, first, count, records, vectors, acc);
      else
        segment_dp4a<T, MODE>(ring + (j % S) * L::STAGE, first, count, records, acc[0]);
    }
    __syncwarp();
    ++consumed;
    // refill the freed stage
    if (ok && more) {
      if (issued / nseg == claimed_count && !claim())
        more = false;
      else
        issue(issued++);
    }
    if (KS == 1 && j % nseg == nseg - 1) {
      // whole rows: write them
      const int tile = claimed[(j / nseg) % 8];
      if constexpr (MODE == MODE_MMA) {
#pragma unroll
        for (int i = 0; i < 2; ++i) {
          const int r0 = tile * ROWS + 16 * i + g, r1 = r0 + 8;
          if (r0 < rows) {
            if (2 * t < vectors) y[(long long)(2 * t) * rows + r0] = acc[i][0];
            if (2 * t + 1 < vectors) y[(long long)(2 * t + 1) * rows + r0] = acc[i][1];
          }
          if (r1 < rows) {
            if (2 * t < vectors) y[(long long)(2 * t) * rows + r1] = acc[i][2];
            if (2 * t + 1 < vectors) y[(long long)(2 * t + 1) * rows + r1] = acc[i][3];
          }
        }
      } else {
        const int row = tile * ROWS + lane;
        if (row < rows) {
#pragma unroll
          for (int v = 0; v < MODE; ++v)
            if (v < vectors) y[(long long)v * rows + row] = acc[0][v];
        }
      }
    }
  }
  if (KS > 1) {
    // this warp's share of its unit's tile, then the shares in order
    float* partial = reinterpret_cast<float*>(smem + L::PARTIAL);
    float* mine = partial + ((kw * GROUPS + slot) * ROWS) * 8;
    if constexpr (MODE == MODE_MMA) {
#pragma unroll
      for (int i = 0; i < 2; ++i) {
        mine[(16 * i + g) * 8 + 2 * t] = acc[i][0];
        mine[(16 * i + g) * 8 + 2 * t + 1] = acc[i][1];
        mine[(16 * i + g + 8) * 8 + 2 * t] = acc[i][2];
        mine[(16 * i + g + 8) * 8 + 2 * t + 1] = acc[i][3];
      }
    } else {
#pragma unroll
      for (int v = 0; v < MODE; ++v) mine[lane * 8 + v] = acc[0][v];
    }
    __syncthreads();
    for (int e = threadIdx.x; e < GROUPS * ROWS * 8; e += blockDim.x) {
      const int gi = e / (ROWS * 8), r = (e / 8) % ROWS, v = e % 8;
      const int row = (blockIdx.x * GROUPS + gi) * ROWS + r;
      if (row < rows && v < vectors) {
        float total = 0.0f;
#pragma unroll
        for (int k = 0; k < KS; ++k) total += partial[((k * GROUPS + gi) * ROWS + r) * 8 + v];
        y[(long long)v * rows + row] = total;
      }
    }
  }
  if (!ok) {
    // let the copies already issued land before the CTA leaves
    volatile int never = 0;
    for (int j = consumed; j < issued; ++j) tc::mbar_wait(&bars[j % S], (j / S) & 1, &never, nullptr);
  }
}

template <typename T, int KS, int S, int WARPS, int MODE>
int launch_mode(const CUtensorMap& wmap, const uint8_t* records, float* y, int rows, int cols,
                int vectors, cudaStream_t stream) {
  using L = RingLayout<T, KS, S, WARPS>;
  static bool configured = false;
  if (!configured) {
    DRIFT_CUDA(cudaFuncSetAttribute(matvec_ring_kernel<T, KS, S, WARPS, MODE>,
                                    cudaFuncAttributeMaxDynamicSharedMemorySize, L::BYTES));
    configured = true;
  }
  const int tiles = (rows + ROWS - 1) / ROWS;
  unsigned grid;
  if (KS == 1)
    grid = unsigned(tiles < sm_count() ? tiles : sm_count());
  else
    grid = unsigned((tiles + (WARPS / KS) - 1) / (WARPS / KS));
  matvec_ring_kernel<T, KS, S, WARPS, MODE><<<grid, WARPS * 32, L::BYTES, stream>>>(
      wmap, records, y, rows, cols, vectors, device_error_word());
  DRIFT_LAUNCHED("matvec_ring");
  return 0;
}

template <typename T, int KS, int S, int WARPS>
int launch_ring(const uint8_t* weight, const uint8_t* records, float* y, int rows, int cols,
                int vectors, cudaStream_t stream) {
  CUtensorMap wmap;
  DRIFT_TRY(encode_word_rows(&wmap, weight, int64_t(cols / 32) * T::BYTES / 4, rows,
                             Ring<T>::SEG / 4, ROWS));
  if (vectors == 1)
    return launch_mode<T, KS, S, WARPS, MODE_DP4A_1>(wmap, records, y, rows, cols, vectors, stream);
  if (vectors == 2)
    return launch_mode<T, KS, S, WARPS, MODE_DP4A_2>(wmap, records, y, rows, cols, vectors, stream);
  return launch_mode<T, KS, S, WARPS, MODE_MMA>(wmap, records, y, rows, cols, vectors, stream);
}

// The configuration of a matrix: the same for every number of vectors, so a
// row's blocks are summed in the same order whatever the batch.
template <typename T>
int ring_dispatch(const uint8_t* weight, const uint8_t* records, float* y, int rows, int cols,
                  int vectors, cudaStream_t stream) {
  const int blocks = cols / 32;
  const int segments = (blocks + SEG_BLOCKS - 1) / SEG_BLOCKS;
  const long long tiles = (rows + ROWS - 1) / ROWS;
  const int sms = sm_count();
  constexpr int WIDE = T::DTYPE == DRIFT_Q8_0 ? 12 : 16;  // warps per CTA (272-byte segments: 12)
  // Many rows: whole tiles per warp, tiles claimed within the CTA's range.
  if (tiles >= 2LL * WIDE * sms)
    return launch_ring<T, 1, 2, WIDE>(weight, records, y, rows, cols, vectors, stream);
  // Fewer rows: split each tile's segments between warps so every SM works.
  int ks = 2;
  while (ks < 8 && ks * 2 <= segments && tiles * ks < 8LL * sms) ks *= 2;
  switch (ks) {
    case 8: return launch_ring<T, 8, 3, 8>(weight, records, y, rows, cols, vectors, stream);
    case 4: return launch_ring<T, 4, 3, 8>(weight, records, y, rows, cols, vectors, stream);
    default: return launch_ring<T, 2, 3, 8>(weight, records, y, rows, cols, vectors, stream);
  }
}

#define DRIFT_RING_REGISTER(T, name, wide)                                                      \
  DRIFT_REGISTER(matvec_ring_##name##_tiles_dp4a1, (matvec_ring_kernel<T, 1, 2, wide, 1>))     \
  DRIFT_REGISTER(matvec_ring_##name##_tiles_dp4a2, (matvec_ring_kernel<T, 1, 2, wide, 2>))     \
  DRIFT_REGISTER(matvec_ring_##name##_tiles_mma, (matvec_ring_kernel<T, 1, 2, wide, 8>))       \
  DRIFT_REGISTER(matvec_ring_##name##_ks2_dp4a1, (matvec_ring_kernel<T, 2, 3, 8, 1>))          \
  DRIFT_REGISTER(matvec_ring_##name##_ks4_dp4a1, (matvec_ring_kernel<T, 4, 3, 8, 1>))          \
  DRIFT_REGISTER(matvec_ring_##name##_ks8_dp4a1, (matvec_ring_kernel<T, 8, 3, 8, 1>))          \
  DRIFT_REGISTER(matvec_ring_##name##_ks2_mma, (matvec_ring_kernel<T, 2, 3, 8, 8>))            \
  DRIFT_REGISTER(matvec_ring_##name##_ks4_mma, (matvec_ring_kernel<T, 4, 3, 8, 8>))            \
  DRIFT_REGISTER(matvec_ring_##name##_ks8_mma, (matvec_ring_kernel<T, 8, 3, 8, 8>))
DRIFT_RING_REGISTER(Q8_0T, q8_0, 12)
DRIFT_RING_REGISTER(Q4_0T, q4_0, 16)
DRIFT_RING_REGISTER(Q4_1T, q4_1, 16)

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
