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

template <typename T, int MT, int KS, int S, int WARPS>
struct RingLayout {
  static constexpr int ROWS = 16 * MT;
  static constexpr int STAGE = ROWS * Ring<T>::PITCH;
  static constexpr int RING = WARPS * S * STAGE;
  static constexpr int BARS = RING;                            // WARPS x S mbarriers
  static constexpr int PARTIAL = BARS + WARPS * S * 8;         // [KS][WARPS/KS][ROWS][8] floats
  static constexpr int COUNTER = PARTIAL + (KS > 1 ? WARPS * ROWS * 8 * 4 : 0);
  static constexpr int BYTES = COUNTER + 16 + 1024;  // + room to align the base to 1024
};

// The products of one 8-block segment held in a stage: acc[i][.] gains the
// blocks' values for rows (16 i + g, 16 i + g + 8) and vectors (2t, 2t + 1),
// each as acc = fmaf(s, value, acc). V1: one vector, whose outputs are the
// first and third of each thread (t = 0); the others are not computed.
template <typename T, int MT, bool V1>
__device__ __forceinline__ void segment_products(const uint8_t* stage, int first_block, int count,
                                                 const uint8_t* __restrict__ records, int vectors,
                                                 float (&acc)[MT][4]) {
  const int lane = threadIdx.x % WARP, g = lane / 4, t = lane % 4;
  const bool have_vector = g < vectors;
  const bool have_v1 = !V1;
  const uint8_t* rec0 = records + (long long)first_block * MMA_RECORD_BYTES;
  const uint8_t* rows_lo[MT];
#pragma unroll
  for (int i = 0; i < MT; ++i) rows_lo[i] = stage + (16 * i + g) * Ring<T>::PITCH;
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
      for (int i = 0; i < MT; ++i) {
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
        acc[i][2] = fmaf(s.x, mma_block_value<T>(p0[2], p1[2], p2[2], d1, m1, sum.x, fsum.x), acc[i][2]);
        if (have_v1) {
          acc[i][1] = fmaf(s.y, mma_block_value<T>(p0[1], p1[1], p2[1], d0, m0, sum.y, fsum.y), acc[i][1]);
          acc[i][3] = fmaf(s.y, mma_block_value<T>(p0[3], p1[3], p2[3], d1, m1, sum.y, fsum.y), acc[i][3]);
        }
      }
    }
  }
}

// Grid (tiles schedule): at most one CTA per SM; `tiles` = ceil(rows / ROWS).
// Grid (split schedule): ceil(tiles / (WARPS / KS)) CTAs, one unit each.
template <typename T, int MT, int KS, int S, int WARPS, bool V1>
__global__ void __launch_bounds__(WARPS * 32, 1)
    matvec_ring_kernel(const __grid_constant__ CUtensorMap wmap,
                       const uint8_t* __restrict__ records, float* __restrict__ y, int rows,
                       int cols, int vectors, int* error) {
  using L = RingLayout<T, MT, KS, S, WARPS>;
  constexpr int ROWS = L::ROWS, GROUPS = WARPS / KS;
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
  const long long row_bytes = (long long)blocks * T::BYTES;
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
  // copy of ROWS rows x SEG bytes (rows past the matrix, and columns past a
  // row, arrive as zeros)
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
  float acc[MT][4];
#pragma unroll
  for (int i = 0; i < MT; ++i) acc[i][0] = acc[i][1] = acc[i][2] = acc[i][3] = 0.0f;
  while (consumed < issued) {
    const int j = consumed;
    const int segment = seg0 + j % nseg;
    if (j % nseg == 0) {
#pragma unroll
      for (int i = 0; i < MT; ++i) acc[i][0] = acc[i][1] = acc[i][2] = acc[i][3] = 0.0f;
    }
    if (ok) ok = tc::mbar_wait_warp(&bars[j % S], (j / S) & 1, abort, error);
    if (ok) {
      const int first = segment * SEG_BLOCKS;
      const int count = blocks - first < SEG_BLOCKS ? blocks - first : SEG_BLOCKS;
      segment_products<T, MT, V1>(ring + (j % S) * L::STAGE, first, count, records, vectors,
                                  acc);
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
    if (j % nseg == nseg - 1) {
      const int tile = claimed[(j / nseg) % 8];
      if (KS == 1) {
        // whole rows: write them
#pragma unroll
        for (int i = 0; i < MT; ++i) {
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
      }
    }
  }
  if (KS > 1) {
    // this warp's share of its unit's tile, then the shares in order
    float* partial = reinterpret_cast<float*>(smem + L::PARTIAL);
    if (nseg == 0) {
#pragma unroll
      for (int i = 0; i < MT; ++i) acc[i][0] = acc[i][1] = acc[i][2] = acc[i][3] = 0.0f;
    }
    float* mine = partial + ((kw * GROUPS + slot) * ROWS) * 8;
#pragma unroll
    for (int i = 0; i < MT; ++i) {
      mine[(16 * i + g) * 8 + 2 * t] = acc[i][0];
      mine[(16 * i + g) * 8 + 2 * t + 1] = acc[i][1];
      mine[(16 * i + g + 8) * 8 + 2 * t] = acc[i][2];
      mine[(16 * i + g + 8) * 8 + 2 * t + 1] = acc[i][3];
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

template <typename T, int MT, int KS, int S, int WARPS>
int launch_ring(const uint8_t* weight, const uint8_t* records, float* y, int rows, int cols,
                int vectors, cudaStream_t stream) {
  using L = RingLayout<T, MT, KS, S, WARPS>;
  CUtensorMap wmap;
  DRIFT_TRY(encode_word_rows(&wmap, weight, int64_t(cols / 32) * T::BYTES / 4, rows,
                             Ring<T>::SEG / 4, L::ROWS));
  static bool configured = false;
  if (!configured) {
    DRIFT_CUDA(cudaFuncSetAttribute(matvec_ring_kernel<T, MT, KS, S, WARPS, true>,
                                    cudaFuncAttributeMaxDynamicSharedMemorySize, L::BYTES));
    DRIFT_CUDA(cudaFuncSetAttribute(matvec_ring_kernel<T, MT, KS, S, WARPS, false>,
                                    cudaFuncAttributeMaxDynamicSharedMemorySize, L::BYTES));
    configured = true;
  }
  const int tiles = (rows + L::ROWS - 1) / L::ROWS;
  unsigned grid;
  if (KS == 1)
    grid = unsigned(tiles < sm_count() ? tiles : sm_count());
  else
    grid = unsigned((tiles + (WARPS / KS) - 1) / (WARPS / KS));
  if (vectors == 1)
    matvec_ring_kernel<T, MT, KS, S, WARPS, true><<<grid, WARPS * 32, L::BYTES, stream>>>(
        wmap, records, y, rows, cols, vectors, device_error_word());
  else
    matvec_ring_kernel<T, MT, KS, S, WARPS, false><<<grid, WARPS * 32, L::BYTES, stream>>>(
        wmap, records, y, rows, cols, vectors, device_error_word());
  DRIFT_LAUNCHED("matvec_ring");
  return 0;
}

// The configuration of a matrix: the same for every number of vectors, so a
// row's blocks are summed in the same order whatever the batch.
template <typename T>
int ring_dispatch(const uint8_t* weight, const uint8_t* records, float* y, int rows, int cols,
                  int vectors, cudaStream_t stream) {
  const int blocks = cols / 32;
  const int segments = (blocks + SEG_BLOCKS - 1) / SEG_BLOCKS;
  const long long tiles16 = (rows + 15) / 16;
  const int sms = sm_count();
  constexpr bool big = T::DTYPE == DRIFT_Q8_0;  // 272-byte segments
  // Many rows: whole tiles per warp, 16 warps per SM (32 rows each when the
  // segments are small enough: x records read once for both halves).
  if ((rows + 31) / 32 >= 16LL * sms) {
    if (big) return launch_ring<T, 1, 1, 3, 16>(weight, records, y, rows, cols, vectors, stream);
    return launch_ring<T, 2, 1, 2, 16>(weight, records, y, rows, cols, vectors, stream);
  }
  if (tiles16 >= 16LL * sms)
    return launch_ring<T, 1, 1, 3, 16>(weight, records, y, rows, cols, vectors, stream);
  // Few rows: split each tile's segments between warps so every SM works.
  int ks = 1;
  while (ks < 8 && ks * 2 <= segments && tiles16 * ks * 2 <= 16LL * sms) ks *= 2;
  if (ks < 2) ks = 2;
  switch (ks) {
    case 8: return launch_ring<T, 1, 8, 3, 8>(weight, records, y, rows, cols, vectors, stream);
    case 4: return launch_ring<T, 1, 4, 4, 8>(weight, records, y, rows, cols, vectors, stream);
    default: return launch_ring<T, 1, 2, 4, 8>(weight, records, y, rows, cols, vectors, stream);
  }
}

#define DRIFT_RING_REGISTER(T, name)                                                          \
  DRIFT_REGISTER(matvec_ring_##name##_mt2_w16, (matvec_ring_kernel<T, 2, 1, 2, 16, false>))   \
  DRIFT_REGISTER(matvec_ring_##name##_mt1_w16, (matvec_ring_kernel<T, 1, 1, 3, 16, false>))   \
  DRIFT_REGISTER(matvec_ring_##name##_ks2, (matvec_ring_kernel<T, 1, 2, 4, 8, false>))        \
  DRIFT_REGISTER(matvec_ring_##name##_ks4, (matvec_ring_kernel<T, 1, 4, 4, 8, false>))        \
  DRIFT_REGISTER(matvec_ring_##name##_ks8, (matvec_ring_kernel<T, 1, 8, 3, 8, false>))
DRIFT_RING_REGISTER(Q8_0T, q8_0)
DRIFT_RING_REGISTER(Q4_0T, q4_0)
DRIFT_RING_REGISTER(Q4_1T, q4_1)

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
