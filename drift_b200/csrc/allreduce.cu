// The tensor-parallel decode step's exchange over NVLink peer memory, fused
// into the kernel that consumes it. A row-split product (o, down: each rank
// sums its own columns' share) writes its partial rows into one of two send
// slots. The next kernel, on every rank, is `add_rms_norm_allreduce`: it
// pushes its partial rows into its lane of the slot on every rank (stores
// over NVLink), waits (bounded) until every rank's lane holds this call's
// rows, sums the ranks' partials in rank order from its own memory -- every
// rank the same bits -- adds the sum to the residual, and normalises,
// writing the next product's x records too. It takes the place of the
// runner's all-reduce followed by addRmsNorm (an NCCL collective and a norm
// launch) with one launch and one crossing of NVLink per value.
//
// Synchronisation: each value travels with its row's call count in one
// 64-bit word (value bits low, count high), stored and loaded whole, so a
// word that shows this call's count holds this call's value -- no fence and
// no separate flag round trip. A CTA (one row) counts its calls in a local
// counter (every rank makes the same calls in the same order, so the counts
// agree) and polls its lanes' words until each shows the count -- at most
// the comm's wait limit (one second unless drift_comm_create names
// another), after which it sets the device error word (code 3) and leaves
// the row as it was. The two slots alternate between consecutive exchanges
// (o, then down), so a lane is pushed into again only after every rank has
// passed the exchange in between, that is, after every rank has finished
// reading it.
#include <cuda_runtime.h>

#include <cstring>

#include "common.cuh"
#include "registry.cuh"
#include "rowwise.cuh"
#include "tc_common.cuh"
#include "x22.cuh"

namespace drift {

int* device_error_word();

namespace {

constexpr int MAX_RANKS = 8;
constexpr int MAX_ROWS = 64;

// The buffer of a rank: two send slots of partial rows (the products write
// them, F32), then per slot a lane per rank of 64-bit words (value, count)
// that the ranks push into, then the local call counts [MAX_ROWS].
struct Comm {
  int rank = 0, world = 1;
  size_t slot_bytes = 0;
  unsigned long long wait_ns = 0;
  uint8_t* local = nullptr;
  uint8_t* peers[MAX_RANKS] = {};
  bool opened[MAX_RANKS] = {};
  // send slot s; rank p's lane of slot s (twice the slot: a word per value)
  size_t send_offset(int s) const { return s * slot_bytes; }
  size_t lane_offset(int s, int p) const { return 2 * slot_bytes + (s * MAX_RANKS + p) * 2 * slot_bytes; }
  size_t counts_offset() const { return 2 * slot_bytes + 2 * MAX_RANKS * 2 * slot_bytes; }
  // a call count per (row, CTA of a row's cluster)
  size_t total() const { return counts_offset() + MAX_ROWS * 8 * 4; }
};

struct ExchangeArgs {
  const float* send;                      // this rank's send slot
  unsigned long long* pushes[MAX_RANKS];  // this rank's lane of the slot on every rank
  const unsigned long long* lanes;        // this rank's lanes of the slot (rank-major)
  unsigned* counts;                       // this rank's call counts
  long long lane_words;                   // words from one rank's lane to the next
  unsigned long long wait_ns;             // how long a row waits for its peers
  int rank, world;
  int* error;
};

__device__ __forceinline__ void store_relaxed_sys(unsigned long long* p, unsigned long long v) {
  asm volatile("st.relaxed.sys.global.b64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}
__device__ __forceinline__ unsigned long long load_relaxed_sys(const unsigned long long* p) {
  unsigned long long v;
  asm volatile("ld.relaxed.sys.global.b64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
  return v;
}

// x[row] += sum over ranks of the slots' row, in rank order; then out =
// rmsNorm(x) and (records) out's x records: rms_norm_kernel's arithmetic.
template <int PER, int THREADS>
__global__ void __launch_bounds__(THREADS) add_rms_norm_allreduce_kernel(
    const __grid_constant__ ExchangeArgs e, float* __restrict__ x, const float* __restrict__ weight,
    float* __restrict__ out, int cols, float epsilon, float weight_offset,
    uint8_t* __restrict__ records) {
  pdl_trigger();  // the next kernel may launch and wait for this one
  pdl_wait();     // this rank's partials (the product before) are written
  __shared__ float partial[32];
  __shared__ unsigned call;
  __shared__ int failed;
  const int row_index = blockIdx.x;
  if (threadIdx.x == 0) {
    call = e.counts[row_index] + 1;
    e.counts[row_index] = call;
    failed = 0;
  }
  __syncthreads();
  const unsigned long long count = (unsigned long long)call << 32;
  static_assert(MAX_RANKS * PER <= 32, "a thread's words fit one bit mask");
  // push this rank's partial row into its lane on every rank (plain stores
  // over NVLink: no round trip to wait for)
  {
    const float* mine = e.send + (long long)row_index * cols;
    unsigned long long own[PER];
#pragma unroll
    for (int i = 0; i < PER; ++i) {
      const int c = threadIdx.x + i * THREADS;
      own[i] = count | (c < cols ? __float_as_uint(mine[c]) : 0u);
    }
    for (int p = 0; p < e.world; ++p) {
      unsigned long long* to = e.pushes[p] + (long long)row_index * cols;
#pragma unroll
      for (int i = 0; i < PER; ++i) {
        const int c = threadIdx.x + i * THREADS;
        if (c < cols) store_relaxed_sys(to + c, own[i]);
      }
    }
  }
  // every rank's words of this row, each polled until it shows this call
  // (a pass's loads all in flight before the first is checked)
  float part[MAX_RANKS][PER];
  unsigned pending = 0;  // bit p PER + i: rank p's value i not yet in
#pragma unroll
  for (int p = 0; p < MAX_RANKS; ++p)
#pragma unroll
    for (int i = 0; i < PER; ++i) {
      part[p][i] = 0.0f;
      if (p < e.world && threadIdx.x + i * THREADS < cols) pending |= 1u << (p * PER + i);
    }
  const uint64_t start = tc::global_ns();
  while (pending) {
#pragma unroll
    for (int p = 0; p < MAX_RANKS; ++p) {
      if (p >= e.world) break;
      const unsigned long long* lane = e.lanes + p * e.lane_words + (long long)row_index * cols;
      unsigned long long w[PER];
#pragma unroll
      for (int i = 0; i < PER; ++i)
        w[i] = (pending >> (p * PER + i)) & 1u ? load_relaxed_sys(lane + threadIdx.x + i * THREADS)
                                               : 0ull;
#pragma unroll
      for (int i = 0; i < PER; ++i) {
        const unsigned bit = 1u << (p * PER + i);
        if ((pending & bit) && unsigned(w[i] >> 32) == call) {
          part[p][i] = __uint_as_float(unsigned(w[i]));
          pending &= ~bit;
        }
      }
    }
    if (!pending) break;
    if (tc::global_ns() - start > e.wait_ns) {
      atomicCAS(e.error, 0, 3);
      failed = 1;
      break;
    }
    __nanosleep(64);
  }
  __syncthreads();
  if (failed) return;
  float* row = x + (long long)row_index * cols;
  float value[PER], w[PER], sum[PER];
#pragma unroll
  for (int i = 0; i < PER; ++i) {
    const int c = threadIdx.x + i * THREADS;
    value[i] = c < cols ? row[c] : 0.0f;
    w[i] = c < cols ? weight[c] : 0.0f;
    sum[i] = 0.0f;
  }
  // summed in rank order
#pragma unroll
  for (int p = 0; p < MAX_RANKS; ++p)
    if (p < e.world) {
#pragma unroll
      for (int i = 0; i < PER; ++i) sum[i] += part[p][i];
    }
#pragma unroll
  for (int i = 0; i < PER; ++i) {
    const int c = threadIdx.x + i * THREADS;
    value[i] = value[i] + sum[i];
    if (c < cols) row[c] = value[i];
  }
  float squares = 0.0f;
#pragma unroll
  for (int i = 0; i < PER; ++i) squares = fmaf(value[i], value[i], squares);
  const float total = block_sum(squares, partial);
  const float scale = 1.0f / sqrtf(total / float(cols) + epsilon);
  float* target = out + (long long)row_index * cols;
#pragma unroll
  for (int i = 0; i < PER; ++i) {
    const int c = threadIdx.x + i * THREADS;
    const float normed = value[i] * scale * (w[i] + weight_offset);
    if (c < cols) target[c] = normed;
    if (records && c < cols) x22_record_block(normed, records, row_index, c / 32, cols / 32);
  }
}

DRIFT_REGISTER(add_rms_norm_allreduce_f32, (add_rms_norm_allreduce_kernel<4, 1024>))

// Rows of more than 1024 values, a cluster of SPLIT CTAs a row: the row's
// exchange and norm spread over SPLIT SMs instead of one. The rms norm
// kernel's 1024 threads (PER values each: columns t + 1024 i) are dealt out
// 128 to a CTA -- CTA j holds threads [128 j, 128 j + 128) -- so each
// thread's sum of squares and each warp's shuffle tree are that kernel's;
// the 32 warp sums meet through distributed shared memory and are added in
// warp order on every CTA: the bits of the one-CTA kernel (and of
// add_rms_norm). Each CTA pushes and polls its own columns with its own call
// count. A wait that runs out in any CTA leaves the whole row as it was:
// the CTAs' outcomes meet at the same cluster barrier as the sums, which
// every CTA reaches.
constexpr int SPLIT = 8, SPLIT_THREADS = 1024 / SPLIT;


template <int PER>
__global__ void __launch_bounds__(SPLIT_THREADS) add_rms_norm_allreduce_cluster_kernel(
    const __grid_constant__ ExchangeArgs e, float* __restrict__ x, const float* __restrict__ weight,
    float* __restrict__ out, int cols, float epsilon, float weight_offset,
    uint8_t* __restrict__ records) {
  pdl_trigger();  // the next kernel may launch and wait for this one
  pdl_wait();     // this rank's partials (the product before) are written
  constexpr int BIG = SPLIT * SPLIT_THREADS;  // the one-CTA kernel's threads
  __shared__ float sums[SPLIT_THREADS / 32];  // this CTA's four warp sums
  __shared__ float failed;                    // 1 when a wait ran out here
  __shared__ unsigned call;
  unsigned j;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(j));
  const int row_index = blockIdx.x / SPLIT;
  const int t = int(j) * SPLIT_THREADS + threadIdx.x;  // the one-CTA kernel's thread
  const int lane = threadIdx.x % 32, warp = threadIdx.x / 32;
  if (threadIdx.x == 0) {
    unsigned* counter = e.counts + row_index * SPLIT + j;
    call = *counter + 1;
    *counter = call;
    failed = 0.0f;
  }
  __syncthreads();
  const unsigned long long count = (unsigned long long)call << 32;
  static_assert(MAX_RANKS * PER <= 32, "a thread's words fit one bit mask");
  {
    const float* mine = e.send + (long long)row_index * cols;
    unsigned long long own[PER];
#pragma unroll
    for (int i = 0; i < PER; ++i) {
      const int c = t + i * BIG;
      own[i] = count | (c < cols ? __float_as_uint(mine[c]) : 0u);
    }
    for (int p = 0; p < e.world; ++p) {
      unsigned long long* to = e.pushes[p] + (long long)row_index * cols;
#pragma unroll
      for (int i = 0; i < PER; ++i) {
        const int c = t + i * BIG;
        if (c < cols) store_relaxed_sys(to + c, own[i]);
      }
    }
  }
  float part[MAX_RANKS][PER];
  unsigned pending = 0;
#pragma unroll
  for (int p = 0; p < MAX_RANKS; ++p)
#pragma unroll
    for (int i = 0; i < PER; ++i) {
      part[p][i] = 0.0f;
      if (p < e.world && t + i * BIG < cols) pending |= 1u << (p * PER + i);
    }
  const uint64_t start = tc::global_ns();
  while (pending) {
#pragma unroll
    for (int p = 0; p < MAX_RANKS; ++p) {
      if (p >= e.world) break;
      const unsigned long long* lane_words = e.lanes + p * e.lane_words + (long long)row_index * cols;
      unsigned long long w[PER];
#pragma unroll
      for (int i = 0; i < PER; ++i)
        w[i] = (pending >> (p * PER + i)) & 1u ? load_relaxed_sys(lane_words + t + i * BIG) : 0ull;
#pragma unroll
      for (int i = 0; i < PER; ++i) {
        const unsigned bit = 1u << (p * PER + i);
        if ((pending & bit) && unsigned(w[i] >> 32) == call) {
          part[p][i] = __uint_as_float(unsigned(w[i]));
          pending &= ~bit;
        }
      }
    }
    if (!pending) break;
    if (tc::global_ns() - start > e.wait_ns) {
      atomicCAS(e.error, 0, 3);
      failed = 1.0f;
      break;
    }
    __nanosleep(64);
  }
  float* row = x + (long long)row_index * cols;
  float value[PER], w[PER], sum[PER];
#pragma unroll
  for (int i = 0; i < PER; ++i) {
    const int c = t + i * BIG;
    value[i] = c < cols ? row[c] : 0.0f;
    w[i] = c < cols ? weight[c] : 0.0f;
    sum[i] = 0.0f;
  }
#pragma unroll
  for (int p = 0; p < MAX_RANKS; ++p)
    if (p < e.world) {
#pragma unroll
      for (int i = 0; i < PER; ++i) sum[i] += part[p][i];
    }
  float squares = 0.0f;
#pragma unroll
  for (int i = 0; i < PER; ++i) {
    value[i] = value[i] + sum[i];
    squares = fmaf(value[i], value[i], squares);
  }
#pragma unroll
  for (int o = 16; o > 0; o /= 2) squares += __shfl_xor_sync(0xffffffffu, squares, o);
  if (lane == 0) sums[warp] = squares;
  __syncthreads();
  cluster_sync();  // every CTA's warp sums and outcome are in
  float total = 0.0f, any_failed = 0.0f;
  for (int w32 = 0; w32 < BIG / 32; ++w32)
    total += cluster_load(&sums[w32 % (SPLIT_THREADS / 32)], unsigned(w32 / (SPLIT_THREADS / 32)));
  for (unsigned r = 0; r < SPLIT; ++r) any_failed += cluster_load(&failed, r);
  cluster_sync();  // every CTA has read the others' before any leaves
  if (any_failed != 0.0f) return;
  const float scale = 1.0f / sqrtf(total / float(cols) + epsilon);
  float* target = out + (long long)row_index * cols;
#pragma unroll
  for (int i = 0; i < PER; ++i) {
    const int c = t + i * BIG;
    if (c < cols) row[c] = value[i];
    const float normed = value[i] * scale * (w[i] + weight_offset);
    if (c < cols) target[c] = normed;
    if (records && c < cols) x22_record_block(normed, records, row_index, c / 32, cols / 32);
  }
}

// (not in the by-name table: it runs only as a cluster launch)

}  // namespace
}  // namespace drift

using namespace drift;

extern "C" {

int drift_comm_create(int rank, int world, size_t slot_bytes, int64_t wait_limit_ns, void** comm,
                      void* handle) {
  if (world < 1 || world > MAX_RANKS || rank < 0 || rank >= world)
    return invalid("comm: rank %d of %d (at most %d ranks)", rank, world, MAX_RANKS);
  if (!comm || !handle) return invalid("comm: no handle to fill");
  if (wait_limit_ns < 0 || wait_limit_ns > 60000000000ll)
    return invalid("comm: a wait limit of %lld ns (0 for one second, at most 60 s)",
                   (long long)wait_limit_ns);
  Comm* c = new Comm;
  c->rank = rank;
  c->world = world;
  c->wait_ns = wait_limit_ns ? (unsigned long long)wait_limit_ns : 1000000000ull;
  c->slot_bytes = (slot_bytes + 255) & ~size_t(255);
  void* memory = nullptr;
  cudaError_t status = cudaMalloc(&memory, c->total());
  if (status == cudaSuccess) status = cudaMemset(memory, 0, c->total());
  cudaIpcMemHandle_t ipc;
  if (status == cudaSuccess) status = cudaIpcGetMemHandle(&ipc, memory);
  if (status != cudaSuccess) {
    if (memory) cudaFree(memory);
    delete c;
    return cuda_status(status, "drift_comm_create");
  }
  c->local = static_cast<uint8_t*>(memory);
  c->peers[rank] = c->local;
  std::memcpy(handle, &ipc, sizeof(ipc));
  *comm = c;
  return 0;
}

size_t drift_comm_handle_bytes(void) { return sizeof(cudaIpcMemHandle_t); }

int drift_comm_open(void* comm, const void* handles) {
  Comm* c = static_cast<Comm*>(comm);
  if (!c || !handles) return invalid("comm: not created");
  const uint8_t* h = static_cast<const uint8_t*>(handles);
  for (int p = 0; p < c->world; ++p) {
    if (p == c->rank || c->opened[p]) continue;
    cudaIpcMemHandle_t ipc;
    std::memcpy(&ipc, h + p * sizeof(ipc), sizeof(ipc));
    void* peer = nullptr;
    DRIFT_CUDA(cudaIpcOpenMemHandle(&peer, ipc, cudaIpcMemLazyEnablePeerAccess));
    c->peers[p] = static_cast<uint8_t*>(peer);
    c->opened[p] = true;
  }
  return 0;
}

int drift_comm_slot(void* comm, int slot, void** pointer) {
  Comm* c = static_cast<Comm*>(comm);
  if (!c || slot < 0 || slot > 1 || !pointer) return invalid("comm: slot %d", slot);
  *pointer = c->local + c->send_offset(slot);
  return 0;
}

int drift_comm_destroy(void* comm) {
  Comm* c = static_cast<Comm*>(comm);
  if (!c) return 0;
  for (int p = 0; p < c->world; ++p)
    if (c->opened[p]) cudaIpcCloseMemHandle(c->peers[p]);
  if (c->local) cudaFree(c->local);
  delete c;
  return 0;
}

int drift_add_rms_norm_allreduce(void* comm, int slot, float* x, const float* weight,
                                 float epsilon, float weight_offset, float* out, int64_t rows,
                                 int64_t cols, void* prepared, drift_stream_t stream) {
  Comm* c = static_cast<Comm*>(comm);
  if (!c || slot < 0 || slot > 1) return invalid("addRmsNorm: no exchange slot %d", slot);
  if (rows < 0 || cols <= 0 || rows > MAX_ROWS || cols > 4096)
    return invalid("addRmsNorm over the exchange: [%lld, %lld] (at most %d rows of 4096)",
                   (long long)rows, (long long)cols, MAX_ROWS);
  if ((size_t)rows * cols * 4 > c->slot_bytes)
    return invalid("addRmsNorm over the exchange: %lld bytes in a slot of %zu",
                   (long long)(rows * cols * 4), c->slot_bytes);
  if (!x || !weight || !out) return invalid("addRmsNorm: a null tensor");
  if (prepared && cols % 32 != 0)
    return invalid("rmsNorm: prepared x needs rows of whole 32-value blocks");
  for (int p = 0; p < c->world; ++p)
    if (!c->peers[p]) return invalid("addRmsNorm: rank %d's buffer is not open", p);
  if (rows == 0) return 0;
  ExchangeArgs e = {};
  e.send = reinterpret_cast<const float*>(c->local + c->send_offset(slot));
  e.lanes = reinterpret_cast<const unsigned long long*>(c->local + c->lane_offset(slot, 0));
  e.lane_words = (long long)(2 * c->slot_bytes / 8);
  for (int p = 0; p < c->world; ++p)
    e.pushes[p] = reinterpret_cast<unsigned long long*>(c->peers[p] + c->lane_offset(slot, c->rank));
  e.counts = reinterpret_cast<unsigned*>(c->local + c->counts_offset());
  e.rank = c->rank;
  e.world = c->world;
  e.wait_ns = c->wait_ns;
  e.error = device_error_word();
  uint8_t* records = static_cast<uint8_t*>(prepared);
  const cudaStream_t s = cudaStream_t(stream);
  const unsigned grid = unsigned(rows);
  const int n = int(cols);
  // rows of more than 1024 values: a cluster of SPLIT CTAs a row, the
  // threads of launch_rms_norm's 1024-thread shape dealt out among them
  if (cols > 1024) {
    cudaLaunchConfig_t config = {};
    config.gridDim = dim3(grid * SPLIT);
    config.blockDim = dim3(SPLIT_THREADS);
    config.stream = s;
    cudaLaunchAttribute attribute[2];
    attribute[0].id = cudaLaunchAttributeClusterDimension;
    attribute[0].val.clusterDim.x = SPLIT;
    attribute[0].val.clusterDim.y = 1;
    attribute[0].val.clusterDim.z = 1;
    attribute[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attribute[1].val.programmaticStreamSerializationAllowed = 1;
    config.attrs = attribute;
    config.numAttrs = 2;
    if (cols <= 2048)
      DRIFT_CUDA(cudaLaunchKernelEx(&config, add_rms_norm_allreduce_cluster_kernel<2>, e, x, weight,
                                    out, n, epsilon, weight_offset, records));
    else
      DRIFT_CUDA(cudaLaunchKernelEx(&config, add_rms_norm_allreduce_cluster_kernel<4>, e, x, weight,
                                    out, n, epsilon, weight_offset, records));
    DRIFT_LAUNCHED("add_rms_norm_allreduce");
    return 0;
  }
  // the shapes of launch_rms_norm (layers.cu), so the norm's bits are its
#define DRIFT_EXCHANGE(PER, THREADS)                                                           \
  DRIFT_CUDA(launch_pdl(add_rms_norm_allreduce_kernel<PER, THREADS>, grid, THREADS, 0, s, e, x, \
                        weight, out, n, epsilon, weight_offset, records))
  if (cols <= 256) DRIFT_EXCHANGE(1, 256);
  else if (cols <= 512) DRIFT_EXCHANGE(2, 256);
  else if (cols <= 1024) DRIFT_EXCHANGE(4, 256);
  else if (cols <= 2048) DRIFT_EXCHANGE(2, 1024);
  else DRIFT_EXCHANGE(4, 1024);
#undef DRIFT_EXCHANGE
  DRIFT_LAUNCHED("add_rms_norm_allreduce");
  return 0;
}

}  // extern "C"
