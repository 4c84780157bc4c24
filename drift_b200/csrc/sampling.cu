// Sampling on the device: each row's argmax and its `count` largest
// candidates (SequenceOps.argmax / candidates, runner/src/drift/runner/ops/
// SequenceOps.scala:14-20; CPU ops/CpuSequence.scala:12-27 and
// ops/Candidates.scala:10-36; GPU kernels/norm.hip:119-153, 322-363), so a
// decode step picks its next tokens without copying 151,936 logits a row to
// the host. With the vocabulary split over ranks, each rank reduces its rows
// to (value, id) pairs and a merge over the gathered pairs picks the same
// tokens on every rank.
//
// Orders (the CPU reference's, bit for bit):
//  - argmax: the first index of the largest value, values compared with `>`
//    from index 0 (CpuSequence.argmax): a NaN never wins, except at index 0,
//    which nothing then replaces. Key: the value's order-keeping bits (NaN
//    lowest; the NaN at global id 0 highest) above the id, lower ids higher.
//  - candidates: Candidates.rank -- larger floats first, -0 as 0, a positive
//    NaN above +inf, a negative NaN below -inf -- then the lower id.
// Both keys are 64-bit (order bits << 32 | ~id): unique per row, so a
// selection by key is exact.
#include <cuda_runtime.h>

#include "common.cuh"
#include "registry.cuh"

namespace drift {

int workspace_reserve(size_t bytes, void** pointer);

namespace {

constexpr int MAX_SAMPLE_ROWS = 4096;
constexpr int CANDIDATE_CHUNK = 4096;  // values a selection CTA takes (the reference's too)
constexpr int MAX_CANDIDATES = 1024;   // SequenceOps.MaximumCandidates
constexpr int SELECT_THREADS = 1024;
constexpr int ARGMAX_THREADS = 256, ARGMAX_SPAN = 8192;  // values an argmax CTA reads

// Per-row state of the launches below, zero between calls: the argmax's best
// key, and the arrival counts that find each row's last CTA (which resets
// them). Operations on one device run as one stream (as the library's other
// device arrays).
__device__ unsigned long long argmax_best[MAX_SAMPLE_ROWS];
__device__ unsigned sample_arrivals[MAX_SAMPLE_ROWS];

__device__ __forceinline__ uint32_t order_bits(float v) {
  const uint32_t bits = __float_as_uint(v == 0.0f ? 0.0f : v);
  return (bits & 0x80000000u) ? ~bits : (bits | 0x80000000u);
}

__device__ __forceinline__ unsigned long long argmax_key(float v, long long id) {
  uint32_t order;
  if (isnan(v)) order = id == 0 ? 0xffffffffu : 0u;
  else order = order_bits(v);
  return (uint64_t(order) << 32) | uint32_t(~uint32_t(id));
}

__device__ __forceinline__ unsigned long long candidate_key(float v, long long id) {
  return (uint64_t(order_bits(v)) << 32) | uint32_t(~uint32_t(id));
}

__device__ __forceinline__ unsigned long long warp_max64(unsigned long long v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const unsigned long long other = __shfl_xor_sync(0xffffffffu, v, o);
    v = other > v ? other : v;
  }
  return v;
}

// ---- argmax -------------------------------------------------------------------------------
// Grid (ceil(width / ARGMAX_SPAN), rows): each CTA the largest key of its
// span, by atomicMax into the row's best; the row's last CTA writes the id
// (and value) and clears the row's state.
__global__ void __launch_bounds__(ARGMAX_THREADS)
    argmax_rows_kernel(const float* __restrict__ values, long long width, long long id_offset,
                       int* __restrict__ ids, float* __restrict__ out_values) {
  pdl_trigger();
  pdl_wait();
  __shared__ unsigned long long warp_best[ARGMAX_THREADS / 32];
  __shared__ bool last;
  const int row = blockIdx.y;
  const float* v = values + (long long)row * width;
  const long long begin = (long long)blockIdx.x * ARGMAX_SPAN;
  const long long end = min(width, begin + ARGMAX_SPAN);
  unsigned long long best = 0;
  for (long long i = begin + threadIdx.x; i < end; i += ARGMAX_THREADS) {
    const unsigned long long key = argmax_key(v[i], i + id_offset);
    best = key > best ? key : best;
  }
  best = warp_max64(best);
  if (threadIdx.x % 32 == 0) warp_best[threadIdx.x / 32] = best;
  __syncthreads();
  if (threadIdx.x == 0) {
    for (int w = 1; w < ARGMAX_THREADS / 32; ++w) best = warp_best[w] > best ? warp_best[w] : best;
    atomicMax(&argmax_best[row], best);
    __threadfence();
    last = atomicAdd(&sample_arrivals[row], 1u) == gridDim.x - 1;
    if (last) {
      __threadfence();
      const unsigned long long winner = atomicExch(&argmax_best[row], 0ull);
      sample_arrivals[row] = 0;
      const long long id = (long long)uint32_t(~uint32_t(winner));
      ids[row] = int(id);
      if (out_values) out_values[row] = v[id - id_offset];
    }
  }
}

// The merge over gathered pairs: rows of n (value, id) pairs, one CTA a row.
__global__ void __launch_bounds__(ARGMAX_THREADS)
    argmax_merge_kernel(const float* __restrict__ values, const int* __restrict__ ids_in, long long n,
                        int* __restrict__ ids, float* __restrict__ out_values) {
  pdl_trigger();
  pdl_wait();
  __shared__ unsigned long long warp_best[ARGMAX_THREADS / 32];
  __shared__ long long at[ARGMAX_THREADS / 32];
  const int row = blockIdx.x;
  unsigned long long best = 0;
  long long best_at = 0;
  for (long long i = threadIdx.x; i < n; i += ARGMAX_THREADS) {
    const unsigned long long key = argmax_key(values[row * n + i], ids_in[row * n + i]);
    if (key > best) best = key, best_at = i;
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const unsigned long long other = __shfl_xor_sync(0xffffffffu, best, o);
    const long long other_at = __shfl_xor_sync(0xffffffffu, best_at, o);
    if (other > best) best = other, best_at = other_at;
  }
  if (threadIdx.x % 32 == 0) warp_best[threadIdx.x / 32] = best, at[threadIdx.x / 32] = best_at;
  __syncthreads();
  if (threadIdx.x == 0) {
    for (int w = 1; w < ARGMAX_THREADS / 32; ++w)
      if (warp_best[w] > best) best = warp_best[w], best_at = at[w];
    ids[row] = ids_in[row * n + best_at];
    if (out_values) out_values[row] = values[row * n + best_at];
  }
}

// ---- selection of the k largest keys (k <= 1024) by one CTA of 1024 threads ----------------
struct Selection {
  unsigned int histogram[256];
  unsigned long long prefix;
  unsigned int remaining;
  unsigned int taken;
  unsigned long long keys[MAX_CANDIDATES];
  int at[MAX_CANDIDATES];  // the item each kept key came from
};

// The k-th largest of n unique keys, by eight passes of 8-bit digits from the
// top: each pass counts the keys that match the digits found so far.
template <typename KeyAt>
__device__ unsigned long long kth_largest(KeyAt key_at, int n, int k, Selection& s) {
  if (threadIdx.x == 0) {
    s.prefix = 0;
    s.remaining = unsigned(k);
  }
  unsigned long long mask = 0;
  for (int pass = 0; pass < 8; ++pass) {
    const int shift = 56 - 8 * pass;
    for (int d = threadIdx.x; d < 256; d += blockDim.x) s.histogram[d] = 0;
    __syncthreads();
    const unsigned long long prefix = s.prefix;
    for (int i = threadIdx.x; i < n; i += blockDim.x) {
      const unsigned long long key = key_at(i);
      if ((key & mask) == prefix) atomicAdd(&s.histogram[(key >> shift) & 255], 1u);
    }
    __syncthreads();
    if (threadIdx.x < 32) {
      // lane l holds digits 255 - 8 l .. 248 - 8 l: the counts above each
      const int lane = threadIdx.x;
      unsigned int counts[8], sum = 0;
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        counts[j] = s.histogram[255 - 8 * lane - j];
        sum += counts[j];
      }
      unsigned int above = sum;  // inclusive scan over lanes (higher digits first)
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const unsigned int other = __shfl_up_sync(0xffffffffu, above, o);
        if (lane >= o) above += other;
      }
      above -= sum;  // keys in digits above this lane's
      const unsigned int remaining = s.remaining;
      int found = -1;
      unsigned int before = 0;
      unsigned int running = above;
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        if (found < 0 && running < remaining && remaining <= running + counts[j]) {
          found = 255 - 8 * lane - j;
          before = running;
        }
        running += counts[j];
      }
      const unsigned int hit = __ballot_sync(0xffffffffu, found >= 0);
      const int owner = __ffs(hit) - 1;
      const int digit = __shfl_sync(0xffffffffu, found, owner);
      const unsigned int skipped = __shfl_sync(0xffffffffu, before, owner);
      if (lane == 0) {
        s.prefix = prefix | ((unsigned long long)digit << shift);
        s.remaining = remaining - skipped;
      }
    }
    mask |= 255ull << shift;
    __syncthreads();
  }
  return s.prefix;
}

// The k keys at or above the k-th largest, into s.keys / s.at (unordered).
template <typename KeyAt>
__device__ void select_largest(KeyAt key_at, int n, int k, Selection& s) {
  const unsigned long long threshold = kth_largest(key_at, n, k, s);
  if (threadIdx.x == 0) s.taken = 0;
  __syncthreads();
  for (int i = threadIdx.x; i < n; i += blockDim.x) {
    const unsigned long long key = key_at(i);
    if (key >= threshold) {
      const unsigned slot = atomicAdd(&s.taken, 1u);
      if (slot < unsigned(k)) {
        s.keys[slot] = key;
        s.at[slot] = i;
      }
    }
  }
  __syncthreads();
}

// s.keys[0..k) (with s.at) into descending order: a bitonic sort over the
// next power of two, padded with the smallest key.
__device__ void sort_descending(int k, Selection& s) {
  int size = 1;
  while (size < k) size <<= 1;
  for (int i = k + threadIdx.x; i < size; i += blockDim.x) {
    s.keys[i] = 0;
    s.at[i] = -1;
  }
  __syncthreads();
  for (int width = 2; width <= size; width <<= 1) {
    for (int half = width >> 1; half > 0; half >>= 1) {
      for (int i = threadIdx.x; i < size; i += blockDim.x) {
        const int j = i ^ half;
        if (j > i) {
          const bool descending = (i & width) == 0;
          const unsigned long long a = s.keys[i], b = s.keys[j];
          if (descending ? a < b : a > b) {
            s.keys[i] = b;
            s.keys[j] = a;
            const int t = s.at[i];
            s.at[i] = s.at[j];
            s.at[j] = t;
          }
        }
      }
      __syncthreads();
    }
  }
}

// One CTA of a row's selection (grid rows x chunks of 1024 threads): it keeps
// its chunk's count largest (key bits, index) pairs in `kept` ([rows][chunks]
// [count], as the runner's candidates_f32 keeps them); the row's last CTA
// (`arrivals[row]`, left at 0) selects among all kept pairs and writes the
// row's candidates, largest first: ids (plus id_offset) and values when `ids`
// is given, else (value bits, index) pairs into `pairs` ([rows][count][2],
// the runner's layout).
__device__ void candidates_block(const float* __restrict__ values, long long width, int count,
                                 long long id_offset, int* __restrict__ kept, unsigned* arrivals,
                                 int* __restrict__ ids, float* __restrict__ out_values, int* pairs,
                                 Selection& s, bool& last) {
  const int chunks = int((width + CANDIDATE_CHUNK - 1) / CANDIDATE_CHUNK);
  const int row = blockIdx.x / chunks, chunk = blockIdx.x % chunks;
  const float* v = values + (long long)row * width;
  const long long first = (long long)chunk * CANDIDATE_CHUNK;
  const int length = int(min((long long)CANDIDATE_CHUNK, width - first));
  const int k = int(min((long long)count, width));
  const int chunk_k = min(k, length);
  int* row_kept = kept + 2LL * row * chunks * count;
  select_largest([&](int i) { return candidate_key(v[first + i], first + i); }, length, chunk_k, s);
  for (int c = threadIdx.x; c < chunk_k; c += blockDim.x) {
    row_kept[2LL * (chunk * count + c)] = int(uint32_t(s.keys[c] >> 32));
    row_kept[2LL * (chunk * count + c) + 1] = int(first + s.at[c]);
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    __threadfence();
    last = atomicAdd(arrivals + row, 1u) == unsigned(chunks - 1);
    if (last) arrivals[row] = 0;
    __threadfence();
  }
  __syncthreads();
  if (!last) return;
  // every chunk but the last keeps k (k <= count <= CANDIDATE_CHUNK); a row
  // of fewer values than count is one chunk
  const int n = (chunks - 1) * count +
                int(min((long long)k, width - (long long)(chunks - 1) * CANDIDATE_CHUNK));
  auto kept_key = [&](int i) {
    const uint32_t order = uint32_t(__ldcg(row_kept + 2LL * i));
    const uint32_t index = uint32_t(__ldcg(row_kept + 2LL * i + 1));
    return (uint64_t(order) << 32) | uint32_t(~index);
  };
  select_largest(kept_key, n, k, s);
  sort_descending(k, s);
  for (int c = threadIdx.x; c < k; c += blockDim.x) {
    const long long index = (long long)uint32_t(~uint32_t(s.keys[c]));
    const float value = v[index];
    if (ids) {
      ids[(long long)row * count + c] = int(index + id_offset);
      if (out_values) out_values[(long long)row * count + c] = value;
    } else {
      pairs[2LL * ((long long)row * count + c)] = __float_as_int(value);
      pairs[2LL * ((long long)row * count + c) + 1] = int(index);
    }
  }
}

__global__ void __launch_bounds__(SELECT_THREADS)
    candidates_kernel(const float* __restrict__ values, long long width, int count,
                      long long id_offset, int* __restrict__ kept, int* __restrict__ ids,
                      float* __restrict__ out_values) {
  pdl_trigger();
  pdl_wait();
  __shared__ Selection s;
  __shared__ bool last;
  candidates_block(values, width, count, id_offset, kept, sample_arrivals, ids, out_values, nullptr,
                   s, last);
}

// The merge over gathered candidates: rows of n (value, id) pairs (ids unique
// in a row), one CTA a row: the row's count largest by the candidates' order.
__global__ void __launch_bounds__(SELECT_THREADS)
    candidates_merge_kernel(const float* __restrict__ values, const int* __restrict__ ids_in,
                            long long n, int count, int* __restrict__ ids,
                            float* __restrict__ out_values) {
  pdl_trigger();
  pdl_wait();
  __shared__ Selection s;
  const long long row = blockIdx.x;
  const float* v = values + row * n;
  const int* g = ids_in + row * n;
  const int k = int(min((long long)count, n));
  select_largest([&](int i) { return candidate_key(v[i], g[i]); }, int(n), k, s);
  sort_descending(k, s);
  for (int c = threadIdx.x; c < k; c += blockDim.x) {
    ids[row * count + c] = g[s.at[c]];
    if (out_values) out_values[row * count + c] = v[s.at[c]];
  }
}

// ---- the runner's kernels by name (norm.hip:119-153, 322-363) ------------------------------
// argmax_f32(values, index, count): one block (of 1024 in the runner's
// dispatch), index[0] the argmax of `count` values.
__global__ void argmax_by_name(const float* __restrict__ values, int* index, int count) {
  __shared__ unsigned long long warp_best[32];
  unsigned long long best = 0;
  for (int i = threadIdx.x; i < count; i += blockDim.x) {
    const unsigned long long key = argmax_key(values[i], i);
    best = key > best ? key : best;
  }
  best = warp_max64(best);
  if (threadIdx.x % 32 == 0) warp_best[threadIdx.x / 32] = best;
  __syncthreads();
  if (threadIdx.x == 0) {
    for (int w = 1; w < int(blockDim.x / 32); ++w) best = warp_best[w] > best ? warp_best[w] : best;
    index[0] = count > 0 ? int(uint32_t(~uint32_t(best))) : 0;
  }
}

// candidates_f32(values, out, width, count, kept, finished): grid rows x
// chunks of 1024, the runner's kept and finished buffers and its out layout.
__global__ void __launch_bounds__(SELECT_THREADS)
    candidates_by_name(const float* __restrict__ values, int* out, int width, int count, int* kept,
                       unsigned* finished) {
  __shared__ Selection s;
  __shared__ bool last;
  candidates_block(values, width, count, 0, kept, finished, nullptr, nullptr, out, s, last);
}

}  // namespace

DRIFT_REGISTER(argmax_rows_f32, argmax_rows_kernel)
DRIFT_REGISTER(argmax_merge_f32, argmax_merge_kernel)
DRIFT_REGISTER(candidates_rows_f32, candidates_kernel)
DRIFT_REGISTER(candidates_merge_f32, candidates_merge_kernel)
DRIFT_REGISTER(argmax_f32, argmax_by_name)
DRIFT_REGISTER(candidates_f32, candidates_by_name)

}  // namespace drift

using namespace drift;

extern "C" {

int drift_argmax(const float* values, int64_t rows, int64_t width, int64_t id_offset, int32_t* ids,
                 float* out_values, drift_stream_t stream) {
  if (rows < 0 || width < 0) return invalid("argmax over [%lld, %lld]", (long long)rows, (long long)width);
  if (rows == 0) return 0;
  if (width == 0) return invalid("argmax of an empty row");
  if (rows > MAX_SAMPLE_ROWS) return invalid("argmax of %lld rows (at most %d)", (long long)rows, MAX_SAMPLE_ROWS);
  if (width + id_offset > 0x7fffffffll || id_offset < 0)
    return invalid("argmax: ids past 2^31 (%lld + %lld)", (long long)width, (long long)id_offset);
  if (!values || !ids) return invalid("argmax: a null tensor");
  const dim3 grid(unsigned((width + ARGMAX_SPAN - 1) / ARGMAX_SPAN), unsigned(rows));
  DRIFT_CUDA(launch_pdl(argmax_rows_kernel, grid, ARGMAX_THREADS, 0, cudaStream_t(stream), values,
                        (long long)width, (long long)id_offset, ids, out_values));
  return 0;
}

int drift_argmax_merge(const float* values, const int32_t* ids_in, int64_t rows, int64_t n,
                       int32_t* ids, float* out_values, drift_stream_t stream) {
  if (rows < 0 || n < 0) return invalid("argmax merge over [%lld, %lld]", (long long)rows, (long long)n);
  if (rows == 0) return 0;
  if (n == 0) return invalid("argmax of an empty row");
  if (!values || !ids_in || !ids) return invalid("argmax merge: a null tensor");
  DRIFT_CUDA(launch_pdl(argmax_merge_kernel, unsigned(rows), ARGMAX_THREADS, 0,
                        cudaStream_t(stream), values, ids_in, (long long)n, ids, out_values));
  return 0;
}

static int candidates_checks(int64_t rows, int64_t width, int count) {
  if (count < 1 || count > MAX_CANDIDATES)
    return invalid("%d candidates, 1 to %d", count, MAX_CANDIDATES);
  if (rows < 0 || width < 0) return invalid("candidates over [%lld, %lld]", (long long)rows, (long long)width);
  if (width > 0x7fffffffll) return invalid("candidates over rows of %lld", (long long)width);
  return 0;
}

size_t drift_candidates_workspace_bytes(int64_t rows, int64_t width, int count) {
  const int64_t chunks = (width + CANDIDATE_CHUNK - 1) / CANDIDATE_CHUNK;
  return size_t(rows) * size_t(chunks) * size_t(count) * 8 + 256;
}

int drift_candidates(const float* values, int64_t rows, int64_t width, int64_t id_offset, int count,
                     int32_t* ids, float* out_values, drift_stream_t stream) {
  DRIFT_TRY(candidates_checks(rows, width, count));
  if (rows == 0) return 0;
  if (width == 0) return invalid("candidates of an empty row");
  if (rows > MAX_SAMPLE_ROWS)
    return invalid("candidates of %lld rows (at most %d)", (long long)rows, MAX_SAMPLE_ROWS);
  if (!values || !ids) return invalid("candidates: a null tensor");
  if (width + id_offset > 0x7fffffffll || id_offset < 0)
    return invalid("candidates: ids past 2^31 (%lld + %lld)", (long long)width, (long long)id_offset);
  void* kept = nullptr;
  DRIFT_TRY(workspace_reserve(drift_candidates_workspace_bytes(rows, width, count), &kept));
  const long long chunks = (width + CANDIDATE_CHUNK - 1) / CANDIDATE_CHUNK;
  DRIFT_CUDA(launch_pdl(candidates_kernel, unsigned(rows * chunks), SELECT_THREADS, 0,
                        cudaStream_t(stream), values, (long long)width, count,
                        (long long)id_offset, static_cast<int*>(kept), ids, out_values));
  return 0;
}

int drift_candidates_merge(const float* values, const int32_t* ids_in, int64_t rows, int64_t n,
                           int count, int32_t* ids, float* out_values, drift_stream_t stream) {
  DRIFT_TRY(candidates_checks(rows, n, count));
  if (rows == 0) return 0;
  if (n == 0) return invalid("candidates of an empty row");
  if (!values || !ids_in || !ids) return invalid("candidates merge: a null tensor");
  DRIFT_CUDA(launch_pdl(candidates_merge_kernel, unsigned(rows), SELECT_THREADS, 0,
                        cudaStream_t(stream), values, ids_in, (long long)n, count, ids, out_values));
  return 0;
}

}  // extern "C"
