// Ops.cacheWrite and Ops.attention for the decode step (ops/AttentionOps.scala:
// 58-64, 113-121), over the reference's paged F16 cache (ops/KvCache.scala:
// 12-23; element indices ops/CpuAttention.scala:163-179): keys [pages][page
// offset][kvHeads][D], values [pages][kvHeads][D][page offset] -- a key row is
// D contiguous halves, a value column (one d, consecutive positions) is
// contiguous within a page.
//
// attention is split-K ("flash decoding"): a CTA takes one key head, the
// query heads that share it (q_heads / kv_heads of them) and 128 consecutive
// keys -- a thread per key for the scores, a thread per dimension for the
// weighted values -- and leaves, per query head, the largest score, the sum
// of exp(score - largest) and the unnormalised weighted sum. A second kernel
// joins the splits (and the sink, if any) per query head. Scores and sums in
// F32 (the CPU reference accumulates in Double; BASELINE's tolerance applies).
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include "common.cuh"
#include "registry.cuh"
#include "rowwise.cuh"

namespace drift {

int workspace_reserve(size_t bytes, void** pointer);
int* device_error_word();

namespace {

constexpr int ATT_THREADS = 128;
constexpr int KEYS = 128;       // keys a split takes
constexpr int MAX_GROUP = 16;   // query heads per key head, at most

__device__ __forceinline__ int64_t key_index(const int* table, int page_size, int kv_heads, int dim,
                                             int position, int head) {
  const int64_t page = table[position / page_size];
  return ((page * page_size + position % page_size) * kv_heads + head) * dim;
}

__device__ __forceinline__ int64_t value_index(const int* table, int page_size, int kv_heads,
                                               int dim, int position, int head, int d) {
  const int64_t page = table[position / page_size];
  return ((page * kv_heads + head) * dim + d) * page_size + position % page_size;
}

// One F32 value of k and v per thread, rounded to F16 to nearest even (as
// Float.floatToFloat16).
__global__ void cache_write_kernel(const float* __restrict__ k, const float* __restrict__ v,
                                   __half* keys, __half* values, const int* __restrict__ table,
                                   int page_size, int kv_heads, int dim, int tokens, int start) {
  pdl_trigger();  // the next kernel may launch and wait for this one
  pdl_wait();     // what the kernels before this one wrote is visible
  const long long total = (long long)tokens * kv_heads * dim;
  for (long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x; i < total;
       i += (long long)gridDim.x * blockDim.x) {
    const int d = int(i % dim), h = int((i / dim) % kv_heads), t = int(i / ((long long)dim * kv_heads));
    const int position = start + t;
    keys[key_index(table, page_size, kv_heads, dim, position, h) + d] = __float2half_rn(k[i]);
    values[value_index(table, page_size, kv_heads, dim, position, h, d)] = __float2half_rn(v[i]);
  }
}

// One launch serves either one sequence's `tokens` queries (the reference's
// call) or, with `positions`, a batch of sequences with one query each (a
// decode step): row z of q is then sequence z at positions[z], seeing keys
// 0..positions[z] through its page table row table + z * table_stride.
// A decode step's attention inputs, fused (the rmsNorm of each query and key
// head, the rope of both, and the cache write of keys and values that the
// dense decoder calls one by one, models/DenseDecoder.scala:830-860): a CTA of
// 256 threads per (head, sequence), thread d holding value d. Slots 0..q_heads
// are query heads, turned into q_out; the rest are key heads, whose turned
// keys and the values go into the sequence's cache at positions[z]. The norm
// and the turn are rms_norm_kernel's and rope_kernel's arithmetic
// (rowwise.cuh), so the results are those kernels' bits. A position outside
// the sequence's page table sets the device error word (code 1) and writes
// nothing.
__global__ void __launch_bounds__(256) attention_inputs_kernel(
    const float* __restrict__ q, const float* __restrict__ k, const float* __restrict__ v,
    int q_heads, int kv_heads, int dim, const float* __restrict__ q_norm,
    const float* __restrict__ k_norm, float epsilon, float weight_offset,
    const int* __restrict__ positions, float theta, int rotary, int layout, float* __restrict__ q_out,
    __half* keys, __half* values, int page_size, const int* __restrict__ tables, int table_stride,
    int* error) {
  pdl_trigger();  // the next kernel may launch and wait for this one
  pdl_wait();     // what the kernels before this one wrote is visible
  __shared__ float partial[32];
  __shared__ float row[256];
  const int slot = blockIdx.x, z = blockIdx.y, d = threadIdx.x;
  const bool query = slot < q_heads;
  const int h = query ? slot : slot - q_heads;
  const float* source = query ? q + ((long long)z * q_heads + h) * dim
                              : k + ((long long)z * kv_heads + h) * dim;
  const float* norm = query ? q_norm : k_norm;
  float value = d < dim ? source[d] : 0.0f;
  if (norm) {
    const float w = d < dim ? norm[d] : 0.0f;
    const float total = block_sum(fmaf(value, value, 0.0f), partial);
    const float scale = 1.0f / sqrtf(total / float(dim) + epsilon);
    value = value * scale * (w + weight_offset);
  }
  if (d < dim) row[d] = value;
  __syncthreads();
  if (d >= dim) return;
  const int position = positions[z];
  const float turned = rope_turn(row, d, position, theta, rotary, layout);
  if (query) {
    q_out[((long long)z * q_heads + h) * dim + d] = turned;
    return;
  }
  if (position < 0 || position >= table_stride * page_size) {
    if (d == 0) atomicCAS(error, 0, 1);
    return;
  }
  const int* table = tables + (long long)z * table_stride;
  keys[key_index(table, page_size, kv_heads, dim, position, h) + d] = __float2half_rn(turned);
  values[value_index(table, page_size, kv_heads, dim, position, h, d)] =
      __float2half_rn(v[((long long)z * kv_heads + h) * dim + d]);
}

struct AttentionArgs {
  const float* q;
  const __half* keys;
  const __half* values;
  const int* table;
  const int* positions;  // batched decode, or nullptr
  float* part_o;   // [rows][q_heads][splits][D]
  float* part_ml;  // [rows][q_heads][splits][2]
  int page_size, kv_heads, q_heads, query_start, key_count, tokens, splits, table_stride;
  float scale;
  int causal, window, has_softcap;
  float softcap;
};

// Row z's page table, key count and query position.
struct Query {
  const int* table;
  int key_count, position;
  __device__ Query(const AttentionArgs& a, int z) {
    if (a.positions) {
      table = a.table + (long long)z * a.table_stride;
      position = a.positions[z];
      key_count = position + 1;
      // a position past the page table (or the launch's key count) sees no keys
      if (position < 0 || key_count > a.table_stride * a.page_size || key_count > a.key_count)
        key_count = 0;
    } else {
      table = a.table;
      position = a.query_start + z;
      key_count = a.key_count;
    }
  }
};

// The visible keys of the query: [lo, hi).
__device__ __forceinline__ void visible(const AttentionArgs& a, const Query& query, int& lo,
                                        int& hi) {
  hi = query.key_count;
  if (a.causal && query.position + 1 < hi) hi = query.position + 1;
  lo = 0;
  if (a.window > 0 && query.position - a.window + 1 > lo) lo = query.position - a.window + 1;
}

// G: query heads per key head, a template so that the unrolled loops hold
// exactly the heads there are (a kernel unrolled for 16 heads but running 4
// spends its time waiting on the instruction cache).
template <int D, int G>
__global__ void __launch_bounds__(ATT_THREADS) attention_split_kernel(const AttentionArgs a) {
  pdl_trigger();  // the next kernel may launch and wait for this one
  pdl_wait();     // what the kernels before this one wrote is visible
  static_assert(D % 8 == 0 && D <= 2 * ATT_THREADS, "head width");
  constexpr int DIMS = (D + ATT_THREADS - 1) / ATT_THREADS;  // dimensions per thread
  constexpr int MAX_GROUP = G;
  __shared__ float qs[MAX_GROUP][D];
  __shared__ float ws[MAX_GROUP][KEYS];
  __shared__ float reduce[MAX_GROUP][ATT_THREADS / 32];
  const int split = blockIdx.x, head = blockIdx.y, t = blockIdx.z;
  const int tid = threadIdx.x, lane = tid % 32, warp = tid / 32;
  const int group = a.q_heads / a.kv_heads;  // <= G
  const Query query(a, t);
  int lo, hi;
  visible(a, query, lo, hi);
  const int k0 = split * KEYS;
  const int first = k0 > lo ? k0 : lo, last = k0 + KEYS < hi ? k0 + KEYS : hi;  // [first, last)

  // the chunk's pages, looked up once
  __shared__ int pages[KEYS / 16 + 2];
  const int page0 = k0 / a.page_size;
  if (tid < KEYS / 16 + 2) {
    const int p = page0 + tid;
    pages[tid] = (long long)p * a.page_size < query.key_count ? query.table[p] : 0;
  }
  for (int i = tid; i < group * D; i += ATT_THREADS)
    qs[i / D][i % D] = a.q[((long long)t * a.q_heads + head * group + i / D) * D + i % D];
  __syncthreads();

  // scores: a thread per key, the key row read in slices of 64 values with
  // every load of a slice issued before its first use
  const int key = k0 + tid;
  const bool seen = key >= first && key < last;
  float score[MAX_GROUP];
#pragma unroll
  for (int g = 0; g < MAX_GROUP; ++g) score[g] = 0.0f;
  if (seen) {
    const long long page = pages[key / a.page_size - page0];
    const uint4* row = reinterpret_cast<const uint4*>(
        a.keys + ((page * a.page_size + key % a.page_size) * a.kv_heads + head) * D);
#pragma unroll
    for (int slice = 0; slice < (D + 63) / 64; ++slice) {
      constexpr int PER = D < 64 ? D / 8 : 8;
      uint4 raw[PER];
#pragma unroll
      for (int c = 0; c < PER; ++c) raw[c] = slice * 8 + c < D / 8 ? row[slice * 8 + c] : make_uint4(0, 0, 0, 0);
#pragma unroll
      for (int c = 0; c < PER; ++c) {
        if (slice * 8 + c >= D / 8) break;
        const __half2* h2 = reinterpret_cast<const __half2*>(&raw[c]);
        float kv[8];
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          const float2 f = __half22float2(h2[i]);
          kv[2 * i] = f.x;
          kv[2 * i + 1] = f.y;
        }
#pragma unroll
        for (int g = 0; g < MAX_GROUP; ++g) {
          if (g < group) {
#pragma unroll
            for (int i = 0; i < 8; ++i)
              score[g] = fmaf(qs[g][8 * (slice * 8 + c) + i], kv[i], score[g]);
          }
        }
      }
    }
  }
  float largest[MAX_GROUP];
#pragma unroll
  for (int g = 0; g < MAX_GROUP; ++g) {
    float s = score[g] * a.scale;
    if (a.has_softcap) s = a.softcap * tanhf(s / a.softcap);
    score[g] = seen ? s : -INFINITY;
    float m = score[g];
#pragma unroll
    for (int o = 16; o > 0; o /= 2) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
    if (lane == 0 && g < group) reduce[g][warp] = m;
  }
  __syncthreads();
#pragma unroll
  for (int g = 0; g < MAX_GROUP; ++g) {
    float m = -INFINITY;
    if (g < group) {
#pragma unroll
      for (int w = 0; w < ATT_THREADS / 32; ++w) m = fmaxf(m, reduce[g][w]);
    }
    largest[g] = m;
  }
  __syncthreads();
#pragma unroll
  for (int g = 0; g < MAX_GROUP; ++g) {
    const float w = seen && g < group ? expf(score[g] - largest[g]) : 0.0f;
    if (g < group) ws[g][tid] = w;
    float s = w;
#pragma unroll
    for (int o = 16; o > 0; o /= 2) s += __shfl_xor_sync(0xffffffffu, s, o);
    if (lane == 0 && g < group) reduce[g][warp] = s;
  }
  __syncthreads();

  // weighted values: a thread per dimension (two for D = 256)
  float acc[MAX_GROUP][DIMS];
#pragma unroll
  for (int g = 0; g < MAX_GROUP; ++g)
#pragma unroll
    for (int j = 0; j < DIMS; ++j) acc[g][j] = 0.0f;
  const bool whole = first == k0 && last == k0 + KEYS;  // a full chunk: 16 runs of 8 keys
#pragma unroll
  for (int j = 0; j < DIMS; ++j) {
    const int d = tid + j * ATT_THREADS;
    if (d >= D) continue;
    if (whole) {
      uint4 raw[KEYS / 8];
#pragma unroll
      for (int r = 0; r < KEYS / 8; ++r) {
        const int p = k0 + 8 * r;
        const long long page = pages[p / a.page_size - page0];  // within the chunk's pages
        raw[r] = *reinterpret_cast<const uint4*>(
            a.values + ((page * a.kv_heads + head) * D + d) * a.page_size + p % a.page_size);
      }
#pragma unroll
      for (int r = 0; r < KEYS / 8; ++r) {
        const __half2* h2 = reinterpret_cast<const __half2*>(&raw[r]);
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          const float2 f = __half22float2(h2[i]);
#pragma unroll
          for (int g = 0; g < MAX_GROUP; ++g) {
            if (g < group) {
              acc[g][j] = fmaf(ws[g][8 * r + 2 * i], f.x, acc[g][j]);
              acc[g][j] = fmaf(ws[g][8 * r + 2 * i + 1], f.y, acc[g][j]);
            }
          }
        }
      }
      continue;
    }
    int p = first;
    // eight keys at a time where they share a page and start on an 8-key
    // boundary (a 16-byte run of one value column)
    while (p < last) {
      if (p % 8 == 0 && p + 8 <= last && (p % a.page_size) + 8 <= a.page_size) {
        const uint4 raw = *reinterpret_cast<const uint4*>(
            a.values + value_index(query.table, a.page_size, a.kv_heads, D, p, head, d));
        const __half2* h2 = reinterpret_cast<const __half2*>(&raw);
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          const float2 f = __half22float2(h2[i]);
#pragma unroll
          for (int g = 0; g < MAX_GROUP; ++g) {
            if (g < group) {
              acc[g][j] = fmaf(ws[g][p - k0 + 2 * i], f.x, acc[g][j]);
              acc[g][j] = fmaf(ws[g][p - k0 + 2 * i + 1], f.y, acc[g][j]);
            }
          }
        }
        p += 8;
      } else {
        const float f = __half2float(
            a.values[value_index(query.table, a.page_size, a.kv_heads, D, p, head, d)]);
#pragma unroll
        for (int g = 0; g < MAX_GROUP; ++g)
          if (g < group) acc[g][j] = fmaf(ws[g][p - k0], f, acc[g][j]);
        ++p;
      }
    }
  }
#pragma unroll
  for (int g = 0; g < MAX_GROUP; ++g) {
    if (g >= group) break;
    const long long at = ((long long)t * a.q_heads + head * group + g) * a.splits + split;
#pragma unroll
    for (int j = 0; j < DIMS; ++j) {
      const int d = tid + j * ATT_THREADS;
      if (d < D) a.part_o[at * D + d] = acc[g][j];
    }
    if (tid == 0) {
      float total = 0.0f;
#pragma unroll
      for (int w = 0; w < ATT_THREADS / 32; ++w) total += reduce[g][w];
      a.part_ml[at * 2] = largest[g];
      a.part_ml[at * 2 + 1] = total;
    }
  }
}

// Joins a query head's splits: out = sum_s o_s e^(m_s - M) / (sum_s l_s
// e^(m_s - M) + e^(sink - M)), M the largest of the m_s and the sink.
template <int D>
__global__ void __launch_bounds__(ATT_THREADS) attention_join_kernel(const AttentionArgs a,
                                                                     const float* sinks,
                                                                     float* out) {
  pdl_trigger();  // the next kernel may launch and wait for this one
  pdl_wait();     // what the kernels before this one wrote is visible
  extern __shared__ float factor[];  // [splits]: e^(m_s - M), 0 for an empty split
  __shared__ float shared_total;
  const int head = blockIdx.x, t = blockIdx.y;
  const long long base = ((long long)t * a.q_heads + head) * a.splits;
  if (threadIdx.x < 32) {
    float largest = -INFINITY;
    for (int s = threadIdx.x; s < a.splits; s += 32)
      if (a.part_ml[(base + s) * 2 + 1] > 0.0f) largest = fmaxf(largest, a.part_ml[(base + s) * 2]);
#pragma unroll
    for (int o = 16; o > 0; o /= 2) largest = fmaxf(largest, __shfl_xor_sync(0xffffffffu, largest, o));
    if (sinks) largest = fmaxf(largest, sinks[head]);
    float total = 0.0f;
    for (int s = threadIdx.x; s < a.splits; s += 32) {
      const float l = a.part_ml[(base + s) * 2 + 1];
      const float f = l > 0.0f ? expf(a.part_ml[(base + s) * 2] - largest) : 0.0f;
      factor[s] = f;
      total += l * f;
    }
#pragma unroll
    for (int o = 16; o > 0; o /= 2) total += __shfl_xor_sync(0xffffffffu, total, o);
    if (threadIdx.x == 0) shared_total = total + (sinks ? expf(sinks[head] - largest) : 0.0f);
  }
  __syncthreads();
  const float total = shared_total;
  for (int d = threadIdx.x; d < D; d += ATT_THREADS) {
    float sum = 0.0f;
    for (int s = 0; s < a.splits; ++s)
      if (factor[s] > 0.0f) sum += a.part_o[(base + s) * D + d] * factor[s];
    out[((long long)t * a.q_heads + head) * D + d] = total > 0.0f ? sum / total : 0.0f;
  }
}

#define DRIFT_ATTENTION_REGISTER(D)                                                   \
  DRIFT_REGISTER(attention_split_d##D##_g4, (attention_split_kernel<D, 4>))           \
  DRIFT_REGISTER(attention_join_d##D, attention_join_kernel<D>)
DRIFT_ATTENTION_REGISTER(64)
DRIFT_ATTENTION_REGISTER(80)
DRIFT_ATTENTION_REGISTER(128)
DRIFT_ATTENTION_REGISTER(256)
DRIFT_REGISTER(cache_write_f16, cache_write_kernel)
DRIFT_REGISTER(attention_inputs_f32, attention_inputs_kernel)

template <int D, int G>
int launch_split(const AttentionArgs& a, cudaStream_t stream) {
  DRIFT_CUDA(launch_pdl(attention_split_kernel<D, G>, dim3(a.splits, a.kv_heads, a.tokens),
                        ATT_THREADS, 0, stream, a));
  DRIFT_LAUNCHED("attention_split");
  return 0;
}

template <int D>
int launch_attention(const AttentionArgs& a, const float* sinks, float* out, cudaStream_t stream) {
  // the key head's query heads, padded up to the next kernel's count (the
  // padding heads' scores are computed and dropped)
  const int group = a.q_heads / a.kv_heads;
  if (group <= 1) DRIFT_TRY((launch_split<D, 1>(a, stream)));
  else if (group <= 2) DRIFT_TRY((launch_split<D, 2>(a, stream)));
  else if (group <= 4) DRIFT_TRY((launch_split<D, 4>(a, stream)));
  else if (group <= 8) DRIFT_TRY((launch_split<D, 8>(a, stream)));
  else DRIFT_TRY((launch_split<D, 16>(a, stream)));
  DRIFT_CUDA(launch_pdl(attention_join_kernel<D>, dim3(a.q_heads, a.tokens), ATT_THREADS,
                        a.splits * sizeof(float), stream, a, sinks, out));
  DRIFT_LAUNCHED("attention_join");
  return 0;
}

int check_cache(int pages, int page_size, int kv_heads, int head_dim, const int32_t* page_table,
                int table_pages, long long positions, const char* call) {
  if (page_size <= 0 || page_size % 16 != 0)
    return invalid("pages of %d tokens: not a multiple of 16", page_size);
  if (head_dim != 64 && head_dim != 80 && head_dim != 128 && head_dim != 256)
    return invalid("%s: heads of %d (kernels take 64, 80, 128, 256)", call, head_dim);
  if (pages <= 0 || kv_heads <= 0) return invalid("%s: an empty cache", call);
  if (!page_table || table_pages <= 0 || (long long)table_pages * page_size < positions)
    return invalid("a page table of %d pages for %lld positions", table_pages, positions);
  return 0;
}

}  // namespace
}  // namespace drift

using namespace drift;

extern "C" {

int drift_cache_write(const float* k, const float* v, int tokens, int kv_heads, int head_dim,
                      void* keys, void* values, int pages, int page_size,
                      const int32_t* page_table, int table_pages, int start,
                      drift_stream_t stream) {
  if (tokens < 0 || start < 0) return invalid("cacheWrite: %d tokens at %d", tokens, start);
  DRIFT_TRY(check_cache(pages, page_size, kv_heads, head_dim, page_table, table_pages,
                        (long long)start + tokens, "cacheWrite"));
  if (tokens == 0) return 0;
  if (!k || !v || !keys || !values) return invalid("cacheWrite: a null tensor");
  if ((reinterpret_cast<uintptr_t>(keys) | reinterpret_cast<uintptr_t>(values)) & 15)
    return invalid("cacheWrite: the cache does not start on a 16-byte boundary");
  const long long total = (long long)tokens * kv_heads * head_dim;
  long long grid = (total + 255) / 256;
  if (grid > 4096) grid = 4096;
  DRIFT_CUDA(launch_pdl(cache_write_kernel, unsigned(grid), 256, 0, cudaStream_t(stream), k, v,
                        static_cast<__half*>(keys), static_cast<__half*>(values), page_table,
                        page_size, kv_heads, head_dim, tokens, start));
  DRIFT_LAUNCHED("cache_write");
  return 0;
}

int drift_attention(const float* q, int tokens, int q_heads, const void* keys, const void* values,
                    int pages, int page_size, int kv_heads, int head_dim,
                    const int32_t* page_table, int table_pages, int query_start, int key_count,
                    float scale, int causal, int window, float softcap, const float* sinks,
                    float* out, drift_stream_t stream) {
  if (tokens < 0 || q_heads <= 0) return invalid("attention: %d tokens of %d heads", tokens, q_heads);
  DRIFT_TRY(check_cache(pages, page_size, kv_heads, head_dim, page_table, table_pages, key_count,
                        "attention"));
  if (q_heads % kv_heads != 0)
    return invalid("attention: %d query heads over %d key heads", q_heads, kv_heads);
  if (q_heads / kv_heads > MAX_GROUP)
    return invalid("attention: %d query heads per key head (at most %d)", q_heads / kv_heads,
                   MAX_GROUP);
  if (query_start < 0 || key_count < 0 ||
      (query_start + tokens > key_count && (causal || window > 0)))
    return invalid("attention: queries at %d..%d past %d keys", query_start,
                   query_start + tokens - 1, key_count);
  if (key_count > (48 * 1024 / 4 - 16) * KEYS)
    return invalid("attention: %d keys (at most %d)", key_count, (48 * 1024 / 4 - 16) * KEYS);
  if (tokens == 0) return 0;
  if (!q || !keys || !values || !out) return invalid("attention: a null tensor");
  if ((reinterpret_cast<uintptr_t>(keys) | reinterpret_cast<uintptr_t>(values)) & 15)
    return invalid("attention: the cache does not start on a 16-byte boundary");
  AttentionArgs a;
  a.q = q;
  a.keys = static_cast<const __half*>(keys);
  a.values = static_cast<const __half*>(values);
  a.table = page_table;
  a.positions = nullptr;
  a.table_stride = 0;
  a.page_size = page_size;
  a.kv_heads = kv_heads;
  a.q_heads = q_heads;
  a.query_start = query_start;
  a.key_count = key_count;
  a.tokens = tokens;
  a.splits = key_count > 0 ? (key_count + KEYS - 1) / KEYS : 1;
  a.scale = scale;
  a.causal = causal;
  a.window = window;
  a.has_softcap = softcap > 0.0f;
  a.softcap = softcap;
  const size_t parts = size_t(tokens) * q_heads * a.splits;
  void* ws = nullptr;
  DRIFT_TRY(workspace_reserve(parts * (head_dim + 2) * sizeof(float), &ws));
  a.part_o = static_cast<float*>(ws);
  a.part_ml = a.part_o + parts * head_dim;
  const cudaStream_t s = cudaStream_t(stream);
  switch (head_dim) {
    case 64: return launch_attention<64>(a, sinks, out, s);
    case 80: return launch_attention<80>(a, sinks, out, s);
    case 128: return launch_attention<128>(a, sinks, out, s);
    default: return launch_attention<256>(a, sinks, out, s);
  }
}

int drift_attention_inputs_decode(const float* q, const float* k, const float* v, int batch,
                                  int q_heads, int kv_heads, int head_dim, const float* q_norm,
                                  const float* k_norm, float epsilon, float weight_offset,
                                  const int32_t* positions, float theta, int rotary, int layout,
                                  float* q_out, void* keys, void* values, int pages,
                                  int page_size, const int32_t* page_tables, int table_stride,
                                  drift_stream_t stream) {
  if (batch < 0 || q_heads <= 0) return invalid("attention inputs: %d sequences of %d heads", batch, q_heads);
  DRIFT_TRY(check_cache(pages, page_size, kv_heads, head_dim, page_tables, table_stride, 0,
                        "attention inputs"));
  if (rotary < 0 || rotary > head_dim || rotary % 2)
    return invalid("rope: %d rotary dimensions in heads of %d", rotary, head_dim);
  if (batch == 0) return 0;
  if (!q || !k || !v || !positions || !q_out || !keys || !values)
    return invalid("attention inputs: a null tensor");
  if ((reinterpret_cast<uintptr_t>(keys) | reinterpret_cast<uintptr_t>(values)) & 15)
    return invalid("attention inputs: the cache does not start on a 16-byte boundary");
  DRIFT_CUDA(launch_pdl(attention_inputs_kernel, dim3(q_heads + kv_heads, batch), 256, 0,
                        cudaStream_t(stream), q, k, v, q_heads, kv_heads, head_dim, q_norm, k_norm,
                        epsilon, weight_offset, positions, theta, rotary, layout, q_out,
                        static_cast<__half*>(keys), static_cast<__half*>(values), page_size,
                        page_tables, table_stride, device_error_word()));
  DRIFT_LAUNCHED("attention_inputs");
  return 0;
}

int drift_attention_decode(const float* q, int batch, int q_heads, const void* keys,
                           const void* values, int pages, int page_size, int kv_heads,
                           int head_dim, const int32_t* page_tables, int table_stride,
                           const int32_t* positions, int max_key_count, float scale, int window,
                           float softcap, const float* sinks, float* out, drift_stream_t stream) {
  if (batch < 0 || q_heads <= 0) return invalid("attention: %d sequences of %d heads", batch, q_heads);
  DRIFT_TRY(check_cache(pages, page_size, kv_heads, head_dim, page_tables, table_stride,
                        max_key_count, "attention"));
  if (q_heads % kv_heads != 0 || q_heads / kv_heads > MAX_GROUP)
    return invalid("attention: %d query heads over %d key heads", q_heads, kv_heads);
  if (max_key_count <= 0 || max_key_count > (48 * 1024 / 4 - 16) * KEYS)
    return invalid("attention: %d keys", max_key_count);
  if (batch == 0) return 0;
  if (!q || !keys || !values || !positions || !out) return invalid("attention: a null tensor");
  if ((reinterpret_cast<uintptr_t>(keys) | reinterpret_cast<uintptr_t>(values)) & 15)
    return invalid("attention: the cache does not start on a 16-byte boundary");
  AttentionArgs a;
  a.q = q;
  a.keys = static_cast<const __half*>(keys);
  a.values = static_cast<const __half*>(values);
  a.table = page_tables;
  a.positions = positions;
  a.table_stride = table_stride;
  a.page_size = page_size;
  a.kv_heads = kv_heads;
  a.q_heads = q_heads;
  a.query_start = 0;
  a.key_count = max_key_count;
  a.tokens = batch;
  a.splits = (max_key_count + KEYS - 1) / KEYS;
  a.scale = scale;
  a.causal = 1;
  a.window = window;
  a.has_softcap = softcap > 0.0f;
  a.softcap = softcap;
  const size_t parts = size_t(batch) * q_heads * a.splits;
  void* ws = nullptr;
  DRIFT_TRY(workspace_reserve(parts * (head_dim + 2) * sizeof(float), &ws));
  a.part_o = static_cast<float*>(ws);
  a.part_ml = a.part_o + parts * head_dim;
  const cudaStream_t s = cudaStream_t(stream);
  switch (head_dim) {
    case 64: return launch_attention<64>(a, sinks, out, s);
    case 80: return launch_attention<80>(a, sinks, out, s);
    case 128: return launch_attention<128>(a, sinks, out, s);
    default: return launch_attention<256>(a, sinks, out, s);
  }
}

}  // extern "C"
