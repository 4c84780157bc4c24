// Ops.cacheWrite and Ops.attention for the decode step (ops/AttentionOps.scala:
// 58-64, 113-121), over the reference's paged F16 cache (ops/KvCache.scala:
// 12-23; element indices ops/CpuAttention.scala:163-179): keys [pages][page
// offset][kvHeads][D], values [pages][kvHeads][D][page offset] -- a key row is
// D contiguous halves, a value column (one d, consecutive positions) is
// contiguous within a page.
//
// attention is split-K ("flash decoding"): a CTA takes one key head, the
// query heads that share it (q_heads / kv_heads of them, at most 16: one
// 16-row tensor-core tile) and 128 consecutive keys (64 for 256-wide heads),
// brings the keys and values into shared memory in one round of asynchronous
// copies, forms scores and weighted values with mma.sync on F16 operands
// (q and the weights as two F16 terms each, so the sums are F32-grade), and
// leaves, per query head, the largest score, the sum of exp(score - largest)
// and the unnormalised weighted sum. The last split of each (row, key head)
// to finish joins the splits (and the sink, if any) for its query heads --
// or, when that is more than 32768 partial floats, a second kernel does. Scores and sums in F32 (the CPU
// reference accumulates in Double; the 1e-4 + 1e-3 |e| tolerance applies).
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include "common.cuh"
#include "registry.cuh"
#include "rowwise.cuh"
#include "x22.cuh"

namespace drift {

int workspace_reserve(size_t bytes, void** pointer);
int* device_error_word();

namespace {

constexpr int SPLIT_THREADS = 256;  // the splits' threads: 8 warps
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
    int q_heads, int kv_heads, int dim, int q_stride, const float* __restrict__ q_norm,
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
  const float* source = query ? q + ((long long)z * q_heads + h) * q_stride
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
  // the join, when the last split of each (row, key head) does it
  int fused_join;
  const float* sinks;
  float* out;
  uint8_t* records;
  const float* gate;
  int gate_stride;
};

// Splits arrived per (row, key head) of a launch whose last split joins;
// zero between launches (the joining CTA clears its entry).
constexpr int MAX_JOINS = 1 << 16;
constexpr int MAX_FUSED_SPLITS = 256;
// The most partial floats (query heads x D x splits) the joining CTA reads:
// past it one CTA per query head (the separate join) is faster -- C4's 4 x
// 128 x 32 joins faster in the last split, C5's 8 x 256 x 64 slower.
constexpr int MAX_FUSED_JOIN_FLOATS = 32768;
__device__ unsigned join_arrivals[MAX_JOINS];

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

// Joins a query head's splits: out = sum_s o_s e^(m_s - M) / (sum_s l_s
// e^(m_s - M) + e^(sink - M)), M the largest of the m_s and the sink.
// With `records` (D a multiple of 32), also the x records of the output rows
// for the product that follows (the o projection): warp w's 32 dimensions
// are one block of the row. With `gate`, the gated attention's output gate:
// value x sigmoid(gate) (the runner's gated(Sigmoid, gate, attended),
// models/HybridBlocks.scala). Called by every thread of the CTA; the
// partials are read at L2 (other CTAs of the same launch may have written
// them).
template <int D, int THREADS>
__device__ void join_head(const AttentionArgs& a, const float* sinks, float* out,
                          uint8_t* records, const float* gate, int gate_stride, int head, int t,
                          float* factor, float* shared_total) {
  const long long base = ((long long)t * a.q_heads + head) * a.splits;
  if (threadIdx.x < 32) {
    float largest = -INFINITY;
    for (int s = threadIdx.x; s < a.splits; s += 32)
      if (__ldcg(a.part_ml + (base + s) * 2 + 1) > 0.0f)
        largest = fmaxf(largest, __ldcg(a.part_ml + (base + s) * 2));
#pragma unroll
    for (int o = 16; o > 0; o /= 2) largest = fmaxf(largest, __shfl_xor_sync(0xffffffffu, largest, o));
    if (sinks) largest = fmaxf(largest, sinks[head]);
    float total = 0.0f;
    for (int s = threadIdx.x; s < a.splits; s += 32) {
      const float l = __ldcg(a.part_ml + (base + s) * 2 + 1);
      const float f = l > 0.0f ? expf(__ldcg(a.part_ml + (base + s) * 2) - largest) : 0.0f;
      factor[s] = f;
      total += l * f;
    }
#pragma unroll
    for (int o = 16; o > 0; o /= 2) total += __shfl_xor_sync(0xffffffffu, total, o);
    if (threadIdx.x == 0) *shared_total = total + (sinks ? expf(sinks[head] - largest) : 0.0f);
  }
  __syncthreads();
  const float total = *shared_total;
  for (int d = threadIdx.x; d < D; d += THREADS) {
    // eight splits' loads in flight at a time, summed in split order
    float sum = 0.0f;
    for (int s0 = 0; s0 < a.splits; s0 += 8) {
      float o[8];
#pragma unroll
      for (int j = 0; j < 8; ++j)
        o[j] = s0 + j < a.splits ? __ldcg(a.part_o + (base + s0 + j) * D + d) : 0.0f;
#pragma unroll
      for (int j = 0; j < 8; ++j)
        if (s0 + j < a.splits && factor[s0 + j] > 0.0f) sum += o[j] * factor[s0 + j];
    }
    float value = total > 0.0f ? sum / total : 0.0f;
    if (gate) {
      const float g = gate[((long long)t * a.q_heads + head) * gate_stride + d];
      value = (1.0f / (1.0f + expf(-g))) * value;
    }
    out[((long long)t * a.q_heads + head) * D + d] = value;
    if constexpr (D % 32 == 0) {
      if (records) x22_record_block(value, records, t, (head * D + d) / 32, a.q_heads * D / 32);
    }
  }
  __syncthreads();  // factor and the total are reused for the next head
}

// A split's tile: KEYS keys of one key head against the (up to 16) query
// heads that share it, as 16-row tensor-core tiles (mma.sync m16n8k16, F16
// operands, F32 sums). The keys and values are F16 in the cache, so they are
// exact operands; q and the weights p are F32, so each goes in as two F16
// terms, hi = f16(x) and lo = f16(x - hi), whose sum holds x to about 2^-22:
// a score is q_hi.k + q_lo.k and an output p_hi.v + p_lo.v, F32 throughout
// after that.
//
// Shared memory: the key rows ([KEYS][D] halves), the value columns
// ([D][KEYS] halves -- the cache's own order within a page), then the q
// fragments, later reused for the p fragments. A fragment load reads one
// 16-byte chunk from each of eight consecutive rows, so chunk c of row r sits
// at chunk c ^ (r mod 8) of its row: the eight reads land on distinct banks.
// (80-wide key rows, ten chunks, are padded by a chunk instead.)
__host__ __device__ constexpr int split_keys(int head_dim) { return head_dim > 128 ? 64 : 128; }

template <int D>
struct SplitTile {
  static constexpr int KEYS = split_keys(D);  // keys of a split
  static constexpr int WARPS = SPLIT_THREADS / 32;
  static constexpr int QW = KEYS / 16;             // warps that score: 16 keys each
  static constexpr int NT = 2;                     // 8-key tiles of a warp's scores
  static constexpr int KQ = D / 16;                // k-steps of q.k
  static constexpr int KP = KEYS / 16;             // k-steps of p.v
  static constexpr int ND = D / 8;                 // 8-wide dimension tiles of p.v
  static constexpr int CH = D / 8;                 // 16-byte chunks of a key row
  static constexpr int RUNS = KEYS / 8;            // 16-byte chunks of a value column
  static constexpr bool KEY_SWIZZLE = CH % 8 == 0;
  static constexpr int KPITCH = KEY_SWIZZLE ? 2 * D : 2 * D + 16;
  static constexpr int VPITCH = 2 * KEYS;
  static constexpr int K_BYTES = KEYS * KPITCH;
  static constexpr int V_BYTES = D * VPITCH;
  static constexpr int QF_BYTES = KQ * 2 * 32 * 16;
  static constexpr int PF_BYTES = KP * 2 * 32 * 16;
  static constexpr int BYTES = K_BYTES + V_BYTES + (QF_BYTES > PF_BYTES ? QF_BYTES : PF_BYTES);
  // byte offsets of chunk c of key row k, and of run r of value column d
  __device__ static int key_chunk(int k, int c) {
    return k * KPITCH + 16 * (KEY_SWIZZLE ? c ^ (k & 7) : c);
  }
  __device__ static int value_chunk(int d, int r) { return d * VPITCH + 16 * (r ^ (d & 7)); }
  static_assert(RUNS % 8 == 0, "value columns of whole 8-chunk groups");
};

__device__ __forceinline__ void cp_async16(void* smem, const void* global) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(
                   static_cast<uint32_t>(__cvta_generic_to_shared(smem))),
               "l"(global)
               : "memory");
}

__device__ __forceinline__ void mma_f16(float (&c)[4], const uint4& a, uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, "
      "{%8,%9}, {%0,%1,%2,%3};"
      : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
      : "r"(a.x), "r"(a.y), "r"(a.z), "r"(a.w), "r"(b0), "r"(b1));
}

// The two F16 terms of a pair of F32 values, packed as (first, second).
__device__ __forceinline__ void split_pair(float x0, float x1, uint32_t& hi, uint32_t& lo) {
  const __half h0 = __float2half_rn(x0), h1 = __float2half_rn(x1);
  const __half l0 = __float2half_rn(x0 - __half2float(h0));
  const __half l1 = __float2half_rn(x1 - __half2float(h1));
  const __half2 h = __halves2half2(h0, h1), l = __halves2half2(l0, l1);
  hi = *reinterpret_cast<const uint32_t*>(&h);
  lo = *reinterpret_cast<const uint32_t*>(&l);
}

// Warp w < KEYS / 16 scores keys [16 w, 16 w + 16) of the split for all 16
// query rows; after the softmax statistics meet in shared memory, it writes
// those keys' weights as one A fragment of the p.v product, and then each of
// the 8 warps takes an eighth of the dimensions of p.v over all of the
// split's keys. Positions outside the visible range are never read from the
// cache: their scores are -inf and their value columns zeros.
// The join of one (row, key head)'s query heads by the split CTA that
// finished last, its threads side by side: warp w takes the factors of heads
// w, w + 8; then each thread sums (head, two dimensions) pairs over the
// splits with sixteen splits' loads in flight; then, with `records`, the x
// records from the values in shared memory. Per output it is join_head's
// arithmetic in join_head's order, so the two give the same bits. `smem`:
// the split's tile, whose keys and values are no longer read.
constexpr int JOIN_GROUP_SPLITS = MAX_GROUP * MAX_FUSED_SPLITS;  // one head's splits, at most
template <int D>
constexpr int join_group_bytes() { return 4 * (MAX_GROUP * MAX_FUSED_SPLITS + MAX_GROUP + MAX_GROUP * D); }

template <int D>
__device__ void join_group(const AttentionArgs& a, int z, int kv_head, int group, uint8_t* smem) {
  float* factor = reinterpret_cast<float*>(smem);        // [group][splits]
  float* total = factor + MAX_GROUP * MAX_FUSED_SPLITS;  // [group]
  float* value = total + MAX_GROUP;                      // [group][D]
  const int S = a.splits;
  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  const float2* ml = reinterpret_cast<const float2*>(a.part_ml);
  for (int q = warp; q < group; q += SPLIT_THREADS / 32) {
    const int head = kv_head * group + q;
    const long long base = ((long long)z * a.q_heads + head) * S;
    float largest = -INFINITY;
    for (int s = lane; s < S; s += 32) {
      const float2 v = __ldcg(ml + base + s);
      if (v.y > 0.0f) largest = fmaxf(largest, v.x);
    }
#pragma unroll
    for (int o = 16; o > 0; o /= 2) largest = fmaxf(largest, __shfl_xor_sync(0xffffffffu, largest, o));
    if (a.sinks) largest = fmaxf(largest, a.sinks[head]);
    float sum = 0.0f;
    for (int s = lane; s < S; s += 32) {
      const float2 v = __ldcg(ml + base + s);
      const float f = v.y > 0.0f ? expf(v.x - largest) : 0.0f;
      factor[q * S + s] = f;
      sum += v.y * f;
    }
#pragma unroll
    for (int o = 16; o > 0; o /= 2) sum += __shfl_xor_sync(0xffffffffu, sum, o);
    if (lane == 0) total[q] = sum + (a.sinks ? expf(a.sinks[head] - largest) : 0.0f);
  }
  __syncthreads();
  constexpr int HALF = D / 2;
  for (int p = threadIdx.x; p < group * HALF; p += SPLIT_THREADS) {
    const int q = p / HALF, d = 2 * (p % HALF);
    const int head = kv_head * group + q;
    const long long base = ((long long)z * a.q_heads + head) * S;
    const float* f = factor + q * S;
    float sum0 = 0.0f, sum1 = 0.0f;
    for (int s0 = 0; s0 < S; s0 += 16) {
      float2 o[16];
#pragma unroll
      for (int j = 0; j < 16; ++j)
        o[j] = s0 + j < S ? __ldcg(reinterpret_cast<const float2*>(a.part_o + (base + s0 + j) * D + d))
                          : make_float2(0.0f, 0.0f);
#pragma unroll
      for (int j = 0; j < 16; ++j)
        if (s0 + j < S && f[s0 + j] > 0.0f) {
          sum0 += o[j].x * f[s0 + j];
          sum1 += o[j].y * f[s0 + j];
        }
    }
    const float t = total[q];
    float v0 = t > 0.0f ? sum0 / t : 0.0f, v1 = t > 0.0f ? sum1 / t : 0.0f;
    const long long at = ((long long)z * a.q_heads + head) * D + d;
    if (a.gate) {
      const float* g = a.gate + ((long long)z * a.q_heads + head) * a.gate_stride + d;
      v0 = (1.0f / (1.0f + expf(-g[0]))) * v0;
      v1 = (1.0f / (1.0f + expf(-g[1]))) * v1;
    }
    a.out[at] = v0;
    a.out[at + 1] = v1;
    value[q * D + d] = v0;
    value[q * D + d + 1] = v1;
  }
  if constexpr (D % 32 == 0) {
    if (a.records) {
      __syncthreads();
      // whole warps: group x D and the stride are multiples of 32
      for (int i = threadIdx.x; i < group * D; i += SPLIT_THREADS) {
        const int head = kv_head * group + i / D, d = i % D;
        x22_record_block(value[i], a.records, z, (head * D + d) / 32, a.q_heads * D / 32);
      }
    }
  }
}

template <int D>
__global__ void __launch_bounds__(SPLIT_THREADS) attention_split_kernel(const AttentionArgs a) {
  pdl_trigger();  // the next kernel may launch and wait for this one
  pdl_wait();     // what the kernels before this one wrote is visible
  using T = SplitTile<D>;
  constexpr int KEYS = T::KEYS;
  extern __shared__ __align__(16) uint8_t tile[];
  uint8_t* ks = tile;
  uint8_t* vs = tile + T::K_BYTES;
  uint4* frags = reinterpret_cast<uint4*>(tile + T::K_BYTES + T::V_BYTES);  // [k-step][hi, lo][lane]
  __shared__ float red_max[T::QW][16], red_sum[T::QW][16];
  const int split = blockIdx.x, head = blockIdx.y, z = blockIdx.z;
  const int tid = threadIdx.x, lane = tid % 32, warp = tid / 32, g = lane / 4, t = lane % 4;
  const int group = a.q_heads / a.kv_heads;  // <= 16
  const Query query(a, z);
  int lo, hi;
  visible(a, query, lo, hi);
  const int k0 = split * KEYS;
  const int first = k0 > lo ? k0 : lo, last = k0 + KEYS < hi ? k0 + KEYS : hi;  // [first, last)
  const int ps = a.page_size;

  // where each visible key's row and each whole visible run of 8 value
  // positions starts in the cache, in 16-byte units (a page is looked up
  // once per key, not once per copy)
  __shared__ unsigned key_at[KEYS], run_at[T::RUNS];
  __shared__ bool run_whole[T::RUNS];
  constexpr unsigned NONE = 0xffffffffu;
  if (tid < KEYS) {
    const int key = k0 + tid;
    unsigned at = NONE;
    if (key >= first && key < last) {
      const long long page = query.table[key / ps];
      at = unsigned((((page * ps + key % ps) * a.kv_heads + head) * D) / 8);
    }
    key_at[tid] = at;
  }
  if (tid < T::RUNS) {
    const int key = k0 + 8 * tid;
    const bool whole = key >= first && key + 8 <= last;
    run_whole[tid] = whole;
    run_at[tid] = whole ? unsigned((((long long)query.table[key / ps] * a.kv_heads + head) * D *
                                        ps + key % ps) / 8)
                        : NONE;
  }
  // q as A fragments, hi and lo: rows past the group are zeros
  const float* q = a.q + ((long long)z * a.q_heads + head * group) * D;
  for (int i = tid; i < T::KQ * 32; i += SPLIT_THREADS) {
    const int kk = i / 32, l = i % 32, row = l / 4, col = 16 * kk + 2 * (l % 4);
    float2 v[4] = {};
    if (row < group) {
      v[0] = make_float2(q[row * D + col], q[row * D + col + 1]);
      v[2] = make_float2(q[row * D + col + 8], q[row * D + col + 9]);
    }
    if (row + 8 < group) {
      v[1] = make_float2(q[(row + 8) * D + col], q[(row + 8) * D + col + 1]);
      v[3] = make_float2(q[(row + 8) * D + col + 8], q[(row + 8) * D + col + 9]);
    }
    uint4 h, w;
    split_pair(v[0].x, v[0].y, h.x, w.x);
    split_pair(v[1].x, v[1].y, h.y, w.y);
    split_pair(v[2].x, v[2].y, h.z, w.z);
    split_pair(v[3].x, v[3].y, h.w, w.w);
    frags[(kk * 2) * 32 + l] = h;
    frags[(kk * 2 + 1) * 32 + l] = w;
  }
  __syncthreads();

  // keys (an invisible key's row is left as it is: its score is never used).
  // Where a row's chunks divide the threads, a thread's chunk column is the
  // same for all its keys, and their starts are read before the copies.
  if constexpr (SPLIT_THREADS % T::CH == 0) {
    constexpr int STEP = SPLIT_THREADS / T::CH, PER = KEYS / STEP;
    const int c = tid % T::CH, k0 = tid / T::CH;
    unsigned at[PER];
#pragma unroll
    for (int j = 0; j < PER; ++j) at[j] = key_at[k0 + STEP * j];
#pragma unroll
    for (int j = 0; j < PER; ++j)
      if (at[j] != NONE)
        cp_async16(ks + T::key_chunk(k0 + STEP * j, c), a.keys + 8 * ((long long)at[j] + c));
  } else {
#pragma unroll 4
    for (int i = tid; i < KEYS * T::CH; i += SPLIT_THREADS) {
      const int k = i / T::CH, c = i % T::CH;
      const unsigned at = key_at[k];
      if (at != NONE) cp_async16(ks + T::key_chunk(k, c), a.keys + 8 * ((long long)at + c));
    }
  }
  asm volatile("cp.async.commit_group;" ::: "memory");  // the keys: group 1
  // values, a 16-byte run of 8 positions of one dimension at a time (a run
  // never crosses a page: pages are multiples of 16 positions); a thread's
  // run r is the same for all its dimensions (RUNS divides the threads)
  const long long column = ps / 8;  // 16-byte units from one dimension to the next
  static_assert(SPLIT_THREADS % T::RUNS == 0, "a thread's run is fixed");
  constexpr int V_STEP = SPLIT_THREADS / T::RUNS;
  const int r = tid % T::RUNS, d0 = tid / T::RUNS;
  const bool whole_run = run_whole[r];
  const unsigned run_start = run_at[r];
#pragma unroll 4
  for (int d = d0; d < D; d += V_STEP) {
    uint8_t* to = vs + T::value_chunk(d, r);
    if (whole_run) {
      cp_async16(to, a.values + 8 * (run_start + d * column));
    } else {
      // a run the visible range cuts or misses: its visible positions one
      // by one, zeros elsewhere (an invisible position's weight is 0, and
      // 0 times whatever the cache holds there must not reach the sum)
      const int key = k0 + 8 * r;
      __align__(16) __half run[8];
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        const int p = key + j;
        run[j] = __float2half_rn(0.0f);
        if (p >= first && p < last) {
          const long long page = query.table[p / ps];
          run[j] = a.values[((page * a.kv_heads + head) * D + d) * ps + p % ps];
        }
      }
      *reinterpret_cast<uint4*>(to) = *reinterpret_cast<const uint4*>(run);
    }
  }
  // the values (group 2) keep coming while the keys are scored
  asm volatile("cp.async.commit_group;\n\tcp.async.wait_group 1;" ::: "memory");
  __syncthreads();

  // scores of this warp's keys: s[j] holds rows (g, g + 8), keys
  // 16 warp + 8 j + (2t, 2t + 1)
  const bool scoring = warp < T::QW;
  float s[T::NT][4];
#pragma unroll
  for (int j = 0; j < T::NT; ++j) s[j][0] = s[j][1] = s[j][2] = s[j][3] = 0.0f;
#pragma unroll
  for (int kk = 0; kk < T::KQ; ++kk) {
    if (!scoring) break;
    const uint4 qh = frags[(kk * 2) * 32 + lane], ql = frags[(kk * 2 + 1) * 32 + lane];
#pragma unroll
    for (int j = 0; j < T::NT; ++j) {
      const int k = 16 * warp + 8 * j + g;
      const uint32_t b0 = *reinterpret_cast<const uint32_t*>(ks + T::key_chunk(k, 2 * kk) + 4 * t);
      const uint32_t b1 =
          *reinterpret_cast<const uint32_t*>(ks + T::key_chunk(k, 2 * kk + 1) + 4 * t);
      mma_f16(s[j], qh, b0, b1);
      mma_f16(s[j], ql, b0, b1);
    }
  }
  float m_lo = -INFINITY, m_hi = -INFINITY;
#pragma unroll
  for (int j = 0; j < T::NT; ++j) {
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const int key = k0 + 16 * warp + 8 * j + 2 * t + (e & 1);
      float v = s[j][e] * a.scale;
      if (a.has_softcap) v = a.softcap * tanhf(v / a.softcap);
      v = key >= first && key < last ? v : -INFINITY;
      s[j][e] = v;
      if (e < 2) m_lo = fmaxf(m_lo, v);
      else m_hi = fmaxf(m_hi, v);
    }
  }
#pragma unroll
  for (int o = 1; o < 4; o *= 2) {
    m_lo = fmaxf(m_lo, __shfl_xor_sync(0xffffffffu, m_lo, o));
    m_hi = fmaxf(m_hi, __shfl_xor_sync(0xffffffffu, m_hi, o));
  }
  if (scoring && t == 0) {
    red_max[warp][g] = m_lo;
    red_max[warp][g + 8] = m_hi;
  }
  __syncthreads();  // every warp is past its q fragments too
  float largest_lo = -INFINITY, largest_hi = -INFINITY;
#pragma unroll
  for (int w = 0; w < T::QW; ++w) {
    largest_lo = fmaxf(largest_lo, red_max[w][g]);
    largest_hi = fmaxf(largest_hi, red_max[w][g + 8]);
  }
  float sum_lo = 0.0f, sum_hi = 0.0f;
#pragma unroll
  for (int j = 0; j < T::NT; ++j) {
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const float m = e < 2 ? largest_lo : largest_hi;
      const float p = s[j][e] == -INFINITY ? 0.0f : expf(s[j][e] - m);
      s[j][e] = p;
      if (e < 2) sum_lo += p;
      else sum_hi += p;
    }
  }
#pragma unroll
  for (int o = 1; o < 4; o *= 2) {
    sum_lo += __shfl_xor_sync(0xffffffffu, sum_lo, o);
    sum_hi += __shfl_xor_sync(0xffffffffu, sum_hi, o);
  }
  if (scoring) {
    if (t == 0) {
      red_sum[warp][g] = sum_lo;
      red_sum[warp][g + 8] = sum_hi;
    }
    // this warp's weights as the A fragment of k-step `warp` (the score
    // tiles 0 and 1 are exactly a 16-key A fragment, lane for lane)
    uint4 h, w;
    split_pair(s[0][0], s[0][1], h.x, w.x);
    split_pair(s[0][2], s[0][3], h.y, w.y);
    split_pair(s[1][0], s[1][1], h.z, w.z);
    split_pair(s[1][2], s[1][3], h.w, w.w);
    frags[(warp * 2) * 32 + lane] = h;
    frags[(warp * 2 + 1) * 32 + lane] = w;
  }
  asm volatile("cp.async.wait_all;" ::: "memory");  // the values are in
  __syncthreads();

  // p.v for this warp's dimension tiles [ND w / 8, ND (w + 1) / 8)
  constexpr int MAXN = (T::ND + T::WARPS - 1) / T::WARPS;
  const int n0 = T::ND * warp / T::WARPS, n1 = T::ND * (warp + 1) / T::WARPS;
  float o[MAXN][4];
#pragma unroll
  for (int n = 0; n < MAXN; ++n) o[n][0] = o[n][1] = o[n][2] = o[n][3] = 0.0f;
#pragma unroll
  for (int kk = 0; kk < T::KP; ++kk) {
    const uint4 ph = frags[(kk * 2) * 32 + lane], pl = frags[(kk * 2 + 1) * 32 + lane];
#pragma unroll
    for (int n = 0; n < MAXN; ++n) {
      if (n0 + n < n1) {
        const int d = 8 * (n0 + n) + g;
        const uint32_t b0 =
            *reinterpret_cast<const uint32_t*>(vs + T::value_chunk(d, 2 * kk) + 4 * t);
        const uint32_t b1 =
            *reinterpret_cast<const uint32_t*>(vs + T::value_chunk(d, 2 * kk + 1) + 4 * t);
        mma_f16(o[n], ph, b0, b1);
        mma_f16(o[n], pl, b0, b1);
      }
    }
  }
  const long long at0 = ((long long)z * a.q_heads + head * group) * a.splits + split;
#pragma unroll
  for (int n = 0; n < MAXN; ++n) {
    if (n0 + n >= n1) break;
    const int d = 8 * (n0 + n) + 2 * t;
    if (g < group)
      *reinterpret_cast<float2*>(a.part_o + (at0 + (long long)g * a.splits) * D + d) =
          make_float2(o[n][0], o[n][1]);
    if (g + 8 < group)
      *reinterpret_cast<float2*>(a.part_o + (at0 + (long long)(g + 8) * a.splits) * D + d) =
          make_float2(o[n][2], o[n][3]);
  }
  if (tid < group) {
    float largest = -INFINITY, total = 0.0f;
#pragma unroll
    for (int w = 0; w < T::QW; ++w) {
      largest = fmaxf(largest, red_max[w][tid]);
      total += red_sum[w][tid];
    }
    a.part_ml[(at0 + (long long)tid * a.splits) * 2] = largest;
    a.part_ml[(at0 + (long long)tid * a.splits) * 2 + 1] = total;
  }
  if (!a.fused_join) return;
  // the last split of this (row, key head) to finish joins its query heads
  static_assert(T::BYTES >= 4 * (MAX_GROUP * MAX_FUSED_SPLITS + MAX_GROUP + MAX_GROUP * D),
                "the join's factors and values fit in the tile");
  __shared__ int joins;
  __syncthreads();  // (every warp is done with the tile)
  unsigned* arrivals = join_arrivals + (long long)z * a.kv_heads + head;
  if (tid == 0) {
    __threadfence();
    joins = atomicAdd(arrivals, 1u) == unsigned(a.splits - 1);
    if (joins) __threadfence();
  }
  __syncthreads();
  if (!joins) return;
  join_group<D>(a, z, head, group, tile);
  if (tid == 0) *arrivals = 0;
}

template <int D>
__global__ void __launch_bounds__(SPLIT_THREADS) attention_join_kernel(const AttentionArgs a,
                                                                       const float* sinks,
                                                                       float* out,
                                                                       uint8_t* records,
                                                                       const float* gate,
                                                                       int gate_stride) {
  pdl_trigger();  // the next kernel may launch and wait for this one
  pdl_wait();     // what the kernels before this one wrote is visible
  extern __shared__ __align__(16) float factor[];
  __shared__ float shared_total;
  // query head blockIdx.x of row blockIdx.y: as a group of one, with every
  // pair of dimensions' sixteen splits in flight; past 4096 splits (the
  // group routine's factor area) one split's loads after another
  if (a.splits <= JOIN_GROUP_SPLITS)
    join_group<D>(a, blockIdx.y, blockIdx.x, 1, reinterpret_cast<uint8_t*>(factor));
  else
    join_head<D, SPLIT_THREADS>(a, sinks, out, records, gate, gate_stride, blockIdx.x,
                                blockIdx.y, factor, &shared_total);
}

#define DRIFT_ATTENTION_REGISTER(D)                                                   \
  DRIFT_REGISTER(attention_split_d##D, attention_split_kernel<D>)                      \
  DRIFT_REGISTER(attention_join_d##D, attention_join_kernel<D>)
DRIFT_ATTENTION_REGISTER(64)
DRIFT_ATTENTION_REGISTER(80)
DRIFT_ATTENTION_REGISTER(128)
DRIFT_ATTENTION_REGISTER(256)
DRIFT_REGISTER(cache_write_f16, cache_write_kernel)
DRIFT_REGISTER(attention_inputs_f32, attention_inputs_kernel)

template <int D>
int launch_attention(const AttentionArgs& a, const float* sinks, float* out, cudaStream_t stream,
                     uint8_t* records = nullptr, const float* gate = nullptr,
                     int gate_stride = 0) {
  // all of L1 as shared memory, so that two or more splits share an SM
  static PerDevice configured;
  DRIFT_TRY(ensure_shared_memory(configured, attention_split_kernel<D>, SplitTile<D>::BYTES, 100));
  // the join in the last split of each (row, key head) when its factors fit
  // in shared memory and the arrival counts in their array; else its own
  // launch
  AttentionArgs args = a;
  args.fused_join = a.splits <= MAX_FUSED_SPLITS && (long long)a.tokens * a.kv_heads <= MAX_JOINS &&
                    (long long)(a.q_heads / a.kv_heads) * D * a.splits <= MAX_FUSED_JOIN_FLOATS;
  args.sinks = sinks;
  args.out = out;
  args.records = records;
  args.gate = gate;
  args.gate_stride = gate_stride;
  DRIFT_CUDA(launch_pdl(attention_split_kernel<D>, dim3(a.splits, a.kv_heads, a.tokens),
                        SPLIT_THREADS, SplitTile<D>::BYTES, stream, args));
  DRIFT_LAUNCHED("attention_split");
  if (args.fused_join) return 0;
  const size_t join_bytes =
      a.splits <= JOIN_GROUP_SPLITS ? join_group_bytes<D>() : a.splits * sizeof(float);
  DRIFT_CUDA(launch_pdl(attention_join_kernel<D>, dim3(a.q_heads, a.tokens), SPLIT_THREADS,
                        join_bytes, stream, args, sinks, out, records, gate, gate_stride));
  DRIFT_LAUNCHED("attention_join");
  return 0;
}

// Keys a split of attention takes, by head width.
int keys_per_split(int head_dim) { return split_keys(head_dim); }

// The most splits the join takes (their factors in 48 KB of shared memory).
constexpr int MAX_SPLITS = 48 * 1024 / 4 - 16;

int check_cache(int pages, int page_size, int kv_heads, int head_dim, const int32_t* page_table,
                int table_pages, long long positions, const char* call) {
  if (page_size <= 0 || page_size % 16 != 0)
    return invalid("pages of %d tokens: not a multiple of 16", page_size);
  if (head_dim != 64 && head_dim != 80 && head_dim != 128 && head_dim != 256)
    return invalid("%s: heads of %d (kernels take 64, 80, 128, 256)", call, head_dim);
  if (pages <= 0 || kv_heads <= 0) return invalid("%s: an empty cache", call);
  // the kernels address the cache in 16-byte units with 32-bit offsets
  if ((long long)pages * page_size * kv_heads * head_dim / 8 >= 0xffffffffll)
    return invalid("%s: a cache of %lld bytes per side (at most 64 GiB)", call,
                   (long long)pages * page_size * kv_heads * head_dim * 2);
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
  if ((long long)key_count > (long long)MAX_SPLITS * keys_per_split(head_dim))
    return invalid("attention: %d keys (at most %d)", key_count,
                   MAX_SPLITS * keys_per_split(head_dim));
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
  const int per_split = keys_per_split(head_dim);
  a.splits = key_count > 0 ? (key_count + per_split - 1) / per_split : 1;
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

static int attention_inputs_decode(const float* q, int q_stride, const float* k, const float* v,
                                   int batch, int q_heads, int kv_heads, int head_dim,
                                   const float* q_norm, const float* k_norm, float epsilon,
                                   float weight_offset, const int32_t* positions, float theta,
                                   int rotary, int layout, float* q_out, void* keys, void* values,
                                   int pages, int page_size, const int32_t* page_tables,
                                   int table_stride, drift_stream_t stream) {
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
                        cudaStream_t(stream), q, k, v, q_heads, kv_heads, head_dim, q_stride,
                        q_norm, k_norm,
                        epsilon, weight_offset, positions, theta, rotary, layout, q_out,
                        static_cast<__half*>(keys), static_cast<__half*>(values), page_size,
                        page_tables, table_stride, device_error_word()));
  DRIFT_LAUNCHED("attention_inputs");
  return 0;
}

int drift_attention_inputs_decode(const float* q, const float* k, const float* v, int batch,
                                  int q_heads, int kv_heads, int head_dim, const float* q_norm,
                                  const float* k_norm, float epsilon, float weight_offset,
                                  const int32_t* positions, float theta, int rotary, int layout,
                                  float* q_out, void* keys, void* values, int pages,
                                  int page_size, const int32_t* page_tables, int table_stride,
                                  drift_stream_t stream) {
  return attention_inputs_decode(q, head_dim, k, v, batch, q_heads, kv_heads, head_dim, q_norm,
                                 k_norm, epsilon, weight_offset, positions, theta, rotary, layout,
                                 q_out, keys, values, pages, page_size, page_tables, table_stride,
                                 stream);
}

int drift_attention_inputs_decode_split(const float* query_and_gate, const float* k,
                                        const float* v, int batch, int q_heads, int kv_heads,
                                        int head_dim, const float* q_norm, const float* k_norm,
                                        float epsilon, float weight_offset,
                                        const int32_t* positions, float theta, int rotary,
                                        int layout, float* q_out, void* keys, void* values,
                                        int pages, int page_size, const int32_t* page_tables,
                                        int table_stride, drift_stream_t stream) {
  return attention_inputs_decode(query_and_gate, 2 * head_dim, k, v, batch, q_heads, kv_heads,
                                 head_dim, q_norm, k_norm, epsilon, weight_offset, positions,
                                 theta, rotary, layout, q_out, keys, values, pages, page_size,
                                 page_tables, table_stride, stream);
}

size_t drift_attention_workspace_bytes(int rows, int q_heads, int head_dim, int key_count) {
  if (rows <= 0 || q_heads <= 0 || head_dim <= 0) return 0;
  const int per_split = keys_per_split(head_dim);
  const size_t splits = key_count > 0 ? size_t(key_count + per_split - 1) / per_split : 1;
  return size_t(rows) * q_heads * splits * (head_dim + 2) * sizeof(float);
}

static int attention_decode(const float* q, int batch, int q_heads, const void* keys,
                            const void* values, int pages, int page_size, int kv_heads,
                            int head_dim, const int32_t* page_tables, int table_stride,
                            const int32_t* positions, int max_key_count, float scale, int window,
                            float softcap, const float* sinks, float* out, uint8_t* records,
                            const float* gate, int gate_stride, drift_stream_t stream) {
  if (batch < 0 || q_heads <= 0) return invalid("attention: %d sequences of %d heads", batch, q_heads);
  DRIFT_TRY(check_cache(pages, page_size, kv_heads, head_dim, page_tables, table_stride,
                        max_key_count, "attention"));
  if (q_heads % kv_heads != 0 || q_heads / kv_heads > MAX_GROUP)
    return invalid("attention: %d query heads over %d key heads", q_heads, kv_heads);
  if (max_key_count <= 0 ||
      (long long)max_key_count > (long long)MAX_SPLITS * keys_per_split(head_dim))
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
  a.splits = (max_key_count + keys_per_split(head_dim) - 1) / keys_per_split(head_dim);
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
    case 64: return launch_attention<64>(a, sinks, out, s, records, gate, gate_stride);
    case 80: return launch_attention<80>(a, sinks, out, s, records, gate, gate_stride);
    case 128: return launch_attention<128>(a, sinks, out, s, records, gate, gate_stride);
    default: return launch_attention<256>(a, sinks, out, s, records, gate, gate_stride);
  }
}

int drift_attention_decode(const float* q, int batch, int q_heads, const void* keys,
                           const void* values, int pages, int page_size, int kv_heads,
                           int head_dim, const int32_t* page_tables, int table_stride,
                           const int32_t* positions, int max_key_count, float scale, int window,
                           float softcap, const float* sinks, float* out, drift_stream_t stream) {
  return attention_decode(q, batch, q_heads, keys, values, pages, page_size, kv_heads, head_dim,
                          page_tables, table_stride, positions, max_key_count, scale, window,
                          softcap, sinks, out, nullptr, nullptr, 0, stream);
}

int drift_attention_decode_prepared(const float* q, int batch, int q_heads, const void* keys,
                                    const void* values, int pages, int page_size, int kv_heads,
                                    int head_dim, const int32_t* page_tables, int table_stride,
                                    const int32_t* positions, int max_key_count, float scale,
                                    int window, float softcap, const float* sinks, float* out,
                                    void* prepared, drift_stream_t stream) {
  if (!prepared) return invalid("attention: no prepared x");
  if (head_dim % 32 != 0) return invalid("attention: prepared x needs heads of whole 32-value blocks");
  return attention_decode(q, batch, q_heads, keys, values, pages, page_size, kv_heads, head_dim,
                          page_tables, table_stride, positions, max_key_count, scale, window,
                          softcap, sinks, out, static_cast<uint8_t*>(prepared), nullptr, 0,
                          stream);
}

int drift_attention_decode_gated(const float* q, int batch, int q_heads, const void* keys,
                                 const void* values, int pages, int page_size, int kv_heads,
                                 int head_dim, const int32_t* page_tables, int table_stride,
                                 const int32_t* positions, int max_key_count, float scale,
                                 int window, float softcap, const float* sinks, float* out,
                                 const float* gate, int gate_stride, void* prepared,
                                 drift_stream_t stream) {
  if (!gate || gate_stride < head_dim) return invalid("attention: no output gate");
  if (prepared && head_dim % 32 != 0)
    return invalid("attention: prepared x needs heads of whole 32-value blocks");
  return attention_decode(q, batch, q_heads, keys, values, pages, page_size, kv_heads, head_dim,
                          page_tables, table_stride, positions, max_key_count, scale, window,
                          softcap, sinks, out, static_cast<uint8_t*>(prepared), gate, gate_stride,
                          stream);
}

}  // extern "C"
