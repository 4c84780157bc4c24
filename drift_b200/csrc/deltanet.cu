// Gated DeltaNet, the hybrid decoder's linear-attention layers (the runner's
// SequenceOps.causalConv / gatedDeltaRule, ops/SequenceOps.scala:60-77, and
// NormalisationOps.gatedRmsNorm; CPU reference ops/CpuSequence.scala:29-158,
// ops/CpuNormalisation.scala:167-178). Every recurrent quantity is F32 here;
// the CPU reference sums in Double, and the results are held to the 1e-4
// absolute + 1e-3 relative bar.
//
// - causal_conv: a thread per channel walks the tokens in order, its window
//   of the last (taps - 1) * dilation inputs in registers; out = SiLU of the
//   taps' sum; the window goes back to the state (and, with a history, the
//   window after every token).
// - gated_delta_rule: per value head h, the state S [D][D] in registers: a
//   CTA of 4 warps takes 32 columns of S (lane = column), warp w the rows
//   [w D / 4, (w + 1) D / 4) -- D / 4 values a thread. Per token: q and k of
//   h's key head into shared memory, L2-normalised (q also by 1/sqrt(D)); g =
//   exp(decay softplus(a + dt_bias)), beta = sigmoid(b); S *= g; delta_j =
//   (v_j - sum_i S_ij k_i) beta; S_ij += k_i delta_j; o_j = sum_i S_ij q_i.
//   The column sums meet across the 4 warps in shared memory. The state is
//   read once and written once per call (and per token with a history): at
//   D = 128, 64 KB per head each way.
// - gated_rms_norm: a row's RMS norm times act(gate) (SiLU or sigmoid),
//   optionally writing the out projection's x records.
#include <cuda_runtime.h>

#include "common.cuh"
#include "registry.cuh"
#include "rowwise.cuh"
#include "x22.cuh"

namespace drift {
namespace {

constexpr int MAX_SPAN = 16;

__global__ void __launch_bounds__(256) causal_conv_kernel(const float* __restrict__ x, int tokens,
                                                          int channels,
                                                          const float* __restrict__ weight,
                                                          int taps, int dilation,
                                                          float* __restrict__ state,
                                                          float* __restrict__ history,
                                                          float* __restrict__ out) {
  pdl_trigger();  // the next kernel may launch and wait for this one
  pdl_wait();     // what the kernels before this one wrote is visible
  const int c = blockIdx.x * blockDim.x + threadIdx.x;
  if (c >= channels) return;
  const int span = (taps - 1) * dilation;
  // sequence blockIdx.y of a decode batch: its own tokens, state and out
  x += (long long)blockIdx.y * tokens * channels;
  out += (long long)blockIdx.y * tokens * channels;
  state += (long long)blockIdx.y * span * channels;
  float window[MAX_SPAN];  // the inputs before the current token, oldest first
#pragma unroll
  for (int i = 0; i < MAX_SPAN; ++i) window[i] = i < span ? state[(long long)i * channels + c] : 0.0f;
  const float* w = weight + (long long)c * taps;
  for (int t = 0; t < tokens; ++t) {
    const float current = x[(long long)t * channels + c];
    // tap i reads (taps - 1 - i) * dilation tokens back: the window's entry
    // span - (taps - 1 - i) * dilation, or the current token for i = taps - 1
    float sum = 0.0f;
    for (int i = 0; i < taps - 1; ++i) {
      const int at = span - (taps - 1 - i) * dilation;
      float seen = 0.0f;
#pragma unroll
      for (int s = 0; s < MAX_SPAN; ++s)
        if (s == at) seen = window[s];
      sum = fmaf(w[i], seen, sum);
    }
    sum = fmaf(w[taps - 1], current, sum);
    out[(long long)t * channels + c] = sum / (1.0f + expf(-sum));
#pragma unroll
    for (int s = 0; s + 1 < MAX_SPAN; ++s)
      if (s + 1 < span) window[s] = window[s + 1];
#pragma unroll
    for (int s = 0; s < MAX_SPAN; ++s)
      if (s == span - 1) window[s] = current;
    if (history)
#pragma unroll
      for (int s = 0; s < MAX_SPAN; ++s)
        if (s < span) history[((long long)t * span + s) * channels + c] = window[s];
  }
#pragma unroll
  for (int s = 0; s < MAX_SPAN; ++s)
    if (s < span) state[(long long)s * channels + c] = window[s];
}

constexpr int RULE_THREADS = 128, RULE_WARPS = 4, RULE_COLUMNS = 32;

__device__ __forceinline__ float block4_sum(float value, float* scratch) {
#pragma unroll
  for (int o = 16; o > 0; o /= 2) value += __shfl_xor_sync(0xffffffffu, value, o);
  const int warp = threadIdx.x / 32;
  if (threadIdx.x % 32 == 0) scratch[warp] = value;
  __syncthreads();
  const float total = ((scratch[0] + scratch[1]) + scratch[2]) + scratch[3];
  __syncthreads();
  return total;
}

template <int D>
__global__ void __launch_bounds__(RULE_THREADS) gated_delta_rule_kernel(
    const float* __restrict__ qkv, int tokens, int key_heads, int value_heads, int tiled,
    const float* __restrict__ a, const float* __restrict__ b, const float* __restrict__ decay,
    const float* __restrict__ dt_bias, float* __restrict__ state, float* __restrict__ history,
    float* __restrict__ out) {
  pdl_trigger();  // the next kernel may launch and wait for this one
  pdl_wait();     // what the kernels before this one wrote is visible
  static_assert(D % RULE_COLUMNS == 0 && D % RULE_WARPS == 0, "head width");
  constexpr int ROWS = D / RULE_WARPS;  // rows of S a thread holds
  constexpr int SLICES = D / RULE_COLUMNS;
  __shared__ float qs[D], ks[D];
  __shared__ float sums[RULE_WARPS][RULE_COLUMNS];
  __shared__ float scratch[RULE_WARPS];
  const int h = blockIdx.x / SLICES, slice = blockIdx.x % SLICES;
  const int lane = threadIdx.x % 32, warp = threadIdx.x / 32;
  {
    // sequence blockIdx.y of a decode batch: its own tokens and state
    const long long z = blockIdx.y;
    qkv += z * tokens * (long long)(2 * key_heads + value_heads) * D;
    a += z * tokens * value_heads;
    b += z * tokens * value_heads;
    out += z * tokens * (long long)value_heads * D;
    state += z * (long long)value_heads * D * D;
  }
  const int j = slice * RULE_COLUMNS + lane, i0 = warp * ROWS;
  const int kh = tiled ? h % key_heads : h / (value_heads / key_heads);
  const long long width = (long long)(2 * key_heads + value_heads) * D;
  float* column = state + ((long long)h * D + i0) * D + j;
  float s[ROWS];
#pragma unroll
  for (int r = 0; r < ROWS; ++r) s[r] = column[(long long)r * D];
  const float rsqrt_d = 1.0f / sqrtf(float(D));
  for (int t = 0; t < tokens; ++t) {
    const float* row = qkv + t * width;
    // q and k of the key head, L2-normalised
    float qq = 0.0f, kk = 0.0f;
    for (int i = threadIdx.x; i < D; i += RULE_THREADS) {
      const float qv = row[(long long)kh * D + i], kv = row[(long long)key_heads * D + kh * D + i];
      qs[i] = qv;
      ks[i] = kv;
      qq = fmaf(qv, qv, qq);
      kk = fmaf(kv, kv, kk);
    }
    const float q_scale = 1.0f / sqrtf(block4_sum(qq, scratch) + 1e-6f) * rsqrt_d;
    const float k_scale = 1.0f / sqrtf(block4_sum(kk, scratch) + 1e-6f);
    const float v = row[2ll * key_heads * D + (long long)h * D + j];
    const float x = a[(long long)t * value_heads + h] + dt_bias[h];
    const float g = expf(decay[h] * (x > 20.0f ? x : log1pf(expf(x))));
    const float beta = 1.0f / (1.0f + expf(-b[(long long)t * value_heads + h]));
    // S *= g; the column's k.S
    float part = 0.0f;
#pragma unroll
    for (int r = 0; r < ROWS; ++r) {
      s[r] *= g;
      part = fmaf(s[r], ks[i0 + r] * k_scale, part);
    }
    sums[warp][lane] = part;
    __syncthreads();
    const float kv = ((sums[0][lane] + sums[1][lane]) + sums[2][lane]) + sums[3][lane];
    const float delta = (v - kv) * beta;
    __syncthreads();  // sums is reused below
    float o = 0.0f;
#pragma unroll
    for (int r = 0; r < ROWS; ++r) {
      s[r] = fmaf(ks[i0 + r] * k_scale, delta, s[r]);
      o = fmaf(s[r], qs[i0 + r] * q_scale, o);
    }
    sums[warp][lane] = o;
    __syncthreads();
    if (warp == 0)
      out[((long long)t * value_heads + h) * D + j] =
          ((sums[0][lane] + sums[1][lane]) + sums[2][lane]) + sums[3][lane];
    if (history) {
      float* kept = history + (((long long)t * value_heads + h) * D + i0) * D + j;
#pragma unroll
      for (int r = 0; r < ROWS; ++r) kept[(long long)r * D] = s[r];
    }
    __syncthreads();  // qs, ks and sums are rewritten for the next token
  }
#pragma unroll
  for (int r = 0; r < ROWS; ++r) column[(long long)r * D] = s[r];
}

// A row of `cols` values (rows are (token, head) pairs of `heads` heads), its
// RMS norm times act(gate); with `records`, the out projection's x records of
// rows [token][heads * cols].
template <int PER>
__global__ void __launch_bounds__(128) gated_rms_norm_kernel(
    const float* __restrict__ x, const float* __restrict__ weight, const float* __restrict__ gate,
    int sigmoid, float epsilon, float* __restrict__ out, int cols, int heads,
    uint8_t* __restrict__ records) {
  pdl_trigger();  // the next kernel may launch and wait for this one
  pdl_wait();     // what the kernels before this one wrote is visible
  __shared__ float partial[32];
  const long long base = (long long)blockIdx.x * cols;
  float value[PER];
  float squares = 0.0f;
#pragma unroll
  for (int i = 0; i < PER; ++i) {
    const int c = threadIdx.x + i * 128;
    value[i] = c < cols ? x[base + c] : 0.0f;
    squares = fmaf(value[i], value[i], squares);
  }
  const float total = block_sum(squares, partial);
  const float scale = 1.0f / sqrtf(total / float(cols) + epsilon);
#pragma unroll
  for (int i = 0; i < PER; ++i) {
    const int c = threadIdx.x + i * 128;
    if (c >= cols) continue;
    const float gv = gate[base + c];
    const float act = sigmoid ? 1.0f / (1.0f + expf(-gv)) : gv / (1.0f + expf(-gv));
    const float normed = value[i] * scale * weight[c] * act;
    out[base + c] = normed;
    if (records) {
      const int token = blockIdx.x / heads, head = blockIdx.x % heads;
      x22_record_block(normed, records, token, (head * cols + c) / 32, heads * cols / 32);
    }
  }
}

// A DeltaNet layer's decode step after its input products, one CTA per
// (value head h, sequence), when every value head has a key head of its own
// (key_heads == value_heads: a CTA then owns its q, k and v channels and
// their convolution state): the causal convolution of the head's 3 D
// channels (causal_conv_kernel's arithmetic), the gated delta rule on its
// D x D state (gated_delta_rule_kernel's: 4 D / 32 warps, warp w the
// columns of slice w % 4 and the rows of group w / 4, the column sums met
// in the same order), then the RMS norm of the head's output times SiLU(z)
// with the out projection's records (gated_rms_norm_kernel's) -- three
// launches' work in one, with the same bits.
constexpr int STEP_D = 128, STEP_THREADS = 4 * STEP_D;  // 16 warps
__global__ void __launch_bounds__(STEP_THREADS) delta_decode_step_kernel(
    const float* __restrict__ qkv, const float* __restrict__ z, int heads,
    const float* __restrict__ conv_weight, int taps, float* __restrict__ conv_states,
    const float* __restrict__ a, const float* __restrict__ b, const float* __restrict__ decay,
    const float* __restrict__ dt_bias, float* __restrict__ states,
    const float* __restrict__ norm_weight, float epsilon, float* __restrict__ out,
    uint8_t* __restrict__ records) {
  pdl_trigger();  // the next kernel may launch and wait for this one
  pdl_wait();     // what the kernels before this one wrote is visible
  constexpr int D = STEP_D, ROWS = D / RULE_WARPS, SLICES = D / RULE_COLUMNS;
  __shared__ float conv[3 * D];  // the head's convolved q, k, v
  __shared__ float sums[RULE_WARPS][SLICES][RULE_COLUMNS];
  __shared__ float o[D];
  __shared__ float partial[32];
  const int h = blockIdx.x, seq = blockIdx.y, tid = threadIdx.x;
  const int channels = 3 * heads * D, span = taps - 1;
  // the convolution: thread t < 3 D takes channel (t / D) (heads D) + h D + t % D
  if (tid < 3 * D) {
    const int c = (tid / D) * heads * D + h * D + tid % D;
    float* state = conv_states + (long long)seq * span * channels;
    float window[MAX_SPAN];
#pragma unroll
    for (int i = 0; i < MAX_SPAN; ++i) window[i] = i < span ? state[(long long)i * channels + c] : 0.0f;
    const float* w = conv_weight + (long long)c * taps;
    const float current = qkv[(long long)seq * channels + c];
    float sum = 0.0f;
    for (int i = 0; i < taps - 1; ++i) {
      const int at = span - (taps - 1 - i);
      float seen = 0.0f;
#pragma unroll
      for (int t = 0; t < MAX_SPAN; ++t)
        if (t == at) seen = window[t];
      sum = fmaf(w[i], seen, sum);
    }
    sum = fmaf(w[taps - 1], current, sum);
    conv[tid] = sum / (1.0f + expf(-sum));
#pragma unroll
    for (int t = 0; t + 1 < MAX_SPAN; ++t)
      if (t + 1 < span) window[t] = window[t + 1];
#pragma unroll
    for (int t = 0; t < MAX_SPAN; ++t)
      if (t == span - 1) window[t] = current;
#pragma unroll
    for (int t = 0; t < MAX_SPAN; ++t)
      if (t < span) state[(long long)t * channels + c] = window[t];
  }
  __syncthreads();
  // the rule: q and k L2-normalised over the first 4 warps, as the rule
  // kernel's 128 threads do
  const int lane = tid % 32, warp = tid / 32;
  const int slice = warp % SLICES, group = warp / SLICES;
  float q_scale = 0.0f, k_scale = 0.0f;
  {
    float qq = 0.0f, kk = 0.0f;
    if (tid < RULE_THREADS) {
      const float qv = conv[tid], kv = conv[D + tid];
      qq = fmaf(qv, qv, qq);
      kk = fmaf(kv, kv, kk);
    }
#pragma unroll
    for (int off = 16; off > 0; off /= 2) {
      qq += __shfl_xor_sync(0xffffffffu, qq, off);
      kk += __shfl_xor_sync(0xffffffffu, kk, off);
    }
    __shared__ float qk_parts[2][RULE_WARPS];
    if (tid < RULE_THREADS && lane == 0) {
      qk_parts[0][warp] = qq;
      qk_parts[1][warp] = kk;
    }
    __syncthreads();
    const float q_total = ((qk_parts[0][0] + qk_parts[0][1]) + qk_parts[0][2]) + qk_parts[0][3];
    const float k_total = ((qk_parts[1][0] + qk_parts[1][1]) + qk_parts[1][2]) + qk_parts[1][3];
    q_scale = 1.0f / sqrtf(q_total + 1e-6f) * (1.0f / sqrtf(float(D)));
    k_scale = 1.0f / sqrtf(k_total + 1e-6f);
  }
  const int j = slice * RULE_COLUMNS + lane, i0 = group * ROWS;
  float* column = states + (((long long)seq * heads + h) * D + i0) * D + j;
  float sv[ROWS];
#pragma unroll
  for (int r = 0; r < ROWS; ++r) sv[r] = column[(long long)r * D];
  const float v = conv[2 * D + j];
  const float x = a[(long long)seq * heads + h] + dt_bias[h];
  const float g = expf(decay[h] * (x > 20.0f ? x : log1pf(expf(x))));
  const float beta = 1.0f / (1.0f + expf(-b[(long long)seq * heads + h]));
  const float* qs = conv;
  const float* ks = conv + D;
  float part = 0.0f;
#pragma unroll
  for (int r = 0; r < ROWS; ++r) {
    sv[r] *= g;
    part = fmaf(sv[r], ks[i0 + r] * k_scale, part);
  }
  sums[group][slice][lane] = part;
  __syncthreads();
  const float kv = ((sums[0][slice][lane] + sums[1][slice][lane]) + sums[2][slice][lane]) +
                   sums[3][slice][lane];
  const float delta = (v - kv) * beta;
  __syncthreads();  // sums is reused below
  float acc = 0.0f;
#pragma unroll
  for (int r = 0; r < ROWS; ++r) {
    sv[r] = fmaf(ks[i0 + r] * k_scale, delta, sv[r]);
    acc = fmaf(sv[r], qs[i0 + r] * q_scale, acc);
  }
  sums[group][slice][lane] = acc;
#pragma unroll
  for (int r = 0; r < ROWS; ++r) column[(long long)r * D] = sv[r];
  __syncthreads();
  if (group == 0)
    o[j] = ((sums[0][slice][lane] + sums[1][slice][lane]) + sums[2][slice][lane]) +
           sums[3][slice][lane];
  __syncthreads();
  // the gated RMS norm of the head's output, over the first 4 warps as
  // gated_rms_norm_kernel's 128 threads
  if (tid < RULE_THREADS) {
    const float value = o[tid];
    float squares = fmaf(value, value, 0.0f);
#pragma unroll
    for (int off = 16; off > 0; off /= 2) squares += __shfl_xor_sync(0xffffffffu, squares, off);
    if (lane == 0) partial[warp] = squares;
    asm volatile("bar.sync 1, %0;" ::"r"(RULE_THREADS));
    float total = 0.0f;
    for (int w = 0; w < RULE_WARPS; ++w) total += partial[w];
    const float scale = 1.0f / sqrtf(total / float(D) + epsilon);
    const long long at = ((long long)seq * heads + h) * D + tid;
    const float gv = z[at];
    const float act = gv / (1.0f + expf(-gv));
    const float normed = value * scale * norm_weight[tid] * act;
    out[at] = normed;
    if (records) x22_record_block(normed, records, seq, (h * D + tid) / 32, heads * D / 32);
  }
}

DRIFT_REGISTER(causal_conv_batched, causal_conv_kernel)
DRIFT_REGISTER(delta_decode_step_d128, delta_decode_step_kernel)
DRIFT_REGISTER(delta_rule_d128, gated_delta_rule_kernel<128>)
DRIFT_REGISTER(gated_rms_norm_records_f32, gated_rms_norm_kernel<1>)

}  // namespace
}  // namespace drift

using namespace drift;

extern "C" {

int drift_causal_conv(const float* x, int tokens, int channels, const float* weight, int taps,
                      int dilation, float* state, float* history, float* out,
                      drift_stream_t stream) {
  if (tokens < 0 || channels < 0) return invalid("causalConv over [%d, %d]", tokens, channels);
  if (taps < 1 || taps > 9 || dilation < 1 || (taps - 1) * dilation > MAX_SPAN)
    return invalid("causalConv: %d taps %d apart (at most 9 taps, a span of %d)", taps, dilation,
                   MAX_SPAN);
  if (tokens == 0 || channels == 0) return 0;
  if (!x || !weight || !out || ((taps > 1) && !state)) return invalid("causalConv: a null tensor");
  DRIFT_CUDA(launch_pdl(causal_conv_kernel, unsigned((channels + 255) / 256), 256, 0,
                        cudaStream_t(stream), x, tokens, channels, weight, taps, dilation, state,
                        history, out));
  DRIFT_LAUNCHED("causal_conv_silu");
  return 0;
}

int drift_gated_delta_rule(const float* qkv, int tokens, int key_heads, int value_heads, int dim,
                           int tiled, const float* a, const float* b, const float* decay,
                           const float* dt_bias, float* state, float* history, float* out,
                           drift_stream_t stream) {
  if (tokens < 0 || key_heads <= 0 || value_heads <= 0 || value_heads % key_heads != 0)
    return invalid("%d value heads over %d key heads", value_heads, key_heads);
  if (dim != 32 && dim != 64 && dim != 128)
    return invalid("gatedDeltaRule: heads of %d (kernels take 32, 64, 128)", dim);
  if (tokens == 0) return 0;
  if (!qkv || !a || !b || !decay || !dt_bias || !state || !out)
    return invalid("gatedDeltaRule: a null tensor");
  const unsigned grid = unsigned(value_heads * (dim / RULE_COLUMNS));
  const cudaStream_t s = cudaStream_t(stream);
  if (dim == 32)
    DRIFT_CUDA(launch_pdl(gated_delta_rule_kernel<32>, grid, RULE_THREADS, 0, s, qkv, tokens,
                          key_heads, value_heads, tiled, a, b, decay, dt_bias, state, history, out));
  else if (dim == 64)
    DRIFT_CUDA(launch_pdl(gated_delta_rule_kernel<64>, grid, RULE_THREADS, 0, s, qkv, tokens,
                          key_heads, value_heads, tiled, a, b, decay, dt_bias, state, history, out));
  else
    DRIFT_CUDA(launch_pdl(gated_delta_rule_kernel<128>, grid, RULE_THREADS, 0, s, qkv, tokens,
                          key_heads, value_heads, tiled, a, b, decay, dt_bias, state, history, out));
  DRIFT_LAUNCHED("delta_rule");
  return 0;
}

int drift_causal_conv_decode(const float* x, int sequences, int channels, const float* weight,
                             int taps, int dilation, float* states, float* out,
                             drift_stream_t stream) {
  if (sequences < 0 || channels < 0 || sequences > 65535)
    return invalid("causalConv over %d sequences of %d channels", sequences, channels);
  if (taps < 1 || taps > 9 || dilation < 1 || (taps - 1) * dilation > MAX_SPAN)
    return invalid("causalConv: %d taps %d apart (at most 9 taps, a span of %d)", taps, dilation,
                   MAX_SPAN);
  if (sequences == 0 || channels == 0) return 0;
  if (!x || !weight || !out || ((taps > 1) && !states)) return invalid("causalConv: a null tensor");
  DRIFT_CUDA(launch_pdl(causal_conv_kernel, dim3(unsigned((channels + 255) / 256), unsigned(sequences)),
                        256, 0, cudaStream_t(stream), x, 1, channels, weight, taps, dilation,
                        states, static_cast<float*>(nullptr), out));
  DRIFT_LAUNCHED("causal_conv_silu");
  return 0;
}

int drift_gated_delta_rule_decode(const float* qkv, int sequences, int key_heads, int value_heads,
                                  int dim, int tiled, const float* a, const float* b,
                                  const float* decay, const float* dt_bias, float* states,
                                  float* out, drift_stream_t stream) {
  if (sequences < 0 || sequences > 65535 || key_heads <= 0 || value_heads <= 0 ||
      value_heads % key_heads != 0)
    return invalid("%d value heads over %d key heads (%d sequences)", value_heads, key_heads,
                   sequences);
  if (dim != 32 && dim != 64 && dim != 128)
    return invalid("gatedDeltaRule: heads of %d (kernels take 32, 64, 128)", dim);
  if (sequences == 0) return 0;
  if (!qkv || !a || !b || !decay || !dt_bias || !states || !out)
    return invalid("gatedDeltaRule: a null tensor");
  const dim3 grid(unsigned(value_heads * (dim / RULE_COLUMNS)), unsigned(sequences));
  const cudaStream_t s = cudaStream_t(stream);
  float* none = nullptr;
  if (dim == 32)
    DRIFT_CUDA(launch_pdl(gated_delta_rule_kernel<32>, grid, RULE_THREADS, 0, s, qkv, 1,
                          key_heads, value_heads, tiled, a, b, decay, dt_bias, states, none, out));
  else if (dim == 64)
    DRIFT_CUDA(launch_pdl(gated_delta_rule_kernel<64>, grid, RULE_THREADS, 0, s, qkv, 1,
                          key_heads, value_heads, tiled, a, b, decay, dt_bias, states, none, out));
  else
    DRIFT_CUDA(launch_pdl(gated_delta_rule_kernel<128>, grid, RULE_THREADS, 0, s, qkv, 1,
                          key_heads, value_heads, tiled, a, b, decay, dt_bias, states, none, out));
  DRIFT_LAUNCHED("delta_rule");
  return 0;
}

int drift_delta_decode_step(const float* qkv, const float* z, int sequences, int key_heads,
                            int value_heads, int dim, int tiled, const float* conv_weight,
                            int taps, float* conv_states, float* convolved, const float* a,
                            const float* b, const float* decay, const float* dt_bias,
                            float* states, const float* norm_weight, float epsilon, float* out,
                            void* prepared, drift_stream_t stream) {
  if (sequences < 0 || sequences > 65535 || key_heads <= 0 || value_heads <= 0 ||
      value_heads % key_heads != 0)
    return invalid("%d value heads over %d key heads (%d sequences)", value_heads, key_heads,
                   sequences);
  if (dim != 32 && dim != 64 && dim != 128)
    return invalid("gatedDeltaRule: heads of %d (kernels take 32, 64, 128)", dim);
  if (taps < 1 || taps > 9 || taps - 1 > MAX_SPAN)
    return invalid("causalConv: %d taps (at most 9)", taps);
  if (sequences == 0) return 0;
  if (!qkv || !z || !conv_weight || (taps > 1 && !conv_states) || !a || !b || !decay ||
      !dt_bias || !states || !norm_weight || !out)
    return invalid("deltaDecodeStep: a null tensor");
  if (prepared && dim % 32 != 0)
    return invalid("gatedRmsNorm: prepared x needs rows of whole heads of 32-value blocks");
  const int channels = (2 * key_heads + value_heads) * dim;
  if (key_heads != value_heads || dim != STEP_D || taps < 2) {
    // the three launches it stands for (the same bits): `convolved` holds
    // the convolution's output between them
    if (!convolved) return invalid("deltaDecodeStep: no room for the convolved channels");
    DRIFT_TRY(drift_causal_conv_decode(qkv, sequences, channels, conv_weight, taps, 1, conv_states,
                                       convolved, stream));
    DRIFT_TRY(drift_gated_delta_rule_decode(convolved, sequences, key_heads, value_heads, dim,
                                            tiled, a, b, decay, dt_bias, states, out, stream));
    return drift_gated_rms_norm(out, norm_weight, z, DRIFT_SILU, epsilon, out,
                                (int64_t)sequences * value_heads, dim, value_heads, prepared,
                                stream);
  }
  DRIFT_CUDA(launch_pdl(delta_decode_step_kernel, dim3(unsigned(value_heads), unsigned(sequences)),
                        STEP_THREADS, 0, cudaStream_t(stream), qkv, z, value_heads, conv_weight,
                        taps, conv_states, a, b, decay, dt_bias, states, norm_weight, epsilon, out,
                        static_cast<uint8_t*>(prepared)));
  DRIFT_LAUNCHED("delta_decode_step");
  return 0;
}

int drift_gated_rms_norm(const float* x, const float* weight, const float* gate, int kind,
                         float epsilon, float* out, int64_t rows, int64_t cols, int heads,
                         void* prepared, drift_stream_t stream) {
  if (kind != DRIFT_SILU && kind != DRIFT_SIGMOID)
    return invalid("gatedRmsNorm gates by SiLU or sigmoid, not activation %d", kind);
  if (rows < 0 || cols <= 0 || cols > 512) return invalid("gatedRmsNorm over rows of %lld (at most 512)", (long long)cols);
  if (rows == 0) return 0;
  if (!x || !weight || !gate || !out) return invalid("gatedRmsNorm: a null tensor");
  if (prepared && (heads <= 0 || rows % heads != 0 || (heads * cols) % 32 != 0 || cols % 32 != 0))
    return invalid("gatedRmsNorm: prepared x needs rows of whole heads of 32-value blocks");
  uint8_t* records = static_cast<uint8_t*>(prepared);
  const int h = heads > 0 ? heads : 1;
  const cudaStream_t s = cudaStream_t(stream);
  const unsigned grid = unsigned(rows);
  if (cols <= 128)
    DRIFT_CUDA(launch_pdl(gated_rms_norm_kernel<1>, grid, 128, 0, s, x, weight, gate,
                          int(kind == DRIFT_SIGMOID), epsilon, out, int(cols), h, records));
  else if (cols <= 256)
    DRIFT_CUDA(launch_pdl(gated_rms_norm_kernel<2>, grid, 128, 0, s, x, weight, gate,
                          int(kind == DRIFT_SIGMOID), epsilon, out, int(cols), h, records));
  else
    DRIFT_CUDA(launch_pdl(gated_rms_norm_kernel<4>, grid, 128, 0, s, x, weight, gate,
                          int(kind == DRIFT_SIGMOID), epsilon, out, int(cols), h, records));
  DRIFT_LAUNCHED("gated_rms_norm_f32");
  return 0;
}

}  // extern "C"
