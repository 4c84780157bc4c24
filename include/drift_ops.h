/*
 * drift_ops.h -- the operator half of libdrift_cuda's C ABI.
 *
 * One entry point per operation of the drift runner's `Ops` API on the
 * quantized-inference hot path. Each does what the runner's HIP backend does
 * for that operation -- check the shapes as `Ops.check*` does, choose a kernel
 * variant by dtype and shape, compute the launch geometry, launch on `stream`
 * -- so a host that calls these needs none of HipLinear/HipNormalisation/
 * HipExperts' dispatch. Every function is asynchronous on `stream`, returns an
 * int status (see drift_runtime.h), and refuses shapes the reference refuses
 * with DRIFT_ERROR_INVALID_ARGUMENT and the reference's message.
 *
 * Conventions, as the reference's (runner/src/drift/runner/ops/Ops.scala:7-13):
 * activations are F32 (this ABI also takes BF16 x for the products, widened
 * exactly); weights are raw GGML blocks, rows of [N, K] row-major with the
 * blocks along K (tensor/Tensor.scala:75-87); `out` is written, never read,
 * and may alias an input for elementwise operations. Pointers are device
 * addresses of the current device.
 *
 * One stream of operations per device at a time: the products' x records
 * (the grow-only workspace), their group sums and arrival counts, and the
 * attention join's arrival counts live in per-device buffers that every call
 * shares, so operations whose kernels overlap on the GPU (calls on different
 * streams, or from different host threads, not ordered by events) race.
 * Calls in one stream, or ordered between streams by events, do not; copies
 * may run on other streams meanwhile (drift_stream_wait_event).
 */
#ifndef DRIFT_OPS_H
#define DRIFT_OPS_H

#include <stddef.h>
#include <stdint.h>

#include "drift_runtime.h"

#ifdef __cplusplus
extern "C" {
#endif

/* Storage types: GGML type ids, as DType.ggmlId gives them
 * (runner/src/drift/runner/tensor/DType.scala:86-175; GgmlQuants.scala). */
#define DRIFT_F32 0
#define DRIFT_F16 1
#define DRIFT_Q4_0 2
#define DRIFT_Q4_1 3
#define DRIFT_Q8_0 8
#define DRIFT_Q4_K 12 /* super-blocks of 256 (tensor/KQuants.scala:99) */
#define DRIFT_Q6_K 14 /* (KQuants.scala:122) */
#define DRIFT_I32 26
#define DRIFT_BF16 30

/* Activation codes (runner/src/drift/runner/ops/Activation.scala:5-19). */
#define DRIFT_SILU 0
#define DRIFT_GELU_TANH 1
#define DRIFT_GELU_ERF 2
#define DRIFT_SIGMOID 3
#define DRIFT_SITU 4

/* RoPE layouts (runner/src/drift/runner/ops/Rope.scala:7-10). */
#define DRIFT_ROPE_NEOX 0
#define DRIFT_ROPE_INTERLEAVED 1

/* Ops.linear (ops/LinearOps.scala:147-150; HIP dispatch ops/HipLinear.scala:
 * 94-276): out[m, n] = x[m, k] . weight[n, k]^T. x is F32 or BF16 [m, k],
 * weight Q8_0/Q4_0/Q4_1 (or F32) [n, k], out F32 [m, n]. Up to 8 rows of x
 * are one pass over the weight; 8 < m < 32 runs passes of 8; m >= 32 is the
 * tensor-core product. Rows must be whole 4-byte words ("rows are not whole
 * words", HipLinear.scala:126-131). */
int drift_linear(int x_dtype, const void* x, int weight_dtype, const void* weight, float* out,
                 int64_t m, int64_t n, int64_t k, drift_stream_t stream);

/* Ops.linears (LinearOps.scala:152-156; HipLinear.scala:104-156): several
 * products of the same x (Q, K and V; gate and up), x prepared once. */
int drift_linears(int x_dtype, const void* x, int count, const int* weight_dtypes,
                  const void* const* weights, float* const* outs, const int64_t* ns, int64_t m,
                  int64_t k, drift_stream_t stream);

/* Ops.embedding (LinearOps.scala:83-87; HipLinear.scala:21-52): out[t] =
 * decode(table[ids[t]]) as F32, bit for bit the CPU decode. An id outside
 * [0, vocab) -- which the reference's CPU backend refuses with "token id ...
 * outside the table" (ops/CpuLinear.scala:19-23) -- leaves that row NaN and
 * sets the device error word (drift_device_error_take). */
int drift_embedding(int table_dtype, const void* table, int64_t vocab, int64_t cols,
                    const int32_t* ids, int64_t count, float* out, drift_stream_t stream);

/* Ops.rmsNorm (ops/NormalisationOps.scala:30-36; HipNormalisation.scala:57-115):
 * out = x / sqrt(mean(x^2) + eps) * (weight + offset), per row of `cols`. */
int drift_rms_norm(const float* x, const float* weight, float epsilon, float weight_offset,
                   float* out, int64_t rows, int64_t cols, drift_stream_t stream);

/* Ops.addRmsNorm (NormalisationOps.scala:42-45; HipNormalisation.scala:117-131):
 * x += y (written back), then out = rmsNorm(x). One launch. */
int drift_add_rms_norm(float* x, const float* y, const float* weight, float epsilon,
                       float weight_offset, float* out, int64_t rows, int64_t cols,
                       drift_stream_t stream);

/* ElementwiseOps.add (ops/CpuElementwise.scala:9-13; kernels add_f32). */
int drift_add(const float* a, const float* b, float* out, int64_t n, drift_stream_t stream);

/* Ops.gated (NormalisationOps.scala:24; HipNormalisation.scala:32-47):
 * out = act(gate) * up; DRIFT_SILU is SwiGLU. */
int drift_gated(int kind, const float* gate, const float* up, float* out, int64_t n,
                drift_stream_t stream);

/* Ops.rope with RopeSections.Single (ops/AttentionOps.scala:42-45;
 * HipAttention.scala:81-104): x [tokens, heads, head_dim] F32, positions I32
 * [tokens]; the first `rotary` values of each head turn in pairs. */
int drift_rope(const float* x, const int32_t* positions, float* out, int tokens, int heads,
               int head_dim, float theta, int rotary, int layout, drift_stream_t stream);

/* Ops.route (ops/ExpertsOps.scala:116-120; HipExperts.scala:19-32): each
 * token's k largest logits (the lower expert first among equals) into ids
 * [tokens, k], their softmax among themselves into weights. k <= 16,
 * experts <= 512 (ExpertsOps.scala:264-267). */
int drift_route(const float* logits, int32_t* ids, float* weights, int tokens, int experts, int k,
                drift_stream_t stream);

/* SequenceOps.argmax (ops/SequenceOps.scala:14; CpuSequence.scala:12-22;
 * HipSequence.scala:15-27, kernels/norm.hip:119-153), per row: ids[r] = the
 * first index of row r's largest value, compared with `>` from index 0 (a NaN
 * never wins except at index 0), plus id_offset (a vocabulary shard's first
 * id: the rule about index 0 is about id 0); out_values[r] (may be NULL) the
 * value. rows <= 4096. */
int drift_argmax(const float* values, int64_t rows, int64_t width, int64_t id_offset, int32_t* ids,
                 float* out_values, drift_stream_t stream);
/* The merge of gathered argmaxes (new: tensor parallelism splits the
 * vocabulary): rows of n (value, id) pairs -> the pair argmax would pick over
 * the whole row, the same on every rank. */
int drift_argmax_merge(const float* values, const int32_t* ids_in, int64_t rows, int64_t n,
                       int32_t* ids, float* out_values, drift_stream_t stream);
/* SequenceOps.candidates (SequenceOps.scala:20; Candidates.of,
 * ops/Candidates.scala:30-35; HipSequence.scala:43-100, norm.hip:322-363):
 * each row's `count` (1 to 1024) largest values, largest first, the lower
 * index first among equals (-0 as 0, a positive NaN above +inf): ids (plus
 * id_offset) and values, [rows][count] (only the first min(count, width) of a
 * row are written). rows <= 4096. Uses the library's scratch
 * (drift_candidates_workspace_bytes). */
int drift_candidates(const float* values, int64_t rows, int64_t width, int64_t id_offset, int count,
                     int32_t* ids, float* out_values, drift_stream_t stream);
size_t drift_candidates_workspace_bytes(int64_t rows, int64_t width, int count);
/* The merge of gathered candidates: rows of n (value, id) pairs with unique
 * ids -> the row's `count` largest by the same order, ids compared as ids. */
int drift_candidates_merge(const float* values, const int32_t* ids_in, int64_t rows, int64_t n,
                           int count, int32_t* ids, float* out_values, drift_stream_t stream);

/* Ops.expertsLinear (ExpertsOps.scala:122-126; HipExperts.scala:76-168): slot
 * s multiplies expert ids[s] of weight [experts, n, k] with x row
 * s / (slots / x_rows), into out [slots, n]. An id outside [0, experts)
 * leaves its slot NaN and sets the device error word. */
int drift_experts_linear(int x_dtype, const void* x, int64_t x_rows, int weight_dtype,
                         const void* weight, int64_t experts, int64_t n, int64_t k,
                         const int32_t* ids, int64_t slots, float* out, drift_stream_t stream);

/* Ops.expertsGatedLinear (ExpertsOps.scala:188-198; HipExperts.scala:478-546):
 * out = silu(gate . x) * (up . x) per slot, one launch. */
int drift_experts_gated_linear(int x_dtype, const void* x, int64_t x_rows, int weight_dtype,
                               const void* gate, const void* up, int64_t experts, int64_t n,
                               int64_t k, const int32_t* ids, int64_t slots, float* out,
                               drift_stream_t stream);

/* Ops.moeCombine (ExpertsOps.scala:128-138; kernels/linear_attention.hip:
 * 286-297, combine.h:10-32): out[t] = residual[t] + sum_j weights[t, j] *
 * expert_out[t*k + j] + sigmoid(shared_input[t] . shared_router) *
 * shared_out[t]. shared_* and residual may be NULL; out may be residual. */
int drift_moe_combine(const float* expert_out, const float* weights, int64_t tokens, int64_t k,
                      int64_t hidden, const float* shared_out, const float* shared_input,
                      const float* shared_router, const float* residual, float* out,
                      drift_stream_t stream);

/* Ops.moeCombineNorm (ExpertsOps.scala:140-152; kernels/norm.hip:43-59):
 * moeCombine into residual, then its RMS norm into normed, one launch. */
int drift_moe_combine_norm(const float* expert_out, const float* weights, int64_t tokens,
                           int64_t k, int64_t hidden, const float* shared_out,
                           const float* shared_input, const float* shared_router, float* residual,
                           const float* norm_weight, float epsilon, float weight_offset,
                           float* normed, drift_stream_t stream);

/* Ops.cacheWrite (ops/AttentionOps.scala:58-64; CPU ops/CpuAttention.scala:
 * 181-210): k, v [tokens, kv_heads, head_dim] F32, rounded to F16 (nearest
 * even), into the paged cache at positions start.. . The cache is the
 * reference's KvCache (ops/KvCache.scala:12-23): keys [pages][page_size]
 * [kv_heads][head_dim] and values [pages][kv_heads][head_dim][page_size], F16,
 * page_size a multiple of 16; page_table I32 [table_pages] maps position /
 * page_size to a page. Cache pointers 16-byte aligned. */
int drift_cache_write(const float* k, const float* v, int tokens, int kv_heads, int head_dim,
                      void* keys, void* values, int pages, int page_size,
                      const int32_t* page_table, int table_pages, int start,
                      drift_stream_t stream);

/* Ops.attention (ops/AttentionOps.scala:113-121; CPU ops/CpuAttention.scala:
 * 215-288): for each token t and query head h, softmax over the visible keys
 * (key < key_count; key <= query_start + t when causal; key > query_start +
 * t - window when window > 0) of scale * q . k (softcapped as softcap *
 * tanh(score / softcap) when softcap > 0; sinks F32 [q_heads] or NULL join the
 * softmax's denominator), times the values. q and out F32 [tokens, q_heads,
 * head_dim]; head_dim 64, 80, 128 or 256; q_heads a multiple of kv_heads, at
 * most 16 query heads per key head. */
int drift_attention(const float* q, int tokens, int q_heads, const void* keys, const void* values,
                    int pages, int page_size, int kv_heads, int head_dim,
                    const int32_t* page_table, int table_pages, int query_start, int key_count,
                    float scale, int causal, int window, float softcap, const float* sinks,
                    float* out, drift_stream_t stream);

/* A decode step's attention inputs in one launch, for `batch` sequences of
 * one new token each (the dense decoder's per-head rmsNorm of q and k, rope of
 * both and cacheWrite, models/DenseDecoder.scala:830-860, fused; no single
 * counterpart in the reference's Ops API). q [batch, q_heads, head_dim], k, v
 * [batch, kv_heads, head_dim] F32; q_norm / k_norm [head_dim] or NULL (no
 * norm); positions I32 [batch] (device) give each token's rope position and
 * cache slot; page_tables I32 [batch, table_stride] (device), row z mapping
 * sequence z's positions to pages. The turned queries go to q_out; keys and
 * values to the cache. Results are bit for bit those of drift_rms_norm,
 * drift_rope and drift_cache_write called in turn. A position outside its
 * page table sets the device error word (code 1). */
int drift_attention_inputs_decode(const float* q, const float* k, const float* v, int batch,
                                  int q_heads, int kv_heads, int head_dim, const float* q_norm,
                                  const float* k_norm, float epsilon, float weight_offset,
                                  const int32_t* positions, float theta, int rotary, int layout,
                                  float* q_out, void* keys, void* values, int pages,
                                  int page_size, const int32_t* page_tables, int table_stride,
                                  drift_stream_t stream);

/* drift_attention for a decode step of `batch` sequences in one launch: row z
 * of q [batch, q_heads, head_dim] is sequence z's token at positions[z]
 * (device), attending causally to its keys 0..positions[z] through page table
 * row z; max_key_count bounds every positions[z] + 1 (a row past it, or past
 * its table, gets zeros). Each row's result is bit for bit drift_attention's
 * for that sequence alone. */
int drift_attention_decode(const float* q, int batch, int q_heads, const void* keys,
                           const void* values, int pages, int page_size, int kv_heads,
                           int head_dim, const int32_t* page_tables, int table_stride,
                           const int32_t* positions, int max_key_count, float scale, int window,
                           float softcap, const float* sinks, float* out, drift_stream_t stream);

/* ---- Gated DeltaNet (the hybrid decoder's linear-attention layers) ---------
 * SequenceOps.causalConv (ops/SequenceOps.scala; CPU ops/CpuSequence.scala:
 * 29-80): x [tokens][channels], weight [channels][taps] (taps <= 9), state
 * [(taps - 1) dilation][channels] (span <= 16, updated), out = SiLU(sum of the
 * taps); history [tokens][span][channels] or NULL. */
int drift_causal_conv(const float* x, int tokens, int channels, const float* weight, int taps,
                      int dilation, float* state, float* history, float* out,
                      drift_stream_t stream);
/* SequenceOps.gatedDeltaRule (CpuSequence.scala:82-158): qkv [tokens][(2
 * key_heads + value_heads) dim], a, b [tokens][value_heads], decay, dt_bias
 * [value_heads], state [value_heads][dim][dim] (updated), out [tokens]
 * [value_heads][dim]; history [tokens][value_heads][dim][dim] or NULL; value
 * head h reads key head h % key_heads when `tiled`, h / (value_heads /
 * key_heads) otherwise (ops/DeltaRule.scala:18-20). dim 32, 64 or 128. */
int drift_gated_delta_rule(const float* qkv, int tokens, int key_heads, int value_heads, int dim,
                           int tiled, const float* a, const float* b, const float* decay,
                           const float* dt_bias, float* state, float* history, float* out,
                           drift_stream_t stream);
/* The decode step of a batch of sequences (new): one token per sequence, each
 * with its own state -- x / qkv rows are the sequences, states [sequences]
 * [span][channels] and [sequences][value_heads][dim][dim]. */
int drift_causal_conv_decode(const float* x, int sequences, int channels, const float* weight,
                             int taps, int dilation, float* states, float* out,
                             drift_stream_t stream);
int drift_gated_delta_rule_decode(const float* qkv, int sequences, int key_heads, int value_heads,
                                  int dim, int tiled, const float* a, const float* b,
                                  const float* decay, const float* dt_bias, float* states,
                                  float* out, drift_stream_t stream);
/* A DeltaNet layer's decode step after its input products (new; the
 * hybrid decoder's causalConv, gatedDeltaRule and gatedRmsNorm of one token
 * per sequence, models/HybridBlocks.scala): qkv [sequences][(2 key_heads +
 * value_heads) dim] through the causal convolution (dilation 1, states
 * [sequences][taps - 1][channels]), the gated delta rule on states
 * [sequences][value_heads][dim][dim], and rmsNorm(core) * norm_weight *
 * SiLU(z) into out [sequences][value_heads][dim] (z the same shape), with the
 * out projection's records into `prepared` (NULL for none). One launch when
 * key_heads == value_heads, dim 128 and taps >= 2; otherwise the three calls
 * it stands for, with `convolved` [sequences][channels] between them. The
 * same bits either way. */
int drift_delta_decode_step(const float* qkv, const float* z, int sequences, int key_heads,
                            int value_heads, int dim, int tiled, const float* conv_weight,
                            int taps, float* conv_states, float* convolved, const float* a,
                            const float* b, const float* decay, const float* dt_bias,
                            float* states, const float* norm_weight, float epsilon, float* out,
                            void* prepared, drift_stream_t stream);
/* NormalisationOps.gatedRmsNorm (CpuNormalisation.scala:167-178): per row of
 * cols (<= 512) values, rmsNorm(x) * weight * act(gate), act DRIFT_SILU or
 * DRIFT_SIGMOID; out may be x. With `prepared` (rows = tokens x heads), the
 * records of out viewed as [tokens][heads * cols] for the out projection. */
int drift_gated_rms_norm(const float* x, const float* weight, const float* gate, int kind,
                         float epsilon, float* out, int64_t rows, int64_t cols, int heads,
                         void* prepared, drift_stream_t stream);

/* Expert parallelism (new): a rank's weight holds experts [first_expert,
 * first_expert + experts) of the model's; `ids` are the model's; a slot whose
 * expert is another rank's gets a row of zeros (drift_experts_linear and
 * drift_experts_gated_linear flag such a slot as an error instead). Id -1
 * names a mixture's shared expert: the rank that holds it puts it first and
 * passes first_expert -1 (its routed experts then start at 0), so the shared
 * expert's slots ride in the routed experts' launches on that rank and are
 * zeros on the others. */
int drift_experts_linear_local(int x_dtype, const void* x, int64_t x_rows, int weight_dtype,
                               const void* weight, int64_t experts, int64_t first_expert,
                               int64_t n, int64_t k, const int32_t* ids, int64_t slots,
                               float* out, const void* prepared, drift_stream_t stream);
/* With shared_tail, the last x_rows slots are a shared expert's, one per x
 * row in order (its weights one more expert of gate and up), the slots
 * before them routed (slots - x_rows) / x_rows to a row: the routed and the
 * shared experts' products in one launch. */
int drift_experts_gated_linear_local(int x_dtype, const void* x, int64_t x_rows, int weight_dtype,
                                     const void* gate, const void* up, int64_t experts,
                                     int64_t first_expert, int64_t n, int64_t k,
                                     const int32_t* ids, int64_t slots, float* out,
                                     const void* prepared, int shared_tail,
                                     drift_stream_t stream);

/* ---- prepared x (new) ------------------------------------------------------
 * A product streams its weights against x's "records" (x per 32-value block as
 * exact 24-bit integer planes and a scale). drift_linear writes them itself; a
 * decode step can have the kernel that produces x write them instead, as the
 * reference's own norm and gated kernels write the quantized x of the product
 * that follows them (rms_norm_f32 / gated_f32 xq, xd, xs outputs,
 * runner/kernels/norm.hip:34-35, elementwise.hip:58-59). The caller owns the
 * buffer: drift_prepared_x_bytes(m, k) bytes for m rows of k values (k a
 * multiple of 32). Results are bit for bit those of the unprepared calls. */
size_t drift_prepared_x_bytes(int64_t m, int64_t k);
/* drift_add_rms_norm (y null: drift_rms_norm), also writing out's records. */
int drift_add_rms_norm_prepared(float* x, const float* y, const float* weight, float epsilon,
                                float weight_offset, float* out, int64_t rows, int64_t cols,
                                void* prepared, drift_stream_t stream);
/* A mixture's whole decode step in one launch (new; the reference's
 * route + expertsGatedLinear + expertsLinear + moeCombineNorm of
 * models/HybridBlocks.scala, its GPU `moe_group*` kernels,
 * runner/kernels/matvec.hip:1816-1933): logits = x . router^T (F32 router
 * [experts][hidden]), the top-k into ids [tokens][k] and route_weights, the
 * routed and shared experts' SwiGLU (gate, up: [experts + 1][ffn][hidden],
 * the shared expert last; x's records in x_prepared) into gated [tokens k +
 * tokens][ffn], their down products (down [experts + 1][hidden][ffn]) into out
 * [tokens k + tokens][hidden], and the combine with the shared expert's
 * sigmoid(x . shared_router) gate into residual [tokens][hidden], then
 * rmsNorm(residual) into normed and its records into prepared (either may be
 * x / x_prepared: they are written last). ids gets tokens k + tokens entries,
 * the shared slots `experts`. The bits of the five separate calls. A
 * cooperative launch of as many CTAs as the device holds at once, its
 * phases separated by grid barriers (each wait bounded: device error 2).
 * hidden <= 2048, whole 32-value blocks; ffn <= 4096; k <= 16; experts <= 512. */
int drift_moe_decode(int weight_dtype, const float* x, const void* x_prepared, const float* router,
                     float* logits, int32_t* ids, float* route_weights, const void* gate,
                     const void* up, const void* down, float* gated, float* out,
                     const float* shared_router, float* residual, const float* norm_weight,
                     float epsilon, float weight_offset, float* normed, void* prepared,
                     int64_t tokens, int64_t experts, int64_t k, int64_t hidden, int64_t ffn,
                     drift_stream_t stream);
/* drift_moe_combine_norm (hidden a multiple of 32), also writing normed's
 * records: the next layer's input, as the reference's moe_combine_norm feeds
 * the next layer's products (norm.hip:43-59). */
int drift_moe_combine_norm_prepared(const float* expert_out, const float* weights, int64_t tokens,
                                    int64_t k, int64_t hidden, const float* shared_out,
                                    const float* shared_input, const float* shared_router,
                                    float* residual, const float* norm_weight, float epsilon,
                                    float weight_offset, float* normed, void* prepared,
                                    drift_stream_t stream);
/* drift_gated over rows x cols values, also writing out's records. */
int drift_gated_prepared(int kind, const float* gate, const float* up, float* out, int64_t rows,
                         int64_t cols, void* prepared, drift_stream_t stream);
/* drift_attention_decode (head_dim a multiple of 32), also writing the
 * records of out viewed as [batch][q_heads * head_dim]. */
int drift_attention_decode_prepared(const float* q, int batch, int q_heads, const void* keys,
                                    const void* values, int pages, int page_size, int kv_heads,
                                    int head_dim, const int32_t* page_tables, int table_stride,
                                    const int32_t* positions, int max_key_count, float scale,
                                    int window, float softcap, const float* sinks, float* out,
                                    void* prepared, drift_stream_t stream);
/* drift_linears over prepared records of F32 x (x itself is still read by
 * the products of 32 rows or more, which take the tensor cores). */
int drift_linears_prepared(int x_dtype, const void* x, const void* prepared, int count,
                           const int* weight_dtypes, const void* const* weights,
                           float* const* outs, const int64_t* ns, int64_t m, int64_t k,
                           drift_stream_t stream);

/* ---- the tensor-parallel exchange over NVLink (new) --------------------------
 * The reference runs one device (native/HipRuntime.scala:40-43); a B200 box
 * runs the decode step tensor-parallel, one process per GPU. Each rank creates
 * a buffer of two slots of `slot_bytes` (CUDA IPC, peer-readable) and a handle
 * of drift_comm_handle_bytes() bytes, gathers every rank's handle (rank
 * order) and opens them. A row-split product writes its partial rows into a
 * slot (drift_comm_slot); drift_add_rms_norm_allreduce then, on every rank,
 * waits for every rank's partials of that slot, adds their sum in rank order
 * to x and writes rmsNorm(x) (and, with `prepared`, its records): the
 * runner's all-reduce and addRmsNorm in one launch. Consecutive exchanges
 * must alternate slots; at most 64 rows of 4096 values.
 * Each row's wait is bounded by `wait_limit_ns` (0: one second; at most 60
 * s). When it runs out -- a rank that skipped or never reached the exchange
 * -- the kernel sets device error code 3, leaves that row's x and out as
 * they were and returns; the ranks' exchange counts then disagree, so every
 * rank synchronizes and destroys the comm (after a host barrier: a peer may
 * still be pushing into this rank's buffer until its own call returns). */
size_t drift_comm_handle_bytes(void);
int drift_comm_create(int rank, int world, size_t slot_bytes, int64_t wait_limit_ns, void** comm,
                      void* handle);
int drift_comm_open(void* comm, const void* handles);
int drift_comm_slot(void* comm, int slot, void** pointer);
int drift_comm_destroy(void* comm);
int drift_add_rms_norm_allreduce(void* comm, int slot, float* x, const float* weight,
                                 float epsilon, float weight_offset, float* out, int64_t rows,
                                 int64_t cols, void* prepared, drift_stream_t stream);

/* The gated attention of the hybrid decoder (models/HybridBlocks.scala:
 * fullAttention): drift_attention_inputs_decode over queryAndGate [batch]
 * [q_heads][2 head_dim], whose first half per head is the query
 * (AttentionOps.attentionInputs' splitHalves, ops/AttentionOps.scala:73-107);
 * and drift_attention_decode whose output is multiplied by sigmoid(gate)
 * (gate + (z q_heads + h) gate_stride + d: the second half of queryAndGate
 * with gate_stride 2 head_dim), as gated(Sigmoid, gate, attended) does, in
 * the join; `prepared` may be NULL. */
int drift_attention_inputs_decode_split(const float* query_and_gate, const float* k,
                                        const float* v, int batch, int q_heads, int kv_heads,
                                        int head_dim, const float* q_norm, const float* k_norm,
                                        float epsilon, float weight_offset,
                                        const int32_t* positions, float theta, int rotary,
                                        int layout, float* q_out, void* keys, void* values,
                                        int pages, int page_size, const int32_t* page_tables,
                                        int table_stride, drift_stream_t stream);
int drift_attention_decode_gated(const float* q, int batch, int q_heads, const void* keys,
                                 const void* values, int pages, int page_size, int kv_heads,
                                 int head_dim, const int32_t* page_tables, int table_stride,
                                 const int32_t* positions, int max_key_count, float scale,
                                 int window, float softcap, const float* sinks, float* out,
                                 const float* gate, int gate_stride, void* prepared,
                                 drift_stream_t stream);

/* The library keeps one grow-only scratch buffer per device for the products'
 * prepared x (as the runner's HIP backend keeps grow-only scratch,
 * ops/HipBase.scala:341-351). Reserving it ahead keeps allocation out of a
 * CUDA graph capture. */
int drift_workspace_reserve(size_t bytes);
/* Bytes of scratch drift_linear needs for m rows of k (new). */
size_t drift_linear_workspace_bytes(int64_t m, int64_t k);
/* Bytes of scratch drift_attention / drift_attention_decode need for `rows`
 * query rows (tokens, or sequences) of q_heads heads over key_count keys
 * (new: the split-K partial sums). */
size_t drift_attention_workspace_bytes(int rows, int q_heads, int head_dim, int key_count);

/* drift_linear, for 1 to 31 rows of x, allocating no device memory. No
 * counterpart in the reference: it exists for hosts that cannot allocate on
 * the call path -- a server whose device memory is all reserved up front, so
 * an allocation mid-step could fail; an FFM host that owns every device
 * buffer through its own allocator and budget; a latency-bound loop that must
 * not let cudaMalloc or cudaFree synchronize the device.
 * Its scratch (the prepared x) is a fixed 1 MiB array in the library's device
 * image: (ceil(m / 8)) * (k / 32) * 896 bytes must fit, i.e. 8 rows of up to
 * 37,440 columns or 31 rows of up to 9,344; larger sizes, and m >= 32, are
 * refused with DRIFT_ERROR_INVALID_ARGUMENT. The first call on a device looks
 * up the array's device address (cudaGetSymbolAddress): make it before any
 * stream capture. Every call shares the array, so calls whose kernels overlap
 * on the GPU (other streams, other threads) race; calls in one stream do not.
 * Each call writes all the scratch it reads, so no state carries over. */
int drift_linear_static(int x_dtype, const void* x, int weight_dtype, const void* weight,
                        float* out, int64_t m, int64_t n, int64_t k, drift_stream_t stream);

/* Reads and clears the current device's error word: 0 if no kernel flagged
 * anything since the last call, else the first flag:
 *   1 = an id outside its table (the row is written as NaN);
 *   2 = a bounded wait inside a kernel gave up (its outputs are incomplete);
 *   3 = the tensor-parallel exchange's wait for a peer rank gave up (the
 *       rows it was exchanging are left as they were: x and out unchanged).
 * Synchronises the device. */
int drift_device_error_take(int* code);

#ifdef __cplusplus
}
#endif

#endif /* DRIFT_OPS_H */
