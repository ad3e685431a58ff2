/*
 * nsrl_b200.h -- C ABI of the B200-native (sm_100a) NSRL integer hot path.
 *
 * This is the drop-in boundary for the reference's nsrl-core kernel API
 * (crates/nsrl-core/src/lib.rs:29-90): the same operations, batched over
 * rows / sequences, on DEVICE buffers, with the reference's arithmetic
 * bit for bit.  Plain pointers and sizes only; `stream` is a cudaStream_t
 * (NULL = the legacy default stream).
 *
 * Conventions shared by every entry point:
 *  - Tensors are row-major and token-major: activations [rows][dim] int16
 *    (Q15), weights [output_dim][input_dim] int8, as in linear.rs:268-271.
 *  - The reference returns `Option::None` both for a bad shape and for an
 *    arithmetic rejection (an i32 prefix overflow in a linear, a logit outside
 *    i32, an all-masked softmax row, an integer rsqrt of 0).  Here shape
 *    errors are detected on the host before any launch and returned as
 *    NSRL_INVALID_SHAPE; arithmetic rejections are detected on the device
 *    and recorded in a caller-owned nsrl_device_status, which
 *    nsrl_status_fetch() turns into NSRL_CORE_REJECTED for the whole call.
 *    Outputs of a rejected call are unspecified, as with `None`.
 *  - Calls are asynchronous on `stream` and allocate nothing: scratch memory
 *    is a caller-owned workspace whose size the matching *_workspace_size()
 *    function returns (the reference's caller-owned *Workspace structs,
 *    e.g. attention.rs:29-36).  Calls are re-entrant per stream.
 */
#ifndef NSRL_B200_H
#define NSRL_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef enum nsrl_status {
  NSRL_OK = 0,
  NSRL_INVALID_SHAPE = 1,  /* validation `None` (shape / parameter rules) */
  NSRL_CORE_REJECTED = 2,  /* arithmetic `None` detected on the device */
  NSRL_CUDA_ERROR = 3,     /* a CUDA runtime/driver call failed */
  NSRL_COMM_TIMEOUT = 4,   /* a collective did not finish before the communicator's deadline */
  NSRL_COMM_ERROR = 5,     /* the communicator reported an error (a peer failed) or was aborted */
} nsrl_status;

/* FixedScale{multiplier, right_shift} (crates/nsrl-core/src/numeric.rs:1-5). */
typedef struct nsrl_fixed_scale {
  int32_t multiplier;
  uint8_t right_shift;
  uint8_t pad[3];
} nsrl_fixed_scale;

/* LinearI16I8Params (crates/nsrl-core/src/linear.rs:6-13); the struct lives
 * in host memory, the arrays it points to in device memory. */
typedef struct nsrl_linear_params {
  const int8_t* weights;          /* [output_dim][input_dim] */
  const int32_t* bias;            /* [output_dim] or NULL */
  const nsrl_fixed_scale* scales; /* [output_dim] */
  size_t input_dim;
  size_t output_dim;
} nsrl_linear_params;

/* Device-resident status written by the kernels of a call.  Reset it with
 * nsrl_status_reset() before a call (or a group of calls); read it with
 * nsrl_status_fetch(). */
typedef struct nsrl_device_status {
  unsigned long long flags;                 /* nonzero = rejected; bits name the cause */
  unsigned long long attention_saturations; /* residual_add saturation count, attention blocks */
  unsigned long long mlp_saturations;       /* residual_add saturation count, MLP blocks */
  unsigned long long reserved[5];
} nsrl_device_status;

/* Clears *status on `stream`. */
nsrl_status nsrl_status_reset(nsrl_device_status* status, void* stream);

/* Synchronises `stream`, copies *status to *host_out (may be NULL) and
 * returns NSRL_CORE_REJECTED if any flag is set, else NSRL_OK. */
nsrl_status nsrl_status_fetch(const nsrl_device_status* status, nsrl_device_status* host_out, void* stream);

/* Text of the last host-side error on this thread ("" if none). */
const char* nsrl_last_error(void);

/* ---------------------------------------------------------------- linear --
 * y[m] = linear_i16_i8_i16_per_channel_checked(x[m], params) for m < rows.
 * Replaces crates/nsrl-core/src/linear.rs:115-126 (generic kernel
 * :228-324; i32 accumulator semantics :144-173) batched over rows.
 * x: [rows][input_dim] int16, y: [rows][output_dim] int16. */
size_t nsrl_linear_workspace_size(size_t rows, size_t input_dim, size_t output_dim);
nsrl_status nsrl_linear_i16_i8_i16(const int16_t* x, size_t rows, const nsrl_linear_params* params, int16_t* y,
                                   void* workspace, size_t workspace_bytes, nsrl_device_status* status,
                                   void* stream);

/* The same linear for callers that cannot allocate device memory.  No
 * counterpart in the reference.  It takes no workspace: it uses a static
 * device scratch array of nsrl_linear_noalloc_scratch_bytes() (16 MiB) that
 * every GPU loading the library holds until exit.  Callers that need it:
 * shims that keep nsrl-core's workspace-free slice signature, and host paths
 * that must not call cudaMalloc / cudaFree (those can synchronise the device,
 * or fail under a memory budget owned by another allocator).  Shapes whose
 * nsrl_linear_workspace_size() exceeds the scratch are rejected with
 * NSRL_INVALID_SHAPE and a message.  The first call on a device looks up the
 * scratch address (cudaGetSymbolAddress) and should come before any stream
 * capture.  That address is cached per device index for the life of the
 * process, so it assumes the device's primary context (the runtime API's):
 * callers that make their own driver-API contexts, or that call
 * cudaDeviceReset after the first call, are not supported.  All calls share
 * the scratch: calls that overlap on the GPU race and must be serialised by
 * the caller. */
size_t nsrl_linear_noalloc_scratch_bytes(void);
nsrl_status nsrl_linear_i16_i8_i16_noalloc(const int16_t* x, size_t rows, const nsrl_linear_params* params,
                                           int16_t* y, nsrl_device_status* status, void* stream);

/* --------------------------------------------------------------- rms norm --
 * y[r] = rms_norm_i16_q15_checked(x[r], gamma, eps) for r < rows.
 * Replaces crates/nsrl-core/src/rms_norm.rs:68-89 batched over rows. */
nsrl_status nsrl_rms_norm_rows(const int16_t* x, size_t rows, size_t dim, const int16_t* gamma, uint64_t eps,
                               int16_t* y, nsrl_device_status* status, void* stream);

/* ------------------------------------------------------------- attention --
 * Causal (or full) multi-head integer self-attention over `batch`
 * independent sequences of seq_len tokens: x and out are [batch*seq_len][d].
 * head_dim = d / heads must be a power of four (attention.rs:1599-1602).
 * Replaces self_attention_i16_q15_checked (attention.rs:727-877), one
 * sequence per reference call. */
size_t nsrl_attention_workspace_size(size_t batch, size_t seq_len, size_t d_model, size_t heads);
nsrl_status nsrl_self_attention(const int16_t* x, size_t batch, size_t seq_len, size_t d_model, size_t heads,
                                int causal, const nsrl_linear_params* q, const nsrl_linear_params* k,
                                const nsrl_linear_params* v, const nsrl_linear_params* o, int16_t* out,
                                void* workspace, size_t workspace_bytes, nsrl_device_status* status,
                                void* stream);

/* y = x + self_attention(rms_norm(x)) with saturating Q15 residual; the
 * residual saturation count is added to status->attention_saturations.
 * Replaces prenorm_attention_residual_block_i16_q15_checked
 * (attention.rs:1522-1583). */
nsrl_status nsrl_prenorm_attention_residual_block(const int16_t* x, size_t batch, size_t seq_len, size_t d_model,
                                                  size_t heads, int causal, const int16_t* rms_gamma,
                                                  uint64_t rms_eps, const nsrl_linear_params* q,
                                                  const nsrl_linear_params* k, const nsrl_linear_params* v,
                                                  const nsrl_linear_params* o, int16_t* y, void* workspace,
                                                  size_t workspace_bytes, nsrl_device_status* status,
                                                  void* stream);

/* ------------------------------------------------------------- gated MLP --
 * y = x + down(gated(up(n), gate(n))), n = rms_norm(x), over `rows` tokens;
 * residual saturations are added to status->mlp_saturations.
 * Replaces prenorm_gated_mlp_residual_block_i16_q15_checked
 * (crates/nsrl-core/src/mlp.rs:541-594). */
size_t nsrl_mlp_workspace_size(size_t rows, size_t d_model, size_t hidden_dim);
nsrl_status nsrl_prenorm_gated_mlp_residual_block(const int16_t* x, size_t rows, size_t d_model,
                                                  size_t hidden_dim, const int16_t* rms_gamma, uint64_t rms_eps,
                                                  const nsrl_linear_params* up, const nsrl_linear_params* gate,
                                                  const nsrl_linear_params* down, int16_t* y, void* workspace,
                                                  size_t workspace_bytes, nsrl_device_status* status,
                                                  void* stream);

/* ---------------------------------------------------- transformer block --
 * The attention block followed by the MLP block with the same RMS gamma and
 * eps -- the loop body of the reference's block benchmark
 * (crates/nsrl-demo/src/bench.rs:288-343).  x and y may not alias. */
size_t nsrl_transformer_block_workspace_size(size_t batch, size_t seq_len, size_t d_model, size_t heads,
                                             size_t hidden_dim);
nsrl_status nsrl_prenorm_transformer_block(const int16_t* x, size_t batch, size_t seq_len, size_t d_model,
                                           size_t heads, size_t hidden_dim, const int16_t* attn_gamma,
                                           const int16_t* mlp_gamma, uint64_t rms_eps,
                                           const nsrl_linear_params* q, const nsrl_linear_params* k,
                                           const nsrl_linear_params* v, const nsrl_linear_params* o,
                                           const nsrl_linear_params* up, const nsrl_linear_params* gate,
                                           const nsrl_linear_params* down, int16_t* y, void* workspace,
                                           size_t workspace_bytes, nsrl_device_status* status, void* stream);

/* ------------------------------------------------------ KV-cache decode --
 * For each sequence b and head h, the single query q[b][h*hd:(h+1)*hd]
 * attends over the first lens[b] cached keys/values of that head:
 * ctx[b][h] = attention_row_i16_q15_checked(q, K[b][:lens[b]], V[b][:lens[b]])
 * (crates/nsrl-core/src/attention.rs:671-725, no mask).
 * q, ctx: [batch][heads*head_dim]; k_cache, v_cache: [batch][max_len][heads*head_dim];
 * lens: [batch] int32 in (0, max_len] (device). */
nsrl_status nsrl_attention_decode(const int16_t* q, const int16_t* k_cache, const int16_t* v_cache,
                                  const int32_t* lens, size_t batch, size_t heads, size_t head_dim, size_t max_len,
                                  int16_t* ctx, nsrl_device_status* status, void* stream);

/* One decode step of a prenorm attention block over a KV cache.  Sequence b
 * has positions[b] cached tokens (device int32); its new token x[b] is
 * normalised, projected, its k and v are written to cache row positions[b],
 * and its query attends over rows 0..positions[b] -- the last row of the
 * causal forward (attention.rs:790, effective_len = token + 1) with earlier
 * keys and values read from the cache instead of recomputed (the reference
 * recomputes, crates/nsrl-train/src/lib.rs:118-130).  y[b] = x[b] +
 * O(context), saturations into status->attention_saturations.  The caller
 * advances positions after every layer of the step.  x, y: [batch][d_model];
 * caches: head-major [batch][heads][max_len][64] int16, 16-byte aligned, so
 * that each head's keys and values stream contiguously (head_dim 64). */
size_t nsrl_decode_block_workspace_size(size_t batch, size_t d_model, size_t heads);
nsrl_status nsrl_prenorm_attention_decode_block(const int16_t* x, size_t batch, size_t d_model, size_t heads,
                                                const int16_t* rms_gamma, uint64_t rms_eps,
                                                const nsrl_linear_params* q, const nsrl_linear_params* k,
                                                const nsrl_linear_params* v, const nsrl_linear_params* o,
                                                int16_t* k_cache, int16_t* v_cache, const int32_t* positions,
                                                size_t max_len, int16_t* y, void* workspace, size_t workspace_bytes,
                                                nsrl_device_status* status, void* stream);

/* ----------------------------------------------- training-step exchange --
 * acc[n][k] += scaled_grad[r][n] * x[r][k] for r < rows, checked i64 adds in
 * row order (zero terms skipped), *sample_count += rows: one call of the
 * reference per row.  Replaces accumulate_linear_weight_gradient_i64_prescaled
 * (crates/nsrl-train-core/src/lib.rs:344-384).  x: [rows][input_dim] int16,
 * scaled_grad: [rows][output_dim] int32, accumulators: [output_dim][input_dim]
 * int64, sample_count: one device uint64.  An overflow rejects the call. */
size_t nsrl_accumulate_workspace_size(size_t input_dim, size_t output_dim);
nsrl_status nsrl_accumulate_linear_weight_gradient_i64(const int16_t* x, const int32_t* scaled_grad, size_t rows,
                                                       size_t input_dim, size_t output_dim, long long* accumulators,
                                                       unsigned long long* sample_count, void* workspace,
                                                       size_t workspace_bytes, nsrl_device_status* status,
                                                       void* stream);

/* Averages the accumulators over *sample_count (round half away from zero),
 * scales by learning_rate, adds the carried residual, rounds with
 * learning_rate_shift, subtracts from the i8 weights with saturation and
 * clears the accumulators and the count.  stats (3 device uint64):
 * {gradient saturations, zero deltas, sum |weight delta|}.  Replaces
 * apply_linear_weight_gradient_i64_to_i8 (crates/nsrl-train-core/src/lib.rs:386-465). */
nsrl_status nsrl_apply_linear_weight_gradient_i64_to_i8(long long* accumulators, long long* residuals, int8_t* weights,
                                                        size_t len, unsigned long long* sample_count,
                                                        int32_t learning_rate, uint8_t learning_rate_shift,
                                                        int carry_residual, unsigned long long* stats,
                                                        nsrl_device_status* status, void* stream);

/* i16 embedding apply (nsrl-train/src/lib.rs:14407-14510): per entry with a
 * nonzero sum or residual, product = round_div(acc, count) * lr + residual,
 * u = rhu(product, shift), residual' = product - (u << shift), e = sat_i16(e - u).
 * stats (3 device uint64, added to): {saturations, zero deltas, sum |delta|}.
 * The accumulators and the count are not cleared (the caller clears the
 * token and position parts together, :14454). */
nsrl_status nsrl_apply_embedding_gradient_i64_to_i16(const long long* accumulators, long long* residuals,
                                                     int16_t* embeddings, size_t len,
                                                     const unsigned long long* sample_count, int32_t learning_rate,
                                                     uint8_t learning_rate_shift, unsigned long long* stats,
                                                     nsrl_device_status* status, void* stream);

/* The movement average of the per-window (serial) training mode
 * (average_mini_transformer_batch_movement, nsrl-train/src/lib.rs:14515-14583):
 * values[i] = sat(base[i] + round_div(values[i] - base[i], divisor)), the
 * movement since the batch's checkpoint `base` divided by the accepted windows
 * (half away from zero).  A tensor that the batch updates through i64
 * accumulators (every tensor of nsrl_train_dp_step) is not averaged. */
nsrl_status nsrl_average_movement_i8(const int8_t* base, int8_t* values, size_t len, uint64_t divisor, void* stream);
nsrl_status nsrl_average_movement_i16(const int16_t* base, int16_t* values, size_t len, uint64_t divisor,
                                      void* stream);

/* Integer Adam (crates/nsrl-train-core/src/lib.rs:276-661): IntegerAdamConfig
 * with beta1 = 1 - 2^-beta1_decay_shift, beta2 = 1 - 2^-beta2_decay_shift. */
typedef struct nsrl_integer_adam_config {
  int32_t learning_rate;
  uint8_t step_shift;
  uint8_t beta1_decay_shift;
  uint8_t beta2_decay_shift;
  uint8_t pad;
  uint64_t epsilon;
} nsrl_integer_adam_config;

/* apply_integer_adam_accumulators_i64_to_i8 / _to_i16 (lib.rs:469-593): per
 * entry g = round_div(acc, count), the moments and the carried residual
 * advance (integer_adam_delta, :602-661), the weight moves by the rounded
 * update with saturation.  Device arrays: moments, residuals [len], *step
 * (uint64, +1 per call with a nonzero count), stats (3 uint64, added to):
 * {saturations, zero deltas, sum |delta|}.  The accumulators are read only. */
nsrl_status nsrl_apply_integer_adam_i64_to_i8(const long long* accumulators, const unsigned long long* sample_count,
                                              int8_t* weights, size_t len, const nsrl_integer_adam_config* config,
                                              long long* first_moments, unsigned long long* second_moments,
                                              long long* update_residuals, unsigned long long* step,
                                              unsigned long long* stats, nsrl_device_status* status, void* stream);
nsrl_status nsrl_apply_integer_adam_i64_to_i16(const long long* accumulators, const unsigned long long* sample_count,
                                               int16_t* weights, size_t len, const nsrl_integer_adam_config* config,
                                               long long* first_moments, unsigned long long* second_moments,
                                               long long* update_residuals, unsigned long long* step,
                                               unsigned long long* stats, nsrl_device_status* status, void* stream);

/* ---------------------------------------------------- training backward --
 * Backward-input linear over rows: dx[m][k] = requantize_i64_to_i16(
 * sum_n g'[m][n] * W[n][k], grad_input_scales[k]) with g' = rhu(g * mult_n,
 * shift_n) from the forward scales of `params` (a g' outside i32 rejects).
 * grad_input_scales: [input_dim] or NULL (identity, as the mini transformer
 * passes them).  Replaces linear_backward_input_i16_i8_i16_per_channel_checked
 * (crates/nsrl-core/src/linear.rs:548-640).  g [rows][output_dim], dx
 * [rows][input_dim] int16. */
size_t nsrl_linear_backward_input_workspace_size(size_t rows, size_t input_dim, size_t output_dim);
nsrl_status nsrl_linear_backward_input(const int16_t* grad_output, size_t rows, const nsrl_linear_params* params,
                                       const nsrl_fixed_scale* grad_input_scales, int16_t* grad_input,
                                       void* workspace, size_t workspace_bytes, nsrl_device_status* status,
                                       void* stream);

/* Gated-MLP backward input with identity grad-input scales (mlp.rs:256-357
 * as the mini transformer calls it, nsrl-train/src/lib.rs:15670-15696):
 * grad_up / grad_gate [rows][hidden] (mlp.rs:172-194), grad_input
 * [rows][d_model] = sat(up^T + gate^T); *saturations (device uint64) +=
 * the saturations of that sum. */
size_t nsrl_gated_mlp_backward_input_workspace_size(size_t rows, size_t d_model, size_t hidden_dim);
nsrl_status nsrl_gated_mlp_backward_input(const int16_t* grad_output, size_t rows, size_t d_model, size_t hidden_dim,
                                          const nsrl_linear_params* up, const nsrl_linear_params* gate,
                                          const nsrl_linear_params* down, const int16_t* forward_up,
                                          const int16_t* forward_gate, int16_t* grad_up, int16_t* grad_gate,
                                          int16_t* grad_input, unsigned long long* saturations, void* workspace,
                                          size_t workspace_bytes, nsrl_device_status* status, void* stream);

/* RMS-norm backward rows (crates/nsrl-core/src/rms_norm.rs:96-170, rows as in
 * nsrl-train/src/lib.rs:15030-15077): grad_input [rows][d] int16; gamma
 * gradients added into gamma_grad [d] int64; *saturations (device uint64)
 * += saturated grad_input values. */
nsrl_status nsrl_rms_norm_backward_rows(const int16_t* x, size_t rows, size_t d, const int16_t* gamma,
                                        const int16_t* grad_output, uint64_t eps, int16_t* grad_input,
                                        long long* gamma_grad, unsigned long long* saturations,
                                        nsrl_device_status* status, void* stream);

/* Causal attention with its probabilities: q, k, v rows of stride ld
 * (sequence b at row b * seq_len, head h at column h * head_dim) -> context
 * [batch*seq_len][d] and P [batch][heads][seq_len][seq_len] int16 (zero above
 * the diagonal).  The forward half of nsrl-train/src/lib.rs:15161-15180 and
 * :15353-15418. */
nsrl_status nsrl_attention_with_probabilities(const int16_t* q, const int16_t* k, const int16_t* v, size_t ld,
                                              size_t batch, size_t seq_len, size_t d_model, size_t heads,
                                              int16_t* context, int16_t* probabilities, nsrl_device_status* status,
                                              void* stream);

/* Softmax-attention backward (nsrl-train/src/lib.rs:16623-16900): from q, k, v
 * (stride ld), P and the context gradient dC [batch*seq_len][d] -> dq, dk, dv
 * [batch*seq_len][d].  Workspace: nsrl_attention_backward_workspace_size. */
size_t nsrl_attention_backward_workspace_size(size_t batch, size_t seq_len, size_t d_model, size_t heads);
nsrl_status nsrl_attention_backward(const int16_t* q, const int16_t* k, const int16_t* v, size_t ld,
                                    const int16_t* probabilities, const int16_t* grad_context, size_t batch,
                                    size_t seq_len, size_t d_model, size_t heads, int16_t* dq, int16_t* dk, int16_t* dv,
                                    void* workspace, size_t workspace_bytes, nsrl_device_status* status, void* stream);

/* i64 weight-gradient accumulation on the tensor cores for int16 gradients:
 * acc[n][k] += g'[r][n] * x[r][k] over r < rows with g' = rhu(g, shift_n)
 * (forward scales with multiplier 1, the reference's tables; another
 * multiplier rejects the call), *sample_count += rows.  The prescale of
 * linear.rs:573-592 followed by accumulate_linear_weight_gradient_i64_prescaled
 * (nsrl-train-core/src/lib.rs:344-384) once per row.  x [rows][input_dim],
 * grad_output [rows][output_dim] int16, accumulators [output_dim][input_dim]. */
size_t nsrl_accumulate_weight_gradient_i16_workspace_size(size_t rows, size_t input_dim, size_t output_dim);
nsrl_status nsrl_accumulate_weight_gradient_i16(const int16_t* x, const int16_t* grad_output, size_t rows,
                                                size_t input_dim, size_t output_dim, const nsrl_fixed_scale* scales,
                                                long long* accumulators, unsigned long long* sample_count,
                                                void* workspace, size_t workspace_bytes, nsrl_device_status* status,
                                                void* stream);

/* ------------------------------------------------- training window step --
 * The map-reduce worker of the reference's mini transformer
 * (nsrl-train/src/lib.rs:7051-7399) for `windows` windows of seq_len bytes on
 * one GPU: embeddings (+ learned positions), the stacked blocks forward with
 * their caches, the byte head on the last position, the softmax gradient,
 * and the backward of every block into i64 gradient accumulators.  The
 * model structs live in host memory; every array they point to is device
 * memory.  Forward multipliers must be 1 (the reference's scale tables). */
typedef struct nsrl_train_layer {
  const int16_t* attn_gamma; /* [d] or NULL: RMS norm disabled (both or neither) */
  const int16_t* mlp_gamma;  /* [d] or NULL */
  nsrl_linear_params lin[7]; /* q, k, v, o [d][d]; up, gate [hidden][d]; down [d][hidden] */
} nsrl_train_layer;

typedef struct nsrl_train_model {
  size_t d_model, heads, hidden_dim, layers, seq_len;
  const int16_t* embeddings; /* [256][d] */
  const int16_t* positions;  /* [seq_len][d], or NULL for the position-free policy */
  const nsrl_train_layer* layer; /* host array of `layers` blocks */
  nsrl_linear_params head;   /* [256][d] byte head */
  int32_t attention_kind;    /* MiniTransformerAttentionKind (lib.rs:1017-1023): 0 base-2
                                softmax, 1 linear (generation and output rows only) */
} nsrl_train_model;

/* Length (int64 elements) of the gradient arena: head [256][d]; per layer
 * q, k, v, o, up, gate, down, rms_attention [d], rms_mlp [d]; token
 * embeddings [256][d]; positions [seq_len][d].  counts: 2 + 9 * layers
 * uint64 (head, 9 per layer in the same order, embeddings). */
size_t nsrl_train_arena_len(const nsrl_train_model* model);
size_t nsrl_train_workspace_size(const nsrl_train_model* model, size_t windows);
/* contexts [windows][seq_len] uint8, targets [windows] uint8, freq_weights
 * [256] int16 or NULL (all 32767).  Adds into arena / counts; stats (4
 * device uint64) += {accepted windows, mlp saturations, attention
 * saturations, residual saturations}.  A rejection anywhere rejects the
 * whole batch (nsrl-train/src/lib.rs:5371-5375). */
nsrl_status nsrl_train_windows(const nsrl_train_model* model, const uint8_t* contexts, const uint8_t* targets,
                               const int16_t* freq_weights, size_t windows, long long* arena,
                               unsigned long long* counts, unsigned long long* stats, void* workspace,
                               size_t workspace_bytes, nsrl_device_status* status, void* stream);

/* ------------------------------------------------ data-parallel step --
 * One training batch of the mini transformer on every rank of a
 * communicator: the reference's map-reduce batch (nsrl-train/src/lib.rs:
 * 6970-7399) with the ranks as its workers, the ordered merge of the
 * workers' i64 accumulators (:7401-7471) as an exact NCCL int64 all-reduce,
 * and the apply of every parameter (:6249-6400 with the shift optimizer, or
 * the integer-Adam batch apply :4270-4465).  Rank r holds window chunk r of
 * the batch, as worker r does in the reference, so the weights after a step
 * are the same for any number of ranks.
 *
 * nsrl_comm is an NCCL communicator (non-blocking, NCCL loaded at run time
 * from libnccl.so.2) whose every wait is bounded by its timeout: a collective
 * still running at the deadline aborts the communicator and the call returns
 * NSRL_COMM_TIMEOUT; an error that NCCL reports (a failed peer) aborts it and
 * returns NSRL_COMM_ERROR.  An aborted communicator fails every later call
 * with NSRL_COMM_ERROR; destroy it and make a new one.  The reference has no
 * communicator (its workers are threads, lib.rs:7012-7047). */
typedef struct nsrl_comm nsrl_comm;
#define NSRL_COMM_ID_BYTES 128

/* Rank 0 makes the id (ncclGetUniqueId) and hands it to every rank. */
nsrl_status nsrl_comm_unique_id(uint8_t id[NSRL_COMM_ID_BYTES]);
/* Joins the communicator on the current CUDA device; timeout_ms bounds the
 * join and every later wait on it (0 = 120 s). */
nsrl_status nsrl_comm_init(nsrl_comm** comm, int nranks, int rank, const uint8_t id[NSRL_COMM_ID_BYTES],
                           uint64_t timeout_ms);
/* Finalises (or, after a failure, aborts) and frees the communicator. */
nsrl_status nsrl_comm_destroy(nsrl_comm* comm);
/* Aborts the communicator now (ncclCommAbort): for a caller that learned on
 * the host that a peer has left; every later step on it fails with
 * NSRL_COMM_ERROR.  Free it with nsrl_comm_destroy. */
nsrl_status nsrl_comm_abort(nsrl_comm* comm);
int nsrl_comm_nranks(const nsrl_comm* comm);
int nsrl_comm_rank(const nsrl_comm* comm);

enum { NSRL_OPTIMIZER_SHIFT = 0, NSRL_OPTIMIZER_INTEGER_ADAM = 1 };
/* MiniTransformerAdamTrainScope (nsrl-train/src/lib.rs:188-195). */
enum {
  NSRL_ADAM_SCOPE_ALL = 0,
  NSRL_ADAM_SCOPE_RMS_NORM = 1,
  NSRL_ADAM_SCOPE_OUTPUT = 2,
  NSRL_ADAM_SCOPE_FINAL_MLP = 3,
  NSRL_ADAM_SCOPE_FINAL_MLP_AND_OUTPUT = 4,
};

/* The learning-rate fields of MiniTransformerMlpTrainConfig (nsrl-train/src/
 * lib.rs:300-390, defaults :86-91: 1, 18, 16, 14, 24, 18, 18) and the
 * optimizer.  The shift optimizer subtracts the batch shift
 * ceil(log2(accepted windows)) from every shift (:13591-13650) and adds the
 * stacked-layer extra shifts (:15454-15495); integer Adam uses `adam`
 * (IntegerAdamConfig) for every tensor in `adam_scope`. */
typedef struct nsrl_train_config {
  int32_t learning_rate;
  uint8_t output_learning_rate_shift;
  uint8_t mlp_learning_rate_shift;
  uint8_t embedding_learning_rate_shift;
  uint8_t attention_learning_rate_shift;
  uint8_t attention_q_learning_rate_shift;
  uint8_t attention_qk_learning_rate_shift;
  uint8_t optimizer;  /* NSRL_OPTIMIZER_* */
  uint8_t adam_scope; /* NSRL_ADAM_SCOPE_* */
  nsrl_integer_adam_config adam;
} nsrl_train_config;

/* Optimizer state carried between steps (device arrays, caller-owned).
 * residuals [nsrl_train_arena_len] int64 (the shift optimizer's carried
 * remainders, arena order).  With integer Adam: adam_* [nsrl_train_adam_state_len]
 * in the reference's flat order (token embeddings, positions, attention and
 * MLP RMS gammas, q, k, v, o, up, gate, down of all layers, output head,
 * lib.rs:1001-1015, :4165-4196) and adam_step (one uint64, +1 per applied
 * batch, :4447-4451); NULL otherwise. */
typedef struct nsrl_train_state {
  long long* residuals;
  long long* adam_first_moments;
  unsigned long long* adam_second_moments;
  long long* adam_update_residuals;
  unsigned long long* adam_step;
} nsrl_train_state;

/* Batch statistics summed over the ranks. */
typedef struct nsrl_train_step_stats {
  uint64_t accepted_windows;
  uint64_t mlp_saturations;
  uint64_t attention_saturations;
  uint64_t residual_saturations;
  uint64_t gradient_saturations; /* of the apply */
  uint64_t zero_deltas;
  uint64_t weight_delta_l1;
} nsrl_train_step_stats;

size_t nsrl_train_adam_state_len(const nsrl_train_model* model);
size_t nsrl_train_dp_workspace_size(const nsrl_train_model* model, size_t windows, int nranks);
/* Runs this rank's `windows` windows (contexts [windows][seq_len] uint8,
 * targets [windows] uint8, freq_weights [256] int16 or NULL), the exchange
 * with the other ranks of `comm` (NULL = one rank) and the apply; the model's
 * weights (i8 linears, i16 embeddings, and with Adam the RMS gammas) are
 * updated in place through its pointers.  The call returns when the step is
 * complete on the device (it waits on `stream`).  It clears `status` first.
 * NSRL_CORE_REJECTED: some rank rejected the batch (lib.rs:5371-5375) or the
 * ordered merge overflowed; the model and the state are unchanged.  Every
 * rank must call it with the same model shapes and config; rank r's windows
 * are chunk r of the batch. */
nsrl_status nsrl_train_dp_step(const nsrl_train_model* model, const uint8_t* contexts, const uint8_t* targets,
                               const int16_t* freq_weights, size_t windows, const nsrl_train_config* config,
                               const nsrl_train_state* state, nsrl_comm* comm, nsrl_train_step_stats* stats,
                               void* workspace, size_t workspace_bytes, nsrl_device_status* status, void* stream);

/* The reference's merge of worker results (mini_transformer_merge_map_reduce_
 * batch_result, nsrl-train/src/lib.rs:7401-7471) as a primitive: parts is
 * [workers][len] int64; out[i] = parts[0][i] + parts[1][i] + ... in worker
 * order, with checked adds for i < checked_len (the i64 accumulators; an
 * overflow rejects the call) and wrapping adds after (the counts).  The
 * data-parallel step uses it when the bound of its all-reduce fails. */
nsrl_status nsrl_merge_worker_parts_i64(const long long* parts, size_t workers, size_t checked_len, size_t len,
                                        long long* out, nsrl_device_status* status, void* stream);

/* The wait of the communicator against a fake clock and fake completion /
 * error reports (no GPU, no NCCL): scenario 0 completes after three polls,
 * 1 never completes, 2 reports a peer error on the third poll.  Returns what
 * the real wait would (NSRL_OK, NSRL_COMM_TIMEOUT, NSRL_COMM_ERROR); *polls
 * and *aborted tell how many polls ran and whether the abort was called. */
nsrl_status nsrl_comm_selftest_wait(int scenario, uint64_t timeout_ms, uint64_t* polls, int* aborted);

/* ------------------------------------------------------ linear attention --
 * Causal (or full) integer linear attention over `batch` sequences of
 * seq_len tokens, x and out [batch*seq_len][d]: q, k, v linears, per head the
 * state S = sum phi(k) v^T and key sums sum phi(k) (phi(x) = x + 32769,
 * checked i64), the projection round_div(phi(q) S, phi(q) . key sums), then
 * the o linear.  Replaces linear_attention_i16_q15_checked
 * (crates/nsrl-core/src/attention.rs:879-1041), one sequence per reference
 * call.  head_dim = d / heads <= 64 (any value, not only powers of four). */
size_t nsrl_linear_attention_workspace_size(size_t batch, size_t seq_len, size_t d_model);
nsrl_status nsrl_linear_attention(const int16_t* x, size_t batch, size_t seq_len, size_t d_model, size_t heads,
                                  int causal, const nsrl_linear_params* q, const nsrl_linear_params* k,
                                  const nsrl_linear_params* v, const nsrl_linear_params* o, int16_t* out,
                                  void* workspace, size_t workspace_bytes, nsrl_device_status* status,
                                  void* stream);

/* One streaming step of `batch` independent streams: row b of x [batch][d]
 * updates stream b's state (state [batch][heads][hd][hd], key_sums
 * [batch][heads][hd], int64, zero at the start of a stream) and projects its
 * query; out [batch][d].  ttt_shift < 0: linear_attention_step_i16_q15_checked
 * (attention.rs:1045-1158); ttt_shift in 0..62: the test-time-training step
 * (:1160-1344), which also adds each stream's sum |state update| to
 * delta_l1[b] (device uint64, may be NULL). */
size_t nsrl_linear_attention_step_workspace_size(size_t batch, size_t d_model);
nsrl_status nsrl_linear_attention_step(const int16_t* x, size_t batch, size_t d_model, size_t heads,
                                       const nsrl_linear_params* q, const nsrl_linear_params* k,
                                       const nsrl_linear_params* v, const nsrl_linear_params* o, long long* state,
                                       long long* key_sums, int ttt_shift, unsigned long long* delta_l1,
                                       int16_t* out, void* workspace, size_t workspace_bytes,
                                       nsrl_device_status* status, void* stream);

/* ------------------------------------------------------------ generation --
 * Byte generation with the mini transformer (softmax attention), the
 * reference's generate_mini_transformer (nsrl-train/src/lib.rs:12702-12800)
 * batched over sequences and kept on the device: every step takes the last
 * seq_len bytes of each context, left-padded with ' ', runs the full forward
 * (:14911-15008), the byte head and its base-2 softmax on the last position
 * (:17455-17490), and picks the next byte (:18979-19100).  The reference's
 * window slides (and its positions shift) every step, so the whole window is
 * recomputed, as the reference does: a KV cache cannot reproduce these
 * steps; nsrl_prenorm_attention_decode_block serves callers whose context
 * does not slide.  `model` is the training model struct (only read). */
typedef struct nsrl_decode_config {
  int32_t strategy;     /* 0: greedy (argmax, lowest index on ties); 1: sample */
  uint32_t top_k;       /* sample among the top_k logits (0 = all 256) */
  uint64_t sample_seed; /* decode_sample_u64 seed (lib.rs:19334-19340) */
} nsrl_decode_config;

size_t nsrl_generate_workspace_size(const nsrl_train_model* model, size_t batch);
/* windows [batch][seq_len] uint8 (device) -> logits_q8 [batch][256] int32
 * and probs_q15 [batch][256] int16 of each window's last position. */
nsrl_status nsrl_mini_transformer_output_rows(const nsrl_train_model* model, const uint8_t* windows, size_t batch,
                                              int32_t* logits_q8, int16_t* probs_q15, void* workspace,
                                              size_t workspace_bytes, nsrl_device_status* status, void* stream);
/* contexts [batch][capacity] uint8 (device) hold each prompt at the start;
 * prompt_lens [batch] (HOST int32, 1..capacity-steps).  Runs `steps` steps:
 * the chosen byte of step i is appended to each context and written to
 * tokens [batch][steps]; pick_logits / pick_probs [batch][steps] (device, or
 * NULL) get its logit and probability.  Asynchronous on `stream`.  The
 * decode options beyond greedy and seeded top-k sampling (priors,
 * penalties, printable filters) are not offered. */
nsrl_status nsrl_mini_transformer_generate(const nsrl_train_model* model, uint8_t* contexts, size_t capacity,
                                           const int32_t* prompt_lens, size_t batch, size_t steps,
                                           const nsrl_decode_config* decode, uint8_t* tokens, int32_t* pick_logits,
                                           int16_t* pick_probs, void* workspace, size_t workspace_bytes,
                                           nsrl_device_status* status, void* stream);

/* Incremental generation with a one-layer linear-attention model without
 * positions: generate_mini_transformer_streaming_linear_nope_with_priors and
 * its TTT variant (nsrl-train/src/lib.rs:12802-12980), batched.  Every
 * prompt byte and then every chosen byte runs one streaming step (the
 * token's embedding, the linear-attention step with the stream's carried
 * state, the residual, the gated MLP, the residual, the byte head); the
 * reference's streaming step applies no RMS norm, and neither does this.
 * All prompts have prompt_len bytes (contexts [batch][capacity], device).
 * ttt_shift < 0: the plain step; else the TTT step with that shift. */
size_t nsrl_generate_streaming_workspace_size(const nsrl_train_model* model, size_t batch);
nsrl_status nsrl_mini_transformer_generate_streaming(const nsrl_train_model* model, uint8_t* contexts,
                                                     size_t capacity, size_t prompt_len, size_t batch, size_t steps,
                                                     const nsrl_decode_config* decode, int ttt_shift,
                                                     uint8_t* tokens, int32_t* pick_logits, int16_t* pick_probs,
                                                     void* workspace, size_t workspace_bytes,
                                                     nsrl_device_status* status, void* stream);

/* The transformer block over HOST buffers (pinned host memory for the
 * overlap): the batch runs in steps of at most `chunk` sequences; the copy
 * in of step i+1, the block of step i and the copy out of step i-1 overlap
 * (two device buffers per direction, two library-owned copy streams per
 * device and thread).  The steps ramp up
 * from chunk / 4 and back down at the end, so that the copy in of the first
 * step and the copy out of the last, the two that nothing hides, are short.  The call is complete on
 * `stream` when y_host holds the output.  No counterpart in the reference
 * (its blocks read host memory); it is nsrl_prenorm_transformer_block for a
 * caller whose activations live on the host.  Workspace:
 * nsrl_transformer_block_host_workspace_size(chunk, ...). */
size_t nsrl_transformer_block_host_workspace_size(size_t chunk, size_t seq_len, size_t d_model, size_t heads,
                                                  size_t hidden_dim);
nsrl_status nsrl_prenorm_transformer_block_host(const int16_t* x_host, size_t batch, size_t chunk, size_t seq_len,
                                                size_t d_model, size_t heads, size_t hidden_dim,
                                                const int16_t* attn_gamma, const int16_t* mlp_gamma, uint64_t rms_eps,
                                                const nsrl_linear_params* q, const nsrl_linear_params* k,
                                                const nsrl_linear_params* v, const nsrl_linear_params* o,
                                                const nsrl_linear_params* up, const nsrl_linear_params* gate,
                                                const nsrl_linear_params* down, int16_t* y_host, void* workspace,
                                                size_t workspace_bytes, nsrl_device_status* status, void* stream);

/* ----------------------------------------------------------- diagnostics --
 * Makes one bounded device wait run out on purpose (no counterpart in the
 * reference, whose kernels never wait on a device barrier).  Every mbarrier
 * wait of the library's kernels gives up after a time limit, sets a
 * WAIT_TIMEOUT bit in the call's status and unwinds, so that a lost arrival
 * ends the call with NSRL_CORE_REJECTED instead of hanging the GPU.  This
 * launches one CTA of 32 threads that wait, with the same loop and a limit of
 * limit_ns (at most 1 s), on a barrier nothing arrives on.  out (3 device
 * uint64): {threads whose wait gave up, whether the call's timeout bit reads
 * as set, nanoseconds waited}. */
nsrl_status nsrl_selftest_bounded_wait(unsigned long long limit_ns, nsrl_device_status* status,
                                       unsigned long long* out, void* stream);

/* Runs the divider of the data-parallel apply over n numerators: out[i] =
 * round_div(num[i], den) (the reference's rounding of an i64 gradient sum by
 * its count, half away from zero), ok[i] = 0 where the reference's checked
 * arithmetic fails.  Device arrays; no counterpart in the reference. */
nsrl_status nsrl_selftest_round_div(const long long* num, size_t n, long long den, long long* out,
                                    unsigned char* ok, void* stream);

/* Runs the element rule of the data-parallel apply's SGD segments over n
 * entries: weights_i8 != 0 is apply_linear_weight_gradient_i64_to_i8 with the
 * residual carried (crates/nsrl-train-core/src/lib.rs:386-465), 0 the i16
 * embedding rule (nsrl-train/src/lib.rs:14457-14510), with the gradient sums,
 * count, learning rate and shift given.  residuals and weights (int8 or
 * int16) are updated in place; stats (3 device uint64, zeroed by the caller)
 * gain {saturations, zero deltas, weight L1}; *bad is set to 1 where the
 * reference's checked arithmetic fails (the apply would be rejected).  The
 * sums are not cleared.  Device arrays; no counterpart in the reference. */
nsrl_status nsrl_selftest_sgd_apply(const long long* sums, long long* residuals, void* weights, int weights_i8,
                                    size_t n, unsigned long long count, int learning_rate, int shift,
                                    unsigned long long* stats, unsigned char* bad, void* stream);

/* ------------------------------------------------- head-sharded forward --
 * The transformer block of nsrl_prenorm_transformer_block (or, without the
 * MLP, nsrl_prenorm_attention_residual_block) split over n ranks, one GPU
 * each, with results identical to the one-GPU block.  The reference computes
 * this block on one CPU (attention.rs:1522-1583, mlp.rs:541-594); the split
 * has no counterpart there.
 *
 * Rank r owns positions [r S/n, (r+1) S/n) of every sequence for the work
 * done token by token -- the RMS norms, the Q|K|V, O, up, gate and down
 * linears, the residual adds -- and heads [r H/n, (r+1) H/n) for attention.
 * The Q|K|V projection of a rank's positions stores each head's q, k and v
 * straight into the exchange buffer of the rank that owns the head, over
 * NVLink (peer stores from the GEMM's epilogue); attention on a rank's heads
 * stores each context row straight into the buffer of the rank that owns the
 * position.  Every value is computed by the same kernel and operation
 * order as on one GPU; only where it is stored changes, so the split is
 * exact.  Weights are whole on every rank.
 *
 * x and y are the rank's rows [batch][S/n][d_model] (position-major within
 * each sequence).  Shape rules: those of the one-GPU block, n <= 8, S and
 * heads multiples of n, head_dim 64 and S <= 16384 (the tensor-core
 * attention); d_model a multiple of 128 keeps the Q|K|V projection on the
 * tensor cores (other sizes use the SIMT linear).
 *
 * Exchange buffers: every rank allocates one buffer of
 * nsrl_shard_exchange_bytes with nsrl_shard_alloc, shares its IPC handle, and
 * opens the others' with nsrl_ipc_open; nsrl_shard_group_create then takes
 * all n buffers (index = rank; its own as allocated).  Every rank must have
 * returned from nsrl_shard_group_create before any rank runs a phase (a host
 * barrier), and all ranks run the same phases in the same order.
 *
 * Synchronisation is on the device: a phase that feeds other ranks ends with
 * a signal (a release store of an epoch count into every rank's signal
 * words); the phase that reads the exchange starts with a wait for every
 * rank's signal of that epoch, bounded by the group's timeout.  A wait that
 * runs out sets NSRL_FLAG_WAIT_TIMEOUT in the status (nsrl_status_fetch then
 * returns NSRL_CORE_REJECTED), and the group is unusable afterwards: destroy
 * it and create a new one on every rank.
 *
 * Status: each rank's status sees its own positions' saturations and its own
 * heads' rejections.  nsrl_shard_status_post followed by
 * nsrl_shard_status_combine adds every other rank's words into the status,
 * so that each rank holds the status of the whole block (flags OR-ed,
 * saturation counts summed); run the pair once per forward, after the last
 * phase. */
typedef struct nsrl_shard_group nsrl_shard_group;
#define NSRL_IPC_HANDLE_BYTES 64

size_t nsrl_shard_exchange_bytes(size_t batch, size_t seq_len, size_t d_model, size_t heads, size_t nranks);
/* cudaMalloc'd, zeroed exchange buffer on the current device; free with nsrl_shard_free. */
nsrl_status nsrl_shard_alloc(size_t bytes, void** buffer);
nsrl_status nsrl_shard_free(void* buffer);
/* CUDA IPC handle of a buffer from nsrl_shard_alloc, and its mapping in another process. */
nsrl_status nsrl_ipc_get_handle(const void* buffer, uint8_t handle[NSRL_IPC_HANDLE_BYTES]);
nsrl_status nsrl_ipc_open(const uint8_t handle[NSRL_IPC_HANDLE_BYTES], void** buffer);
nsrl_status nsrl_ipc_close(void* buffer);

/* Binds rank `rank` of `nranks` to the shape and the n exchange buffers (as
 * mapped in this process), zeroes its own buffer's header and synchronises
 * the device.  timeout_ms bounds every device wait (0 = 10 s). */
nsrl_status nsrl_shard_group_create(nsrl_shard_group** group, int nranks, int rank, void* const* exchange,
                                    size_t exchange_bytes, size_t batch, size_t seq_len, size_t d_model,
                                    size_t heads, uint64_t timeout_ms);
nsrl_status nsrl_shard_group_destroy(nsrl_shard_group* group);

/* Scratch of the three phases on one rank (MLP hidden size hidden_dim; 0 when
 * the MLP is left out). */
size_t nsrl_sharded_block_workspace_size(const nsrl_shard_group* group, size_t hidden_dim);

/* Phase 1: n = rms_norm(x) (or x itself with rms_gamma NULL), the Q|K|V
 * projection of the rank's positions into the head owners' buffers, signal. */
nsrl_status nsrl_sharded_block_qkv(const nsrl_shard_group* group, const int16_t* x, const int16_t* rms_gamma,
                                   uint64_t rms_eps, const nsrl_linear_params* q, const nsrl_linear_params* k,
                                   const nsrl_linear_params* v, const nsrl_linear_params* o, void* workspace,
                                   size_t workspace_bytes, nsrl_device_status* status, void* stream);
/* Phase 2: wait, causal attention of the rank's heads over all positions into
 * the position owners' buffers, signal.  o is the block's output projection:
 * the context's row L1 norms are kept when its i32 prefix check needs them. */
nsrl_status nsrl_sharded_block_attention(const nsrl_shard_group* group, const nsrl_linear_params* o, void* workspace,
                                         size_t workspace_bytes, nsrl_device_status* status, void* stream);
/* Phase 3: wait, h = x + O(context) for the rank's positions, then (up not
 * NULL) y = h + down(gated(up(n), gate(n))) with n = rms_norm(h), else y = h. */
nsrl_status nsrl_sharded_block_output(const nsrl_shard_group* group, const int16_t* x, const nsrl_linear_params* o,
                                      const int16_t* mlp_gamma, uint64_t rms_eps, const nsrl_linear_params* up,
                                      const nsrl_linear_params* gate, const nsrl_linear_params* down, size_t hidden_dim,
                                      int16_t* y, void* workspace, size_t workspace_bytes,
                                      nsrl_device_status* status, void* stream);
/* The three phases in order: one transformer block (MLP when up is not NULL),
 * each signal fused with the wait that follows it (one launch), which needs
 * every rank's phases to run at the same time: ranks in separate processes,
 * one GPU each.  Ranks emulated on one GPU call the phases one by one. */
nsrl_status nsrl_sharded_transformer_block(const nsrl_shard_group* group, const int16_t* x,
                                           const int16_t* attn_gamma, const int16_t* mlp_gamma, uint64_t rms_eps,
                                           const nsrl_linear_params* q, const nsrl_linear_params* k,
                                           const nsrl_linear_params* v, const nsrl_linear_params* o,
                                           const nsrl_linear_params* up, const nsrl_linear_params* gate,
                                           const nsrl_linear_params* down, size_t hidden_dim, int16_t* y,
                                           void* workspace, size_t workspace_bytes, nsrl_device_status* status,
                                           void* stream);
/* Posts this rank's status words to every rank and signals; then (combine)
 * waits and adds the other ranks' posted words into *status.  The pair in
 * one launch, for ranks in separate processes: nsrl_shard_status_allreduce. */
nsrl_status nsrl_shard_status_post(const nsrl_shard_group* group, const nsrl_device_status* status, void* stream);
nsrl_status nsrl_shard_status_combine(const nsrl_shard_group* group, nsrl_device_status* status, void* stream);
nsrl_status nsrl_shard_status_allreduce(const nsrl_shard_group* group, nsrl_device_status* status, void* stream);

/* ------------------------------------------------------------ profiling --
 * Per-launch CUDA-event timing of the library's own kernels (no counterpart
 * in the reference, whose only timer is a wall clock around the block loop,
 * crates/nsrl-demo/src/bench.rs:285).  While enabled, every kernel launch of
 * the library is bracketed by two events on its stream and recorded with its
 * algorithmic work (integer ops) and algorithmic HBM bytes.  Reading
 * synchronises the device. */
void nsrl_profile_enable(int enable);
void nsrl_profile_reset(void);
size_t nsrl_profile_count(void);
/* Entry i: kernel name (static string), duration in ms, algorithmic ops and bytes. */
nsrl_status nsrl_profile_entry(size_t i, const char** name, float* ms, double* ops, double* bytes);

#ifdef __cplusplus
}
#endif

#endif /* NSRL_B200_H */
