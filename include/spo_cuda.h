/*
 * libspo_cuda — C ABI of the B200-native (sm_100a) SPO learner step.
 *
 * This is the drop-in boundary for the hot path of josedanielchg/spo-mojo: the
 * Mojo functions of its networks/ layer (Linear, MLP, actor, actor_loss, optim)
 * as called by the learner's update() (demos/train_spo.mojo:417-554,
 * demos/train_critic.mojo:280-363). Each entry point below names the reference
 * function it replaces (path:line within the reference project). A Mojo caller
 * binds them with external_call; the Python ctypes harness in
 * spo_mojo_b200/ffi.py binds the same symbols.
 *
 * Conventions
 *   - Every function returns an int status: SPO_OK (0) or a negative SPO_ERR_*;
 *     spo_last_error_string() describes the last failure of the calling thread.
 *     Bad shapes, null pointers, misalignment and short workspaces are rejected on
 *     the host before anything is launched (the reference raises Error in the same
 *     places, e.g. networks/actor.mojo:156-165).
 *   - All tensors are caller-owned device pointers to row-major float32; W is stored
 *     [in, out] (networks/linear.mojo:7-11). Pointers that are read with vector
 *     loads must be 16-byte aligned (the functions say which).
 *   - `stream` is a cudaStream_t (NULL = the legacy default stream). Work is
 *     enqueued in order on that stream and nothing synchronises the host, except
 *     spo_learner_create, which zeroes a few bytes of its workspace.
 *   - Nothing in the hot path allocates: functions that need scratch take a
 *     caller-allocated `workspace` sized by the matching *_workspace_size query.
 *   - Gradients are OVERWRITTEN, not accumulated (as the reference's kernels do).
 *   - Thread-compatible: concurrent calls need distinct workspaces.
 */
#ifndef SPO_CUDA_H_
#define SPO_CUDA_H_

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define SPO_ABI_VERSION 3

#if defined(__GNUC__)
#define SPO_API __attribute__((visibility("default")))
#else
#define SPO_API
#endif

typedef void* spo_stream_t; /* cudaStream_t */

/* status codes */
#define SPO_OK 0
#define SPO_ERR_ARG (-1)         /* null pointer / invalid argument */
#define SPO_ERR_SHAPE (-2)       /* dimension out of range */
#define SPO_ERR_ALIGN (-3)       /* pointer or stride not 16-byte aligned */
#define SPO_ERR_WORKSPACE (-4)   /* workspace too small */
#define SPO_ERR_CUDA (-5)        /* CUDA runtime error */
#define SPO_ERR_NCCL (-6)        /* NCCL error */
#define SPO_ERR_UNSUPPORTED (-7) /* shape the fused path does not cover */
#define SPO_ERR_TIMEOUT (-8)     /* a bounded wait gave up */

#define SPO_ACT_NONE 0
#define SPO_ACT_RELU 1

#define SPO_MAX_LAYERS 8
#define SPO_ALIGN_FLOATS 64 /* each tensor of a flat parameter buffer starts on 256 B */

/* loss statistics (scaled sums: batch means when scale = 1 / global batch) */
#define SPO_NUM_STATS 8
#define SPO_STAT_ACTOR_LOSS 0  /* CE + alpha * KL(pi_old || pi) */
#define SPO_STAT_CE 1          /* -sum q log pi          networks/actor_loss.mojo:40-65 */
#define SPO_STAT_ENTROPY 2     /* H(q)                   networks/actor_loss.mojo:105-116 */
#define SPO_STAT_KL_Q 3        /* KL(q || pi)            networks/actor_loss.mojo:119-124 */
#define SPO_STAT_KL_OLD 4      /* KL(pi_old || pi) */
#define SPO_STAT_CRITIC_LOSS 5 /* 0.5 (V - t)^2          demos/train_critic.mojo:317-327 */

/* learner report (written by spo_learner_apply) */
#define SPO_REPORT_SIZE 16
#define SPO_REPORT_NORM_ACTOR 0  /* global gradient norms (only when clipping) */
#define SPO_REPORT_NORM_CRITIC 1
#define SPO_REPORT_CLIP_ACTOR 4  /* global-norm clip scales */
#define SPO_REPORT_CLIP_CRITIC 5
#define SPO_REPORT_DLOG_ALPHA 8  /* dual gradient */
#define SPO_REPORT_STEP 9        /* Adam step just taken */

typedef struct spo_mlp_desc {
  int32_t num_layers;                /* Linear layers L, 1..SPO_MAX_LAYERS */
  int32_t dims[SPO_MAX_LAYERS + 1];  /* d0 .. dL */
} spo_mlp_desc;

SPO_API int32_t spo_abi_version(void);
SPO_API const char* spo_last_error_string(void);

/* ------------------------------------------------------------------ Linear
 * linear_forward  networks/linear.mojo:86-95 (kernel :37-84), with the ReLU of
 * networks/mlp.mojo:34-46 fused when act == SPO_ACT_RELU.
 * y[m x n] = act(x[m x k] W[k x n] + b[n]). */
SPO_API int spo_linear_fwd(spo_stream_t stream, float* y, const float* x, const float* w,
                   const float* b, int64_t m, int64_t k, int64_t n, int32_t act);

/* linear_backward  networks/linear.mojo:170-193 (kernels :120-167).
 * dW = x^T dy, db = sum_rows dy, dx = (dy W^T) [* (relu_src > 0) when relu_src is
 * given: relu_backward_kernel networks/mlp.mojo:155-166]. dx may be NULL (the
 * reference computes it and drops it for the first layer, :176-178). */
SPO_API size_t spo_linear_bwd_workspace_size(int64_t m, int64_t k, int64_t n);
SPO_API int spo_linear_bwd(spo_stream_t stream, float* dw, float* db, float* dx, const float* x,
                   const float* w, const float* dy, const float* relu_src, int64_t m,
                   int64_t k, int64_t n, void* workspace, size_t workspace_bytes);

/* No counterpart in the reference. spo_linear_bwd for callers that cannot allocate
 * device memory — e.g. a host framework that pre-reserves nearly all of the GPU's memory
 * for its own pool, so cudaMalloc has nothing left to give — and so cannot provide a
 * workspace. It allocates nothing: its scratch is one static 8 MiB device array that
 * every GPU loading this library keeps until the process exits. Limits: k*n + 256*n must
 * not exceed 2,097,152 floats (larger shapes return SPO_ERR_WORKSPACE; use
 * spo_linear_bwd). The first call on a device looks the array's address up (once, with
 * that device current); make that first call before any stream capture. The address is
 * kept for the life of the process: after cudaDeviceReset (or any teardown of the
 * device's primary context) it is stale, so do not call this function again in a process
 * that has reset the device. All calls share
 * the array, so calls whose work overlaps on the GPU (other streams, other threads)
 * race: serialise them. Nothing in the array needs clearing between calls. */
SPO_API int spo_linear_bwd_noalloc(spo_stream_t stream, float* dw, float* db, float* dx,
                                   const float* x, const float* w, const float* dy,
                                   const float* relu_src, int64_t m, int64_t k, int64_t n);

/* relu networks/mlp.mojo:34-46 and relu_backward_kernel :155-166 (in place). */
SPO_API int spo_relu(spo_stream_t stream, float* a, int64_t n);
SPO_API int spo_relu_bwd(spo_stream_t stream, float* grad, const float* act, int64_t n);

/* ------------------------------------------------------------------ MLP
 * CriticParams (networks/mlp.mojo:50-81) generalised to L layers as views into ONE
 * flat buffer: w1, b1, w2, b2, ... each starting on SPO_ALIGN_FLOATS. Offsets are
 * written to w_off[L], b_off[L]; *total = padded length in floats. */
SPO_API int spo_mlp_param_layout(const spo_mlp_desc* desc, int64_t* w_off, int64_t* b_off,
                         int64_t* total);

/* CriticCache (networks/mlp.mojo:84-102): floats needed for the post-ReLU
 * activations a1 .. a_{L-1} of m rows, stored layer after layer. */
SPO_API int64_t spo_mlp_acts_size(const spo_mlp_desc* desc, int64_t m);

/* critic_forward networks/mlp.mojo:105-123 (and the actor's MLP part,
 * networks/actor.mojo:74-87): out[m x dL]; acts receives a1 .. a_{L-1}. */
SPO_API int spo_mlp_fwd(spo_stream_t stream, const spo_mlp_desc* desc, const float* params,
                const float* x, int64_t m, float* acts, float* out);

/* backward_from_dvalue networks/mlp.mojo:236-275: all layer gradients into the flat
 * `grads` buffer (same layout as params) from dout = dL/d(out) [m x dL]. `acts`
 * must come from spo_mlp_fwd with the same x and params (networks/mlp.mojo:218-221). */
SPO_API size_t spo_mlp_bwd_workspace_size(const spo_mlp_desc* desc, int64_t m);
SPO_API int spo_mlp_bwd(spo_stream_t stream, const spo_mlp_desc* desc, const float* params,
                const float* x, const float* acts, const float* dout, int64_t m,
                float* grads, void* workspace, size_t workspace_bytes);

/* ------------------------------------------------------------------ softmax / actor
 * mask_logits_kernel networks/actor.mojo:50-71: logits[i] = -FLT_MAX where mask[i] == 0. */
SPO_API int spo_mask_logits(spo_stream_t stream, float* logits, const float* mask, int64_t n);
/* softmax_rows / log_softmax_rows / logsumexp_rows ops/softmax.mojo:58-135. */
SPO_API int spo_softmax_rows(spo_stream_t stream, float* out, const float* in, int64_t rows,
                     int32_t cols);
SPO_API int spo_log_softmax_rows(spo_stream_t stream, float* out, const float* in, int64_t rows,
                         int32_t cols);
SPO_API int spo_logsumexp_rows(spo_stream_t stream, float* out, const float* in, int64_t rows,
                       int32_t cols);

/* ------------------------------------------------------------------ actor loss
 * cross_entropy_rows networks/actor_loss.mojo:68-79 (skips q == 0),
 * entropy_rows :133-139, kl_rows :142-148, logits_grad_kernel :168-191,
 * value_loss_grad_kernel networks/mlp.mojo:141-152. */
SPO_API int spo_cross_entropy_rows(spo_stream_t stream, float* loss, const float* q,
                           const float* log_pi, int64_t rows, int32_t cols);
SPO_API int spo_entropy_rows(spo_stream_t stream, float* h, const float* q, int64_t rows,
                     int32_t cols);
SPO_API int spo_kl_rows(spo_stream_t stream, float* kl, const float* ce, const float* h,
                int64_t rows);
SPO_API int spo_logits_grad(spo_stream_t stream, float* dz, const float* pi, const float* q,
                    const float* mask, int64_t n, float scale);
SPO_API int spo_value_loss_grad(spo_stream_t stream, float* dv, const float* v,
                        const float* target, int64_t n, float scale);

/* Fused output heads: the last Linear layer + masked softmax + eq-11 loss
 * (+ alpha*KL(pi_old || pi) when logits_old != NULL, alpha = softplus(*log_alpha))
 * + dz + the last layer's backward, in one pass. Replaces actor_logits/actor_probs
 * (networks/actor.mojo:74-103), log_softmax_rows, cross_entropy/entropy/kl rows and
 * actor_backward (networks/actor_loss.mojo:194-214) down to the layer below; for the
 * critic, the last linear_forward + value_loss_grad_kernel + critic_backward's first
 * layer (networks/mlp.mojo:212-233).
 *   act [m x h] post-ReLU input (16 B aligned, h % 4 == 0, h <= 1024), w [h x a], b [a]
 *   a = 9 (actor) or 1 (critic)
 *   outputs (each optional unless noted): logits_out (masked logits / V), pi_out,
 *   dz_out [m x a]; dact [m x h] = (dz W^T) * (act > 0); dw [h x a], db [a] (required);
 *   dbact [h] = column sums of dact; stats [SPO_NUM_STATS] (required). */
SPO_API size_t spo_head_workspace_size(int64_t m, int32_t h, int32_t a);
SPO_API int spo_actor_head_fwd_bwd(spo_stream_t stream, const float* act, const float* w,
                           const float* b, int64_t m, int32_t h, int32_t a,
                           const float* mask, const float* q, const float* logits_old,
                           const float* log_alpha, float scale, float* logits_out,
                           float* pi_out, float* dz_out, float* dact, float* dw, float* db,
                           float* dbact, float* stats, void* workspace,
                           size_t workspace_bytes);
SPO_API int spo_critic_head_fwd_bwd(spo_stream_t stream, const float* act, const float* w,
                            const float* b, int64_t m, int32_t h, const float* target,
                            float scale, float* v_out, float* dv_out, float* dact, float* dw,
                            float* db, float* dbact, float* stats, void* workspace,
                            size_t workspace_bytes);

/* Loss on caller-held outputs, for a caller that runs its own forward (the reference's
 * actor_backward networks/actor_loss.mojo:194-214 starts from the logits; critic_backward
 * networks/mlp.mojo:212-233 from V). Deterministic: per-CTA partial sums in the workspace
 * (spo_loss_workspace_size bytes) are added in a fixed order.
 *
 * spo_actor_loss_fwd_bwd: mask_logits_kernel (networks/actor.mojo:50-71), log_softmax_rows
 * (ops/softmax.mojo:101-135), cross_entropy/entropy/kl rows (networks/actor_loss.mojo:40-148)
 * and logits_grad_kernel (:168-191) in one pass over logits [rows x a] (a <= 32), plus the
 * alpha*KL(pi_old || pi) term when logits_old != NULL (alpha = softplus(*log_alpha)):
 *   dz [rows x a] = ((pi - q) + alpha (pi - pi_old)) * scale, 0 where mask == 0
 *   loss_stats[SPO_STAT_ACTOR_LOSS .. SPO_STAT_KL_OLD] = scale * sums over rows
 *   *dlog_alpha (optional, device) = sigmoid(log_alpha) * (eps_kl - loss_stats[SPO_STAT_KL_OLD])
 * mask may be NULL (every action legal); log_alpha is a device scalar (NULL: 0 when
 * logits_old is NULL). Only the listed stats slots are written. scale is normally 1 / rows
 * (the reference's 1/m).
 * spo_value_loss_fwd_bwd: value_loss_grad_kernel networks/mlp.mojo:141-152 and the loss of
 * demos/train_critic.mojo:317-327 over n values: dv = (v - target) * scale,
 * loss_stats[SPO_STAT_CRITIC_LOSS] = scale * sum 0.5 (v - target)^2 (the only slot written). */
SPO_API size_t spo_loss_workspace_size(void);
SPO_API int spo_actor_loss_fwd_bwd(spo_stream_t stream, const float* logits, const float* mask,
                                   const float* q, const float* logits_old, const float* log_alpha,
                                   float eps_kl, int64_t rows, int32_t a, float scale, float* dz,
                                   float* loss_stats, float* dlog_alpha, void* workspace,
                                   size_t workspace_bytes);
SPO_API int spo_value_loss_fwd_bwd(spo_stream_t stream, const float* v, const float* target, int64_t n,
                                   float scale, float* dv, float* loss_stats, void* workspace,
                                   size_t workspace_bytes);

/* ------------------------------------------------------------------ optimiser
 * sum_squares networks/optim.mojo:115-130 without the host round trip: *out (device)
 * = sum x^2. global_clip_scale :133-142 is a pure host function. */
SPO_API size_t spo_sum_squares_workspace_size(void);
SPO_API int spo_sum_squares(spo_stream_t stream, const float* x, int64_t n, float* out,
                    void* workspace, size_t workspace_bytes);
SPO_API float spo_global_clip_scale(float total_sq, float max_norm);

/* adam_step networks/optim.mojo:172-187 (kernel :75-99) over a flat buffer:
 * g' = g * grad_scale; m = b1 m + (1-b1) g'; v = b2 v + (1-b2) g'^2;
 * p -= lr * (m / (1 - b1^step)) / (sqrt(v / (1 - b2^step)) + eps).
 * p, g, m, v 16-byte aligned; step >= 1. */
SPO_API int spo_adam_flat(spo_stream_t stream, float* p, const float* g, float* m, float* v,
                  int64_t n, float lr, float b1, float b2, float eps, int32_t step,
                  float grad_scale);

/* ema_update networks/optim.mojo:163-169 (kernel :145-160):
 * target = tau * online + (1 - tau) * target. */
SPO_API int spo_ema(spo_stream_t stream, float* target, const float* online, int64_t n, float tau);

/* truncated_gae rl_utils/multistep.mojo:72-82 (kernel :40-69), batch-major [B, T]. */
SPO_API int spo_truncated_gae(spo_stream_t stream, float* adv, float* targets, const float* reward,
                      const float* discount, const float* v_tm1, const float* v_t,
                      const float* truncation, int64_t batch, int32_t t_len, float lambda);

/* ------------------------------------------------------------------ compute peaks
 * No reference counterpart. Measured peaks of the two arithmetic paths of this library on
 * the current device: tf32_flops = tcgen05.mma.kind::tf32 128x128x8 issued back to back
 * from shared memory, one CTA per SM; fp32_flops = packed FFMA2 chains on every SM.
 * FLOP/s; a few tens of ms of GPU time. */
SPO_API int spo_measure_peaks(spo_stream_t stream, double* tf32_flops, double* fp32_flops);

/* ------------------------------------------------------------------ replay buffer, device side
 * TrajectoryBuffer.sample_indices rl_utils/buffer.mojo:138-152: idx[i] =
 * rand_bits(seed, stream_id, i) % count (ops/rng.mojo:43-58), i < n, with replacement.
 * count == 0 is rejected ("the buffer is empty"). */
SPO_API int spo_replay_sample(spo_stream_t stream, int32_t* idx, int64_t n, int64_t count, uint32_t seed,
                              uint32_t stream_id);

/* TrajectoryBuffer.gather / gather_steps / gather_bootstrap / gather_q
 * rl_utils/buffer.mojo:154-211: dst[k, :] = src[idx[k], :] for k < n, span floats per
 * sequence, in the order of idx, repeats allowed. An index outside [0, count) gives a zero
 * row and sets *err (optional) to 1 (the reference raises on the host). */
SPO_API int spo_replay_gather(spo_stream_t stream, float* dst, const float* src, const int32_t* idx,
                              int64_t n, int64_t span, int64_t count, int32_t* err);

/* ttt_encode_obs_kernel envs/tictactoe.mojo:449-480 and ttt_legal_mask_from_obs_kernel
 * :577-597: board cells [n x 9] coded +1 agent / -1 rival / 0 empty -> obs [n x 27], the
 * plane-major 0/1 planes [empty | agent | rival], and mask [n x 9] (optional) = empty. */
SPO_API int spo_encode_obs(spo_stream_t stream, float* obs, float* mask, const float* cells, int64_t n);

/* ------------------------------------------------------------------ tensor-core GEMM
 * The hidden-layer products of linear_forward / linear_backward
 * (networks/linear.mojo:37-167) on sm_100a tensor cores (tcgen05, TF32 inputs, fp32
 * accumulation) at near-fp32 accuracy through the 3xTF32 split: every operand is a pair
 * of TF32 values (hi, lo) with hi = round-to-nearest TF32 of x and lo = the same rounding
 * of x - hi (spo_split_tf32), and C = lo_A hi_B + hi_A lo_B + hi_A hi_B.
 *   SPO_TC_FWD     C = relu(A B^T + bias) -> (c_hi, c_lo) split, A [m x k], B [n x k]
 *   SPO_TC_DX      C = (A B^T) * (mask > 0) -> (c_hi, c_lo), column sums -> colsum
 *   SPO_TC_DX_F32  as SPO_TC_DX, C written as plain fp32 to c_hi
 *   SPO_TC_DW      C = A^T B from A [k x m], B [k x n], rows of k split in chunks of
 *                  k_chunk, one fp32 partial per chunk -> c_part [splits][m x n]
 * Shapes: n % 128 == 0; FWD/DX: k % 32 == 0, n <= 1024 for DX; DW: m % 128 == 0.
 * Plain fp32 operands: with a_lo == NULL, A is plain fp32 in a_hi and the kernel splits it
 * into its TF32 halves in shared memory (forward, dX: B must be a pair; dW: b_lo == NULL
 * too, both operands plain fp32). With c_lo == NULL, SPO_TC_FWD writes plain fp32 (and
 * c_bits when set).
 * colsum receives [grid][n] partials (grid from spo_tc_gemm_shape). All pointers
 * 16-byte aligned. err (optional) receives a nonzero code if a bounded wait of the
 * kernel gave up (the kernel then returns without hanging).
 * ReLU masks packed one bit per element (row-major [m x n/32] 32-bit words, bit j of
 * word w = column 32 w + j; 8-byte aligned): SPO_TC_FWD writes c_bits (bit = output > 0)
 * when it is set; SPO_TC_DX* read mask_bits instead of mask when it is set. */
#define SPO_TC_FWD 0
#define SPO_TC_DX 1
#define SPO_TC_DX_F32 2
#define SPO_TC_DW 3
typedef struct spo_tc_gemm_desc {
  int32_t kind;
  const float* a_hi;
  const float* a_lo;
  const float* b_hi;
  const float* b_lo;
  int64_t m, n, k, k_chunk;
  const float* bias;
  const float* mask;
  float* c_hi;
  float* c_lo;
  float* c_part;
  float* colsum;
  int32_t* err;
  const uint32_t* mask_bits;
  uint32_t* c_bits;
} spo_tc_gemm_desc;
SPO_API int spo_tc_gemm_shape(const spo_tc_gemm_desc* desc, int32_t* grid, int32_t* splits);
SPO_API int spo_tc_gemm(spo_stream_t stream, const spo_tc_gemm_desc* desc);
/* No reference counterpart: a test of the kernel's failure path. Runs spo_tc_gemm with the
 * operands of each CTA's first k-block never loaded and every bounded wait limited to
 * wait_us microseconds (1 .. 2,000,000; spo_tc_gemm waits up to 2 s). The MMA issuer's wait
 * for the missing stage runs out: the kernel stops its roles, waits (bounded) for the copies
 * and MMAs it issued, frees its tensor memory, writes a nonzero code to *desc->err (required)
 * and returns. The output is undefined; the device stays usable. */
SPO_API int spo_tc_gemm_withheld(spo_stream_t stream, const spo_tc_gemm_desc* desc, int64_t wait_us);
/* hi/lo split of n floats; keep_positive: positive x never get hi == 0 (ReLU outputs). */
SPO_API int spo_split_tf32(spo_stream_t stream, float* hi, float* lo, const float* x, int64_t n,
                           int32_t keep_positive);

/* ------------------------------------------------------------------ learner step
 * One M-step update of the actor and/or critic, demos/train_spo.mojo:417-554 and
 * demos/train_critic.mojo:280-363 (minus target construction): forward, loss,
 * backward, per-network global-norm clip (optional) and Adam, with the log_alpha dual.
 *
 * Flat buffers (params, grads, adam_m, adam_v) share one layout:
 *   [actor tensors | critic tensors | log_alpha slot | statistics slot]
 * given by spo_learner_layout. Gradients and loss statistics are contiguous so a
 * data-parallel caller reduces them with ONE all-reduce between
 * spo_learner_backward and spo_learner_apply. */
typedef struct spo_learner_desc {
  spo_mlp_desc actor;   /* num_layers == 0: no actor */
  spo_mlp_desc critic;  /* num_layers == 0: no critic */
  int64_t max_rows;     /* largest batch (rows on this rank) per call */
  float lr_actor, lr_critic, beta1, beta2, adam_eps;
  float max_grad_norm;  /* <= 0 or inf: no clip (reference: 0.5, demos/train_spo.mojo:68) */
  float kl_eps;         /* dual target epsilon */
  int32_t use_kl;       /* alpha * KL(pi_old || pi) term (needs batch.logits_old) */
  int32_t dual;         /* update log_alpha with the dual gradient */
  int32_t engine;       /* 0: tensor cores (3xTF32 tcgen05) for the hidden x hidden layers
                           when every hidden width is a multiple of 128 and <= 1024;
                           1: CUDA cores (fp32 FMA) for every layer */
} spo_learner_desc;

typedef struct spo_learner_layout {
  int64_t actor_offset, actor_size;   /* floats; size = padded flat size */
  int64_t critic_offset, critic_size;
  int64_t alpha_index;                /* log_alpha */
  int64_t stats_offset;               /* SPO_NUM_STATS loss statistics (in grads) */
  int64_t total;                      /* length of every flat buffer */
  int64_t actor_w_off[SPO_MAX_LAYERS], actor_b_off[SPO_MAX_LAYERS];
  int64_t critic_w_off[SPO_MAX_LAYERS], critic_b_off[SPO_MAX_LAYERS];
} spo_learner_layout;

typedef struct spo_batch {
  const float* obs;        /* [rows x d0] */
  const float* mask;       /* [rows x A] 1 legal / 0 illegal (actor) */
  const float* q;          /* [rows x A] target policy (actor) */
  const float* logits_old; /* [rows x A] pi_old logits (actor, use_kl) */
  const float* target;     /* [rows] critic targets */
  int64_t rows;
  /* Board cells [rows x 9] (+1 agent / -1 rival / 0 empty), used when obs is null: the
   * first layers read the 27-wide [empty | agent | rival] encoding of the cells
   * (ttt_encode_obs_kernel, envs/tictactoe.mojo:449-480) and, when mask is null too, the
   * actor's legal mask is the empty plane (envs/tictactoe.mojo:577-597). */
  const float* cells;
} spo_batch;

typedef struct spo_train_state {
  float* params;   /* flat, learner layout */
  float* grads;    /* flat, learner layout (gradients + statistics) */
  float* adam_m;
  float* adam_v;
  int32_t* step;   /* device counter of Adam steps taken (starts at 0) */
  float* report;   /* device [SPO_REPORT_SIZE] or NULL */
} spo_train_state;

typedef struct spo_learner* spo_learner_t;

SPO_API int spo_learner_layout_of(const spo_learner_desc* desc, spo_learner_layout* out);
SPO_API size_t spo_learner_workspace_size(const spo_learner_desc* desc);
SPO_API int spo_learner_create(const spo_learner_desc* desc, void* workspace, size_t workspace_bytes,
                       spo_learner_t* out);
SPO_API int spo_learner_destroy(spo_learner_t learner);
/* Forward + loss + backward: writes grads (and the statistics slot). grad_scale is
 * 1 / (global batch rows): 1 / batch->rows on one GPU. */
SPO_API int spo_learner_backward(spo_learner_t learner, spo_stream_t stream, const spo_batch* batch,
                         float grad_scale, const spo_train_state* state);
/* Optional clip, Adam over the flat buffers, dual update; increments *step. */
SPO_API int spo_learner_apply(spo_learner_t learner, spo_stream_t stream, const spo_train_state* state);
/* The activation cache of the last forward (CriticCache a1, a2, ...,
 * networks/mlp.mojo:84-102): device pointers to the post-ReLU activations of hidden layer
 * `layer` (0-based, [rows x d_{layer+1}]) of network `which` (0 actor, 1 critic). With the
 * tensor-core engine the activations that feed tensor-core products are stored as TF32
 * hi/lo pairs (value = hi + lo) and *lo is set; otherwise (the CUDA-core engine, and the
 * last hidden layer, which only the fused head reads) *lo is NULL and *hi is the plain
 * fp32 value. Valid until the next call on the learner. */
SPO_API int spo_learner_cache(spo_learner_t learner, int32_t which, int32_t layer,
                              const float** hi, const float** lo);
/* Reads (synchronously) and clears the learner's device error word: 0 when every
 * bounded wait of its kernels completed since the last call (tensor-core GEMM waits 1-6,
 * a grid-barrier wait of the one-launch step 16, its weight copies 17; a step whose wait
 * ran out applied no update). */
SPO_API int spo_learner_status(spo_learner_t learner, int32_t* device_error);
/* Batches of at most max_rows rows run the whole step (or the backward of
 * spo_learner_backward) as ONE cooperative launch whose phases are separated by grid-wide
 * barriers, instead of ~10 dependent launches; 0 turns that off. The default is
 * min(8192, desc.max_rows) when every network has 2-4 layers, an input at most 32 wide,
 * hidden widths that are multiples of 32 up to 256, at most 65,536 parameters, and its
 * weights, biases and a 32-row block of activations fit in 220 KB of shared memory (else
 * 0, and nonzero values are refused). Results agree with the multi-launch path within the
 * fp32 tolerances; the reduction order of the partial sums differs, so the two are not
 * bit-identical. The first such step on a parameter buffer copies the tensor maps of its
 * weights into the workspace (stream-ordered); under stream capture that step is refused
 * (SPO_ERR_UNSUPPORTED): run one step on the buffer before capturing.
 * No reference counterpart (the reference's update() is ~35 launches,
 * demos/train_spo.mojo:417-554). */
SPO_API int spo_learner_set_small_rows(spo_learner_t learner, int64_t max_rows);
/* No reference counterpart: a test of the one-launch step's failure path. Runs the
 * one-launch step of spo_learner_step on batch (which must take it: 1 <= rows <= the
 * small-rows limit) with the first CTA's arrival at the first grid-wide barrier withheld
 * and every barrier wait limited to wait_us microseconds (1 .. 2,000,000; the step itself
 * waits up to 2 s). The other CTAs' waits run out: the step is aborted (no gradient is
 * written, no parameter, moment or step counter changes), the learner's error word gets a
 * nonzero code (spo_learner_status) and the barrier words are reset for the next step. */
SPO_API int spo_learner_step_withheld(spo_learner_t learner, spo_stream_t stream, const spo_batch* batch,
                                      const spo_train_state* state, int64_t wait_us);
/* backward (grad_scale = 1 / rows) + apply. */
SPO_API int spo_learner_step(spo_learner_t learner, spo_stream_t stream, const spo_batch* batch,
                     const spo_train_state* state);
/* Forward only of one network of the learner (inference for the search heads,
 * envs/tictactoe_actor.mojo:148-171 / tictactoe_critic.mojo:193-232): out [rows x dL];
 * for the actor, pi_out (optional) receives the masked softmax. which: 0 actor,
 * 1 critic. */
SPO_API int spo_learner_forward(spo_learner_t learner, spo_stream_t stream, int32_t which,
                        const float* params, const float* obs, const float* mask, int64_t rows,
                        float* out, float* pi_out);

/* ------------------------------------------------------------------ data parallel
 * One process per GPU. The caller shares the 128-byte unique id (e.g. through
 * torch.distributed) and creates a communicator per rank; spo_allreduce_sum is an
 * in-place float32 sum (ncclAllReduce) on `stream`. */
typedef struct spo_comm* spo_comm_t;
#define SPO_COMM_ID_BYTES 128
SPO_API int spo_comm_get_unique_id(void* id_out);
SPO_API int spo_comm_init(spo_comm_t* out, const void* id, int32_t nranks, int32_t rank);
SPO_API int spo_comm_destroy(spo_comm_t comm);
SPO_API int spo_allreduce_sum(spo_comm_t comm, spo_stream_t stream, float* buf, int64_t n);

#ifdef __cplusplus
}
#endif

#endif /* SPO_CUDA_H_ */
