// Internal kernel interfaces of libspo_cuda (not part of the C ABI).
#pragma once

#include "spo_common.cuh"

namespace spo {

// ---------------------------------------------------------------- loss statistics
// Slots of the statistics vector (scaled sums: means when scale = 1/batch).
enum StatSlot : int {
  kStatActorLoss = 0,   // CE + alpha * KL(pi_old || pi)
  kStatCE = 1,          // -sum q log pi              (networks/actor_loss.mojo:40-65)
  kStatEntropy = 2,     // H(q)                        (networks/actor_loss.mojo:105-116)
  kStatKLq = 3,         // KL(q || pi) = CE - H(q)     (networks/actor_loss.mojo:119-124)
  kStatKLold = 4,       // KL(pi_old || pi)
  kStatCriticLoss = 5,  // 0.5 (V - t)^2               (demos/train_critic.mojo:317-327)
  kStats = 8,
};

// ---------------------------------------------------------------- fused head
enum HeadMode : int { kHeadActor = 0, kHeadCritic = 1 };

struct HeadParams {
  const float* act;        // [M x H] post-ReLU input of the last Linear layer
  const float* act_lo;     // optional: lo half when act is stored as a TF32 hi/lo pair
  const float* W;          // [H x A]
  const float* b;          // [A]
  int64_t M;
  int H, A;
  int mode;                // kHeadActor / kHeadCritic
  int rows_per_tile;       // set by head_launch
  const float* mask;       // actor: [M x A] 1 legal / 0 illegal (null: all legal)
  const float* cells;      // actor, mask null: board cells [M x 9]; legal = empty (0)
  const float* q;          // actor: [M x A] target policy
  const float* z_old;      // actor: [M x A] pi_old logits, or null (no KL term)
  const float* log_alpha;  // actor: device scalar, or null (use alpha_host)
  float alpha_host;
  const float* target;     // critic: [M x A]
  float scale;             // gradient scale (1 / global batch)
  float* out_logits;       // optional [M x A]: masked logits (actor) or V (critic)
  float* out_pi;           // optional [M x A]: pi (actor)
  float* dz_out;           // optional [M x A]: dL/dz
  float* dX;               // optional [M x H]: (dz W^T) * [act > 0]
  float* dX_lo;            // optional: write dX as a TF32 hi/lo pair (dX = hi)
  float* dW_part;          // [grid][H x A]
  float* db_part;          // [grid][A]
  float* dbx_part;         // optional [grid][H]: column sums of dX
  float* stats_part;       // optional [grid][kStats]
};

int head_rows_per_tile(int64_t M, int H, bool has_lo, int A);
size_t head_smem_bytes(int H, int A, bool has_lo);
int head_grid(const HeadParams& p);  // CTAs of the launch = partial-sum slots written
int head_launch(HeadParams p, int grid, cudaStream_t s);

// ---------------------------------------------------------------- losses on caller-held outputs
// (loss.cu). part: [loss_parts_max()][kStats] floats of scratch.
int64_t loss_parts_max();
int actor_loss_launch(const float* z, const float* mask, const float* q, const float* z_old,
                      const float* log_alpha, float eps_kl, int64_t rows, int A, float scale, float* dz,
                      float* stats, float* dlog_alpha, float* part, cudaStream_t s);
int value_loss_launch(const float* v, const float* target, int64_t n, float scale, float* dv, float* stats,
                      float* part, cudaStream_t s);

// ---------------------------------------------------------------- partial-sum reduction
constexpr int kMaxSegs = 80;

struct ReduceSeg {
  const float* src;        // parts x part_stride floats
  float* dst;              // count floats
  int64_t count;
  int64_t part_stride;
  int32_t parts;
};

struct ReduceParams {
  ReduceSeg seg[kMaxSegs];
  int nseg;
};

int reduce_launch(const ReduceParams& p, cudaStream_t s);

// ---------------------------------------------------------------- optimiser
constexpr int kMaxGroups = 4;
constexpr int kSumsqParts = 128;  // CTAs of the sum-of-squares pass

struct AdamGroup {
  int64_t begin, end;      // [begin, end) in the flat buffers, multiples of 4
  float lr;
  float max_norm;          // clip when finite and > 0
};

struct AdamParams {
  float* p;
  float* g;
  float* m;
  float* v;
  AdamGroup grp[kMaxGroups];
  int ngrp;
  float b1, b2, eps;
  float grad_scale;        // multiplies every gradient (1 in the learner)
  const float* sumsq_part; // [ngrp][kSumsqParts] or null (no clipping)
  int* step;               // device step counter (t = *step + 1) or null
  unsigned* ticket;        // completion counter for the step update (with step)
  int host_step;           // used when step == null
  int64_t alpha_index;     // flat index of log_alpha, or -1
  const float* kl_stat;    // device: mean KL(pi_old || pi) of the batch (global)
  float kl_eps;
  float* report;           // optional device [kReportSize]
};

enum ReportSlot : int {
  kRepNorm0 = 0,           // per-group global norms (kMaxGroups)
  kRepClip0 = 4,           // per-group clip scales (kMaxGroups)
  kRepDlogAlpha = 8,
  kRepStep = 9,
  kReportSize = 16,
};

int sumsq_groups_launch(const float* g, const AdamGroup* grp, int ngrp, float* part,
                        cudaStream_t s);
int adam_launch(const AdamParams& p, int64_t n, cudaStream_t s);
int sumsq_launch(const float* x, int64_t n, float* part, float* out, cudaStream_t s);
int ema_launch(float* target, const float* online, int64_t n, float tau, cudaStream_t s);

// ---------------------------------------------------------------- row-wise kernels
int mask_logits_launch(float* logits, const float* mask, int64_t n, cudaStream_t s);
int softmax_rows_launch(float* out, const float* in, int64_t rows, int cols, int mode,
                        cudaStream_t s);  // mode 0 softmax, 1 log_softmax, 2 logsumexp
int ce_rows_launch(float* out, const float* q, const float* log_pi, int64_t rows, int cols,
                   cudaStream_t s);
int entropy_rows_launch(float* out, const float* q, int64_t rows, int cols, cudaStream_t s);
int kl_rows_launch(float* out, const float* ce, const float* h, int64_t rows, cudaStream_t s);
int logits_grad_launch(float* dz, const float* pi, const float* q, const float* mask,
                       int64_t n, float scale, cudaStream_t s);
int value_grad_launch(float* dv, const float* v, const float* t, int64_t n, float scale,
                      cudaStream_t s);
int relu_launch(float* a, int64_t n, cudaStream_t s);
int relu_bwd_launch(float* g, const float* act, int64_t n, cudaStream_t s);
// part[c][n] = sum of rows [c*per, (c+1)*per) of x [rows x n], per = ceil(rows / chunks).
// Rows of a first layer's input: x [rows x k] fp32, or (x null) board cells [rows x 9]
// coded +1 agent / -1 rival / 0 empty, read as the 27-wide [empty | agent | rival] planes.
struct LayerInput {
  const float* x;
  const float* cells;
};

// y = relu(x W + b) for inputs at most 32 wide (input_layer.cu): y fp32, or a TF32 hi/lo
// pair (y = hi) when y_lo is set; bits (optional): packed y > 0, [rows x n/32] words.
bool fwd_skinny_ok(int64_t k, int64_t n);
int fwd_skinny_launch(LayerInput in, const float* w, const float* b, int64_t rows, int64_t k, int64_t n,
                      float* y, float* y_lo, uint32_t* bits, cudaStream_t s);

// The first layer on tensor cores: input rows [rows x k] (k <= 32) padded to 32 columns as
// plain fp32 (lo null) or TF32 hi/lo pairs, and W [k x n] as W^T [n x 32] hi/lo pairs
// (zeros past k).
int pad_split_input_launch(LayerInput in, int64_t k, int64_t rows, float* hi, float* lo, cudaStream_t s);
int split_weights_t_pad_launch(const float* w, int64_t k, int64_t n, float* wt_hi, float* wt_lo, cudaStream_t s);

// dW = x^T dY for inputs at most 32 wide (input_layer.cu): per-chunk partials
// part[chunk][k x n], *parts chunks (at most dw_skinny_max_parts()).
bool dw_skinny_ok(int64_t k, int64_t n);
int64_t dw_skinny_max_parts();
int dw_skinny_launch(LayerInput in, const float* dy, int64_t rows, int64_t k, int64_t n, float* part,
                     int* parts, cudaStream_t s);

int colsum_part_launch(const float* x, int64_t rows, int64_t n, int64_t chunks, float* part,
                       cudaStream_t s);
// peaks.cu: measured TF32 tensor and FP32 FMA peaks (FLOP/s)
int measure_peaks(double* tf32_flops, double* fp32_flops, cudaStream_t s);

// replay.cu: replay sampling / gather and observation encoding
int replay_sample_launch(int32_t* idx, int64_t n, int64_t count, uint32_t seed, uint32_t stream,
                         cudaStream_t s);
int replay_gather_launch(float* dst, const float* src, const int32_t* idx, int64_t n, int64_t span,
                         int64_t count, int* err, cudaStream_t s);
int encode_obs_launch(float* obs, float* mask, const float* cells, int64_t n, cudaStream_t s);

int gae_launch(float* adv, float* targets, const float* r, const float* discount,
               const float* v_tm1, const float* v_t, const float* trunc, int64_t batch,
               int t_len, float lambda, cudaStream_t s);

}  // namespace spo
