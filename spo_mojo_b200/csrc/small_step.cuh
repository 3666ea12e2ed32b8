// The one-launch learner step for small batches (small_step.cu): parameters and limits.
#pragma once

#include "kernels.cuh"

namespace spo {

constexpr int kSmallMaxLayers = 4;     // Linear layers per network
constexpr int kSmallMaxHidden = 256;   // hidden widths: multiples of 32, at most this
constexpr int kSmallMaxIn = 32;        // input width
constexpr int kSmallMaxA = 9;          // output width (9 actions, or 1 value)
constexpr int kSmallMaxS = 16;         // row chunks of a dW product
constexpr int64_t kSmallDefaultRows = 8192;

__host__ __device__ inline int64_t ceil_div_dev(int64_t a, int64_t b) { return (a + b - 1) / b; }

struct SmallNet {
  int L;                               // Linear layers (0: no such network)
  int dims[kSmallMaxLayers + 1];
  int mode;                            // 0 actor (9 actions), 1 critic (1 value)
  const float* W[kSmallMaxLayers];     // W_l [d_l x d_{l+1}], b_l: views of the params
  const float* b[kSmallMaxLayers];
  float* act[kSmallMaxLayers - 1];     // post-ReLU a_l [rows x d_{l+1}]
  float* dz[2];                        // gradients flowing down, ping-pong [rows x <= max width]
  float* pw[kSmallMaxLayers];          // dW partials [S_l][d_l x d_{l+1}]
  float* pb[kSmallMaxLayers];          // db partials [S_l][d_{l+1}]
  int S[kSmallMaxLayers];              // row chunks of layer l's dW
  float* pstats;                       // loss statistics per CTA [grid][kStats]
};

struct SmallStepParams {
  SmallNet net[2];                     // actor, critic
  const float* obs;                    // [rows x d0], or null: cells
  const float* cells;                  // [rows x 9] board cells
  const float* mask;                   // actor [rows x 9] (null: the empty cells)
  const float* q;
  const float* z_old;                  // pi_old logits (null: no KL term)
  const float* target;                 // critic [rows]
  const float* log_alpha;
  int64_t rows;
  float scale;                         // gradient scale (1 / global batch)
  ReduceParams red;                    // partials -> flat gradients
  int apply;                           // clip (optional) and Adam after the backward
  int clip;
  AdamParams adam;
  int64_t total;                       // length of the flat buffers
  float* sumsq;                        // [kMaxGroups][grid]
  unsigned* sync;                      // [0] barrier arrivals, [1] exits, [2] abort; zero between launches
  int* err;                            // learner error word
  uint64_t wait_ns;                    // limit of every barrier wait
};

int small_step_grid();                 // CTAs of a launch (all co-resident), 0 if unavailable
int small_step_launch(const SmallStepParams& p, int grid, cudaStream_t s);

}  // namespace spo
