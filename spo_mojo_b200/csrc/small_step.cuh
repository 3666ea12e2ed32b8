// The one-launch learner step for small batches (small_step.cu): parameters and limits.
#pragma once

#include <cuda.h>

#include "spo_cuda.h"
#include "kernels.cuh"

namespace spo {

constexpr int kSmallMaxLayers = 4;     // Linear layers per network
constexpr int kSmallMaxHidden = 256;   // hidden widths: multiples of 32, at most this
constexpr int kSmallMaxIn = 32;        // input width
constexpr int kSmallMaxA = 9;          // output width (9 actions, or 1 value)
constexpr int64_t kSmallMaxParams = 65536;   // weights + biases per network (partials per CTA)
constexpr int64_t kSmallDefaultRows = 8192;
constexpr size_t kSmallMaxSmem = 220 * 1024;   // dynamic shared memory of every launch

struct SmallNet {
  int L;                               // Linear layers (0: no such network)
  int dims[kSmallMaxLayers + 1];
  int mode;                            // 0 actor (9 actions), 1 critic (1 value)
  const float* W[kSmallMaxLayers];     // W_l [d_l x d_{l+1}], b_l: views of the params
  const float* b[kSmallMaxLayers];
  float* pw[kSmallMaxLayers];          // dW partials [parts][d_l x d_{l+1}]
  float* pb[kSmallMaxLayers];          // db partials [parts][d_{l+1}]
  float* pstats;                       // loss statistics [parts][kStats]
  float* gact[kSmallMaxLayers - 1];    // the activation cache a_l [rows x d_{l+1}] (or null)
};

struct SmallStepParams {
  SmallNet net[2];                     // actor, critic
  // [2][kSmallMaxLayers - 1] in device memory: per network, its hidden layers' W_l
  // [d_l x d_{l+1}] as boxes of 32 columns x wrows rows (32 for the first layer, d_l after
  // it), 128-byte swizzle, zero fill past d_l (kept out of the launch parameters, whose
  // size every launch pays for)
  const CUtensorMap* wmap;
  const float* obs;                    // [rows x d0], or null: cells
  const float* cells;                  // [rows x 9] board cells
  const float* mask;                   // actor [rows x 9] (null: the empty cells)
  const float* q;
  const float* z_old;                  // pi_old logits (null: no KL term)
  const float* target;                 // critic [rows]
  const float* log_alpha;
  int64_t rows;
  int64_t rows_per_cta;                // CTA c owns rows [c * rows_per_cta, ...)
  int parts;                           // CTAs with rows (= partials per sum)
  float scale;                         // gradient scale (1 / global batch)
  ReduceParams red;                    // partials -> flat gradients
  int64_t seg_start[kMaxSegs];         // first reduced element of each segment
  int64_t flat_index[kMaxSegs];        // its index in the flat buffers
  int64_t total_red;                   // reduced elements
  int apply;                           // clip (optional) and Adam after the backward
  int clip;
  AdamParams adam;
  int64_t total;                       // length of the flat buffers
  float* sumsq;                        // [kMaxGroups][grid]
  unsigned* sync;                      // [0] barrier arrivals (bit 30: abort), [1] exits; zero between launches
  int* err;                            // learner error word
  uint64_t wait_ns;                    // limit of every barrier wait
  uint32_t withhold;                   // a test of the bounded waits: 1 + the CTA whose first
                                       // barrier arrival is withheld (0: none)
};

// Dynamic shared memory of the nets' row blocks (the largest of the given networks).
size_t small_step_smem(const spo_mlp_desc* nets, int count);
int small_step_grid();                 // CTAs of a launch (all co-resident), 0 if unavailable
int small_step_launch(const SmallStepParams& p, int grid, size_t smem, cudaStream_t s);
// The tensor map of hidden layer l's W (rows d_l, columns d_{l+1}) for the small step.
int small_weight_map(CUtensorMap* m, const float* W, int l, int rows, int cols);

}  // namespace spo
