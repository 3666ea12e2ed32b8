// Row-wise and elementwise kernels behind the reference-shaped entry points
// (the pieces the fused head combines; exposed so a caller can run the reference's
// step-by-step composition). The softmax family: one thread per row up to 16 columns,
// one warp per row beyond; one thread per row or element for the rest.
//
//   mask_logits_kernel        networks/actor.mojo:50-71
//   softmax_rows / log_softmax_rows / logsumexp_rows   ops/softmax.mojo:29-135
//   cross_entropy_rows_kernel networks/actor_loss.mojo:40-65
//   entropy_rows_kernel       networks/actor_loss.mojo:105-116
//   kl_rows_kernel            networks/actor_loss.mojo:119-124
//   logits_grad_kernel        networks/actor_loss.mojo:168-191
//   value_loss_grad_kernel    networks/mlp.mojo:141-152
//   relu_kernel / relu_backward_kernel   networks/mlp.mojo:34-46, 155-166
//   gae_kernel                rl_utils/multistep.mojo:40-69
#include "kernels.cuh"

namespace spo {

namespace {

constexpr int kThreads = 256;

int blocks(int64_t n) {
  return (int)std::max<int64_t>(1, std::min<int64_t>(ceil_div(n, kThreads), 16LL * sm_count()));
}

#define GRID_STRIDE(i, n)                                                     \
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < (n); \
       i += (int64_t)gridDim.x * blockDim.x)

__global__ void mask_logits_kernel(float* logits, const float* mask, int64_t n) {
  GRID_STRIDE(i, n) {
    if (mask[i] == 0.f) logits[i] = kNegInf;
  }
}

// One warp per row; mode 0 = softmax, 1 = log_softmax, 2 = logsumexp (one value per row).
__global__ void softmax_rows_kernel(float* out, const float* in, int64_t rows, int cols, int mode) {
  const int lane = threadIdx.x & 31;
  const int64_t warp = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int64_t nwarps = ((int64_t)gridDim.x * blockDim.x) >> 5;
  for (int64_t r = warp; r < rows; r += nwarps) {
    const float* a = in + r * cols;
    float mx = kNegInf;
    for (int c = lane; c < cols; c += 32) mx = fmaxf(mx, a[c]);
    mx = warp_max(mx);
    float s = 0.f;
    for (int c = lane; c < cols; c += 32) s += expf(a[c] - mx);
    s = warp_sum(s);
    if (mode == 2) {
      if (lane == 0) out[r] = mx + logf(s);
    } else if (mode == 1) {
      const float lse = mx + logf(s);
      for (int c = lane; c < cols; c += 32) out[r * cols + c] = a[c] - lse;
    } else {
      for (int c = lane; c < cols; c += 32) out[r * cols + c] = expf(a[c] - mx) / s;
    }
  }
}

// The same for rows of at most kThreadCols columns (the 9 actions): one row per thread,
// its maximum and sum taken serially in column order with no exchange between lanes.
constexpr int kThreadCols = 16;
__global__ void softmax_rows_thread_kernel(float* out, const float* in, int64_t rows, int cols, int mode) {
  GRID_STRIDE(r, rows) {
    const float* a = in + r * cols;
    float v[kThreadCols];
    float mx = kNegInf;
#pragma unroll
    for (int c = 0; c < kThreadCols; ++c) {
      v[c] = c < cols ? a[c] : kNegInf;
      mx = fmaxf(mx, v[c]);
    }
    float s = 0.f;
#pragma unroll
    for (int c = 0; c < kThreadCols; ++c)
      if (c < cols) s += expf(v[c] - mx);
    if (mode == 2) {
      out[r] = mx + logf(s);
    } else if (mode == 1) {
      const float lse = mx + logf(s);
#pragma unroll
      for (int c = 0; c < kThreadCols; ++c)
        if (c < cols) out[r * cols + c] = v[c] - lse;
    } else {
#pragma unroll
      for (int c = 0; c < kThreadCols; ++c)
        if (c < cols) out[r * cols + c] = expf(v[c] - mx) / s;
    }
  }
}

__global__ void ce_rows_kernel(float* out, const float* q, const float* lp, int64_t rows, int cols) {
  GRID_STRIDE(r, rows) {
    float acc = 0.f;
    for (int a = 0; a < cols; ++a) {
      const float w = q[r * cols + a];
      if (w != 0.f) acc += w * lp[r * cols + a];
    }
    out[r] = -acc;
  }
}

__global__ void entropy_rows_kernel(float* out, const float* q, int64_t rows, int cols) {
  GRID_STRIDE(r, rows) {
    float acc = 0.f;
    for (int a = 0; a < cols; ++a) {
      const float w = q[r * cols + a];
      if (w > 0.f) acc += w * logf(w);
    }
    out[r] = -acc;
  }
}

__global__ void kl_rows_kernel(float* out, const float* ce, const float* h, int64_t rows) {
  GRID_STRIDE(r, rows) out[r] = ce[r] - h[r];
}

__global__ void logits_grad_kernel(float* dz, const float* pi, const float* q, const float* mask,
                                   int64_t n, float scale) {
  GRID_STRIDE(i, n) dz[i] = (mask != nullptr && mask[i] == 0.f) ? 0.f : (pi[i] - q[i]) * scale;
}

__global__ void value_grad_kernel(float* dv, const float* v, const float* t, int64_t n, float scale) {
  GRID_STRIDE(i, n) dv[i] = (v[i] - t[i]) * scale;
}

__global__ void relu_kernel(float* a, int64_t n) {
  GRID_STRIDE(i, n) {
    if (a[i] < 0.f) a[i] = 0.f;
  }
}

__global__ void relu_bwd_kernel(float* g, const float* act, int64_t n) {
  GRID_STRIDE(i, n) {
    if (act[i] <= 0.f) g[i] = 0.f;
  }
}

__global__ void gae_kernel(float* adv, float* targets, const float* r, const float* disc,
                           const float* v_tm1, const float* v_t, const float* trunc,
                           int64_t batch, int t_len, float lambda) {
  GRID_STRIDE(b, batch) {
    float acc = 0.f;
    for (int i = t_len - 1; i >= 0; --i) {
      const int64_t idx = b * t_len + i;
      const float delta = r[idx] + disc[idx] * v_t[idx] - v_tm1[idx];
      acc = delta + disc[idx] * lambda * acc * (1.f - trunc[idx]);
      adv[idx] = acc;
      targets[idx] = v_tm1[idx] + acc;
    }
  }
}

__global__ void colsum_part_kernel(const float* x, int64_t rows, int64_t n, int64_t per,
                                   float* part) {
  __shared__ float sh[8][33];
  const int64_t col = (int64_t)blockIdx.x * 32 + threadIdx.x;
  const int64_t r0 = (int64_t)blockIdx.y * per;
  const int64_t r1 = min(rows, r0 + per);
  float acc = 0.f;
  if (col < n)
    for (int64_t r = r0 + threadIdx.y; r < r1; r += 8) acc += x[r * n + col];
  sh[threadIdx.y][threadIdx.x] = acc;
  __syncthreads();
  if (threadIdx.y == 0 && col < n) {
    float t = 0.f;
#pragma unroll
    for (int y = 0; y < 8; ++y) t += sh[y][threadIdx.x];
    part[(int64_t)blockIdx.y * n + col] = t;
  }
}

}  // namespace

int colsum_part_launch(const float* x, int64_t rows, int64_t n, int64_t chunks, float* part,
                       cudaStream_t s) {
  if (n <= 0 || chunks <= 0) return kOk;
  const int64_t per = ceil_div(std::max<int64_t>(rows, 1), chunks);
  colsum_part_kernel<<<dim3((unsigned)ceil_div(n, 32), (unsigned)chunks), dim3(32, 8), 0, s>>>(
      x, rows, n, per, part);
  SPO_LAUNCH_CHECK();
  return kOk;
}

#define LAUNCH_1D(kernel, n, ...)                         \
  do {                                                    \
    if ((n) <= 0) return kOk;                             \
    kernel<<<blocks(n), kThreads, 0, s>>>(__VA_ARGS__);   \
    SPO_LAUNCH_CHECK();                                   \
    return kOk;                                           \
  } while (0)

int mask_logits_launch(float* logits, const float* mask, int64_t n, cudaStream_t s) {
  LAUNCH_1D(mask_logits_kernel, n, logits, mask, n);
}

int softmax_rows_launch(float* out, const float* in, int64_t rows, int cols, int mode,
                        cudaStream_t s) {
  if (rows <= 0) return kOk;
  if (cols <= kThreadCols) {
    softmax_rows_thread_kernel<<<blocks(rows), kThreads, 0, s>>>(out, in, rows, cols, mode);
    SPO_LAUNCH_CHECK();
    return kOk;
  }
  const int64_t warps_per_block = kThreads / 32;
  const int grid = (int)std::min<int64_t>(ceil_div(rows, warps_per_block), 16LL * sm_count());
  softmax_rows_kernel<<<grid, kThreads, 0, s>>>(out, in, rows, cols, mode);
  SPO_LAUNCH_CHECK();
  return kOk;
}

int ce_rows_launch(float* out, const float* q, const float* lp, int64_t rows, int cols, cudaStream_t s) {
  LAUNCH_1D(ce_rows_kernel, rows, out, q, lp, rows, cols);
}

int entropy_rows_launch(float* out, const float* q, int64_t rows, int cols, cudaStream_t s) {
  LAUNCH_1D(entropy_rows_kernel, rows, out, q, rows, cols);
}

int kl_rows_launch(float* out, const float* ce, const float* h, int64_t rows, cudaStream_t s) {
  LAUNCH_1D(kl_rows_kernel, rows, out, ce, h, rows);
}

int logits_grad_launch(float* dz, const float* pi, const float* q, const float* mask, int64_t n,
                       float scale, cudaStream_t s) {
  LAUNCH_1D(logits_grad_kernel, n, dz, pi, q, mask, n, scale);
}

int value_grad_launch(float* dv, const float* v, const float* t, int64_t n, float scale,
                      cudaStream_t s) {
  LAUNCH_1D(value_grad_kernel, n, dv, v, t, n, scale);
}

int relu_launch(float* a, int64_t n, cudaStream_t s) { LAUNCH_1D(relu_kernel, n, a, n); }

int relu_bwd_launch(float* g, const float* act, int64_t n, cudaStream_t s) {
  LAUNCH_1D(relu_bwd_kernel, n, g, act, n);
}

int gae_launch(float* adv, float* targets, const float* r, const float* discount,
               const float* v_tm1, const float* v_t, const float* trunc, int64_t batch,
               int t_len, float lambda, cudaStream_t s) {
  LAUNCH_1D(gae_kernel, batch, adv, targets, r, discount, v_tm1, v_t, trunc, batch, t_len, lambda);
}

}  // namespace spo
