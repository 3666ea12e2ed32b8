// The losses on caller-held outputs: the actor's equation-11 loss on logits (with the
// alpha*KL(pi_old || pi) term and the log_alpha dual gradient) and the critic's 0.5*MSE
// on values, each with its gradient and its batch statistics, for a caller that runs its
// own forward (the reference's actor_backward and critic_backward start from logits / V,
// networks/actor_loss.mojo:194-214, networks/mlp.mojo:212-233).
//
// Actor: nine actions, one row per thread; other widths, one warp per row with lane a
// holding action a (A <= 32). Per row, in the order of the fused head's loss phase:
//   z_m = z, or -FLT_MAX where mask == 0            mask_logits_kernel, networks/actor.mojo:50-71
//   log pi = z_m - logsumexp(z_m), pi = softmax(z_m)  ops/softmax.mojo:58-135
//   ce  = -sum_{q != 0} q log pi                      networks/actor_loss.mojo:40-65
//   H   = -sum_{q > 0} q log q                        networks/actor_loss.mojo:105-116
//   kl_old = sum_{pi_old > 0} pi_old (log pi_old - log pi)   (no reference code)
//   dz  = ((pi - q) + alpha (pi - pi_old)) * scale, 0 where illegal
//                                                    logits_grad_kernel, networks/actor_loss.mojo:168-191
// Critic: one thread per value, dV = (V - t) * scale, loss += 0.5 (V - t)^2 * scale
// (value_loss_grad_kernel, networks/mlp.mojo:141-152).
// Each CTA writes its scaled partial sums to a workspace slot; one CTA then adds the slots
// in a fixed order (deterministic) and writes the statistics and the dual gradient
// sigmoid(log_alpha) * (eps_kl - mean KL(pi_old || pi)).
#include <algorithm>

#include "spo_common.cuh"
#include "kernels.cuh"

namespace spo {

namespace {

constexpr int kThreads = 256;
constexpr int kWarps = kThreads / 32;

__device__ __forceinline__ float softplus_f(float x) { return log1pf(expf(-fabsf(x))) + fmaxf(x, 0.f); }

// Butterfly sums (max) of N values at once: the same xor order per value as warp_sum
// (warp_max), the N exchanges of a level issued together instead of N dependent chains.
template <int N>
__device__ __forceinline__ void warp_sum_n(float (&v)[N]) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1)
#pragma unroll
    for (int j = 0; j < N; ++j) v[j] += __shfl_xor_sync(0xffffffffu, v[j], o);
}
template <int N>
__device__ __forceinline__ void warp_max_n(float (&v)[N]) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1)
#pragma unroll
    for (int j = 0; j < N; ++j) v[j] = fmaxf(v[j], __shfl_xor_sync(0xffffffffu, v[j], o));
}

struct LossParams {
  const float* z;        // actor: logits [rows x A]; critic: V [rows]
  const float* mask;     // actor: [rows x A] or null (all legal)
  const float* q;        // actor: [rows x A]
  const float* z_old;    // actor: [rows x A] or null (no KL term)
  const float* log_alpha;
  const float* target;   // critic: [rows]
  int64_t rows;
  int A;
  float scale;
  float* dz;             // [rows x A] / [rows]
  float* part;           // [grid][kStats]
};

__global__ void __launch_bounds__(kThreads) actor_loss_rows_kernel(const LossParams p) {
  __shared__ float red[kWarps][kStats];
  pdl_wait();
  pdl_trigger();
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const float alpha = p.z_old != nullptr ? softplus_f(__ldg(p.log_alpha)) : 0.f;
  float st[kStats] = {};
  const bool valid = lane < p.A;
  for (int64_t r = (int64_t)blockIdx.x * kWarps + warp; r < p.rows; r += (int64_t)gridDim.x * kWarps) {
    const int64_t o = r * p.A + lane;
    const float mk = valid ? (p.mask ? __ldg(p.mask + o) : 1.f) : 0.f;
    const bool legal = valid && mk != 0.f;
    const float qv = valid ? __ldg(p.q + o) : 0.f;
    // the softmax of z and, with pi_old, of its logits: their reductions side by side
    // (each value in the same xor order as alone)
    const bool has_old = p.z_old != nullptr;
    float mxs[2] = {legal ? __ldg(p.z + o) : kNegInf, (has_old && legal) ? __ldg(p.z_old + o) : kNegInf};
    const float zm = mxs[0], zo = mxs[1];
    warp_max_n(mxs);
    const float mx = mxs[0], mxo = mxs[1];
    float ss[2] = {valid ? expf(zm - mx) : 0.f, (has_old && valid) ? expf(zo - mxo) : 0.f};
    const float e = ss[0], eo = ss[1];
    warp_sum_n(ss);
    const float s = ss[0], so = ss[1];
    const float pi = e * (1.f / s);
    const float lp = zm - (mx + logf(s));
    float po = 0.f, klo_t = 0.f;
    if (has_old) {
      po = eo * (1.f / so);
      if (valid && po > 0.f) klo_t = po * ((zo - (mxo + logf(so))) - lp);
    }
    float sums[3] = {(valid && qv != 0.f) ? -qv * lp : 0.f, (valid && qv > 0.f) ? -qv * logf(qv) : 0.f, klo_t};
    warp_sum_n(sums);
    const float ce = sums[0], hq = sums[1], klo = sums[2];
    if (valid) p.dz[o] = legal ? ((pi - qv) + alpha * (pi - po)) * p.scale : 0.f;
    st[kStatActorLoss] += (ce + alpha * klo) * p.scale;
    st[kStatCE] += ce * p.scale;
    st[kStatEntropy] += hq * p.scale;
    st[kStatKLq] += (ce - hq) * p.scale;
    st[kStatKLold] += klo * p.scale;
  }
  if (lane == 0)
#pragma unroll
    for (int k = 0; k < kStats; ++k) red[warp][k] = st[k];
  __syncthreads();
  if (threadIdx.x < kStats) {
    float v = 0.f;
#pragma unroll
    for (int w = 0; w < kWarps; ++w) v += red[w][threadIdx.x];
    p.part[(int64_t)blockIdx.x * kStats + threadIdx.x] = v;
  }
}

// The same loss with one row per thread, for a fixed action count NA: a row's logits,
// mask, targets and pi_old logits come from consecutive words (a warp reads 32 adjacent
// rows, whose lines the later words of each row then hit in L1), and the row's maxima and
// sums are taken serially in action order, with no exchange between lanes. Per element
// the same expressions as the kernel above; the statistics are reduced over the warp and
// then the CTA's warps in order.
template <int NA>
__global__ void __launch_bounds__(kThreads) actor_loss_row_per_thread_kernel(const LossParams p) {
  __shared__ float red[kWarps][kStats];
  pdl_wait();
  pdl_trigger();
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const bool has_old = p.z_old != nullptr;
  const float alpha = has_old ? softplus_f(__ldg(p.log_alpha)) : 0.f;
  float st[kStats] = {};
  for (int64_t r = (int64_t)blockIdx.x * kThreads + threadIdx.x; r < p.rows; r += (int64_t)gridDim.x * kThreads) {
    const int64_t o = r * NA;
    float zm[NA], zo[NA], qv[NA];
    bool legal[NA];
#pragma unroll
    for (int a = 0; a < NA; ++a) {
      const float mk = p.mask ? __ldg(p.mask + o + a) : 1.f;
      legal[a] = mk != 0.f;
      qv[a] = __ldg(p.q + o + a);
      zm[a] = legal[a] ? __ldg(p.z + o + a) : kNegInf;
      zo[a] = (has_old && legal[a]) ? __ldg(p.z_old + o + a) : kNegInf;
    }
    float mx = zm[0], mxo = zo[0];
#pragma unroll
    for (int a = 1; a < NA; ++a) {
      mx = fmaxf(mx, zm[a]);
      mxo = fmaxf(mxo, zo[a]);
    }
    float e[NA], eo[NA], s = 0.f, so = 0.f;
#pragma unroll
    for (int a = 0; a < NA; ++a) {
      e[a] = expf(zm[a] - mx);
      s += e[a];
      eo[a] = has_old ? expf(zo[a] - mxo) : 0.f;
      so += eo[a];
    }
    const float inv_s = 1.f / s, lse = mx + logf(s);
    const float inv_so = has_old ? 1.f / so : 0.f, lseo = has_old ? mxo + logf(so) : 0.f;
    float ce = 0.f, hq = 0.f, klo = 0.f;
#pragma unroll
    for (int a = 0; a < NA; ++a) {
      const float pi = e[a] * inv_s;
      const float lp = zm[a] - lse;
      float po = 0.f;
      if (has_old) {
        po = eo[a] * inv_so;
        if (po > 0.f) klo += po * ((zo[a] - lseo) - lp);
      }
      if (qv[a] != 0.f) ce += -qv[a] * lp;
      if (qv[a] > 0.f) hq += -qv[a] * logf(qv[a]);
      p.dz[o + a] = legal[a] ? ((pi - qv[a]) + alpha * (pi - po)) * p.scale : 0.f;
    }
    st[kStatActorLoss] += (ce + alpha * klo) * p.scale;
    st[kStatCE] += ce * p.scale;
    st[kStatEntropy] += hq * p.scale;
    st[kStatKLq] += (ce - hq) * p.scale;
    st[kStatKLold] += klo * p.scale;
  }
  warp_sum_n(st);
  if (lane == 0)
#pragma unroll
    for (int k = 0; k < kStats; ++k) red[warp][k] = st[k];
  __syncthreads();
  if (threadIdx.x < kStats) {
    float v = 0.f;
#pragma unroll
    for (int w = 0; w < kWarps; ++w) v += red[w][threadIdx.x];
    p.part[(int64_t)blockIdx.x * kStats + threadIdx.x] = v;
  }
}

__global__ void __launch_bounds__(kThreads) value_loss_rows_kernel(const LossParams p) {
  __shared__ float red[kWarps];
  pdl_wait();
  pdl_trigger();
  float acc = 0.f;
  for (int64_t i = (int64_t)blockIdx.x * kThreads + threadIdx.x; i < p.rows; i += (int64_t)gridDim.x * kThreads) {
    const float d = __ldg(p.z + i) - __ldg(p.target + i);
    p.dz[i] = d * p.scale;
    acc += 0.5f * d * d * p.scale;
  }
  acc = warp_sum(acc);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = acc;
  __syncthreads();
  if (threadIdx.x == 0) {
    float v = 0.f;
#pragma unroll
    for (int w = 0; w < kWarps; ++w) v += red[w];
    p.part[(int64_t)blockIdx.x * kStats + kStatCriticLoss] = v;
  }
}

// Statistics slots [first, last) = the sum of the parts in part order; the dual gradient
// (actor, optional) from the summed KL(pi_old || pi).
__global__ void loss_finish_kernel(const float* part, int parts, int first, int last, float* stats,
                                   const float* log_alpha, float eps_kl, float* dlog_alpha) {
  __shared__ float kl;
  pdl_wait();
  pdl_trigger();
  const int s = first + (int)threadIdx.x;
  if (s < last) {
    float v = 0.f;
    for (int g = 0; g < parts; ++g) v += part[(int64_t)g * kStats + s];
    stats[s] = v;
    if (s == kStatKLold) kl = v;
  }
  __syncthreads();
  if (threadIdx.x == 0 && dlog_alpha != nullptr) {
    const float la = log_alpha ? *log_alpha : 0.f;
    const float klv = (first <= kStatKLold && kStatKLold < last) ? kl : 0.f;
    dlog_alpha[0] = (1.f / (1.f + expf(-la))) * (eps_kl - klv);
  }
}

int loss_grid(int64_t rows_or_n, int per_cta) {
  return (int)std::max<int64_t>(1, std::min<int64_t>(ceil_div(rows_or_n, per_cta), loss_parts_max()));
}

}  // namespace

int64_t loss_parts_max() { return 4LL * sm_count(); }

int actor_loss_launch(const float* z, const float* mask, const float* q, const float* z_old,
                      const float* log_alpha, float eps_kl, int64_t rows, int A, float scale, float* dz,
                      float* stats, float* dlog_alpha, float* part, cudaStream_t s) {
  LossParams p{};
  p.z = z;
  p.mask = mask;
  p.q = q;
  p.z_old = z_old;
  p.log_alpha = log_alpha;
  p.rows = rows;
  p.A = A;
  p.scale = scale;
  p.dz = dz;
  p.part = part;
  // nine actions (the board's cells): one row per thread; other widths: one row per warp
  const bool per_thread = A == 9;
  const int grid = rows > 0 ? loss_grid(rows, per_thread ? kThreads : kWarps) : 0;
  if (grid > 0) {
    if (per_thread)
      SPO_CUDA_TRY(launch_pdl(actor_loss_row_per_thread_kernel<9>, dim3(grid), dim3(kThreads), 0, s, 0u, p));
    else
      SPO_CUDA_TRY(launch_pdl(actor_loss_rows_kernel, dim3(grid), dim3(kThreads), 0, s, 0u, p));
  }
  SPO_CUDA_TRY(launch_pdl(loss_finish_kernel, dim3(1), dim3(32), 0, s, 0u, (const float*)part, grid,
                          (int)kStatActorLoss, (int)kStatKLold + 1, stats, log_alpha, eps_kl, dlog_alpha));
  return kOk;
}

int value_loss_launch(const float* v, const float* target, int64_t n, float scale, float* dv, float* stats,
                      float* part, cudaStream_t s) {
  LossParams p{};
  p.z = v;
  p.target = target;
  p.rows = n;
  p.scale = scale;
  p.dz = dv;
  p.part = part;
  const int grid = n > 0 ? loss_grid(n, kThreads) : 0;
  if (grid > 0) SPO_CUDA_TRY(launch_pdl(value_loss_rows_kernel, dim3(grid), dim3(kThreads), 0, s, 0u, p));
  SPO_CUDA_TRY(launch_pdl(loss_finish_kernel, dim3(1), dim3(32), 0, s, 0u, (const float*)part, grid,
                          (int)kStatCriticLoss, (int)kStatCriticLoss + 1, stats, (const float*)nullptr, 0.f,
                          (float*)nullptr));
  return kOk;
}

}  // namespace spo
