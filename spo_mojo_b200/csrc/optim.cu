// Optimiser-side kernels: deterministic reduction of per-CTA partial gradients,
// grouped sum of squares (global-norm clip), fused flat Adam, and the EMA update.
//
// Reference (networks/optim.mojo):
//   sum_squares + host sum   :48-73, 115-130  -> sumsq_groups_kernel (no host sync)
//   global_clip_scale        :133-142         -> computed per group inside adam_kernel
//   adam_step_kernel         :75-99           -> adam_kernel over ONE flat buffer
//   adam_step bias correction on the host :172-187 -> from a device step counter
//   ema_kernel               :145-160         -> ema_kernel (float4)
#include "kernels.cuh"

namespace spo {

namespace {

constexpr int kThreads = 256;

// ---------------------------------------------------------------- reduction
// The work is the segments' 32-element chunks, numbered segment after segment; block b
// takes chunks b, b + grid, ... (so a small step's few chunks spread over many blocks
// instead of each block walking every segment). For a chunk, the block's 8 warps split
// the parts (warp g sums parts g, g + 8, ..., four chains), so that a segment with few
// elements and many parts still has enough loads in flight. The 8 group sums are then
// added in group order: the result does not depend on scheduling or on the grid.
constexpr int kRedCols = 32;
constexpr int kRedGroups = kThreads / kRedCols;

__host__ __device__ inline int64_t red_chunks(const ReduceSeg& sg) { return (sg.count + kRedCols - 1) / kRedCols; }

__global__ void __launch_bounds__(kThreads) reduce_kernel(const ReduceParams P) {
  __shared__ float gsum[kRedGroups][kRedCols + 1];
  pdl_wait();
  pdl_trigger();
  const int c = threadIdx.x % kRedCols, g = threadIdx.x / kRedCols;
  int s = 0;
  int64_t base = 0;  // number of the first chunk of segment s
  for (int64_t gch = blockIdx.x;; gch += gridDim.x) {
    while (s < P.nseg && gch >= base + red_chunks(P.seg[s])) base += red_chunks(P.seg[s++]);
    if (s >= P.nseg) break;  // block-uniform
    const ReduceSeg sg = P.seg[s];
    const int64_t i = (gch - base) * kRedCols + c;
    // this group's parts k = g, g + G, g + 2G, ... (G = kRedGroups), eight loads in flight:
    // the j-th of a round goes to accumulator j, the eight combine in a fixed tree
    float a[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
    if (i < sg.count) {
      const float* src = sg.src + i;
      for (int k = g; k < sg.parts; k += 8 * kRedGroups) {
        float v[8];
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          const int kk = k + j * kRedGroups;
          v[j] = kk < sg.parts ? __ldg(src + (int64_t)kk * sg.part_stride) : 0.f;
        }
#pragma unroll
        for (int j = 0; j < 8; ++j) a[j] += v[j];
      }
    }
    gsum[g][c] = ((a[0] + a[1]) + (a[2] + a[3])) + ((a[4] + a[5]) + (a[6] + a[7]));
    __syncthreads();
    if (g == 0 && i < sg.count) {
      float v = gsum[0][c];
#pragma unroll
      for (int q = 1; q < kRedGroups; ++q) v += gsum[q][c];
      sg.dst[i] = v;
    }
    __syncthreads();
  }
}

__device__ __forceinline__ float block_sum(float v, float* sh) {
  v = warp_sum(v);
  const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
  if (lane == 0) sh[w] = v;
  __syncthreads();
  float r = 0.f;
  if (threadIdx.x < 32) {
    r = threadIdx.x < (blockDim.x >> 5) ? sh[threadIdx.x] : 0.f;
    r = warp_sum(r);
  }
  __syncthreads();
  return r;  // valid in thread 0
}

// ---------------------------------------------------------------- sum of squares
struct SumsqGroups {
  const float* g;
  int64_t begin[kMaxGroups], end[kMaxGroups];
  int ngrp;
  float* part;  // [ngrp][kSumsqParts]
};

__global__ void __launch_bounds__(kThreads) sumsq_groups_kernel(const SumsqGroups P) {
  __shared__ float sh[32];
  pdl_wait();
  pdl_trigger();
  for (int gi = 0; gi < P.ngrp; ++gi) {
    float acc = 0.f;
    const int64_t b4 = P.begin[gi] / 4, e4 = P.end[gi] / 4;
    const float4* g4 = reinterpret_cast<const float4*>(P.g);
    for (int64_t i = b4 + (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < e4;
         i += (int64_t)gridDim.x * blockDim.x) {
      const float4 v = __ldg(g4 + i);
      acc += v.x * v.x + v.y * v.y + v.z * v.z + v.w * v.w;
    }
    const float tot = block_sum(acc, sh);
    if (threadIdx.x == 0) P.part[gi * kSumsqParts + blockIdx.x] = tot;
  }
}

__global__ void __launch_bounds__(kThreads) sumsq_flat_kernel(const float* x, int64_t n, float* part) {
  __shared__ float sh[32];
  float acc = 0.f;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n;
       i += (int64_t)gridDim.x * blockDim.x) {
    const float v = __ldg(x + i);
    acc += v * v;
  }
  const float tot = block_sum(acc, sh);
  if (threadIdx.x == 0) part[blockIdx.x] = tot;
}

__global__ void __launch_bounds__(kThreads) sum_parts_kernel(const float* part, int n, float* out) {
  __shared__ float sh[32];
  float acc = 0.f;
  for (int i = threadIdx.x; i < n; i += blockDim.x) acc += part[i];
  const float tot = block_sum(acc, sh);
  if (threadIdx.x == 0) *out = tot;
}

// ---------------------------------------------------------------- Adam
__device__ __forceinline__ float adam_one(float& p, float g, float& m, float& v, float lr,
                                          float b1, float b2, float eps, float bc1,
                                          float bc2) {
  m = b1 * m + (1.f - b1) * g;
  v = b2 * v + (1.f - b2) * g * g;
  const float mh = m * bc1, vh = v * bc2;
  p = p - lr * mh / (sqrtf(vh) + eps);
  return p;
}

__global__ void __launch_bounds__(kThreads) adam_kernel(const AdamParams P, int64_t n) {
  __shared__ float s_clip[kMaxGroups];
  __shared__ float s_norm[kMaxGroups];
  __shared__ int s_t;
  pdl_wait();
  pdl_trigger();
  if (threadIdx.x == 0) s_t = P.step ? (*P.step + 1) : P.host_step;
  if (threadIdx.x < kMaxGroups) {
    float clip = 1.f, norm = 0.f;
    const int gi = threadIdx.x;
    const float mn = gi < P.ngrp ? P.grp[gi].max_norm : 0.f;
    if (gi < P.ngrp && P.sumsq_part && mn > 0.f && isfinite(mn)) {
      float s = 0.f;
      for (int k = 0; k < kSumsqParts; ++k) s += P.sumsq_part[gi * kSumsqParts + k];
      norm = sqrtf(s);
      if (norm > mn) clip = mn / norm;
    }
    s_clip[threadIdx.x] = clip;
    s_norm[threadIdx.x] = norm;
  }
  __syncthreads();
  const int t = s_t;
  const float bc1 = 1.f / (1.f - powf(P.b1, (float)t));
  const float bc2 = 1.f / (1.f - powf(P.b2, (float)t));

  const int64_t n4 = n / 4;
  float4* p4 = reinterpret_cast<float4*>(P.p);
  float4* g4 = reinterpret_cast<float4*>(P.g);
  float4* m4 = reinterpret_cast<float4*>(P.m);
  float4* v4 = reinterpret_cast<float4*>(P.v);
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n4;
       i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t e = 4 * i;
    int gi = -1;
#pragma unroll
    for (int k = 0; k < kMaxGroups; ++k)
      if (k < P.ngrp && e >= P.grp[k].begin && e < P.grp[k].end) gi = k;
    if (gi < 0) continue;
    const float lr = P.grp[gi].lr;
    const float sc = s_clip[gi] * P.grad_scale;
    float4 pv = p4[i], gv = g4[i], mv = m4[i], vv = v4[i];
    if (P.alpha_index >= e && P.alpha_index < e + 4) {
      // Dual gradient: d/dlog_alpha of softplus(log_alpha) * (eps - mean KL(pi_old||pi))
      float* pa = &pv.x + (P.alpha_index - e);
      float* ga = &gv.x + (P.alpha_index - e);
      const float la = *pa;
      *ga = (1.f / (1.f + expf(-la))) * (P.kl_eps - __ldg(P.kl_stat));
      g4[i] = gv;
      if (P.report) P.report[kRepDlogAlpha] = *ga;
    }
    adam_one(pv.x, gv.x * sc, mv.x, vv.x, lr, P.b1, P.b2, P.eps, bc1, bc2);
    adam_one(pv.y, gv.y * sc, mv.y, vv.y, lr, P.b1, P.b2, P.eps, bc1, bc2);
    adam_one(pv.z, gv.z * sc, mv.z, vv.z, lr, P.b1, P.b2, P.eps, bc1, bc2);
    adam_one(pv.w, gv.w * sc, mv.w, vv.w, lr, P.b1, P.b2, P.eps, bc1, bc2);
    p4[i] = pv;
    m4[i] = mv;
    v4[i] = vv;
  }
  // Tail (n not a multiple of 4; only the standalone single-group call reaches it).
  if (blockIdx.x == 0 && threadIdx.x < (n & 3)) {
    const int64_t e = n4 * 4 + threadIdx.x;
    int gi = -1;
    for (int k = 0; k < P.ngrp; ++k)
      if (e >= P.grp[k].begin && e < P.grp[k].end) gi = k;
    if (gi >= 0) {
      float pv = P.p[e], mv = P.m[e], vv = P.v[e];
      adam_one(pv, P.g[e] * s_clip[gi] * P.grad_scale, mv, vv, P.grp[gi].lr, P.b1, P.b2,
               P.eps, bc1, bc2);
      P.p[e] = pv;
      P.m[e] = mv;
      P.v[e] = vv;
    }
  }

  if (P.step) {
    __syncthreads();
    if (threadIdx.x == 0) {
      __threadfence();
      const unsigned prev = atomicAdd(P.ticket, 1u);
      if (prev == gridDim.x - 1) {
        *P.step = t;
        *P.ticket = 0u;
        if (P.report) {
          for (int k = 0; k < kMaxGroups; ++k) {
            P.report[kRepNorm0 + k] = s_norm[k];
            P.report[kRepClip0 + k] = s_clip[k];
          }
          P.report[kRepStep] = (float)t;
        }
        __threadfence();
      }
    }
  }
}

// ---------------------------------------------------------------- EMA
// optax.incremental_update rounds each product before the add (no fused multiply-add),
// which the reference's goldens record; the explicit _rn intrinsics keep that order.
__device__ __forceinline__ float ema_one(float t, float o, float tau, float keep) {
  return __fadd_rn(__fmul_rn(tau, o), __fmul_rn(keep, t));
}

__global__ void __launch_bounds__(kThreads) ema_kernel(float* target, const float* online,
                                                        int64_t n, float tau) {
  const int64_t n4 = n / 4;
  float4* t4 = reinterpret_cast<float4*>(target);
  const float4* o4 = reinterpret_cast<const float4*>(online);
  const bool vec = ((reinterpret_cast<uintptr_t>(target) | reinterpret_cast<uintptr_t>(online)) & 15) == 0;
  const int64_t gs = (int64_t)gridDim.x * blockDim.x;
  const int64_t gt = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  const float keep = 1.f - tau;
  if (vec) {
    for (int64_t i = gt; i < n4; i += gs) {
      float4 t = t4[i];
      const float4 o = __ldg(o4 + i);
      t.x = ema_one(t.x, o.x, tau, keep);
      t.y = ema_one(t.y, o.y, tau, keep);
      t.z = ema_one(t.z, o.z, tau, keep);
      t.w = ema_one(t.w, o.w, tau, keep);
      t4[i] = t;
    }
    for (int64_t i = 4 * n4 + gt; i < n; i += gs) target[i] = ema_one(target[i], online[i], tau, keep);
  } else {
    for (int64_t i = gt; i < n; i += gs) target[i] = ema_one(target[i], online[i], tau, keep);
  }
}

int grid_for(int64_t n, int per_thread = 1) {
  const int64_t want = ceil_div(std::max<int64_t>(n, 1), (int64_t)kThreads * per_thread);
  return (int)std::min<int64_t>(want, 4LL * sm_count());
}

}  // namespace

int reduce_launch(const ReduceParams& p, cudaStream_t s) {
  int64_t total = 0;  // chunks over all segments
  for (int i = 0; i < p.nseg; ++i) total += red_chunks(p.seg[i]);
  if (p.nseg == 0) return kOk;
  // every block resident at once (the occupancy of this kernel, asked once per device)
  static int per_sm[64] = {};
  int dev = 0;
  SPO_CUDA_TRY(cudaGetDevice(&dev));
  if (dev >= 0 && dev < 64 && per_sm[dev] == 0) {
    int n = 0;
    if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&n, reduce_kernel, kThreads, 0) != cudaSuccess || n < 1) {
      (void)cudaGetLastError();
      n = 4;
    }
    per_sm[dev] = n;
  }
  const int64_t resident = (int64_t)(dev >= 0 && dev < 64 ? per_sm[dev] : 4) * sm_count();
  const int grid = (int)std::min<int64_t>(total, resident);
  SPO_CUDA_TRY(launch_pdl(reduce_kernel, dim3(std::max(grid, 1)), dim3(kThreads), 0, s, 0u, p));
  return kOk;
}

int sumsq_groups_launch(const float* g, const AdamGroup* grp, int ngrp, float* part,
                        cudaStream_t s) {
  SumsqGroups P{};
  P.g = g;
  P.ngrp = ngrp;
  P.part = part;
  for (int i = 0; i < ngrp; ++i) {
    P.begin[i] = grp[i].begin;
    P.end[i] = grp[i].end;
  }
  SPO_CUDA_TRY(launch_pdl(sumsq_groups_kernel, dim3(kSumsqParts), dim3(kThreads), 0, s, 0u, P));
  return kOk;
}

int adam_launch(const AdamParams& p, int64_t n, cudaStream_t s) {
  SPO_CHECK_ARG(aligned16(p.p) && aligned16(p.g) && aligned16(p.m) && aligned16(p.v), kErrAlign,
                "adam: buffers must be 16-byte aligned");
  SPO_CUDA_TRY(launch_pdl(adam_kernel, dim3(grid_for(n / 4 + 1)), dim3(kThreads), 0, s, 0u, p, n));
  return kOk;
}

int sumsq_launch(const float* x, int64_t n, float* part, float* out, cudaStream_t s) {
  sumsq_flat_kernel<<<kSumsqParts, kThreads, 0, s>>>(x, n, part);
  SPO_LAUNCH_CHECK();
  sum_parts_kernel<<<1, kThreads, 0, s>>>(part, kSumsqParts, out);
  SPO_LAUNCH_CHECK();
  return kOk;
}

int ema_launch(float* target, const float* online, int64_t n, float tau, cudaStream_t s) {
  if (n == 0) return kOk;
  ema_kernel<<<grid_for(n, 4), kThreads, 0, s>>>(target, online, n, tau);
  SPO_LAUNCH_CHECK();
  return kOk;
}

}  // namespace spo
