// The whole learner step of a small batch in ONE launch: forward, loss, backward, the
// fixed-order reduction of the partial sums into the flat gradient buffer and (optionally)
// the clip and Adam.
//
// A small step (the reference's own scale: 256 boards, 27-128-128-9) costs ~10 dependent
// launches of a few microseconds each when run as separate kernels. Here every CTA owns a
// contiguous block of rows and runs, for each network, the whole per-row chain of its rows
// on chip: the activations of every layer, the loss and the gradients flowing down stay in
// shared memory (32 rows at a time), and only the weight gradients, which sum over all
// rows, leave the CTA as one partial per CTA. One grid-wide barrier then separates that
// from the reduction of the partials (each sum in CTA order: deterministic), which with
// Adam fused per element finishes the step (a clipped step needs the global norm first:
// two more barriers).
//
//   forward   a_l = relu(a_{l-1} W_l + b_l)   linear_forward + relu, networks/linear.mojo:37-95,
//                                             networks/mlp.mojo:34-46
//   loss      logits / V, the masked softmax, eq-11 cross entropy, alpha*KL(pi_old || pi),
//             dz (networks/actor_loss.mojo:40-191); 0.5*MSE and dV (networks/mlp.mojo:141-152)
//   backward  dW_l += a_{l-1}^T dz_l and db_l += sum dz_l over the CTA's rows;
//             dz_{l-1} = (dz_l W_l^T) * [a_{l-1} > 0]   (linear_backward
//             networks/linear.mojo:120-193, relu_backward_kernel networks/mlp.mojo:155-166)
//   reduce    partials -> flat gradients, gaps zeroed, loss statistics, then Adam
//             (networks/optim.mojo:75-187) with the dual gradient of log_alpha
//
// Every grid barrier wait is bounded (wait_ns); on expiry the CTA raises a shared abort
// word, records a code in the learner's error word and goes to the exit; the others see
// the abort word in their own waits. The last CTA to leave resets the barrier words for
// the next launch and, after a complete Adam phase, advances the step counter.
#include <algorithm>
#include <cmath>

#include "spo_common.cuh"
#include "kernels.cuh"
#include "small_step.cuh"

namespace spo {

namespace {

constexpr int kT = 256;      // threads per CTA
constexpr int kW = kT / 32;  // warps per CTA
constexpr int kR = 32;       // rows held in shared memory at a time
constexpr int kErrGridWait = 16;

__device__ __forceinline__ uint64_t now_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

__device__ __forceinline__ unsigned ld_acquire(const unsigned* p) {
  unsigned v;
  asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

// Data that other CTAs write during the launch (partials, gradients, parameters in the
// Adam phase) is read through L2 (.cg): never a stale L1 line. Weights are read before any
// write to them in the launch, through L1.
__device__ __forceinline__ float ldcg(const float* p) { return __ldcg(p); }

__device__ __forceinline__ float softplus_f(float x) { return log1pf(expf(-fabsf(x))) + fmaxf(x, 0.f); }

// Grid-wide barrier: every CTA arrives, then waits (bounded) until all have. false when
// the step was aborted.
__device__ bool grid_barrier(unsigned& target, const SmallStepParams& P) {
  __shared__ int s_ok;
  __syncthreads();
  target += gridDim.x;
  if (threadIdx.x == 0) {
    __threadfence();
    atomicAdd(P.sync + 0, 1u);
    int ok = 1;
    const uint64_t t0 = now_ns();
    while (ld_acquire(P.sync + 0) < target) {
      if (ld_acquire(P.sync + 2) != 0u) {
        ok = 0;
        break;
      }
      if (now_ns() - t0 > P.wait_ns) {
        atomicExch(P.sync + 2, 1u);
        if (P.err) atomicCAS(P.err, 0, kErrGridWait);
        ok = 0;
        break;
      }
    }
    __threadfence();
    s_ok = ok;
  }
  __syncthreads();
  return s_ok != 0;
}

// ---------------------------------------------------------------- per-block steps
// Shared-memory rows: stride = width rounded up to 4 (float4 access).
__device__ __forceinline__ int pad4(int n) { return (n + 3) & ~3; }

// Shared-memory copies of global data issued as asynchronous 16-byte copies (L2 only),
// every thread's share in flight at once; the caller waits with copies_wait().
__device__ __forceinline__ void cp16(float* dst, const float* src) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(static_cast<uint32_t>(__cvta_generic_to_shared(dst))),
               "l"(src)
               : "memory");
}
__device__ __forceinline__ void copies_wait() {
  asm volatile("cp.async.commit_group;\n\tcp.async.wait_group 0;" ::: "memory");
}
// n4 float4 from src (16-byte aligned) to dst, all threads of the CTA.
__device__ __forceinline__ void stage16(float* dst, const float* src, int n4) {
  for (int e = threadIdx.x; e < n4; e += kT) cp16(dst + 4 * e, src + 4 * e);
}

// out[R x N] = relu(in[R x K] W[K x N] + b) (in: stride ks; out: stride N), N % 32 == 0;
// also to gout (the activation cache in global memory, stride N) when given. W comes into
// shared memory (ws, wcap floats) a chunk of whole rows at a time, every thread issuing its
// share of the 16-byte loads before any is used.
__device__ void block_forward(const float* in, int ks, int K, const float* W, const float* b, int N, float* out,
                              float* gout, int R, float* ws, int wcap) {
  const int cg = N / 4, rg = kT / cg, t = threadIdx.x;
  const int c = 4 * (t % cg), r0 = t / cg;
  const bool active = r0 < rg;   // threads past the last full row group (256 % cg != 0) only stage
  constexpr int kMaxRows = kR / 4;
  float acc[kMaxRows][4] = {};
  const int nr = active ? (R - r0 + rg - 1) / rg : 0;   // rows r0, r0 + rg, ... of this thread
  const int rc = max(4, min(K, wcap / N) & ~3);   // W rows per chunk
  for (int kc = 0; kc < K; kc += rc) {
    const int kn = min(rc, K - kc);
    __syncthreads();   // the previous chunk's readers are done
    stage16(ws, W + (int64_t)kc * N, kn * N / 4);
    copies_wait();
    __syncthreads();
    for (int k = 0; k < kn; ++k) {
      const float4 w = *reinterpret_cast<const float4*>(ws + k * N + c);
#pragma unroll
      for (int j = 0; j < kMaxRows; ++j) {
        if (j >= nr) break;
        const float a = in[(r0 + j * rg) * ks + kc + k];
        acc[j][0] = fmaf(a, w.x, acc[j][0]);
        acc[j][1] = fmaf(a, w.y, acc[j][1]);
        acc[j][2] = fmaf(a, w.z, acc[j][2]);
        acc[j][3] = fmaf(a, w.w, acc[j][3]);
      }
    }
  }
  if (!active) return;
  const float4 bb = *reinterpret_cast<const float4*>(b + c);
#pragma unroll
  for (int j = 0; j < kMaxRows; ++j) {
    if (j >= nr) break;
    const int r = r0 + j * rg;
    float4 y;
    y.x = fmaxf(acc[j][0] + bb.x, 0.f);
    y.y = fmaxf(acc[j][1] + bb.y, 0.f);
    y.z = fmaxf(acc[j][2] + bb.z, 0.f);
    y.w = fmaxf(acc[j][3] + bb.w, 0.f);
    *reinterpret_cast<float4*>(out + r * N + c) = y;
    if (gout) __stcg(reinterpret_cast<float4*>(gout + (int64_t)r * N + c), y);
  }
}

// out[R x K] = (dz[R x N] W[K x N]^T) * [act > 0] (dz: stride zs; act, out: stride K),
// K % 32 == 0 (a hidden width), N any (9 or 1 for the last layer). W comes into shared
// memory transposed, a chunk of its columns at a time: wt[n][k], row stride K + 4.
__device__ void block_dx(const float* dz, int zs, int N, const float* W, int K, const float* act, float* out,
                         int R, float* wt, int wcap) {
  const int cg = K / 4, rg = kT / cg, t = threadIdx.x;
  const int c = 4 * (t % cg), r0 = t / cg;
  const bool active = r0 < rg;
  constexpr int kMaxRows = kR / 4;
  float acc[kMaxRows][4] = {};
  const int nr = active ? (R - r0 + rg - 1) / rg : 0;
  const int ws = K + 4;
  const int nc = max(1, min(N, wcap / ws));   // W columns per chunk
  for (int n0 = 0; n0 < N; n0 += nc) {
    const int nn = min(nc, N - n0);
    __syncthreads();
    // 8 loads in flight per thread, then their transposed stores
    for (int e0 = t; e0 < K * nn; e0 += 8 * kT) {
      float v[8];
#pragma unroll
      for (int u = 0; u < 8; ++u) {
        const int e = e0 + u * kT;
        if (e < K * nn) {
          const int k = e / nn, n = e - k * nn;
          v[u] = W[(int64_t)k * N + n0 + n];
        }
      }
#pragma unroll
      for (int u = 0; u < 8; ++u) {
        const int e = e0 + u * kT;
        if (e < K * nn) {
          const int k = e / nn, n = e - k * nn;
          wt[n * ws + k] = v[u];
        }
      }
    }
    __syncthreads();
    for (int n = 0; n < nn; ++n) {
      const float4 w = *reinterpret_cast<const float4*>(wt + n * ws + c);
#pragma unroll
      for (int j = 0; j < kMaxRows; ++j) {
        if (j >= nr) break;
        const float z = dz[(r0 + j * rg) * zs + n0 + n];
        acc[j][0] = fmaf(z, w.x, acc[j][0]);
        acc[j][1] = fmaf(z, w.y, acc[j][1]);
        acc[j][2] = fmaf(z, w.z, acc[j][2]);
        acc[j][3] = fmaf(z, w.w, acc[j][3]);
      }
    }
  }
  if (!active) return;
#pragma unroll
  for (int j = 0; j < kMaxRows; ++j) {
    if (j >= nr) break;
    const int r = r0 + j * rg;
    const float4 m = *reinterpret_cast<const float4*>(act + r * K + c);
    float4 y;
    y.x = m.x > 0.f ? acc[j][0] : 0.f;
    y.y = m.y > 0.f ? acc[j][1] : 0.f;
    y.z = m.z > 0.f ? acc[j][2] : 0.f;
    y.w = m.w > 0.f ? acc[j][3] : 0.f;
    *reinterpret_cast<float4*>(out + r * K + c) = y;
  }
}

// pw[K x N] (+)= in[R x K]^T dz[R x N] and pb[N] (+)= sum of the rows of dz, over this
// block's R rows (in: stride ks >= pad4(K), zero past K; dz: stride zs >= pad4(N)).
__device__ void block_dw(const float* in, int ks, int K, const float* dz, int zs, int N, int R, float* pw,
                         float* pb, bool first) {
  const int gk = (K + 3) / 4, gn = (N + 3) / 4;
  for (int gi = threadIdx.x; gi < gk * gn; gi += kT) {
    const int k0 = 4 * (gi / gn), n0 = 4 * (gi % gn);
    float acc[4][4] = {};
    for (int r = 0; r < R; ++r) {
      const float4 a = *reinterpret_cast<const float4*>(in + r * ks + k0);
      const float4 z = *reinterpret_cast<const float4*>(dz + r * zs + n0);
      const float av[4] = {a.x, a.y, a.z, a.w}, zv[4] = {z.x, z.y, z.z, z.w};
#pragma unroll
      for (int i = 0; i < 4; ++i)
#pragma unroll
        for (int j = 0; j < 4; ++j) acc[i][j] = fmaf(av[i], zv[j], acc[i][j]);
    }
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      if (k0 + i >= K) break;
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        if (n0 + j >= N) break;
        float* p = pw + (int64_t)(k0 + i) * N + n0 + j;
        __stcg(p, first ? acc[i][j] : ldcg(p) + acc[i][j]);
      }
    }
  }
  for (int n = threadIdx.x; n < N; n += kT) {
    float s = 0.f;
    for (int r = 0; r < R; ++r) s += dz[r * zs + n];
    __stcg(pb + n, first ? s : ldcg(pb + n) + s);
  }
}

// Logits / V of rows [0, R) of the block, the row losses and dz (into dz, stride zs); the
// statistics accumulate in st (lane 0 of each warp).
__device__ void block_loss(const SmallStepParams& P, const SmallNet& n, const float* act, int64_t row0, int R,
                           float* dz, int zs, const float* W, float (&st)[kStats]) {
  const int L = n.L, H = n.dims[L - 1], A = n.dims[L];   // W: the last layer's [H x A] in shared memory
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const bool actor = n.mode == 0;
  const float alpha = (actor && P.z_old) ? softplus_f(*P.log_alpha) : 0.f;
  const bool valid = lane < A;
  const float bias = valid ? n.b[L - 1][lane] : 0.f;
  for (int r = warp; r < R; r += kW) {
    const int64_t row = row0 + r;
    float part[kSmallMaxA] = {};
    for (int h = lane; h < H; h += 32) {
      const float a = act[r * H + h];
#pragma unroll
      for (int j = 0; j < kSmallMaxA; ++j)
        if (j < A) part[j] = fmaf(a, W[h * A + j], part[j]);
    }
    float z = 0.f;
#pragma unroll
    for (int j = 0; j < kSmallMaxA; ++j) {
      if (j >= A) break;
      const float s = warp_sum(part[j]);
      if (lane == j) z = s;
    }
    z += bias;
    if (!actor) {
      const float d = z - P.target[row];   // meaningful in lane 0
      if (lane < zs) dz[r * zs + lane] = lane == 0 ? d * P.scale : 0.f;
      if (lane == 0) st[kStatCriticLoss] += 0.5f * d * d * P.scale;
      continue;
    }
    const int64_t o = row * A + lane;
    const float mk = valid ? (P.mask ? P.mask[o] : (P.cells[row * 9 + lane] == 0.f ? 1.f : 0.f)) : 0.f;
    const bool legal = valid && mk != 0.f;
    const float qv = valid ? P.q[o] : 0.f;
    const float zm = legal ? z : kNegInf;
    const float mx = warp_max(zm);
    const float e = valid ? expf(zm - mx) : 0.f;
    const float s = warp_sum(e);
    const float pi = e * (1.f / s);
    const float lp = zm - (mx + logf(s));
    float po = 0.f, klo_t = 0.f;
    if (P.z_old) {
      const float zo = legal ? P.z_old[o] : kNegInf;
      const float mxo = warp_max(zo);
      const float eo = valid ? expf(zo - mxo) : 0.f;
      const float so = warp_sum(eo);
      po = eo * (1.f / so);
      if (valid && po > 0.f) klo_t = po * ((zo - (mxo + logf(so))) - lp);
    }
    const float ce = warp_sum((valid && qv != 0.f) ? -qv * lp : 0.f);
    const float hq = warp_sum((valid && qv > 0.f) ? -qv * logf(qv) : 0.f);
    const float klo = warp_sum(klo_t);
    if (lane < zs) dz[r * zs + lane] = legal ? ((pi - qv) + alpha * (pi - po)) * P.scale : 0.f;
    if (lane == 0) {
      st[kStatActorLoss] += (ce + alpha * klo) * P.scale;
      st[kStatCE] += ce * P.scale;
      st[kStatEntropy] += hq * P.scale;
      st[kStatKLq] += (ce - hq) * P.scale;
      st[kStatKLold] += klo * P.scale;
    }
  }
}

// Shared memory of one network's row block, in floats: x [kR x 32] | a_0 .. a_{L-2}
// [kR x d_{l+1}] | dz ping-pong 2 x [kR x dmax] | the last layer's W [H x A] | a weight
// staging area (the rest, up to kSmallMaxSmem).
__host__ __device__ inline int small_base_floats(const int* dims, int L) {
  int f = kR * 32, dmax = (dims[L] + 3) & ~3;
  for (int l = 1; l < L; ++l) {
    f += kR * dims[l];
    dmax = dims[l] > dmax ? dims[l] : dmax;
  }
  return f + 2 * kR * dmax + ((dims[L - 1] * dims[L] + 3) & ~3);
}

// One network over this CTA's rows [rb, re), 32 rows at a time.
__device__ void net_rows(const SmallStepParams& P, const SmallNet& n, int64_t rb, int64_t re, float* sm,
                         float* red) {
  const int L = n.L, d0 = n.dims[0];
  const int part = blockIdx.x;
  float* xs = sm;
  float* acts[kSmallMaxLayers - 1];
  float* p = xs + kR * 32;
  int dmax = pad4(n.dims[L]);
  for (int l = 0; l + 1 < L; ++l) {
    acts[l] = p;
    p += kR * n.dims[l + 1];
    dmax = max(dmax, n.dims[l + 1]);
  }
  float* dzb[2] = {p, p + kR * dmax};
  float* hw = p + 2 * kR * dmax;
  float* ws = hw + pad4(n.dims[L - 1] * n.dims[L]);
  const int wcap = (int)(kSmallMaxSmem / sizeof(float)) - small_base_floats(n.dims, L);
  // the last layer's W: H x A floats, a multiple of 4 (H % 32 == 0), 16-byte aligned
  stage16(hw, n.W[L - 1], n.dims[L - 1] * n.dims[L] / 4);
  copies_wait();
  float st[kStats] = {};
  bool first = true;
  for (int64_t r0 = rb; r0 < re; r0 += kR, first = false) {
    const int R = (int)min((int64_t)kR, re - r0);
    // input rows (zero past d0); board cells expand to the plane-major planes
    {
      float v[kR * 32 / kT];   // this thread's 4 input values, loaded together
#pragma unroll
      for (int u = 0; u < kR * 32 / kT; ++u) {
        const int e = threadIdx.x + u * kT, r = e >> 5, f = e & 31;
        v[u] = 0.f;
        if (r < R && f < d0) {
          const int64_t row = r0 + r;
          v[u] = P.obs ? P.obs[row * d0 + f] : P.cells[row * 9 + (f % 9)];
        }
      }
#pragma unroll
      for (int u = 0; u < kR * 32 / kT; ++u) {
        const int e = threadIdx.x + u * kT, r = e >> 5, f = e & 31;
        float x = v[u];
        if (!P.obs && r < R && f < d0) {   // cell code -> the plane's 0/1 value
          const int plane = f / 9;
          x = (plane == 0 ? x == 0.f : (plane == 1 ? x == 1.f : x == -1.f)) ? 1.f : 0.f;
        }
        xs[e] = x;
      }
    }
    __syncthreads();
    for (int l = 0; l + 1 < L; ++l) {
      block_forward(l == 0 ? xs : acts[l - 1], l == 0 ? 32 : n.dims[l], n.dims[l], n.W[l], n.b[l], n.dims[l + 1],
                    acts[l], n.gact[l] ? n.gact[l] + r0 * n.dims[l + 1] : nullptr, R, ws, wcap);
      __syncthreads();
    }
    int zs = pad4(n.dims[L]);   // row stride of the gradient in dzb[cur]: its layer's width
    block_loss(P, n, acts[L - 2], r0, R, dzb[0], zs, hw, st);
    __syncthreads();
    int cur = 0;
    for (int l = L - 1; l >= 0; --l) {
      const float* in = l == 0 ? xs : acts[l - 1];
      const int ks = l == 0 ? 32 : n.dims[l];
      block_dw(in, ks, n.dims[l], dzb[cur], zs, n.dims[l + 1], R, n.pw[l] + (int64_t)part * n.dims[l] * n.dims[l + 1],
               n.pb[l] + (int64_t)part * n.dims[l + 1], first);
      if (l >= 1) block_dx(dzb[cur], zs, n.dims[l + 1], n.W[l], n.dims[l], acts[l - 1], dzb[cur ^ 1], R, ws, wcap);
      __syncthreads();
      zs = n.dims[l];
      cur ^= 1;
    }
  }
  // the statistics of this CTA's rows
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  if (lane == 0)
#pragma unroll
    for (int k = 0; k < kStats; ++k) red[warp * kStats + k] = st[k];
  __syncthreads();
  if (threadIdx.x < kStats) {
    float v = 0.f;
#pragma unroll
    for (int w = 0; w < kW; ++w) v += red[w * kStats + threadIdx.x];
    __stcg(n.pstats + (int64_t)part * kStats + threadIdx.x, v);
  }
  __syncthreads();
}

__device__ __forceinline__ void adam_one(float& p, float g, float& m, float& v, float lr, float b1, float b2,
                                         float eps, float bc1, float bc2) {
  m = b1 * m + (1.f - b1) * g;
  v = b2 * v + (1.f - b2) * g * g;
  p = p - lr * (m * bc1) / (sqrtf(v * bc2) + eps);
}

// sum over k < parts of src[k * stride] with 8 loads in flight: part k goes to partial sum
// k % 8 and the eight are combined in a fixed order (deterministic).
__device__ __forceinline__ float sum_parts(const float* src, int parts, int64_t stride) {
  float a[8] = {};
  int k = 0;
  for (; k + 8 <= parts; k += 8) {
#pragma unroll
    for (int u = 0; u < 8; ++u) a[u] += ldcg(src + (int64_t)(k + u) * stride);
  }
  for (int u = 0; k < parts; ++k, ++u) a[u] += ldcg(src + (int64_t)k * stride);
  return ((a[0] + a[1]) + (a[2] + a[3])) + ((a[4] + a[5]) + (a[6] + a[7]));
}

// Reduced value of flat element e (the segment it falls in, its parts in order).
__device__ __forceinline__ float reduced(const SmallStepParams& P, int64_t e, int& si) {
  while (si + 1 < P.red.nseg && e >= P.seg_start[si + 1]) ++si;
  const ReduceSeg& sg = P.red.seg[si];
  const int64_t i = e - P.seg_start[si];
  return sum_parts(sg.src + i, sg.parts, sg.part_stride);
}

__global__ void __launch_bounds__(kT, 1) small_step_kernel(const __grid_constant__ SmallStepParams P) {
  extern __shared__ __align__(16) float sm[];
  __shared__ float red[kW * kStats];
  __shared__ float s_clip[kMaxGroups], s_norm[kMaxGroups];
  __shared__ float s_sq[kW];
  unsigned target = 0;
  bool ok = true;
  const AdamParams& ap = P.adam;

  // ---- rows: forward, loss, backward; per-CTA partial sums
  if (blockIdx.x < P.parts) {
    const int64_t rb = (int64_t)blockIdx.x * P.rows_per_cta;
    const int64_t re = min(rb + P.rows_per_cta, P.rows);
    for (int i = 0; i < 2; ++i)
      if (P.net[i].L) net_rows(P, P.net[i], rb, re, sm, red);
  }
  ok = grid_barrier(target, P);

  // ---- partial sums -> flat gradients (each in CTA order), Adam fused per element
  int t_step = 0;
  float bc1 = 1.f, bc2 = 1.f;
  if (ok && P.apply) {
    t_step = *ap.step + 1;
    bc1 = 1.f / (1.f - powf(ap.b1, (float)t_step));
    bc2 = 1.f / (1.f - powf(ap.b2, (float)t_step));
    if (threadIdx.x < kMaxGroups) {
      s_clip[threadIdx.x] = 1.f;
      s_norm[threadIdx.x] = 0.f;
    }
    __syncthreads();
  }
  const bool fuse = P.apply && !P.clip;
  if (ok) {
    int si = 0;
    for (int64_t e = (int64_t)blockIdx.x * kT + threadIdx.x; e < P.total_red; e += (int64_t)gridDim.x * kT) {
      const float g = reduced(P, e, si);
      const int64_t fe = P.flat_index[si] + (e - P.seg_start[si]);   // element of the flat buffers
      __stcg(P.red.seg[si].dst + (e - P.seg_start[si]), g);
      if (!fuse || fe < 0) continue;
      int gi = -1;
#pragma unroll
      for (int k = 0; k < kMaxGroups; ++k)
        if (k < ap.ngrp && fe >= ap.grp[k].begin && fe < ap.grp[k].end) gi = k;
      if (gi < 0) continue;
      float gv = g;
      if (fe == ap.alpha_index) {
        // dual gradient: sigmoid(log_alpha) * (eps - mean KL(pi_old || pi)), the KL from the
        // actor's per-CTA statistics in the same order as its own reduced slot
        const float kl = sum_parts(P.net[0].pstats + kStatKLold, P.parts, kStats);
        gv = (1.f / (1.f + expf(-ldcg(ap.p + fe)))) * (ap.kl_eps - kl);
        __stcg(ap.g + fe, gv);
        if (ap.report) ap.report[kRepDlogAlpha] = gv;
      }
      float p = ldcg(ap.p + fe), m = ldcg(ap.m + fe), v = ldcg(ap.v + fe);
      adam_one(p, gv, m, v, ap.grp[gi].lr, ap.b1, ap.b2, ap.eps, bc1, bc2);
      __stcg(ap.p + fe, p);
      __stcg(ap.m + fe, m);
      __stcg(ap.v + fe, v);
    }
  }
  // ---- clipped step: global norms of the reduced gradients, then Adam
  if (ok && P.apply && P.clip) {
    ok = grid_barrier(target, P);
    if (ok) {
      for (int gi = 0; gi < ap.ngrp; ++gi) {
        float acc = 0.f;
        for (int64_t e = ap.grp[gi].begin + (int64_t)blockIdx.x * kT + threadIdx.x; e < ap.grp[gi].end;
             e += (int64_t)gridDim.x * kT) {
          const float v = ldcg(ap.g + e);
          acc += v * v;
        }
        acc = warp_sum(acc);
        if ((threadIdx.x & 31) == 0) s_sq[threadIdx.x >> 5] = acc;
        __syncthreads();
        if (threadIdx.x == 0) {
          float v = 0.f;
          for (int w = 0; w < kW; ++w) v += s_sq[w];
          __stcg(P.sumsq + (int64_t)gi * gridDim.x + blockIdx.x, v);
        }
        __syncthreads();
      }
      ok = grid_barrier(target, P);
    }
    if (ok) {
      if (threadIdx.x < kMaxGroups) {
        float clip = 1.f, norm = 0.f;
        const int gi = threadIdx.x;
        const float mn = gi < ap.ngrp ? ap.grp[gi].max_norm : 0.f;
        if (gi < ap.ngrp && mn > 0.f && isfinite(mn)) {
          float s = 0.f;
          for (unsigned k = 0; k < gridDim.x; ++k) s += ldcg(P.sumsq + (int64_t)gi * gridDim.x + k);
          norm = sqrtf(s);
          if (norm > mn) clip = mn / norm;
        }
        s_clip[gi] = clip;
        s_norm[gi] = norm;
      }
      __syncthreads();
      for (int64_t e = (int64_t)blockIdx.x * kT + threadIdx.x; e < P.total; e += (int64_t)gridDim.x * kT) {
        int gi = -1;
#pragma unroll
        for (int k = 0; k < kMaxGroups; ++k)
          if (k < ap.ngrp && e >= ap.grp[k].begin && e < ap.grp[k].end) gi = k;
        if (gi < 0) continue;
        float gv = ldcg(ap.g + e);
        if (e == ap.alpha_index) {
          gv = (1.f / (1.f + expf(-ldcg(ap.p + e)))) * (ap.kl_eps - ldcg(ap.kl_stat));
          __stcg(ap.g + e, gv);
          if (ap.report) ap.report[kRepDlogAlpha] = gv;
        }
        float p = ldcg(ap.p + e), m = ldcg(ap.m + e), v = ldcg(ap.v + e);
        adam_one(p, gv * s_clip[gi], m, v, ap.grp[gi].lr, ap.b1, ap.b2, ap.eps, bc1, bc2);
        __stcg(ap.p + e, p);
        __stcg(ap.m + e, m);
        __stcg(ap.v + e, v);
      }
    }
  }
  // ---- exit: the last CTA out resets the barrier words (and advances the step)
  __syncthreads();
  if (threadIdx.x == 0) {
    __threadfence();
    const unsigned prev = atomicAdd(P.sync + 1, 1u);
    if (prev == gridDim.x - 1) {
      const bool done = ld_acquire(P.sync + 2) == 0u;
      if (done && P.apply) {
        *ap.step = t_step;
        if (ap.report) {
          for (int k = 0; k < kMaxGroups; ++k) {
            ap.report[kRepNorm0 + k] = s_norm[k];
            ap.report[kRepClip0 + k] = s_clip[k];
          }
          ap.report[kRepStep] = (float)t_step;
        }
      }
      P.sync[0] = 0u;
      P.sync[2] = 0u;
      __threadfence();
      P.sync[1] = 0u;
      __threadfence();
    }
  }
}

}  // namespace

size_t small_step_smem(const spo_mlp_desc* nets, int count) {
  // the base of every network plus room to stage at least 4 rows (forward) and 1 column
  // (dX, stride <= 260) of its weights; the launch takes all kSmallMaxSmem bytes
  size_t most = 0;
  for (int i = 0; i < count; ++i) {
    const spo_mlp_desc& d = nets[i];
    if (d.num_layers < 2) continue;
    int wneed = 4 * 256;
    for (int l = 0; l < d.num_layers; ++l) wneed = std::max(wneed, 4 * d.dims[l + 1]);
    most = std::max(most, (size_t)(small_base_floats(d.dims, d.num_layers) + wneed) * sizeof(float));
  }
  return most;
}

int small_step_grid() {
  static int cached[64] = {};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return 0;
  if (!cached[dev]) {
    if (cudaFuncSetAttribute(small_step_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             (int)kSmallMaxSmem) != cudaSuccess) {
      (void)cudaGetLastError();
      return 0;
    }
    int per_sm = 0;
    if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, small_step_kernel, kT, kSmallMaxSmem) !=
            cudaSuccess ||
        per_sm < 1) {
      (void)cudaGetLastError();
      return 0;
    }
    cached[dev] = sm_count();   // one CTA per SM: all co-resident
  }
  return cached[dev];
}

int small_step_launch(const SmallStepParams& p, int grid, size_t smem, cudaStream_t s) {
  cudaLaunchConfig_t cfg{};
  cfg.gridDim = dim3((unsigned)grid);
  cfg.blockDim = dim3(kT);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeCooperative;
  attr[0].val.cooperative = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  SPO_CUDA_TRY(cudaLaunchKernelEx(&cfg, small_step_kernel, p));
  return kOk;
}

}  // namespace spo
