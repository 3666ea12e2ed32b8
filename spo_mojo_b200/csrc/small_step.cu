// The whole learner step of a small batch in ONE launch: forward, loss, backward, the
// fixed-order reduction of the partial sums into the flat gradient buffer and (optionally)
// the clip and Adam, as phases of one cooperative kernel separated by grid-wide barriers.
//
// A small step (the reference's own scale: 256 boards, 27-128-128-9) is a chain of ~10
// dependent launches of a few microseconds each when run as separate kernels; here the
// launches become phases and each phase boundary costs one grid barrier (an atomic arrive
// and an acquire spin, bounded in time) instead of a launch.
//
// Phases (each network's work is spread over all CTAs, items taken grid-stride):
//   F_l   a_l = relu(in W_l + b_l), l = 0..L-2, in = x (or board cells expanded to the
//         27-wide planes) for l = 0: items of 32 rows x 64 columns, k in chunks of 32
//         staged in shared memory, 2 x 4 outputs per thread (linear_forward + relu,
//         networks/linear.mojo:37-95, networks/mlp.mojo:34-46)
//   H     logits / V of the last layer, one warp per row, then the loss of the row and
//         dz = dL/dz (the actor's masked softmax, eq-11 cross entropy, alpha*KL(pi_old||pi),
//         networks/actor_loss.mojo:40-191; the critic's 0.5*MSE, networks/mlp.mojo:141-152);
//         per-CTA sums of the loss statistics
//   B_l   l = L-1..0: dW_l = in^T dz_l over row chunks (items of 32 x 32 outputs and one
//         chunk of rows, one partial per chunk), db_l with it, and for l >= 1
//         dz_{l-1} = (dz_l W_l^T) * [a_{l-1} > 0] (items of 32 rows x 64 columns)
//         (linear_backward networks/linear.mojo:120-193, relu_backward_kernel
//         networks/mlp.mojo:155-166)
//   R     partials -> flat gradients, each sum in part order (deterministic), the
//         alignment gaps zeroed, the statistics slots
//   C     (clipping only) per-CTA sums of squares of each network's gradients
//   A     (apply only) Adam over the flat buffer with the dual gradient of log_alpha
//         (networks/optim.mojo:75-187)
// Data written in one phase and read in a later one is read with ld.global.cg (L2, never
// a stale L1 line). Every barrier wait is bounded (wait_ns); on expiry the CTA raises a
// shared abort word, records a code in the learner's error word and skips to the exit,
// and the other CTAs see the abort word in their next wait. The last CTA to leave resets
// the barrier words for the next launch (and, after a complete Adam phase, advances the
// step counter).
#include <algorithm>
#include <cmath>

#include "spo_common.cuh"
#include "kernels.cuh"
#include "small_step.cuh"

namespace spo {

namespace {

constexpr int kT = 256;      // threads per CTA
constexpr int kW = kT / 32;  // warps per CTA
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

// Loads of data another CTA wrote earlier in this launch (or that this launch writes
// later): through L2.
__device__ __forceinline__ float ldg(const float* p) { return __ldcg(p); }
__device__ __forceinline__ float4 ldg4(const float* p) { return __ldcg(reinterpret_cast<const float4*>(p)); }

__device__ __forceinline__ float softplus_f(float x) { return log1pf(expf(-fabsf(x))) + fmaxf(x, 0.f); }

struct Sync {
  unsigned target = 0;
};

// Grid-wide barrier: every CTA arrives, then waits (bounded) until all have. false when
// the step was aborted.
__device__ bool grid_barrier(Sync& g, const SmallStepParams& P) {
  __shared__ int s_ok;
  __syncthreads();
  g.target += gridDim.x;
  if (threadIdx.x == 0) {
    __threadfence();
    atomicAdd(P.sync + 0, 1u);
    int ok = 1;
    const uint64_t t0 = now_ns();
    while (ld_acquire(P.sync + 0) < g.target) {
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

// ---------------------------------------------------------------- shared memory
struct FwdSmem {
  float x[32][33];   // [row][k]
  float w[32][64];   // [k][col]
};
struct DwSmem {
  float a[32][33];   // [row][k]
  float z[32][32];   // [row][n]
};
union Smem {
  FwdSmem f;
  DwSmem d;
  float hw[kSmallMaxHidden * 9];   // last layer's W for the head
  float red[kW][kStats + 4];
};

// value of input feature f of row r of a first layer: x, or the board cells expanded to
// the plane-major [empty | agent | rival] planes (envs/tictactoe.mojo:449-480)
__device__ __forceinline__ float in0(const SmallStepParams& P, int64_t r, int f, int k) {
  if (P.obs) return ldg(P.obs + r * k + f);
  const float c = ldg(P.cells + r * 9 + (f % 9));
  const int plane = f / 9;
  return (plane == 0 ? c == 0.f : (plane == 1 ? c == 1.f : c == -1.f)) ? 1.f : 0.f;
}

// ---------------------------------------------------------------- forward items
// out[B x N] = relu(in[B x K] W[K x N] + b) for one 32-row x 64-column item.
__device__ void fwd_item(const SmallStepParams& P, const float* in, bool first, int K, const float* W,
                         const float* bias, int N, float* out, int64_t r0, int c0, Smem& sm) {
  const int t = threadIdx.x, ty = t >> 4, tx = t & 15;
  float acc[2][4] = {};
  for (int kc = 0; kc < K; kc += 32) {
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const int e = t + kT * j, r = e >> 5, k = e & 31;
      const int64_t row = r0 + r;
      float v = 0.f;
      if (row < P.rows && kc + k < K) v = first ? in0(P, row, kc + k, K) : ldg(in + row * K + kc + k);
      sm.f.x[r][k] = v;
    }
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const int e = t + kT * j, k = e >> 6, c = e & 63;
      sm.f.w[k][c] = (kc + k < K && c0 + c < N) ? ldg(W + (int64_t)(kc + k) * N + c0 + c) : 0.f;
    }
    __syncthreads();
#pragma unroll 8
    for (int k = 0; k < 32; ++k) {
      const float a0 = sm.f.x[2 * ty][k], a1 = sm.f.x[2 * ty + 1][k];
      const float4 w = *reinterpret_cast<const float4*>(&sm.f.w[k][4 * tx]);
      acc[0][0] = fmaf(a0, w.x, acc[0][0]);
      acc[0][1] = fmaf(a0, w.y, acc[0][1]);
      acc[0][2] = fmaf(a0, w.z, acc[0][2]);
      acc[0][3] = fmaf(a0, w.w, acc[0][3]);
      acc[1][0] = fmaf(a1, w.x, acc[1][0]);
      acc[1][1] = fmaf(a1, w.y, acc[1][1]);
      acc[1][2] = fmaf(a1, w.z, acc[1][2]);
      acc[1][3] = fmaf(a1, w.w, acc[1][3]);
    }
    __syncthreads();
  }
  const int c = c0 + 4 * tx;
  if (c >= N) return;   // N is a multiple of 32: a 4-column group is all in or all out
  const float4 b = ldg4(bias + c);
#pragma unroll
  for (int i = 0; i < 2; ++i) {
    const int64_t row = r0 + 2 * ty + i;
    if (row >= P.rows) continue;
    float4 y;
    y.x = fmaxf(acc[i][0] + b.x, 0.f);
    y.y = fmaxf(acc[i][1] + b.y, 0.f);
    y.z = fmaxf(acc[i][2] + b.z, 0.f);
    y.w = fmaxf(acc[i][3] + b.w, 0.f);
    __stcg(reinterpret_cast<float4*>(out + row * N + c), y);
  }
}

// ---------------------------------------------------------------- dX items
// out[B x K] = (dz[B x N] W[K x N]^T) * [act > 0] for one 32-row x 64-column item.
__device__ void dx_item(const SmallStepParams& P, const float* dz, int N, const float* W, int K,
                        const float* act, float* out, int64_t r0, int c0, Smem& sm) {
  const int t = threadIdx.x, ty = t >> 4, tx = t & 15;
  float acc[2][4] = {};
  for (int nc = 0; nc < N; nc += 32) {
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const int e = t + kT * j, r = e >> 5, n = e & 31;
      const int64_t row = r0 + r;
      sm.f.x[r][n] = (row < P.rows && nc + n < N) ? ldg(dz + row * N + nc + n) : 0.f;
    }
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const int e = t + kT * j, c = e >> 5, n = e & 31;   // W[c0 + c][nc + n] -> w[n][c]
      sm.f.w[n][c] = (nc + n < N && c0 + c < K) ? ldg(W + (int64_t)(c0 + c) * N + nc + n) : 0.f;
    }
    __syncthreads();
#pragma unroll 8
    for (int n = 0; n < 32; ++n) {
      const float a0 = sm.f.x[2 * ty][n], a1 = sm.f.x[2 * ty + 1][n];
      const float4 w = *reinterpret_cast<const float4*>(&sm.f.w[n][4 * tx]);
      acc[0][0] = fmaf(a0, w.x, acc[0][0]);
      acc[0][1] = fmaf(a0, w.y, acc[0][1]);
      acc[0][2] = fmaf(a0, w.z, acc[0][2]);
      acc[0][3] = fmaf(a0, w.w, acc[0][3]);
      acc[1][0] = fmaf(a1, w.x, acc[1][0]);
      acc[1][1] = fmaf(a1, w.y, acc[1][1]);
      acc[1][2] = fmaf(a1, w.z, acc[1][2]);
      acc[1][3] = fmaf(a1, w.w, acc[1][3]);
    }
    __syncthreads();
  }
  const int c = c0 + 4 * tx;
  if (c >= K) return;
#pragma unroll
  for (int i = 0; i < 2; ++i) {
    const int64_t row = r0 + 2 * ty + i;
    if (row >= P.rows) continue;
    const float4 m = ldg4(act + row * K + c);
    float4 y;
    y.x = m.x > 0.f ? acc[i][0] : 0.f;
    y.y = m.y > 0.f ? acc[i][1] : 0.f;
    y.z = m.z > 0.f ? acc[i][2] : 0.f;
    y.w = m.w > 0.f ? acc[i][3] : 0.f;
    __stcg(reinterpret_cast<float4*>(out + row * K + c), y);
  }
}

// ---------------------------------------------------------------- dW items
// Partial of dW[K x N] = in^T dz over rows [rb, re) for a 32 x 32 block at (k0, n0); with
// k0 == 0 also the partial column sums of dz (db).
__device__ void dw_item(const SmallStepParams& P, const float* in, bool first, int K, const float* dz, int N,
                        int64_t rb, int64_t re, int k0, int n0, float* pw, float* pb, Smem& sm) {
  const int t = threadIdx.x, kk = t >> 3, nn = (t & 7) * 4;
  float acc[4] = {}, db[4] = {};
  for (int64_t rs = rb; rs < re; rs += 32) {
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const int e = t + kT * j, r = e >> 5, c = e & 31;
      const int64_t row = rs + r;
      const bool okr = row < re;
      sm.d.a[r][c] = (okr && k0 + c < K) ? (first ? in0(P, row, k0 + c, K) : ldg(in + row * K + k0 + c)) : 0.f;
      sm.d.z[r][c] = (okr && n0 + c < N) ? ldg(dz + row * N + n0 + c) : 0.f;
    }
    __syncthreads();
#pragma unroll 8
    for (int r = 0; r < 32; ++r) {
      const float a = sm.d.a[r][kk];
      const float4 z = *reinterpret_cast<const float4*>(&sm.d.z[r][nn]);
      acc[0] = fmaf(a, z.x, acc[0]);
      acc[1] = fmaf(a, z.y, acc[1]);
      acc[2] = fmaf(a, z.z, acc[2]);
      acc[3] = fmaf(a, z.w, acc[3]);
      db[0] += z.x;
      db[1] += z.y;
      db[2] += z.z;
      db[3] += z.w;
    }
    __syncthreads();
  }
  if (k0 + kk < K)
#pragma unroll
    for (int j = 0; j < 4; ++j)
      if (n0 + nn + j < N) __stcg(pw + (int64_t)(k0 + kk) * N + n0 + nn + j, acc[j]);
  if (k0 == 0 && kk == 0)
#pragma unroll
    for (int j = 0; j < 4; ++j)
      if (n0 + nn + j < N) __stcg(pb + n0 + nn + j, db[j]);
}

// ---------------------------------------------------------------- head (loss rows)
// Logits / V of one network's last layer, the row loss and dz, one warp per row; the
// statistics' per-CTA sums into net.pstats[blockIdx.x].
__device__ void head_phase(const SmallStepParams& P, const SmallNet& n, Smem& sm) {
  const int L = n.L, H = n.dims[L - 1], A = n.dims[L];
  const float* act = n.act[L - 2];
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  for (int i = threadIdx.x; i < H * A; i += kT) sm.hw[i] = ldg(n.W[L - 1] + i);
  __syncthreads();
  const bool actor = n.mode == 0;
  const float alpha = (actor && P.z_old) ? softplus_f(ldg(P.log_alpha)) : 0.f;
  const bool valid = lane < A;
  const float bias = valid ? ldg(n.b[L - 1] + lane) : 0.f;
  float st[kStats] = {};
  float* dzo = n.dz[0];
  for (int64_t r = (int64_t)blockIdx.x * kW + warp; r < P.rows; r += (int64_t)gridDim.x * kW) {
    float part[kSmallMaxA] = {};
    for (int h = lane; h < H; h += 32) {
      const float a = ldg(act + r * H + h);
#pragma unroll
      for (int j = 0; j < kSmallMaxA; ++j)
        if (j < A) part[j] = fmaf(a, sm.hw[h * A + j], part[j]);
    }
    float z = 0.f;
#pragma unroll
    for (int j = 0; j < kSmallMaxA; ++j) {
      if (j >= A) break;
      const float s = warp_sum(part[j]);
      if (lane == j) z = s;
    }
    z += bias;
    const int64_t o = r * A + lane;
    if (!actor) {
      if (lane == 0) {
        const float d = z - ldg(P.target + r);
        __stcg(dzo + r, d * P.scale);
        st[kStatCriticLoss] += 0.5f * d * d * P.scale;
      }
      continue;
    }
    // the masked softmax, loss terms and dz of the row (lane = action)
    const float mk = valid ? (P.mask ? ldg(P.mask + o) : (ldg(P.cells + r * 9 + lane) == 0.f ? 1.f : 0.f)) : 0.f;
    const bool legal = valid && mk != 0.f;
    const float qv = valid ? ldg(P.q + o) : 0.f;
    const float zm = legal ? z : kNegInf;
    const float mx = warp_max(zm);
    const float e = valid ? expf(zm - mx) : 0.f;
    const float s = warp_sum(e);
    const float pi = e * (1.f / s);
    const float lp = zm - (mx + logf(s));
    float po = 0.f, klo_t = 0.f;
    if (P.z_old) {
      const float zo = legal ? ldg(P.z_old + o) : kNegInf;
      const float mxo = warp_max(zo);
      const float eo = valid ? expf(zo - mxo) : 0.f;
      const float so = warp_sum(eo);
      po = eo * (1.f / so);
      if (valid && po > 0.f) klo_t = po * ((zo - (mxo + logf(so))) - lp);
    }
    const float ce = warp_sum((valid && qv != 0.f) ? -qv * lp : 0.f);
    const float hq = warp_sum((valid && qv > 0.f) ? -qv * logf(qv) : 0.f);
    const float klo = warp_sum(klo_t);
    if (valid) __stcg(dzo + o, legal ? ((pi - qv) + alpha * (pi - po)) * P.scale : 0.f);
    if (lane == 0) {
      st[kStatActorLoss] += (ce + alpha * klo) * P.scale;
      st[kStatCE] += ce * P.scale;
      st[kStatEntropy] += hq * P.scale;
      st[kStatKLq] += (ce - hq) * P.scale;
      st[kStatKLold] += klo * P.scale;
    }
  }
  __syncthreads();   // sm.hw is reused below
  if (lane == 0)
#pragma unroll
    for (int k = 0; k < kStats; ++k) sm.red[warp][k] = st[k];
  __syncthreads();
  if (threadIdx.x < kStats) {
    float v = 0.f;
#pragma unroll
    for (int w = 0; w < kW; ++w) v += sm.red[w][threadIdx.x];
    __stcg(n.pstats + (int64_t)blockIdx.x * kStats + threadIdx.x, v);
  }
  __syncthreads();
}

__device__ __forceinline__ void adam_one(float& p, float g, float& m, float& v, float lr, float b1, float b2,
                                         float eps, float bc1, float bc2) {
  m = b1 * m + (1.f - b1) * g;
  v = b2 * v + (1.f - b2) * g * g;
  p = p - lr * (m * bc1) / (sqrtf(v * bc2) + eps);
}

__global__ void __launch_bounds__(kT) small_step_kernel(const __grid_constant__ SmallStepParams P) {
  __shared__ __align__(16) Smem sm;
  __shared__ float s_clip[kMaxGroups], s_norm[kMaxGroups];
  __shared__ int s_t;
  Sync g;
  bool ok = true;

  // ---- forward, layer by layer (both networks in each phase)
  int maxl = 0;
  for (int i = 0; i < 2; ++i) maxl = max(maxl, P.net[i].L);
  for (int l = 0; l + 1 < maxl && ok; ++l) {
    int items[2] = {0, 0};
    for (int i = 0; i < 2; ++i) {
      const SmallNet& n = P.net[i];
      if (l + 1 < n.L) items[i] = (int)(ceil_div_dev(P.rows, 32) * ((n.dims[l + 1] + 63) / 64));
    }
    for (int it = blockIdx.x; it < items[0] + items[1]; it += gridDim.x) {
      const int i = it < items[0] ? 0 : 1;
      const int j = it - (i ? items[0] : 0);
      const SmallNet& n = P.net[i];
      const int N = n.dims[l + 1], ct = (N + 63) / 64;
      fwd_item(P, l == 0 ? nullptr : n.act[l - 1], l == 0, n.dims[l], n.W[l], n.b[l], N, n.act[l],
               (int64_t)(j / ct) * 32, (j % ct) * 64, sm);
    }
    ok = grid_barrier(g, P);
  }
  // ---- loss rows
  if (ok) {
    for (int i = 0; i < 2; ++i)
      if (P.net[i].L) head_phase(P, P.net[i], sm);
    ok = grid_barrier(g, P);
  }
  // ---- backward, layer by layer from the top
  int cur[2] = {0, 0};
  for (int l = maxl - 1; l >= 0 && ok; --l) {
    int nw[2] = {0, 0}, nx[2] = {0, 0};
    for (int i = 0; i < 2; ++i) {
      const SmallNet& n = P.net[i];
      const int ll = l - (maxl - n.L);   // networks of fewer layers run their top layers later
      if (!n.L || ll < 0) continue;
      nw[i] = ((n.dims[ll] + 31) / 32) * ((n.dims[ll + 1] + 31) / 32) * n.S[ll];
      if (ll >= 1) nx[i] = (int)(ceil_div_dev(P.rows, 32) * ((n.dims[ll] + 63) / 64));
    }
    const int total = nw[0] + nx[0] + nw[1] + nx[1];
    for (int it = blockIdx.x; it < total; it += gridDim.x) {
      int j = it, i = 0;
      if (j >= nw[0] + nx[0]) {
        j -= nw[0] + nx[0];
        i = 1;
      }
      const SmallNet& n = P.net[i];
      const int ll = l - (maxl - n.L);
      const int K = n.dims[ll], N = n.dims[ll + 1];
      const float* dz = n.dz[cur[i]];
      if (j < nw[i]) {
        const int kb = (K + 31) / 32, nb = (N + 31) / 32;
        const int s = j / (kb * nb), rem = j % (kb * nb);
        const int64_t cs = ceil_div_dev(P.rows, n.S[ll]);
        const int64_t rb = min((int64_t)s * cs, P.rows), re = min(rb + cs, P.rows);
        dw_item(P, ll == 0 ? nullptr : n.act[ll - 1], ll == 0, K, dz, N, rb, re, (rem / nb) * 32,
                (rem % nb) * 32, n.pw[ll] + (int64_t)s * K * N, n.pb[ll] + (int64_t)s * N, sm);
      } else {
        j -= nw[i];
        const int ct = (K + 63) / 64;
        dx_item(P, dz, N, n.W[ll], K, n.act[ll - 1], n.dz[cur[i] ^ 1], (int64_t)(j / ct) * 32, (j % ct) * 64, sm);
      }
    }
    for (int i = 0; i < 2; ++i)
      if (P.net[i].L && l - (maxl - P.net[i].L) >= 1) cur[i] ^= 1;
    ok = grid_barrier(g, P);
  }
  // ---- partial sums -> flat gradient buffer (each sum in part order)
  if (ok) {
    for (int si = 0; si < P.red.nseg; ++si) {
      const ReduceSeg sg = P.red.seg[si];
      for (int64_t e = (int64_t)blockIdx.x * kT + threadIdx.x; e < sg.count; e += (int64_t)gridDim.x * kT) {
        float v = 0.f;
        for (int k = 0; k < sg.parts; ++k) v += ldg(sg.src + (int64_t)k * sg.part_stride + e);
        __stcg(sg.dst + e, v);
      }
    }
    if (P.apply) ok = grid_barrier(g, P);
  }
  // ---- (clipping) per-CTA sums of squares of each group's gradients
  const AdamParams& ap = P.adam;
  if (ok && P.apply && P.clip) {
    __shared__ float s_sq[kW];
    for (int gi = 0; gi < ap.ngrp; ++gi) {
      float acc = 0.f;
      for (int64_t e = ap.grp[gi].begin + (int64_t)blockIdx.x * kT + threadIdx.x; e < ap.grp[gi].end;
           e += (int64_t)gridDim.x * kT) {
        const float v = ldg(ap.g + e);
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
    ok = grid_barrier(g, P);
  }
  // ---- Adam over the flat buffer
  if (ok && P.apply) {
    if (threadIdx.x == 0) s_t = *ap.step + 1;
    if (threadIdx.x < kMaxGroups) {
      float clip = 1.f, norm = 0.f;
      const int gi = threadIdx.x;
      const float mn = gi < ap.ngrp ? ap.grp[gi].max_norm : 0.f;
      if (P.clip && gi < ap.ngrp && mn > 0.f && isfinite(mn)) {
        float s = 0.f;
        for (unsigned k = 0; k < gridDim.x; ++k) s += ldg(P.sumsq + (int64_t)gi * gridDim.x + k);
        norm = sqrtf(s);
        if (norm > mn) clip = mn / norm;
      }
      s_clip[gi] = clip;
      s_norm[gi] = norm;
    }
    __syncthreads();
    const int t = s_t;
    const float bc1 = 1.f / (1.f - powf(ap.b1, (float)t));
    const float bc2 = 1.f / (1.f - powf(ap.b2, (float)t));
    for (int64_t e = (int64_t)blockIdx.x * kT + threadIdx.x; e < P.total; e += (int64_t)gridDim.x * kT) {
      int gi = -1;
#pragma unroll
      for (int k = 0; k < kMaxGroups; ++k)
        if (k < ap.ngrp && e >= ap.grp[k].begin && e < ap.grp[k].end) gi = k;
      if (gi < 0) continue;
      float gv = ldg(ap.g + e);
      if (e == ap.alpha_index) {
        // dual gradient of log_alpha: sigmoid(log_alpha) * (eps - mean KL(pi_old || pi))
        gv = (1.f / (1.f + expf(-ldg(ap.p + e)))) * (ap.kl_eps - ldg(ap.kl_stat));
        __stcg(ap.g + e, gv);
        if (ap.report) ap.report[kRepDlogAlpha] = gv;
      }
      float p = ldg(ap.p + e), m = ldg(ap.m + e), v = ldg(ap.v + e);
      adam_one(p, gv * s_clip[gi], m, v, ap.grp[gi].lr, ap.b1, ap.b2, ap.eps, bc1, bc2);
      __stcg(ap.p + e, p);
      __stcg(ap.m + e, m);
      __stcg(ap.v + e, v);
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
        const int t = *ap.step + 1;
        *ap.step = t;
        if (ap.report) {
          for (int k = 0; k < kMaxGroups; ++k) {
            ap.report[kRepNorm0 + k] = s_norm[k];
            ap.report[kRepClip0 + k] = s_clip[k];
          }
          ap.report[kRepStep] = (float)t;
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

int small_step_grid() {
  static int cached[64] = {};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return 0;
  if (!cached[dev]) {
    int per_sm = 0;
    if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, small_step_kernel, kT, 0) != cudaSuccess ||
        per_sm < 1) {
      (void)cudaGetLastError();
      return 0;
    }
    cached[dev] = sm_count();   // one CTA per SM: all co-resident
  }
  return cached[dev];
}

int small_step_launch(const SmallStepParams& p, int grid, cudaStream_t s) {
  cudaLaunchConfig_t cfg{};
  cfg.gridDim = dim3((unsigned)grid);
  cfg.blockDim = dim3(kT);
  cfg.dynamicSmemBytes = 0;
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
