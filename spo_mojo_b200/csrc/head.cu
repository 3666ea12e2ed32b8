// Fused output head of the learner step: the last Linear layer, the loss, its
// gradient, and the last layer's backward, in one pass over the activations.
//
// Reference chain replaced (one launch instead of ~9):
//   linear_forward of the last layer      networks/linear.mojo:37-95
//   mask_logits_kernel                    networks/actor.mojo:50-71
//   softmax_rows / log_softmax_rows       ops/softmax.mojo:58-135
//   cross_entropy / entropy / kl rows     networks/actor_loss.mojo:40-148
//   logits_grad_kernel (dz)               networks/actor_loss.mojo:168-191
//   value_loss_grad_kernel (dV)           networks/mlp.mojo:141-152
//   linear_backward of the last layer     networks/linear.mojo:120-193
//   relu_backward_kernel below it         networks/mlp.mojo:155-166
// plus the alpha*KL(pi_old || pi) term (no reference code):
//   loss_row += alpha * sum_{pi_old > 0} pi_old (log pi_old - log pi)
//   dz       += alpha * (pi - pi_old) * scale,   alpha = softplus(log_alpha)
//
// Work split. A CTA walks row tiles of R rows (grid-stride), two CTAs per SM. For each tile:
//   1. the activations act[R x H] (and their lo halves) are copied into shared memory
//      with cp.async, three tiles ahead of the one being computed when act is plain fp32
//      (one ahead with lo halves), so enough bytes are in flight to cover HBM latency;
//   2. one warp per row computes z = act W + b: lane l takes h = l + 32 m, W rows come
//      from shared memory padded to AP = 12 columns (three conflict-free float4 reads),
//      and a transpose-reduce leaves z_a in lane a. Lanes 0..A-1 then evaluate the
//      masked softmax, the loss terms and dz of action a together (shuffle reductions
//      over the actions), and the lane writes the combined act (hi + lo) back in place;
//   3. each thread owns a fixed pair of adjacent columns h, h+1 of act (when H < 512, the
//      256 / (H/2) row groups of the CTA split the rows) and, over its rows, accumulates
//      dW[h, :] += act[r, h] dz[r, :] and writes dX[r, h] = (dz[r] . W[h, :]) * [act > 0]
//      as one 8-byte store per output (packed FFMA2 over action pairs), accumulating the
//      column sums of dX (the bias gradient of the layer below). Row groups' partial sums
//      are added in group order at the end.
// Partial sums (dW, db, column sums, loss statistics) go to per-CTA slots that a
// deterministic reduction adds up.
#include <algorithm>
#include <mutex>
#include <set>
#include <utility>

#include "spo_common.cuh"
#include "kernels.cuh"

namespace spo {

namespace {

constexpr int kHeadThreads = 256;
constexpr int kHeadMaxHJ = 4;  // H <= 1024
constexpr int kNW = kHeadThreads / 32;

template <int A>
__host__ __device__ constexpr int padded_actions() { return A == 1 ? 1 : (A + 3) & ~3; }

// Tile buffers: the copies run NB - 1 tiles ahead. With lo halves 2 (the lo buffers take
// the room); fp32 input: the critic (one output) 4 tiles of 4096 activations, the actor 2
// of 8192 (two rows per warp in its logits phase; measured 2.11 vs 2.78 ms for
// 1,048,576 rows at H = 512 against 4 x 4096, while the critic measured 1.05 vs 1.13 ms the other way round).
__host__ __device__ constexpr int head_buffers(bool has_lo, int A) { return has_lo ? 2 : (A == 1 ? 4 : 2); }

__device__ __forceinline__ float softplus_f(float x) {
  return log1pf(expf(-fabsf(x))) + fmaxf(x, 0.f);
}

__device__ __forceinline__ void cp_async4(float* dst, const float* src) {
  asm volatile("cp.async.ca.shared.global [%0], [%1], 4;" ::"r"(static_cast<uint32_t>(__cvta_generic_to_shared(dst))),
               "l"(src)
               : "memory");
}

__device__ __forceinline__ void cp_async16(float* dst, const float* src) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(static_cast<uint32_t>(__cvta_generic_to_shared(dst))),
               "l"(src)
               : "memory");
}

// Max / sum over the 16 lanes of each half-warp (lanes 16-31 mirror lanes 0-15).
__device__ __forceinline__ float half_max(float v) {
#pragma unroll
  for (int o = 8; o >= 1; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}
__device__ __forceinline__ float half_sum(float v) {
#pragma unroll
  for (int o = 8; o >= 1; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}
// The same for N values at once: the N exchanges of a level issued together.
template <int N>
__device__ __forceinline__ void half_max_n(float (&v)[N]) {
#pragma unroll
  for (int o = 8; o >= 1; o >>= 1)
#pragma unroll
    for (int j = 0; j < N; ++j) v[j] = fmaxf(v[j], __shfl_xor_sync(0xffffffffu, v[j], o));
}
template <int N>
__device__ __forceinline__ void half_sum_n(float (&v)[N]) {
#pragma unroll
  for (int o = 8; o >= 1; o >>= 1)
#pragma unroll
    for (int j = 0; j < N; ++j) v[j] += __shfl_xor_sync(0xffffffffu, v[j], o);
}

template <int A, int NJ>
__global__ void __launch_bounds__(kHeadThreads, 2)
head_kernel(const HeadParams p) {
  constexpr int AP = padded_actions<A>();
  extern __shared__ __align__(16) float sm[];
  pdl_wait();
  pdl_trigger();
  const int H = p.H;
  const int R = p.rows_per_tile;
  const bool has_lo = p.act_lo != nullptr;
  const int NB = head_buffers(has_lo, A);  // tile buffers: copies run NB - 1 tiles ahead
  float* Ws = sm;                          // [H][AP]
  float* abuf = Ws + H * AP;               // [NB][R][H] (act; hi + lo after phase 2)
  float* lbuf = abuf + NB * R * H;         // [2][R][H] lo halves (NB == 2)
  float* dzs = lbuf + (has_lo ? 2 * R * H : 0);  // [R][AP]
  float* red = dzs + R * AP;               // [kNW][AP + kStats]
  // per-row loss inputs of the tile buffers, copied with the activations:
  // [NB][3][R][A] = (q or critic target, mask or board cells, pi_old logits)
  float* rinb = red + kNW * (AP + kStats);

  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;

  for (int i = tid; i < H * AP; i += kHeadThreads) {
    const int h = i / AP, a = i % AP;
    Ws[i] = a < A ? __ldg(p.W + (int64_t)h * A + a) : 0.f;
  }
  // phase 2 lane roles: action a of this lane (A == 9: lanes 0-8 and their mirrors 16-24)
  const int la = lane & 15;
  const bool lvalid = la < A;
  const float lbias = A == 1 ? __ldg(p.b) : (lvalid ? __ldg(p.b + la) : 0.f);
  float alpha = p.alpha_host;
  if (p.log_alpha != nullptr) alpha = softplus_f(__ldg(p.log_alpha));

  // Phase 3 ownership: column pair c = cp0 + 256 j (columns 2c, 2c + 1) in row group rg.
  const int G2 = H >> 1;
  const int RG = G2 >= kHeadThreads ? 1 : kHeadThreads / G2;
  const int rg = G2 >= kHeadThreads ? 0 : tid / G2;
  const int cp0 = G2 >= kHeadThreads ? tid : tid % G2;
  const bool p3 = rg < RG;
  constexpr int A2 = (A + 1) / 2;  // action pairs (packed FFMA2); the odd one pads with 0
  float2 wp[NJ][2][A2];            // W[h + c][2 i], W[h + c][2 i + 1]
  float2 dw[NJ][2][A2];
  float2 dbx[NJ];
#pragma unroll
  for (int j = 0; j < NJ; ++j) {
    const int h = 2 * (cp0 + j * kHeadThreads);
    dbx[j] = make_float2(0.f, 0.f);
#pragma unroll
    for (int c = 0; c < 2; ++c)
#pragma unroll
      for (int i = 0; i < A2; ++i) {
        const bool ok = p3 && h + c < H;
        const float w0 = ok ? __ldg(p.W + (int64_t)(h + c) * A + 2 * i) : 0.f;
        const float w1 = ok && 2 * i + 1 < A ? __ldg(p.W + (int64_t)(h + c) * A + 2 * i + 1) : 0.f;
        wp[j][c][i] = make_float2(w0, w1);
        dw[j][c][i] = make_float2(0.f, 0.f);
      }
  }
  float dbl = 0.f;  // db of action la (A == 9) or of the output (A == 1, lane 0)
  float st[kStats];
#pragma unroll
  for (int s = 0; s < kStats; ++s) st[s] = 0.f;

  const int64_t tiles = (p.M + R - 1) / R;
  // copies of tile t into buffer b (an empty group past the last tile)
  auto issue = [&](int64_t t, int b) {
    if (t < tiles) {
      const int64_t r0 = t * R;
      const int n4 = (int)min((int64_t)R, p.M - r0) * H / 4;
      const float* src = p.act + r0 * H;
      float* dst = abuf + b * R * H;
      for (int i = tid; i < n4; i += kHeadThreads) cp_async16(dst + 4 * i, src + 4 * i);
      if (has_lo) {
        const float* slo = p.act_lo + r0 * H;
        float* dlo = lbuf + b * R * H;
        for (int i = tid; i < n4; i += kHeadThreads) cp_async16(dlo + 4 * i, slo + 4 * i);
      }
      const int ne = (int)min((int64_t)R, p.M - r0) * A;
      float* base = rinb + b * 3 * R * A;
      const float* s0 = p.mode == kHeadCritic ? p.target : p.q;
      const float* s1 = p.mode == kHeadCritic ? nullptr : (p.mask ? p.mask : p.cells);
      const float* s2 = p.mode == kHeadCritic ? nullptr : p.z_old;
      for (int e = tid; e < ne; e += kHeadThreads) {
        cp_async4(base + e, s0 + r0 * A + e);
        if (s1) cp_async4(base + R * A + e, s1 + r0 * A + e);  // cells rows are 9 wide = A
        if (s2) cp_async4(base + 2 * R * A + e, s2 + r0 * A + e);
      }
    }
    asm volatile("cp.async.commit_group;" ::: "memory");
  };
  for (int i = 0; i + 1 < NB; ++i) issue(blockIdx.x + (int64_t)i * gridDim.x, i);
  int it = 0;
  for (int64_t t = blockIdx.x; t < tiles; t += gridDim.x, ++it) {
    const int64_t r0 = t * R;
    const int rows = (int)min((int64_t)R, p.M - r0);
    // buffer (it + NB - 1) % NB was released by the barrier that ended the previous tile
    issue(t + (int64_t)(NB - 1) * gridDim.x, (it + NB - 1) % NB);
    // this tile's group is complete when at most NB - 1 younger groups are pending
    if (NB == 4)
      asm volatile("cp.async.wait_group 3;" ::: "memory");
    else
      asm volatile("cp.async.wait_group 1;" ::: "memory");
    __syncthreads();  // this tile's copies (every thread's) have landed; W staged
    const int bi = it % NB;
    float* ahi = abuf + bi * R * H;
    const float* alo = lbuf + (it & 1) * R * H;
    const float* rq = rinb + bi * 3 * R * A;  // q (actor) / target (critic)
    const float* rm = rq + R * A;                   // mask, or board cells
    const float* rz = rq + 2 * R * A;               // pi_old logits
    const bool from_cells = !p.mask && p.cells;

    // 2. Logits, loss and dz per row. A == 1: one warp per row. Otherwise a warp takes two
    //    rows (r, r + 8) per pass, so each W read from shared memory serves both rows (the
    //    W reads, three float4 per column and lane, are what bounds this phase).
    if constexpr (A == 1) {
      for (int r = warp; r < rows; r += kNW) {
        float* arow = ahi + r * H;
        const float* lrow = alo + r * H;
        const int64_t row = r0 + r;
        float z = 0.f;
        for (int h = lane; h < H; h += 32) {
          float av = arow[h];
          if (has_lo) {
            av += lrow[h];
            arow[h] = av;
          }
          z = fmaf(av, Ws[h], z);
        }
        z = warp_sum(z) + lbias;
        if (lane == 0) {
          float dz;
          if (p.mode == kHeadCritic) {
            const float d = z - rq[r];
            dz = d * p.scale;
            st[kStatCriticLoss] += 0.5f * d * d * p.scale;
          } else {
            // one action: pi = 1 where legal, log pi = 0
            const float mk = p.mask ? rm[r] : (from_cells ? (rm[r] == 0.f ? 1.f : 0.f) : 1.f);
            const float qv = rq[r];
            const float zm = mk == 0.f ? kNegInf : z;
            const float e = expf(zm - zm), pi = e / e, lp = zm - (zm + logf(e));
            float po = 0.f, klo = 0.f;
            if (p.z_old != nullptr) {
              const float zo = mk == 0.f ? kNegInf : rz[r];
              const float eo = expf(zo - zo);
              po = eo / eo;
              if (po > 0.f) klo = po * ((zo - (zo + logf(eo))) - lp);
            }
            const float ce = qv != 0.f ? -qv * lp : 0.f;
            const float hq = qv > 0.f ? -qv * logf(qv) : 0.f;
            dz = mk == 0.f ? 0.f : ((pi - qv) + alpha * (pi - po)) * p.scale;
            st[kStatActorLoss] += (ce + alpha * klo) * p.scale;
            st[kStatCE] += ce * p.scale;
            st[kStatEntropy] += hq * p.scale;
            st[kStatKLq] += (ce - hq) * p.scale;
            st[kStatKLold] += klo * p.scale;
            if (p.out_pi) p.out_pi[row] = pi;
            z = zm;
          }
          if (p.out_logits) p.out_logits[row] = z;
          if (p.dz_out) p.dz_out[row] = dz;
          dzs[r] = dz;
          dbl += dz;
        }
      }
    } else {
      for (int r = warp; r < rows; r += 2 * kNW) {
        const int r2 = r + kNW;
        const bool two = r2 < rows;  // warp-uniform
        float* arow0 = ahi + r * H;
        float* arow1 = ahi + (two ? r2 : r) * H;
        const float* lrow0 = alo + r * H;
        const float* lrow1 = alo + (two ? r2 : r) * H;
        // action pairs as packed FFMA2 (two fp32 fma.rn each: the fmaf results)
        float2 zp2[2][8];
#pragma unroll
        for (int a = 0; a < 8; ++a) zp2[0][a] = zp2[1][a] = make_float2(0.f, 0.f);
        for (int h = lane; h < H; h += 32) {
          float av0 = arow0[h], av1 = arow1[h];
          if (has_lo) {
            av0 += lrow0[h];
            av1 += lrow1[h];
            arow0[h] = av0;
            if (two) arow1[h] = av1;
          }
          const float2 aa0 = make_float2(av0, av0), aa1 = make_float2(av1, av1);
          const float4* w4 = reinterpret_cast<const float4*>(Ws + h * AP);
#pragma unroll
          for (int c = 0; c < AP / 4; ++c) {
            const float4 w = w4[c];
            const float2 wa = make_float2(w.x, w.y), wb = make_float2(w.z, w.w);
            zp2[0][2 * c] = __ffma2_rn(aa0, wa, zp2[0][2 * c]);
            zp2[0][2 * c + 1] = __ffma2_rn(aa0, wb, zp2[0][2 * c + 1]);
            zp2[1][2 * c] = __ffma2_rn(aa1, wa, zp2[1][2 * c]);
            zp2[1][2 * c + 1] = __ffma2_rn(aa1, wb, zp2[1][2 * c + 1]);
          }
        }
        // transpose-reduce each row: lane L ends with the sum of its row's zp[L & 15] over
        // its half of the warp
        float zr[2];
#pragma unroll
        for (int k = 0; k < 2; ++k) {
          float zp[16];
#pragma unroll
          for (int a = 0; a < 8; ++a) {
            zp[2 * a] = zp2[k][a].x;
            zp[2 * a + 1] = zp2[k][a].y;
          }
#pragma unroll
          for (int o = 8; o >= 1; o >>= 1) {
            const bool upper = (lane & o) != 0;
#pragma unroll
            for (int i = 0; i < o; ++i) {
              const float send = upper ? zp[i] : zp[i + o];
              const float keep = upper ? zp[i + o] : zp[i];
              zp[i] = keep + __shfl_xor_sync(0xffffffffu, send, o);
            }
          }
          zr[k] = zp[0];
        }
        // one exchange completes both rows: lanes 0-15 hold row r, lanes 16-31 row r2, so
        // the masked softmax, the loss terms and dz below run once for the two rows
        const bool up = lane >= 16;
        const float zv = (up ? zr[1] : zr[0]) + __shfl_xor_sync(0xffffffffu, up ? zr[0] : zr[1], 16) + lbias;
        const int rr = up ? r2 : r;
        const bool rvalid = !up || two;     // no second row in the last pass of an odd count
        const bool lv = lvalid && rvalid;
        const int64_t row = r0 + rr;

      float dz = 0.f;
      if (p.mode == kHeadCritic) {
        const float d = lv ? zv - rq[rr * A + la] : 0.f;
        dz = d * p.scale;
        const float l2 = half_sum(0.5f * d * d * p.scale);
        if (la == 0 && rvalid) st[kStatCriticLoss] += l2;
        if (p.out_logits && lv) p.out_logits[row * A + la] = zv;
      } else {
        float mk = 1.f, qv = 0.f;
        if (lv) {
          const float m = rm[rr * A + la];
          mk = p.mask ? m : (from_cells ? (m == 0.f ? 1.f : 0.f) : 1.f);
          qv = rq[rr * A + la];
        }
        // the softmax of z and, with pi_old, of its logits: their half-warp reductions side
        // by side (each value in the same xor order as alone)
        const bool has_old = p.z_old != nullptr;
        float mxs[2] = {(!lv || mk == 0.f) ? kNegInf : zv,
                        (!has_old || !lv || mk == 0.f) ? kNegInf : rz[rr * A + la]};
        const float zm = mxs[0], zo = mxs[1];
        half_max_n(mxs);
        const float mx = mxs[0], mxo = mxs[1];
        float ss[2] = {lv ? expf(zm - mx) : 0.f, (has_old && lv) ? expf(zo - mxo) : 0.f};
        const float e = ss[0], eo = ss[1];
        half_sum_n(ss);
        const float s = ss[0], so = ss[1];
        const float inv_s = 1.f / s;
        const float lse = mx + logf(s);
        const float pi = e * inv_s;
        const float lp = zm - lse;
        float po = 0.f, klo_t = 0.f;
        if (has_old) {
          const float inv_so = 1.f / so, lseo = mxo + logf(so);
          po = eo * inv_so;
          if (lv && po > 0.f) klo_t = po * ((zo - lseo) - lp);
        }
        float sums[3] = {(lv && qv != 0.f) ? -qv * lp : 0.f, (lv && qv > 0.f) ? -qv * logf(qv) : 0.f, klo_t};
        half_sum_n(sums);
        const float ce = sums[0], hq = sums[1], klo = sums[2];
        dz = (!lv || mk == 0.f) ? 0.f : ((pi - qv) + alpha * (pi - po)) * p.scale;
        if (la == 0 && rvalid) {
          st[kStatActorLoss] += (ce + alpha * klo) * p.scale;
          st[kStatCE] += ce * p.scale;
          st[kStatEntropy] += hq * p.scale;
          st[kStatKLq] += (ce - hq) * p.scale;
          st[kStatKLold] += klo * p.scale;
        }
        if (lv) {
          if (p.out_logits) p.out_logits[row * A + la] = zm;
          if (p.out_pi) p.out_pi[row * A + la] = pi;
        }
      }
      if (lv) {
        if (p.dz_out) p.dz_out[row * A + la] = dz;
        dbl += dz;
      }
      if (la < AP && rvalid) dzs[rr * AP + la] = dz;  // dz is 0 on the padding lanes
      }
    }
    __syncthreads();

    // 3. Column pairs: dW, dX (ReLU-masked), column sums of dX.
#pragma unroll
    for (int j = 0; j < NJ; ++j) {
      const int h = 2 * (cp0 + j * kHeadThreads);
      if (!p3 || h >= H) continue;
      for (int r = rg; r < rows; r += RG) {
        const float2 av = *reinterpret_cast<const float2*>(ahi + r * H + h);
        float d[AP];
        if constexpr (A == 1) {
          d[0] = dzs[r];
        } else {
#pragma unroll
          for (int c = 0; c < AP / 4; ++c) {
            const float4 v = reinterpret_cast<const float4*>(dzs + r * AP)[c];
            d[4 * c] = v.x;
            d[4 * c + 1] = v.y;
            d[4 * c + 2] = v.z;
            d[4 * c + 3] = v.w;
          }
        }
        float g[2];
#pragma unroll
        for (int c = 0; c < 2; ++c) {
          const float a = c ? av.y : av.x;
          if constexpr (A == 1) {
            dw[j][c][0].x = fmaf(a, d[0], dw[j][c][0].x);
            g[c] = d[0] * wp[j][c][0].x;
          } else {
            const float2 aa = make_float2(a, a);
            float2 gg = make_float2(0.f, 0.f);
#pragma unroll
            for (int i = 0; i < A2; ++i) {
              const float2 dd = make_float2(d[2 * i], d[2 * i + 1]);
              dw[j][c][i] = __ffma2_rn(aa, dd, dw[j][c][i]);
              gg = __ffma2_rn(dd, wp[j][c][i], gg);
            }
            g[c] = gg.x + gg.y;
          }
          g[c] = a > 0.f ? g[c] : 0.f;
        }
        dbx[j].x += g[0];
        dbx[j].y += g[1];
        const int64_t o = (r0 + r) * H + h;
        if (p.dX_lo) {
          float h0, l0, h1, l1;
          tf32_split(g[0], h0, l0);
          tf32_split(g[1], h1, l1);
          *reinterpret_cast<float2*>(p.dX + o) = make_float2(h0, h1);
          *reinterpret_cast<float2*>(p.dX_lo + o) = make_float2(l0, l1);
        } else if (p.dX) {
          *reinterpret_cast<float2*>(p.dX + o) = make_float2(g[0], g[1]);
        }
      }
    }
    __syncthreads();  // the tile's buffer and dzs are free for the next copies / rows
  }
  asm volatile("cp.async.wait_group 0;" ::: "memory");

  // Per-CTA partials. Row groups 1.. hand their sums to group 0 through shared memory,
  // one group at a time (fixed order).
  __syncthreads();
  float* xs = abuf;  // [H x A] dW, then [H] column sums
  for (int gsrc = 1; gsrc < RG; ++gsrc) {
    if (rg == gsrc) {
#pragma unroll
      for (int j = 0; j < NJ; ++j) {
        const int h = 2 * (cp0 + j * kHeadThreads);
        if (h >= H) continue;
#pragma unroll
        for (int c = 0; c < 2; ++c) {
#pragma unroll
          for (int a = 0; a < A; ++a) xs[(h + c) * A + a] = (a & 1) ? dw[j][c][a / 2].y : dw[j][c][a / 2].x;
          xs[H * A + h + c] = c ? dbx[j].y : dbx[j].x;
        }
      }
    }
    __syncthreads();
    if (rg == 0) {
#pragma unroll
      for (int j = 0; j < NJ; ++j) {
        const int h = 2 * (cp0 + j * kHeadThreads);
        if (h >= H) continue;
#pragma unroll
        for (int c = 0; c < 2; ++c) {
#pragma unroll
          for (int a = 0; a < A; ++a) {
            if (a & 1)
              dw[j][c][a / 2].y += xs[(h + c) * A + a];
            else
              dw[j][c][a / 2].x += xs[(h + c) * A + a];
          }
          if (c)
            dbx[j].y += xs[H * A + h + c];
          else
            dbx[j].x += xs[H * A + h + c];
        }
      }
    }
    __syncthreads();
  }
  const int64_t cta = blockIdx.x;
  if (rg == 0) {
#pragma unroll
    for (int j = 0; j < NJ; ++j) {
      const int h = 2 * (cp0 + j * kHeadThreads);
      if (h >= H) continue;
#pragma unroll
      for (int c = 0; c < 2; ++c) {
#pragma unroll
        for (int a = 0; a < A; ++a)
          p.dW_part[cta * H * A + (int64_t)(h + c) * A + a] = (a & 1) ? dw[j][c][a / 2].y : dw[j][c][a / 2].x;
        if (p.dbx_part) p.dbx_part[cta * H + h + c] = c ? dbx[j].y : dbx[j].x;
      }
    }
  }
  __syncthreads();
  constexpr int RW = AP + kStats;
  // lanes 16-31 hold the sums of the second row of each pair (zero where unused)
  dbl += __shfl_xor_sync(0xffffffffu, dbl, 16);
#pragma unroll
  for (int s = 0; s < kStats; ++s) st[s] += __shfl_xor_sync(0xffffffffu, st[s], 16);
  if (lane < A) red[warp * RW + lane] = dbl;
  if (lane == 0)
#pragma unroll
    for (int s = 0; s < kStats; ++s) red[warp * RW + AP + s] = st[s];
  __syncthreads();
  if (tid < A) {
    float v = 0.f;
#pragma unroll
    for (int w = 0; w < kNW; ++w) v += red[w * RW + tid];
    p.db_part[cta * A + tid] = v;
  } else if (tid >= AP && tid < AP + kStats && p.stats_part) {
    float v = 0.f;
#pragma unroll
    for (int w = 0; w < kNW; ++w) v += red[w * RW + tid];
    p.stats_part[cta * kStats + (tid - AP)] = v;
  }
}

template <int A>
int launch_a(const HeadParams& p, int grid, size_t smem, cudaStream_t s) {
  void (*k)(const HeadParams);
  const int nj = (p.H / 2 + kHeadThreads - 1) / kHeadThreads;  // column pairs per thread
  k = nj <= 1 ? head_kernel<A, 1> : head_kernel<A, 2>;
  // opt in once per device and instantiation to the largest size any H needs, so that no
  // attribute call happens while a stream is being captured into a graph
  static std::mutex mu;
  static std::set<std::pair<int, const void*>> opted;
  int dev = 0;
  SPO_CUDA_TRY(cudaGetDevice(&dev));
  {
    std::lock_guard<std::mutex> lk(mu);
    if (!opted.count({dev, (const void*)k})) {
      size_t most = 0;
      for (int h = 4; h <= kHeadThreads * kHeadMaxHJ; h += 4)
        most = std::max({most, head_smem_bytes(h, A, true), head_smem_bytes(h, A, false)});
      SPO_CUDA_TRY(cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)most));
      opted.insert({dev, (const void*)k});
    }
  }
  SPO_CUDA_TRY(launch_pdl(k, dim3(grid), dim3(kHeadThreads), smem, s, 0u, p));
  return kOk;
}

}  // namespace

// Activations per tile buffer: 4096 (16 KB), or 8192 (32 KB, two rows per warp in the
// logits phase at H = 512) for the actor's fp32 input; at most 64 rows (the per-row loss
// inputs of narrow layers stay small): two CTAs per SM. Shared memory is sized for these.
static int head_default_rows(int H, bool has_lo, int A) {
  return std::max(1, std::min(64, (has_lo || A == 1 ? 4096 : 8192) / H));
}

// Rows per tile for a batch of M rows: the default, unless that leaves fewer tiles than
// SMs (small batches), where a CTA would walk its tile's rows one pass after another while
// most SMs idle; then about one tile per SM, never fewer than 8 rows for the actor (its
// warps take rows r and r + 8 in one pass) or 2 for the critic, never more than the default.
int head_rows_per_tile(int64_t M, int H, bool has_lo, int A) {
  const int def = head_default_rows(H, has_lo, A);
  const int64_t sms = sm_count();
  if (ceil_div(std::max<int64_t>(M, 1), (int64_t)def) >= sms) return def;
  const int64_t least = A == 1 ? 2 : 8;
  return (int)std::min<int64_t>(def, std::max<int64_t>(least, ceil_div(M, sms)));
}

size_t head_smem_bytes(int H, int A, bool has_lo) {
  const int R = head_default_rows(H, has_lo, A);
  const int AP = A == 1 ? 1 : (A + 3) & ~3;
  const size_t nb = head_buffers(has_lo, A);
  return sizeof(float) * ((size_t)H * AP + (nb + (has_lo ? 2 : 0)) * (size_t)R * H + (size_t)R * AP +
                          (size_t)kNW * (AP + kStats) + 3 * nb * (size_t)R * A);
}

int head_grid(const HeadParams& p) {
  const int64_t tiles = ceil_div(p.M, (int64_t)head_rows_per_tile(p.M, p.H, p.act_lo != nullptr, p.A));
  const int64_t cap = 2LL * sm_count();
  return (int)std::max<int64_t>(1, std::min<int64_t>(tiles, cap));
}

int head_launch(HeadParams p, int grid, cudaStream_t s) {
  SPO_CHECK_ARG(p.H > 0 && p.H <= kHeadThreads * kHeadMaxHJ && p.H % 4 == 0, kErrShape,
                "head: hidden width must be a multiple of 4 and at most 1024");
  SPO_CHECK_ARG(aligned16(p.act) && (!p.act_lo || aligned16(p.act_lo)), kErrAlign,
                "head: activations must be 16-byte aligned");
  SPO_CHECK_ARG(!p.dX_lo || p.dX, kErrArg, "head: dX_lo needs dX");
  SPO_CHECK_ARG(reinterpret_cast<uintptr_t>(p.dX) % 8 == 0 && reinterpret_cast<uintptr_t>(p.dX_lo) % 8 == 0,
                kErrAlign, "head: dX must be 8-byte aligned");
  SPO_CHECK_ARG(p.A == 1 || p.A == 9, kErrUnsupported, "head: output width must be 1 or 9");
  SPO_CHECK_ARG(!p.cells || p.mask || p.A == 9, kErrUnsupported, "head: board cells need 9 actions");
  SPO_CHECK_ARG(p.mode == kHeadCritic ? p.target != nullptr : p.q != nullptr, kErrArg,
                "head: missing loss inputs");
  p.rows_per_tile = head_rows_per_tile(p.M, p.H, p.act_lo != nullptr, p.A);
  const size_t smem = head_smem_bytes(p.H, p.A, p.act_lo != nullptr);
  if (p.M == 0) return kOk;
  return p.A == 9 ? launch_a<9>(p, grid, smem, s) : launch_a<1>(p, grid, smem, s);
}

}  // namespace spo
