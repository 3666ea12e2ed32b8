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
// Work split. A CTA walks row tiles of R rows (grid-stride). For each tile:
//   1. the post-ReLU activations act[R x H] are staged in shared memory (float4);
//   2. one warp per row computes z = act W + b (lanes split H, butterfly sum), then
//      lane 0 evaluates the masked softmax, the loss terms and dz for that row;
//   3. each thread owns fixed columns h of act and, over the R rows, accumulates
//      dW[h, :] += act[r, h] dz[r, :] and writes dX[r, h] = (dz[r] . W[h, :]) * [act > 0],
//      accumulating the column sums of dX (the bias gradient of the layer below).
// Partial sums (dW, db, column sums, loss statistics) go to per-CTA slots that a
// deterministic reduction adds up.
#include "spo_common.cuh"
#include "kernels.cuh"

namespace spo {

namespace {

constexpr int kHeadThreads = 256;
constexpr int kHeadMaxHJ = 4;  // H <= 1024

__device__ __forceinline__ float softplus_f(float x) {
  return log1pf(expf(-fabsf(x))) + fmaxf(x, 0.f);
}

template <int A>
__global__ void __launch_bounds__(kHeadThreads)
head_kernel(const HeadParams p) {
  extern __shared__ __align__(16) float sm[];
  const int H = p.H;
  const int R = p.rows_per_tile;
  float* Ws = sm;                          // [H][A]
  float* as = Ws + ((H * A + 3) & ~3);     // [R][H]
  float* dzs = as + R * H;                 // [R][A]
  float* red = dzs + R * A;                // scratch for the final reductions

  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  constexpr int NW = kHeadThreads / 32;

  for (int i = tid; i < H * A; i += kHeadThreads) Ws[i] = __ldg(p.W + i);
  float bias[A];
#pragma unroll
  for (int a = 0; a < A; ++a) bias[a] = __ldg(p.b + a);
  float alpha = p.alpha_host;
  if (p.log_alpha != nullptr) alpha = softplus_f(__ldg(p.log_alpha));

  // Thread-owned columns h = tid + 256 j.
  float wreg[kHeadMaxHJ][A];
  float dw[kHeadMaxHJ][A];
  float dbx[kHeadMaxHJ];
#pragma unroll
  for (int j = 0; j < kHeadMaxHJ; ++j) {
    const int h = tid + j * kHeadThreads;
    dbx[j] = 0.f;
#pragma unroll
    for (int a = 0; a < A; ++a) {
      wreg[j][a] = h < H ? __ldg(p.W + (int64_t)h * A + a) : 0.f;
      dw[j][a] = 0.f;
    }
  }
  // Per-warp (lane 0) accumulators: db of the last layer and the loss statistics.
  float dbl[A];
#pragma unroll
  for (int a = 0; a < A; ++a) dbl[a] = 0.f;
  float st[kStats];
#pragma unroll
  for (int s = 0; s < kStats; ++s) st[s] = 0.f;

  const int64_t tiles = (p.M + R - 1) / R;
  const int hv = H / 4;
  for (int64_t t = blockIdx.x; t < tiles; t += gridDim.x) {
    const int64_t r0 = t * R;
    const int rows = (int)min((int64_t)R, p.M - r0);
    __syncthreads();  // previous tile fully consumed
    {
      const float4* src = reinterpret_cast<const float4*>(p.act + r0 * H);
      float4* dst = reinterpret_cast<float4*>(as);
      const int n4 = rows * hv;
      if (p.act_lo) {
        const float4* slo = reinterpret_cast<const float4*>(p.act_lo + r0 * H);
        for (int i = tid; i < n4; i += kHeadThreads) {
          float4 a = __ldg(src + i);
          const float4 b = __ldg(slo + i);
          a.x += b.x; a.y += b.y; a.z += b.z; a.w += b.w;
          dst[i] = a;
        }
      } else {
        for (int i = tid; i < n4; i += kHeadThreads) dst[i] = __ldg(src + i);
      }
    }
    __syncthreads();

    // 2. One warp per row: logits, loss, dz.
    for (int r = warp; r < rows; r += NW) {
      float z[A];
#pragma unroll
      for (int a = 0; a < A; ++a) z[a] = 0.f;
      const float* arow = as + r * H;
      for (int h = lane; h < H; h += 32) {
        const float av = arow[h];
#pragma unroll
        for (int a = 0; a < A; ++a) z[a] = fmaf(av, Ws[h * A + a], z[a]);
      }
#pragma unroll
      for (int a = 0; a < A; ++a) z[a] = warp_sum(z[a]) + bias[a];

      if (lane == 0) {
        const int64_t row = r0 + r;
        float dz[A];
        if (p.mode == kHeadCritic) {
#pragma unroll
          for (int a = 0; a < A; ++a) {
            const float d = z[a] - __ldg(p.target + row * A + a);
            dz[a] = d * p.scale;
            st[kStatCriticLoss] += 0.5f * d * d * p.scale;
            if (p.out_logits) p.out_logits[row * A + a] = z[a];
          }
        } else {
          float mk[A], q[A], zm[A];
          float mx = kNegInf;
#pragma unroll
          for (int a = 0; a < A; ++a) {
            mk[a] = p.mask ? __ldg(p.mask + row * A + a) : 1.f;
            q[a] = __ldg(p.q + row * A + a);
            zm[a] = mk[a] == 0.f ? kNegInf : z[a];
            mx = fmaxf(mx, zm[a]);
          }
          float e[A], s = 0.f;
#pragma unroll
          for (int a = 0; a < A; ++a) { e[a] = expf(zm[a] - mx); s += e[a]; }
          const float inv_s = 1.f / s;
          const float lse = mx + logf(s);
          float ce = 0.f, hq = 0.f, pi[A], lp[A];
#pragma unroll
          for (int a = 0; a < A; ++a) {
            pi[a] = e[a] * inv_s;
            lp[a] = zm[a] - lse;
            if (q[a] != 0.f) ce -= q[a] * lp[a];
            if (q[a] > 0.f) hq -= q[a] * logf(q[a]);
          }
          float klo = 0.f, po[A];
          if (p.z_old != nullptr) {
            float zo[A], mxo = kNegInf;
#pragma unroll
            for (int a = 0; a < A; ++a) {
              zo[a] = mk[a] == 0.f ? kNegInf : __ldg(p.z_old + row * A + a);
              mxo = fmaxf(mxo, zo[a]);
            }
            float so = 0.f;
#pragma unroll
            for (int a = 0; a < A; ++a) { po[a] = expf(zo[a] - mxo); so += po[a]; }
            const float inv_so = 1.f / so, lseo = mxo + logf(so);
#pragma unroll
            for (int a = 0; a < A; ++a) {
              po[a] *= inv_so;
              if (po[a] > 0.f) klo += po[a] * ((zo[a] - lseo) - lp[a]);
            }
          } else {
#pragma unroll
            for (int a = 0; a < A; ++a) po[a] = 0.f;
          }
#pragma unroll
          for (int a = 0; a < A; ++a)
            dz[a] = mk[a] == 0.f ? 0.f : ((pi[a] - q[a]) + alpha * (pi[a] - po[a])) * p.scale;
          st[kStatActorLoss] += (ce + alpha * klo) * p.scale;
          st[kStatCE] += ce * p.scale;
          st[kStatEntropy] += hq * p.scale;
          st[kStatKLq] += (ce - hq) * p.scale;
          st[kStatKLold] += klo * p.scale;
          if (p.out_logits)
#pragma unroll
            for (int a = 0; a < A; ++a) p.out_logits[row * A + a] = zm[a];
          if (p.out_pi)
#pragma unroll
            for (int a = 0; a < A; ++a) p.out_pi[row * A + a] = pi[a];
        }
#pragma unroll
        for (int a = 0; a < A; ++a) {
          dzs[r * A + a] = dz[a];
          dbl[a] += dz[a];
          if (p.dz_out) p.dz_out[row * A + a] = dz[a];
        }
      }
    }
    __syncthreads();

    // 3. Thread-owned columns: dW, dX (ReLU-masked), column sums of dX.
#pragma unroll
    for (int j = 0; j < kHeadMaxHJ; ++j) {
      const int h = tid + j * kHeadThreads;
      if (h >= H) continue;
      for (int r = 0; r < rows; ++r) {
        const float av = as[r * H + h];
        float g = 0.f;
#pragma unroll
        for (int a = 0; a < A; ++a) {
          const float d = dzs[r * A + a];
          dw[j][a] = fmaf(av, d, dw[j][a]);
          g = fmaf(d, wreg[j][a], g);
        }
        g = av > 0.f ? g : 0.f;
        if (p.dX_lo) {
          float hi, lo;
          tf32_split(g, hi, lo);
          p.dX[(r0 + r) * H + h] = hi;
          p.dX_lo[(r0 + r) * H + h] = lo;
        } else if (p.dX) {
          p.dX[(r0 + r) * H + h] = g;
        }
        dbx[j] += g;
      }
    }
  }

  // Per-CTA partials.
  const int64_t cta = blockIdx.x;
#pragma unroll
  for (int j = 0; j < kHeadMaxHJ; ++j) {
    const int h = tid + j * kHeadThreads;
    if (h >= H) continue;
#pragma unroll
    for (int a = 0; a < A; ++a) p.dW_part[cta * H * A + (int64_t)h * A + a] = dw[j][a];
    if (p.dbx_part) p.dbx_part[cta * H + h] = dbx[j];
  }
  __syncthreads();
  if (lane == 0) {
#pragma unroll
    for (int a = 0; a < A; ++a) red[warp * (A + kStats) + a] = dbl[a];
#pragma unroll
    for (int s = 0; s < kStats; ++s) red[warp * (A + kStats) + A + s] = st[s];
  }
  __syncthreads();
  if (tid < A + kStats) {
    float v = 0.f;
#pragma unroll
    for (int w = 0; w < NW; ++w) v += red[w * (A + kStats) + tid];
    if (tid < A) p.db_part[cta * A + tid] = v;
    else if (p.stats_part) p.stats_part[cta * kStats + (tid - A)] = v;
  }
}

}  // namespace

int head_rows_per_tile(int H) { return H > 512 ? 16 : (H > 256 ? 32 : 64); }

size_t head_smem_bytes(int H, int A) {
  const int R = head_rows_per_tile(H);
  const int NW = kHeadThreads / 32;
  return sizeof(float) * ((size_t)((H * A + 3) & ~3) + (size_t)R * H + (size_t)R * A +
                          (size_t)NW * (A + kStats));
}

int head_grid(int64_t M, int H) {
  const int64_t tiles = ceil_div(M, head_rows_per_tile(H));
  const int64_t cap = 2LL * sm_count();
  return (int)std::max<int64_t>(1, std::min<int64_t>(tiles, cap));
}

int head_launch(HeadParams p, int grid, cudaStream_t s) {
  SPO_CHECK_ARG(p.H > 0 && p.H <= kHeadThreads * kHeadMaxHJ && p.H % 4 == 0, kErrShape,
                "head: hidden width must be a multiple of 4 and at most 1024");
  SPO_CHECK_ARG(aligned16(p.act) && (!p.act_lo || aligned16(p.act_lo)), kErrAlign,
                "head: activations must be 16-byte aligned");
  SPO_CHECK_ARG(!p.dX_lo || p.dX, kErrArg, "head: dX_lo needs dX");
  SPO_CHECK_ARG(p.A == 1 || p.A == 9, kErrUnsupported, "head: output width must be 1 or 9");
  SPO_CHECK_ARG(p.mode == kHeadCritic ? p.target != nullptr : p.q != nullptr, kErrArg,
                "head: missing loss inputs");
  p.rows_per_tile = head_rows_per_tile(p.H);
  const size_t smem = head_smem_bytes(p.H, p.A);
  if (p.M == 0) return kOk;
  if (p.A == 9) {
    SPO_CUDA_TRY(cudaFuncSetAttribute(head_kernel<9>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
    head_kernel<9><<<grid, kHeadThreads, smem, s>>>(p);
  } else {
    SPO_CUDA_TRY(cudaFuncSetAttribute(head_kernel<1>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
    head_kernel<1><<<grid, kHeadThreads, smem, s>>>(p);
  }
  SPO_LAUNCH_CHECK();
  return kOk;
}

}  // namespace spo
