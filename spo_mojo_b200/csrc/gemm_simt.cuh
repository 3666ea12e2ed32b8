// FP32 CUDA-core GEMM for the learner's Linear layers, with the epilogues fused.
//
//   C[M x N] = A[M x K] . B[K x N]   (fp32 in, fp32 FMA accumulation, fp32 out)
//
// One template covers the three products of a Linear layer
// (networks/linear.mojo:37-167 computes them with three separate kernels):
//   forward  y  = x W + b (+ReLU)      A = x   (row-major), B = W   (row-major)
//   dX       dZ = (dY W^T) * [a > 0]   A = dY  (row-major), B = W^T (W row-major)
//   dW       dW = x^T dY               A = x^T (x row-major), B = dY, split over rows
// and, optionally, per-CTA column sums of the stored C (the bias gradient of the
// layer below, whose input gradient this kernel produces).
//
// Tiling: BM x BN output tile per CTA, BK-deep k-steps double-buffered through
// shared memory (register-staged prefetch), TM x TN outputs per thread read as
// float4 fragments from k-major shared tiles. The grid's y dimension strides over
// M tiles (persistent in M, so column sums need one partial per blockIdx.y), the z
// dimension splits K into chunks that write separate partial outputs (dW).
#pragma once

#include "spo_common.cuh"

namespace spo {

enum : int { OP_ROW = 0, OP_COL = 1 };
// EPI_BIAS_RELU_SPLIT: bias + ReLU written as a TF32 hi/lo pair (C = hi, C2 = lo), the
// operand format of the tensor-core layers that consume it.
enum : int { EPI_STORE = 0, EPI_BIAS = 1, EPI_BIAS_RELU = 2, EPI_RELU_MASK = 3, EPI_BIAS_RELU_SPLIT = 4 };

struct GemmParams {
  const float* A;
  const float* B;
  float* C;
  float* C2;               // EPI_BIAS_RELU_SPLIT: lo half, same layout as C
  const float* bias;       // EPI_BIAS*: [N]
  const float* mask;       // EPI_RELU_MASK: keep C where mask[m * ldm + n] > 0
  float* colsum;           // optional: [gridDim.y][N] column sums of the stored C
  int64_t M, N, K;
  int64_t lda, ldb, ldc, ldm;
  int64_t k_chunk;         // K extent per blockIdx.z (multiple of BK)
  int64_t c_split_stride;  // offset of blockIdx.z's partial C
  int vec_c;               // C / mask rows can be accessed as float4
};

// A(m,k): OP_ROW -> A[m*lda + k], OP_COL -> A[k*lda + m]
// B(k,n): OP_ROW -> B[k*ldb + n], OP_COL -> B[n*ldb + k]
template <int BM, int BN, int BK, int TM, int TN, int AOP, int BOP, bool VA, bool VB, int EPI>
__global__ void __launch_bounds__((BM / TM) * (BN / TN), (BM * BN >= 128 * 128) ? 2 : 1)
gemm_simt_kernel(const GemmParams p) {
  constexpr int TX = BN / TN, TY = BM / TM, NT = TX * TY;
  constexpr int PAD = 4;
  constexpr int AS = BM + PAD, BS = BN + PAD;
  constexpr int A_ELEMS = BM * BK / NT, B_ELEMS = BK * BN / NT;
  constexpr int A_OPS = VA ? A_ELEMS / 4 : A_ELEMS;
  constexpr int B_OPS = VB ? B_ELEMS / 4 : B_ELEMS;
  static_assert(TM % 4 == 0 && TN % 4 == 0, "thread tile must be float4 fragments");
  static_assert((BM * BK) % NT == 0 && (BK * BN) % NT == 0, "tile/threads mismatch");
  static_assert(!VA || A_ELEMS % 4 == 0, "vector A load");
  static_assert(!VB || B_ELEMS % 4 == 0, "vector B load");
  static_assert(BN * TY <= 2 * BK * (AS + BS), "column-sum scratch must fit");

  __shared__ __align__(16) float smem[2 * BK * AS + 2 * BK * BS];
  float* As = smem;
  float* Bs = smem + 2 * BK * AS;

  const int tid = threadIdx.x;
  const int tx = tid % TX, ty = tid / TX;
  const int64_t n0 = (int64_t)blockIdx.x * BN;
  const int64_t m_tiles = (p.M + BM - 1) / BM;
  const int64_t kbeg = (int64_t)blockIdx.z * p.k_chunk;
  const int64_t kend = min(p.K, kbeg + p.k_chunk);
  const int nk = kend > kbeg ? (int)((kend - kbeg + BK - 1) / BK) : 0;
  float* C = p.C + (int64_t)blockIdx.z * p.c_split_stride;

  float ra[A_ELEMS];
  float rb[B_ELEMS];
  float cs[TN];
#pragma unroll
  for (int j = 0; j < TN; ++j) cs[j] = 0.f;

  for (int64_t mt = blockIdx.y; mt < m_tiles; mt += gridDim.y) {
    const int64_t m0 = mt * BM;

    auto load_a = [&](int64_t k0) {
#pragma unroll
      for (int i = 0; i < A_OPS; ++i) {
        const int f = tid + i * NT;
        if (VA) {
          int ml, kl;
          if (AOP == OP_ROW) { ml = f / (BK / 4); kl = (f % (BK / 4)) * 4; }
          else               { kl = f / (BM / 4); ml = (f % (BM / 4)) * 4; }
          const int64_t m = m0 + ml, k = k0 + kl;
          float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
          if (m < p.M && k < kend) {
            const float* src = AOP == OP_ROW ? p.A + m * p.lda + k : p.A + k * p.lda + m;
            v = __ldg(reinterpret_cast<const float4*>(src));
          }
          ra[4 * i + 0] = v.x; ra[4 * i + 1] = v.y; ra[4 * i + 2] = v.z; ra[4 * i + 3] = v.w;
        } else {
          int ml, kl;
          if (AOP == OP_ROW) { ml = f / BK; kl = f % BK; }
          else               { kl = f / BM; ml = f % BM; }
          const int64_t m = m0 + ml, k = k0 + kl;
          float v = 0.f;
          if (m < p.M && k < kend)
            v = __ldg(AOP == OP_ROW ? p.A + m * p.lda + k : p.A + k * p.lda + m);
          ra[i] = v;
        }
      }
    };
    auto store_a = [&](int buf) {
      float* dst = As + buf * BK * AS;
#pragma unroll
      for (int i = 0; i < A_OPS; ++i) {
        const int f = tid + i * NT;
        if (VA) {
          if (AOP == OP_ROW) {
            const int ml = f / (BK / 4), kl = (f % (BK / 4)) * 4;
#pragma unroll
            for (int j = 0; j < 4; ++j) dst[(kl + j) * AS + ml] = ra[4 * i + j];
          } else {
            const int kl = f / (BM / 4), ml = (f % (BM / 4)) * 4;
            *reinterpret_cast<float4*>(dst + kl * AS + ml) =
                make_float4(ra[4 * i], ra[4 * i + 1], ra[4 * i + 2], ra[4 * i + 3]);
          }
        } else {
          int ml, kl;
          if (AOP == OP_ROW) { ml = f / BK; kl = f % BK; }
          else               { kl = f / BM; ml = f % BM; }
          dst[kl * AS + ml] = ra[i];
        }
      }
    };
    auto load_b = [&](int64_t k0) {
#pragma unroll
      for (int i = 0; i < B_OPS; ++i) {
        const int f = tid + i * NT;
        if (VB) {
          int nl, kl;
          if (BOP == OP_ROW) { kl = f / (BN / 4); nl = (f % (BN / 4)) * 4; }
          else               { nl = f / (BK / 4); kl = (f % (BK / 4)) * 4; }
          const int64_t n = n0 + nl, k = k0 + kl;
          float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
          if (n < p.N && k < kend) {
            const float* src = BOP == OP_ROW ? p.B + k * p.ldb + n : p.B + n * p.ldb + k;
            v = __ldg(reinterpret_cast<const float4*>(src));
          }
          rb[4 * i + 0] = v.x; rb[4 * i + 1] = v.y; rb[4 * i + 2] = v.z; rb[4 * i + 3] = v.w;
        } else {
          int nl, kl;
          if (BOP == OP_ROW) { kl = f / BN; nl = f % BN; }
          else               { nl = f / BK; kl = f % BK; }
          const int64_t n = n0 + nl, k = k0 + kl;
          float v = 0.f;
          if (n < p.N && k < kend)
            v = __ldg(BOP == OP_ROW ? p.B + k * p.ldb + n : p.B + n * p.ldb + k);
          rb[i] = v;
        }
      }
    };
    auto store_b = [&](int buf) {
      float* dst = Bs + buf * BK * BS;
#pragma unroll
      for (int i = 0; i < B_OPS; ++i) {
        const int f = tid + i * NT;
        if (VB) {
          if (BOP == OP_ROW) {
            const int kl = f / (BN / 4), nl = (f % (BN / 4)) * 4;
            *reinterpret_cast<float4*>(dst + kl * BS + nl) =
                make_float4(rb[4 * i], rb[4 * i + 1], rb[4 * i + 2], rb[4 * i + 3]);
          } else {
            const int nl = f / (BK / 4), kl = (f % (BK / 4)) * 4;
#pragma unroll
            for (int j = 0; j < 4; ++j) dst[(kl + j) * BS + nl] = rb[4 * i + j];
          }
        } else {
          int nl, kl;
          if (BOP == OP_ROW) { kl = f / BN; nl = f % BN; }
          else               { nl = f / BK; kl = f % BK; }
          dst[kl * BS + nl] = rb[i];
        }
      }
    };

    float acc[TM][TN];
#pragma unroll
    for (int i = 0; i < TM; ++i)
#pragma unroll
      for (int j = 0; j < TN; ++j) acc[i][j] = 0.f;

    if (nk > 0) {
      load_a(kbeg);
      load_b(kbeg);
      store_a(0);
      store_b(0);
      __syncthreads();
      for (int t = 0; t < nk; ++t) {
        const int cur = t & 1;
        if (t + 1 < nk) {
          load_a(kbeg + (int64_t)(t + 1) * BK);
          load_b(kbeg + (int64_t)(t + 1) * BK);
        }
        const float* a_s = As + cur * BK * AS;
        const float* b_s = Bs + cur * BK * BS;
#pragma unroll
        for (int kk = 0; kk < BK; ++kk) {
          float a[TM], b[TN];
#pragma unroll
          for (int c = 0; c < TM / 4; ++c) {
            const float4 v = *reinterpret_cast<const float4*>(a_s + kk * AS + c * TY * 4 + ty * 4);
            a[4 * c] = v.x; a[4 * c + 1] = v.y; a[4 * c + 2] = v.z; a[4 * c + 3] = v.w;
          }
#pragma unroll
          for (int c = 0; c < TN / 4; ++c) {
            const float4 v = *reinterpret_cast<const float4*>(b_s + kk * BS + c * TX * 4 + tx * 4);
            b[4 * c] = v.x; b[4 * c + 1] = v.y; b[4 * c + 2] = v.z; b[4 * c + 3] = v.w;
          }
#pragma unroll
          for (int i = 0; i < TM; ++i)
#pragma unroll
            for (int j = 0; j < TN; ++j) acc[i][j] = fmaf(a[i], b[j], acc[i][j]);
        }
        if (t + 1 < nk) {
          store_a(cur ^ 1);
          store_b(cur ^ 1);
        }
        __syncthreads();
      }
    }

    // Epilogue: bias / ReLU / ReLU-mask, store, column sums.
#pragma unroll
    for (int i = 0; i < TM; ++i) {
      const int64_t row = m0 + (i / 4) * TY * 4 + ty * 4 + (i % 4);
      if (row >= p.M) continue;
#pragma unroll
      for (int cj = 0; cj < TN / 4; ++cj) {
        const int64_t col0 = n0 + cj * TX * 4 + tx * 4;
        float v[4] = {acc[i][cj * 4], acc[i][cj * 4 + 1], acc[i][cj * 4 + 2], acc[i][cj * 4 + 3]};
        const bool full = p.vec_c && col0 + 3 < p.N;
        float lo[4] = {0.f, 0.f, 0.f, 0.f};
        if (EPI == EPI_BIAS || EPI == EPI_BIAS_RELU || EPI == EPI_BIAS_RELU_SPLIT) {
#pragma unroll
          for (int j = 0; j < 4; ++j) {
            if (col0 + j < p.N) v[j] += __ldg(p.bias + col0 + j);
            if (EPI != EPI_BIAS) v[j] = v[j] > 0.f ? v[j] : 0.f;
            if (EPI == EPI_BIAS_RELU_SPLIT) tf32_split_pos(v[j], v[j], lo[j]);
          }
        } else if (EPI == EPI_RELU_MASK) {
          if (full) {
            const float4 mk = __ldg(reinterpret_cast<const float4*>(p.mask + row * p.ldm + col0));
            v[0] = mk.x > 0.f ? v[0] : 0.f;
            v[1] = mk.y > 0.f ? v[1] : 0.f;
            v[2] = mk.z > 0.f ? v[2] : 0.f;
            v[3] = mk.w > 0.f ? v[3] : 0.f;
          } else {
#pragma unroll
            for (int j = 0; j < 4; ++j)
              if (col0 + j < p.N) v[j] = __ldg(p.mask + row * p.ldm + col0 + j) > 0.f ? v[j] : 0.f;
          }
        }
        if (full) {
          *reinterpret_cast<float4*>(C + row * p.ldc + col0) = make_float4(v[0], v[1], v[2], v[3]);
          if (EPI == EPI_BIAS_RELU_SPLIT)
            *reinterpret_cast<float4*>(p.C2 + row * p.ldc + col0) = make_float4(lo[0], lo[1], lo[2], lo[3]);
        } else {
#pragma unroll
          for (int j = 0; j < 4; ++j)
            if (col0 + j < p.N) {
              C[row * p.ldc + col0 + j] = v[j];
              if (EPI == EPI_BIAS_RELU_SPLIT) p.C2[row * p.ldc + col0 + j] = lo[j];
            }
        }
#pragma unroll
        for (int j = 0; j < 4; ++j)
          if (col0 + j < p.N) cs[cj * 4 + j] += v[j];
      }
    }
  }

  if (p.colsum != nullptr) {
    __syncthreads();
#pragma unroll
    for (int cj = 0; cj < TN / 4; ++cj)
#pragma unroll
      for (int j = 0; j < 4; ++j) smem[ty * BN + cj * TX * 4 + tx * 4 + j] = cs[cj * 4 + j];
    __syncthreads();
    for (int c = tid; c < BN; c += NT) {
      float s = 0.f;
#pragma unroll 4
      for (int y = 0; y < TY; ++y) s += smem[y * BN + c];
      const int64_t col = n0 + c;
      if (col < p.N) p.colsum[(int64_t)blockIdx.y * p.N + col] = s;
    }
  }
}

// Tile shapes: "big" 128x128 (8x8 per thread), "small" 64x64 (4x4 per thread).
enum GemmTile : int { TILE_BIG = 0, TILE_SMALL = 1 };

struct GemmShape {
  int bm, bn, bk;
};
inline GemmShape gemm_shape(int tile) {
  return tile == TILE_BIG ? GemmShape{128, 128, 8} : GemmShape{64, 64, 16};
}

// Host dispatch (gemm_simt.cu). grid.z splits K with p.k_chunk; grid.y strides M.
int gemm_simt_launch(int tile, int aop, int bop, int epi, GemmParams p, dim3 grid,
                     cudaStream_t s);

// Picks the tile for an M x N output.
inline int gemm_pick_tile(int64_t M, int64_t N) {
  return (M >= 128 && N >= 128 && M * N >= (int64_t)128 * 128 * 96) ? TILE_BIG : TILE_SMALL;
}

}  // namespace spo
