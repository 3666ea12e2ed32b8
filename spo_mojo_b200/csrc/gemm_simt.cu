// Instantiations and runtime dispatch of the FP32 CUDA-core GEMM (gemm_simt.cuh).
#include "gemm_simt.cuh"

namespace spo {

namespace {

template <int BM, int BN, int BK, int TM, int TN, int AOP, int BOP, int EPI>
int launch_v(const GemmParams& p, dim3 grid, cudaStream_t s, bool va, bool vb) {
  constexpr int NT = (BM / TM) * (BN / TN);
  if (va && vb)
    gemm_simt_kernel<BM, BN, BK, TM, TN, AOP, BOP, true, true, EPI><<<grid, NT, 0, s>>>(p);
  else if (va)
    gemm_simt_kernel<BM, BN, BK, TM, TN, AOP, BOP, true, false, EPI><<<grid, NT, 0, s>>>(p);
  else if (vb)
    gemm_simt_kernel<BM, BN, BK, TM, TN, AOP, BOP, false, true, EPI><<<grid, NT, 0, s>>>(p);
  else
    gemm_simt_kernel<BM, BN, BK, TM, TN, AOP, BOP, false, false, EPI><<<grid, NT, 0, s>>>(p);
  SPO_LAUNCH_CHECK();
  return kOk;
}

template <int BM, int BN, int BK, int TM, int TN>
int launch_tile(int aop, int bop, int epi, const GemmParams& p, dim3 grid, cudaStream_t s,
                bool va, bool vb) {
  if (aop == OP_ROW && bop == OP_ROW) {
    if (epi == EPI_BIAS) return launch_v<BM, BN, BK, TM, TN, OP_ROW, OP_ROW, EPI_BIAS>(p, grid, s, va, vb);
    if (epi == EPI_BIAS_RELU) return launch_v<BM, BN, BK, TM, TN, OP_ROW, OP_ROW, EPI_BIAS_RELU>(p, grid, s, va, vb);
    if (epi == EPI_BIAS_RELU_SPLIT) return launch_v<BM, BN, BK, TM, TN, OP_ROW, OP_ROW, EPI_BIAS_RELU_SPLIT>(p, grid, s, va, vb);
  } else if (aop == OP_ROW && bop == OP_COL) {
    if (epi == EPI_STORE) return launch_v<BM, BN, BK, TM, TN, OP_ROW, OP_COL, EPI_STORE>(p, grid, s, va, vb);
    if (epi == EPI_RELU_MASK) return launch_v<BM, BN, BK, TM, TN, OP_ROW, OP_COL, EPI_RELU_MASK>(p, grid, s, va, vb);
  } else if (aop == OP_COL && bop == OP_ROW) {
    if (epi == EPI_STORE) return launch_v<BM, BN, BK, TM, TN, OP_COL, OP_ROW, EPI_STORE>(p, grid, s, va, vb);
  }
  return set_error(kErrUnsupported, "gemm_simt: unsupported operand/epilogue combination");
}

}  // namespace

int gemm_simt_launch(int tile, int aop, int bop, int epi, GemmParams p, dim3 grid,
                     cudaStream_t s) {
  p.vec_c = aligned16(p.C) && p.ldc % 4 == 0 && p.N % 4 == 0 && p.c_split_stride % 4 == 0 &&
            (epi != EPI_RELU_MASK || (aligned16(p.mask) && p.ldm % 4 == 0));
  // Vector (float4) operand loads need the contiguous extent, the leading dimension
  // and the base pointer to be multiples of 4 floats.
  const bool va = aligned16(p.A) && p.lda % 4 == 0 &&
                  (aop == OP_ROW ? p.K % 4 == 0 : p.M % 4 == 0);
  const bool vb = aligned16(p.B) && p.ldb % 4 == 0 &&
                  (bop == OP_ROW ? p.N % 4 == 0 : p.K % 4 == 0);
  if (grid.x == 0 || grid.y == 0 || grid.z == 0) return kOk;
  if (tile == TILE_BIG) return launch_tile<128, 128, 8, 8, 8>(aop, bop, epi, p, grid, s, va, vb);
  return launch_tile<64, 64, 16, 4, 4>(aop, bop, epi, p, grid, s, va, vb);
}

}  // namespace spo
