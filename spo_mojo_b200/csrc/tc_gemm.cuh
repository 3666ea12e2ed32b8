// Tensor-core (tcgen05, sm_100a) GEMM of the learner's hidden layers, fp32-accurate
// through the 3xTF32 split, with the learner epilogues fused.
//
// Every fp32 operand x is held as a pair of exact TF32 values (hi, lo):
// hi = rna_tf32(x), lo = rna_tf32(x - hi), so x - hi - lo is below 2^-22 |x| and
// unbiased. Then
//   x . y ~= lo_x hi_y + hi_x lo_y + hi_x hi_y
// (the dropped lo_x lo_y term is ~2^-24 relative), accumulated in fp32 in tensor
// memory: the published error-compensated "3xTF32" method (the scheme CUTLASS calls
// 3xTF32; Ootomo & Yokota 2022). Products of hi/lo halves are exact in the tensor core,
// so the result carries near-fp32 error instead of TF32's 2^-11. The accumulator is
// folded into an fp32 running sum every few k-blocks (4 for the forward, 8 for dX and dW)
// to bound the error of the tensor memory accumulation.
#pragma once

#include <cuda.h>

#include "spo_common.cuh"

namespace spo {

enum TcKind : int {
  TC_FWD = 0,      // C = relu(A B + bias), written as (hi, lo)
  TC_DX = 1,       // C = (A B) * [mask > 0], written as (hi, lo), column sums
  TC_DX_F32 = 2,   // same, written as plain fp32
  TC_DW = 3,       // split-K partial tiles of A^T-style products (both operands MN-major)
};

struct TcGemmArgs {
  int kind;
  // Operand arrays (each a hi/lo pair). Layout in memory:
  //   TC_FWD/TC_DX: A row-major [M x K] (pitch K), B row-major [N x K] (pitch K)
  //   TC_DW:        A row-major [K x M] (pitch M), B row-major [K x N] (pitch N)
  const float* a_hi;
  const float* a_lo;
  const float* b_hi;
  const float* b_lo;
  int64_t M, N, K;
  int64_t k_chunk;         // TC_DW: rows of K per split (multiple of 32)
  const float* bias;       // TC_FWD: [N]
  const float* mask;       // TC_DX*: [M x N] (pitch N), keep where > 0
  float* c_hi;             // [M x N] (pitch N): hi or fp32 result
  float* c_lo;             // [M x N] (pitch N): lo (TC_DX; TC_FWD: null = fp32 into c_hi)
  float* c_part;           // TC_DW: [splits][M x N]
  float* colsum;           // TC_DX*: [grid][N] column sums (optional)
  int* err;                // device error word (bounded waits), optional
  // ReLU mask packed one bit per element: row-major [M x N/32] 32-bit words, bit j of
  // word w of a row = column 32 w + j.
  const uint32_t* mask_bits;  // TC_DX*: used instead of mask when set (bit = keep)
  uint32_t* c_bits;           // TC_FWD: optional output, bit = (output > 0)
  // Tests of the timeout path only: the limit of every bounded wait (0: 2 s) and
  // 1 + the k-block whose operands the producer never loads (0: none).
  uint64_t wait_ns;
  uint32_t withhold;
};

// Launch configuration queries (host).
int tc_gemm_grid(const TcGemmArgs& a);     // CTAs the launch will use (= colsum parts)
int tc_gemm_splits(const TcGemmArgs& a);   // TC_DW partial count
int64_t tc_gemm_tiles(int kind, int64_t M, int64_t N);  // output tiles (units per split)
int tc_gemm_slots(int kind, int64_t N);     // units that run at once (SMs or CTA pairs)
bool tc_gemm_supported(int kind, int64_t M, int64_t N, int64_t K);
// 2-D fp32 tensor map of a row-major [outer x inner] array (host; error code, kOk).
int make_map(CUtensorMap* m, const float* ptr, uint64_t inner, uint64_t outer, uint32_t box_inner,
             uint32_t box_outer, CUtensorMapSwizzle swz);
int tc_gemm_launch(const TcGemmArgs& a, cudaStream_t s);

// hi/lo split of n floats (elementwise); keep_positive: a positive x never gets hi == 0
// (so hi > 0 <=> x > 0, the ReLU mask test).
int split_tf32_launch(const float* x, float* hi, float* lo, int64_t n, bool keep_positive,
                      cudaStream_t s);
// hi[i] += lo[i] (back to plain fp32, in place).
int combine_tf32_launch(float* hi, const float* lo, int64_t n, cudaStream_t s);
// W [K x N] -> Wt_hi/Wt_lo [N x K] (transposed) and W_hi/W_lo [K x N].
int split_weights_launch(const float* w, int64_t K, int64_t N, float* wt_hi, float* wt_lo,
                         float* w_hi, float* w_lo, cudaStream_t s);

}  // namespace spo
