// The first layer of the learner's MLPs, whose input is narrow: x [rows x k] with k <= 32
// (the 27-wide board encoding). The CUDA-core GEMM tiles waste most of a 64- or 128-wide
// tile on k = 27; these kernels stream the wide side once, at the HBM rate.
//
// Forward (linear_forward + relu, networks/linear.mojo:37-95, networks/mlp.mojo:34-46):
// y = relu(x W + b), W [k x n]. CTA = 128 threads over 512 columns: thread t keeps its 4
// columns of W (k x 4 values) and of b in registers and walks the rows of its CTA; the
// rows of x are staged in shared memory and read as broadcasts. Each row's outputs leave
// as one float4 per thread (2 KB contiguous per CTA), optionally as a TF32 hi/lo pair and
// with the packed ReLU mask (bit j of word w = column 32 w + j).
//
// Both kernels can take board cells [rows x 9] (+1 agent / -1 rival / 0 empty) instead of
// x: the cells are staged and expanded in shared memory into the 27-wide plane-major
// [empty | agent | rival] rows (envs/tictactoe.mojo:449-480), the observation encoding
// fused into the first layer's load stage.
//
// Weight gradient: dW[k x n] = x^T dY summed over rows, dY [rows x n].
// CTA = 256 threads over one chunk of rows and 512 columns: thread t owns the 4 columns
// 4 (t % 128) .. +3 of its column block and one half of the k features (t / 128: 16
// feature slots, or 14 when k <= 28), so its accumulators are [half of k] x 4. With fewer
// columns (n / 4 dividing 128) the spare threads take interleaved rows of the same
// columns and hand their sums over at the end. Rows are walked in blocks of kRows: the block's x rows
// are staged in shared memory (zero-padded to 32 features) and read as broadcasts, the dY
// float4 of each row is loaded straight from global memory, 8 rows in flight per thread.
// Each CTA writes its partial [k x n] tile to part[chunk]; a deterministic reduction adds
// the chunks (linear_backward's dW, networks/linear.mojo:120-167).
#include <cmath>

#include "spo_common.cuh"
#include "kernels.cuh"

namespace spo {

namespace {

constexpr int kThreads = 256;
constexpr int kCols = 512;       // columns per CTA (128 threads x float4)
constexpr int kMaxK = 32;
constexpr int kRows = 64;        // rows staged per block
constexpr int kUnroll = 8;
constexpr int kCells = 9;        // board cells per row (cells input)
constexpr int kPadK = 32;        // input width of the first layer on tensor cores

__device__ __forceinline__ void cp_async4(float* dst, const float* src) {
  asm volatile("cp.async.ca.shared.global [%0], [%1], 4;" ::"r"(static_cast<uint32_t>(__cvta_generic_to_shared(dst))),
               "l"(src)
               : "memory");
}

// Double-buffered staging of the rows of x [rows x k] (k <= kMaxK) in shared memory.
// Columns k..kMaxK-1 stay zero (cleared once); a block of kRows rows is copied with
// 4-byte cp.async (consecutive threads take consecutive elements: coalesced), one block
// ahead of the one being consumed.
struct XStage {
  float (*xs)[kRows][kMaxK];  // [2][kRows][kMaxK]
  float (*cs)[kRows][kCells];  // [2][kRows][kCells] staged board cells (cells != null)
  const float* x;
  const float* cells;
  int k;
  int64_t r_begin, r_end;
  __device__ void clear(int tid, int nthreads) {
    for (int e = tid; e < 2 * kRows * kMaxK; e += nthreads) (&xs[0][0][0])[e] = 0.f;
  }
  // issue the copies of block b (rows r_begin + b*kRows ..) into buffer b & 1
  __device__ void issue(int64_t b, int tid, int nthreads) {
    const int64_t rb = r_begin + b * kRows;
    if (rb < r_end) {
      const int nr = (int)min((int64_t)kRows, r_end - rb);
      if (cells) {
        float* buf = &cs[b & 1][0][0];
        const float* src = cells + rb * kCells;
        for (int e = tid; e < nr * kCells; e += nthreads) cp_async4(buf + e, src + e);
      } else {
        float (*buf)[kMaxK] = xs[b & 1];
        const float* src = x + rb * k;
        for (int e = tid; e < nr * k; e += nthreads) {
          const int r = e / k, i = e - r * k;
          cp_async4(&buf[r][i], src + e);
        }
      }
    }
    asm volatile("cp.async.commit_group;" ::: "memory");
  }
  // cells only: expand staged block b into its x rows (call between two barriers)
  __device__ void expand(int64_t b, int nr, int tid, int nthreads) {
    float (*dst)[kMaxK] = xs[b & 1];
    const float* src = &cs[b & 1][0][0];
    for (int e = tid; e < nr * kCells; e += nthreads) {
      const int r = e / kCells, c = e - r * kCells;
      const float v = src[e];
      dst[r][c] = v == 0.f ? 1.f : 0.f;
      dst[r][kCells + c] = v == 1.f ? 1.f : 0.f;
      dst[r][2 * kCells + c] = v == -1.f ? 1.f : 0.f;
    }
  }
  __device__ static void wait_prev() { asm volatile("cp.async.wait_group 1;" ::: "memory"); }
};

// KH features per thread: 16 (any k <= 32), or 14 when k <= 28 (the 27-wide board input:
// 28 feature slots instead of 32, one in eight packed FMAs fewer; the x pairs of the
// second half start at feature 14 and are read as float2).
template <int KH>
__global__ void __launch_bounds__(kThreads, 2)
dw_skinny_kernel(const float* __restrict__ x, const float* __restrict__ cells, const float* __restrict__ dy,
                 int64_t rows, int k, int64_t n, int64_t chunk, float* __restrict__ part) {
  __shared__ __align__(16) float xs2[2][kRows][kMaxK];
  __shared__ __align__(16) float cs2[2][kRows][kCells];
  pdl_wait();
  pdl_trigger();
  const int tid = threadIdx.x;
  const int half = tid / 128;
  // Fewer than 512 columns: the 128 threads of a half split into RS row subgroups of n/4
  // column threads each (subgroup s takes rows s, s + RS, ... of every block); their sums
  // are added in subgroup order at the end.
  const int rs = (n < kCols && 128 % (n / 4) == 0) ? (int)(128 / (n / 4)) : 1;
  const int per = 128 / rs, ct = (tid % 128) % per, rsub = (tid % 128) / per;
  const int64_t col = (int64_t)blockIdx.y * kCols + 4 * ct;
  const bool col_ok = col < n;
  const int64_t r_begin = (int64_t)blockIdx.x * chunk;
  const int64_t r_end = min(rows, r_begin + chunk);
  const int i0 = half * KH;

  // per column, adjacent features as packed pairs: one FFMA2 (two fp32 fma.rn, the same
  // results as fmaf) per pair; the x pairs come straight from the staged float4 reads and
  // only the dY value is broadcast into a pair
  float2 acc[4][KH / 2];
#pragma unroll
  for (int q = 0; q < 4; ++q)
#pragma unroll
    for (int i = 0; i < KH / 2; ++i) acc[q][i] = make_float2(0.f, 0.f);

  XStage st{xs2, cs2, x, cells, k, r_begin, r_end};
  st.clear(tid, kThreads);
  __syncthreads();
  st.issue(0, tid, kThreads);
  int64_t blk = 0;
  for (int64_t rb = r_begin; rb < r_end; rb += kRows, ++blk) {
    const int nr = (int)min((int64_t)kRows, r_end - rb);
    st.issue(blk + 1, tid, kThreads);  // the buffer it fills was released by the last barrier
    XStage::wait_prev();
    __syncthreads();
    if (cells) {
      st.expand(blk, nr, tid, kThreads);
      __syncthreads();
    }
    float (*xs)[kMaxK] = xs2[blk & 1];
    if (col_ok) {
      for (int r0 = rsub; r0 < nr; r0 += kUnroll * rs) {
        float4 g[kUnroll];
#pragma unroll
        for (int u = 0; u < kUnroll; ++u)
          g[u] = r0 + u * rs < nr ? __ldg(reinterpret_cast<const float4*>(dy + (rb + r0 + u * rs) * n + col))
                                  : make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
        for (int u = 0; u < kUnroll; ++u) {
          const int xr_row = min(r0 + u * rs, kRows - 1);   // past nr: dY is zero there
          const float gv[4] = {g[u].x, g[u].y, g[u].z, g[u].w};
          if constexpr (KH == 16) {
            const float4* xr = reinterpret_cast<const float4*>(&xs[xr_row][i0]);
#pragma unroll
            for (int q = 0; q < 4; ++q) {
              const float2 gg = make_float2(gv[q], gv[q]);
#pragma unroll
              for (int c = 0; c < KH / 4; ++c) {
                const float4 xv = xr[c];
                acc[q][2 * c] = __ffma2_rn(make_float2(xv.x, xv.y), gg, acc[q][2 * c]);
                acc[q][2 * c + 1] = __ffma2_rn(make_float2(xv.z, xv.w), gg, acc[q][2 * c + 1]);
              }
            }
          } else {
            const float2* xr = reinterpret_cast<const float2*>(&xs[xr_row][i0]);
#pragma unroll
            for (int q = 0; q < 4; ++q) {
              const float2 gg = make_float2(gv[q], gv[q]);
#pragma unroll
              for (int c = 0; c < KH / 2; ++c) acc[q][c] = __ffma2_rn(xr[c], gg, acc[q][c]);
            }
          }
        }
      }
    }
    __syncthreads();  // buffer blk & 1 is consumed before block blk + 2 is copied into it
  }
  asm volatile("cp.async.wait_group 0;" ::: "memory");
  if (rs > 1) {
    // row subgroups 1 .. rs-1 hand their sums to subgroup 0 through shared memory (the
    // staging buffers are free now), one subgroup and one column of the 4 at a time
    float* buf = &xs2[0][0][0];   // [2 halves][per][KH]
    for (int s = 1; s < rs; ++s) {
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        __syncthreads();
        if (rsub == s)
#pragma unroll
          for (int i = 0; i < KH / 2; ++i) {
            buf[(half * per + ct) * KH + 2 * i] = acc[q][i].x;
            buf[(half * per + ct) * KH + 2 * i + 1] = acc[q][i].y;
          }
        __syncthreads();
        if (rsub == 0)
#pragma unroll
          for (int i = 0; i < KH / 2; ++i) {
            acc[q][i].x += buf[(half * per + ct) * KH + 2 * i];
            acc[q][i].y += buf[(half * per + ct) * KH + 2 * i + 1];
          }
      }
    }
    if (rsub != 0) return;
  }
  if (!col_ok) return;
  float* out = part + (int64_t)blockIdx.x * k * n;
#pragma unroll
  for (int i = 0; i < KH; ++i) {
    const int f = i0 + i;
    if (f < k) {
      auto pick = [&](int q) { return (i & 1) ? acc[q][i / 2].y : acc[q][i / 2].x; };
      *reinterpret_cast<float4*>(out + (int64_t)f * n + col) = make_float4(pick(0), pick(1), pick(2), pick(3));
    }
  }
}

constexpr int kFwdThreads = 128;

__global__ void __launch_bounds__(kFwdThreads, 3)
fwd_skinny_kernel(const float* __restrict__ x, const float* __restrict__ cells, const float* __restrict__ w,
                  const float* __restrict__ b, int64_t rows, int k, int64_t n, int64_t chunk, float* __restrict__ y,
                  float* __restrict__ y_lo, uint32_t* __restrict__ bits) {
  __shared__ __align__(16) float xs2[2][kRows][kMaxK];
  __shared__ __align__(16) float cs2[2][kRows][kCells];
  pdl_wait();
  pdl_trigger();
  const int tid = threadIdx.x, lane = tid & 31;
  const int64_t col = (int64_t)blockIdx.y * kCols + 4 * tid;
  const bool col_ok = col < n;
  float wr[kMaxK][4];
#pragma unroll
  for (int i = 0; i < kMaxK; ++i) {
    const float4 v = (col_ok && i < k) ? __ldg(reinterpret_cast<const float4*>(w + (int64_t)i * n + col))
                                      : make_float4(0.f, 0.f, 0.f, 0.f);
    wr[i][0] = v.x; wr[i][1] = v.y; wr[i][2] = v.z; wr[i][3] = v.w;
  }
  const float4 bv = col_ok ? __ldg(reinterpret_cast<const float4*>(b + col)) : make_float4(0.f, 0.f, 0.f, 0.f);
  const int64_t r_begin = (int64_t)blockIdx.x * chunk;
  const int64_t r_end = min(rows, r_begin + chunk);
  XStage st{xs2, cs2, x, cells, k, r_begin, r_end};
  st.clear(tid, kFwdThreads);
  __syncthreads();
  st.issue(0, tid, kFwdThreads);
  int64_t blk = 0;
  for (int64_t rb = r_begin; rb < r_end; rb += kRows, ++blk) {
    const int nr = (int)min((int64_t)kRows, r_end - rb);
    st.issue(blk + 1, tid, kFwdThreads);
    XStage::wait_prev();
    __syncthreads();
    if (cells) {
      st.expand(blk, nr, tid, kFwdThreads);
      __syncthreads();
    }
    float (*xs)[kMaxK] = xs2[blk & 1];
    for (int r = 0; r < nr; ++r) {
      // products summed in k order from zero, then the bias (the CUDA-core GEMM's order)
      float a0 = 0.f, a1 = 0.f, a2 = 0.f, a3 = 0.f;
      const float4* xr = reinterpret_cast<const float4*>(xs[r]);
#pragma unroll
      for (int c = 0; c < kMaxK / 4; ++c) {
        const float4 xv = xr[c];
        const float xa[4] = {xv.x, xv.y, xv.z, xv.w};
#pragma unroll
        for (int t = 0; t < 4; ++t) {
          a0 = fmaf(xa[t], wr[4 * c + t][0], a0);
          a1 = fmaf(xa[t], wr[4 * c + t][1], a1);
          a2 = fmaf(xa[t], wr[4 * c + t][2], a2);
          a3 = fmaf(xa[t], wr[4 * c + t][3], a3);
        }
      }
      float v[4] = {a0 + bv.x, a1 + bv.y, a2 + bv.z, a3 + bv.w};
#pragma unroll
      for (int t = 0; t < 4; ++t) v[t] = v[t] > 0.f ? v[t] : 0.f;
      const int64_t row = rb + r;
      if (col_ok) {
        if (y_lo) {
          float h[4], l[4];
#pragma unroll
          for (int t = 0; t < 4; ++t) tf32_split_pos(v[t], h[t], l[t]);
          *reinterpret_cast<float4*>(y + row * n + col) = make_float4(h[0], h[1], h[2], h[3]);
          *reinterpret_cast<float4*>(y_lo + row * n + col) = make_float4(l[0], l[1], l[2], l[3]);
        } else {
          *reinterpret_cast<float4*>(y + row * n + col) = make_float4(v[0], v[1], v[2], v[3]);
        }
      }
      if (bits) {
        // 8 threads cover 32 columns: OR their nibbles, the first of them stores the word
        uint32_t m = ((v[0] > 0.f ? 1u : 0u) | (v[1] > 0.f ? 2u : 0u) | (v[2] > 0.f ? 4u : 0u) |
                      (v[3] > 0.f ? 8u : 0u)) << (4 * (lane & 7));
        m |= __shfl_xor_sync(0xffffffffu, m, 1);
        m |= __shfl_xor_sync(0xffffffffu, m, 2);
        m |= __shfl_xor_sync(0xffffffffu, m, 4);
        if ((lane & 7) == 0 && col_ok) bits[row * (n / 32) + col / 32] = m;
      }
    }
    __syncthreads();  // buffer blk & 1 is consumed before block blk + 2 is copied into it
  }
  asm volatile("cp.async.wait_group 0;" ::: "memory");
}

// Tensor-core operands of the first layer: the input rows padded to kPadK columns (zeros
// past k), as plain fp32 (lo null) or TF32 hi/lo pairs, and W^T [n x kPadK] as hi/lo
// pairs. One thread per element.
__global__ void pad_split_input_kernel(const float* __restrict__ x, const float* __restrict__ cells, int k,
                                       int64_t rows, float* __restrict__ hi, float* __restrict__ lo) {
  pdl_wait();
  pdl_trigger();
  const int64_t gs = (int64_t)gridDim.x * blockDim.x;
  for (int64_t e = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; e < rows * kPadK; e += gs) {
    const int64_t r = e / kPadK;
    const int c = (int)(e - r * kPadK);
    float v = 0.f;
    if (c < k) {
      if (cells) {
        const int cell = c % kCells, plane = c / kCells;
        const float cv = __ldg(cells + r * kCells + cell);
        v = (plane == 0 ? cv == 0.f : (plane == 1 ? cv == 1.f : cv == -1.f)) ? 1.f : 0.f;
      } else {
        v = __ldg(x + r * k + c);
      }
    }
    if (lo) {
      float h, l;
      tf32_split(v, h, l);
      hi[e] = h;
      lo[e] = l;
    } else {
      hi[e] = v;   // plain fp32: the tensor-core kernel splits it
    }
  }
}

__global__ void split_weights_t_pad_kernel(const float* __restrict__ w, int k, int64_t n, float* __restrict__ wt_hi,
                                           float* __restrict__ wt_lo) {
  pdl_wait();
  pdl_trigger();
  const int64_t gs = (int64_t)gridDim.x * blockDim.x;
  for (int64_t e = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; e < n * kPadK; e += gs) {
    const int64_t col = e / kPadK;
    const int i = (int)(e - col * kPadK);
    const float v = i < k ? __ldg(w + (int64_t)i * n + col) : 0.f;
    float h, l;
    tf32_split(v, h, l);
    wt_hi[e] = h;
    wt_lo[e] = l;
  }
}

}  // namespace

bool dw_skinny_ok(int64_t k, int64_t n) { return k >= 1 && k <= kMaxK && n >= 4 && n % 4 == 0; }

bool fwd_skinny_ok(int64_t k, int64_t n) { return k >= 1 && k <= kMaxK && n >= 4 && n % 4 == 0; }

int pad_split_input_launch(LayerInput in, int64_t k, int64_t rows, float* hi, float* lo, cudaStream_t s) {
  SPO_CHECK_ARG(k >= 1 && k <= kPadK, kErrUnsupported, "pad_split_input: input wider than 32");
  SPO_CHECK_ARG(!in.cells || k == 3 * kCells, kErrShape, "pad_split_input: board cells need a 27-wide input");
  if (rows <= 0) return kOk;
  const int grid = (int)std::min<int64_t>(ceil_div(rows * kPadK, 256), 8LL * sm_count());
  SPO_CUDA_TRY(launch_pdl(pad_split_input_kernel, dim3(grid), dim3(256), 0, s, 0u, in.x, in.cells, (int)k, rows, hi,
                          lo));
  return kOk;
}

int split_weights_t_pad_launch(const float* w, int64_t k, int64_t n, float* wt_hi, float* wt_lo, cudaStream_t s) {
  SPO_CHECK_ARG(k >= 1 && k <= kPadK && n >= 1, kErrUnsupported, "split_weights_t_pad: bad shape");
  const int grid = (int)std::min<int64_t>(ceil_div(n * kPadK, 256), 8LL * sm_count());
  SPO_CUDA_TRY(launch_pdl(split_weights_t_pad_kernel, dim3(grid), dim3(256), 0, s, 0u, w, (int)k, n, wt_hi, wt_lo));
  return kOk;
}

int fwd_skinny_launch(LayerInput in, const float* w, const float* b, int64_t rows, int64_t k, int64_t n,
                      float* y, float* y_lo, uint32_t* bits, cudaStream_t s) {
  SPO_CHECK_ARG(!in.cells || k == 3 * kCells, kErrShape, "fwd_skinny: board cells need a 27-wide input layer");
  SPO_CHECK_ARG(fwd_skinny_ok(k, n), kErrUnsupported, "fwd_skinny: k <= 32 and n % 4 == 0");
  SPO_CHECK_ARG(aligned16(w) && aligned16(b) && aligned16(y) && (!y_lo || aligned16(y_lo)), kErrAlign,
                "fwd_skinny: W, b and outputs must be 16-byte aligned");
  SPO_CHECK_ARG(!bits || n % 32 == 0, kErrUnsupported, "fwd_skinny: packed mask needs n % 32 == 0");
  if (rows <= 0) return kOk;
  const int64_t col_blocks = ceil_div(n, kCols);
  const int64_t want = std::max<int64_t>(1, 3LL * sm_count() / col_blocks);
  int64_t chunk = std::max<int64_t>(kRows, ceil_div(ceil_div(rows, want), kRows) * kRows);
  // A CTA walks its rows one after another: when that leaves fewer CTAs than SMs (small
  // batches), shorter chunks of 8-row multiples spread the rows over about three CTAs per
  // SM (the kernel's residency).
  if (ceil_div(rows, chunk) < sm_count())
    chunk = std::max<int64_t>(8, ceil_div(ceil_div(rows, want), (int64_t)8) * 8);
  dim3 grid((unsigned)ceil_div(rows, chunk), (unsigned)col_blocks);
  SPO_CUDA_TRY(launch_pdl(fwd_skinny_kernel, grid, dim3(kFwdThreads), 0, s, 0u, in.x, in.cells, w, b, rows, (int)k, n,
                          chunk, y, y_lo, bits));
  return kOk;
}

int64_t dw_skinny_max_parts() { return 4LL * sm_count(); }

int64_t dw_skinny_chunk(int64_t rows, int64_t n) {
  // enough chunks for ~4 CTAs per SM, each at least a few row blocks long
  const int64_t col_blocks = ceil_div(n, kCols);
  const int64_t want = std::max<int64_t>(1, dw_skinny_max_parts() / col_blocks);
  const int64_t r = std::max<int64_t>(rows, 1);
  const int64_t chunk = std::max<int64_t>(4 * kRows, ceil_div(ceil_div(r, want), kRows) * kRows);
  if (ceil_div(r, chunk) >= sm_count()) return chunk;
  // Small batches (fewer chunks than SMs): a CTA walks its rows kUnroll at a time, each
  // step waiting on memory, while the reduction that adds the partials gets deeper with
  // their number; chunks of about sqrt(rows / 4) rows (kUnroll multiples) balance the two.
  // Never more than `want` partials (the workspace holds dw_skinny_max_parts()).
  int64_t c = (int64_t)std::ceil(std::sqrt((double)r / 4.0));
  c = std::max<int64_t>(c, ceil_div(r, want));
  return std::max<int64_t>(kUnroll, ceil_div(c, (int64_t)kUnroll) * kUnroll);
}

int dw_skinny_launch(LayerInput in, const float* dy, int64_t rows, int64_t k, int64_t n, float* part,
                     int* parts, cudaStream_t s) {
  SPO_CHECK_ARG(!in.cells || k == 3 * kCells, kErrShape, "dw_skinny: board cells need a 27-wide input layer");
  SPO_CHECK_ARG(dw_skinny_ok(k, n), kErrUnsupported, "dw_skinny: k <= 32 and n % 4 == 0");
  SPO_CHECK_ARG(aligned16(dy) && aligned16(part), kErrAlign, "dw_skinny: dY and part must be 16-byte aligned");
  const int64_t chunk = dw_skinny_chunk(rows, n);
  const int64_t p = rows > 0 ? ceil_div(rows, chunk) : 0;
  if (parts) *parts = (int)p;
  if (p == 0) return kOk;
  dim3 grid((unsigned)p, (unsigned)ceil_div(n, kCols));
  SPO_CUDA_TRY(launch_pdl(k <= 28 ? dw_skinny_kernel<14> : dw_skinny_kernel<16>, grid, dim3(kThreads), 0, s, 0u, in.x,
                          in.cells, dy, rows, (int)k, n, chunk, part));
  return kOk;
}

}  // namespace spo
