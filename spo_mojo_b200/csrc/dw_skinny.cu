// Weight gradient of a layer with a narrow input: dW[k x n] = x^T dY summed over rows,
// x [rows x k] with k <= 32 (the 27-wide board encoding of the first layer), dY
// [rows x n]. The CUDA-core GEMM tiles waste most of a 64- or 128-row tile on k = 27 and
// re-read dY per tile; this kernel streams dY once, at the HBM rate.
//
// CTA = 256 threads over one chunk of rows and 512 columns: thread t owns the 4 columns
// 4 (t % 128) .. +3 of its column block and one half of the k features (t / 128), so its
// accumulators are [half of k] x 4. Rows are walked in blocks of kRows: the block's x rows
// are staged in shared memory (zero-padded to 32 features) and read as broadcasts, the dY
// float4 of each row is loaded straight from global memory, 8 rows in flight per thread.
// Each CTA writes its partial [k x n] tile to part[chunk]; a deterministic reduction adds
// the chunks (linear_backward's dW, networks/linear.mojo:120-167).
#include "spo_common.cuh"
#include "kernels.cuh"

namespace spo {

namespace {

constexpr int kThreads = 256;
constexpr int kCols = 512;       // columns per CTA (128 threads x float4)
constexpr int kMaxK = 32;
constexpr int kHalf = kMaxK / 2;  // features per thread
constexpr int kRows = 64;        // rows staged per block
constexpr int kUnroll = 8;

__global__ void __launch_bounds__(kThreads, 2)
dw_skinny_kernel(const float* __restrict__ x, const float* __restrict__ dy, int64_t rows, int k, int64_t n,
                 int64_t chunk, float* __restrict__ part) {
  __shared__ __align__(16) float xs[kRows][kMaxK];
  const int tid = threadIdx.x;
  const int half = tid / 128;
  const int64_t col = (int64_t)blockIdx.y * kCols + 4 * (tid % 128);
  const bool col_ok = col < n;
  const int64_t r_begin = (int64_t)blockIdx.x * chunk;
  const int64_t r_end = min(rows, r_begin + chunk);
  const int i0 = half * kHalf;

  float acc[kHalf][4];
#pragma unroll
  for (int i = 0; i < kHalf; ++i)
#pragma unroll
    for (int j = 0; j < 4; ++j) acc[i][j] = 0.f;

  for (int64_t rb = r_begin; rb < r_end; rb += kRows) {
    const int nr = (int)min((int64_t)kRows, r_end - rb);
    __syncthreads();  // the previous block's x rows are consumed
    for (int e = tid; e < kRows * kMaxK; e += kThreads) {
      const int r = e / kMaxK, i = e % kMaxK;
      xs[r][i] = (r < nr && i < k) ? __ldg(x + (rb + r) * k + i) : 0.f;
    }
    __syncthreads();
    if (col_ok) {
      for (int r0 = 0; r0 < nr; r0 += kUnroll) {
        float4 g[kUnroll];
#pragma unroll
        for (int u = 0; u < kUnroll; ++u)
          g[u] = r0 + u < nr ? __ldg(reinterpret_cast<const float4*>(dy + (rb + r0 + u) * n + col))
                             : make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
        for (int u = 0; u < kUnroll; ++u) {
          const float4* xr = reinterpret_cast<const float4*>(&xs[r0 + u][i0]);
#pragma unroll
          for (int c = 0; c < kHalf / 4; ++c) {
            const float4 xv = xr[c];
            const float xa[4] = {xv.x, xv.y, xv.z, xv.w};
#pragma unroll
            for (int t = 0; t < 4; ++t) {
              float* a = acc[4 * c + t];
              a[0] = fmaf(xa[t], g[u].x, a[0]);
              a[1] = fmaf(xa[t], g[u].y, a[1]);
              a[2] = fmaf(xa[t], g[u].z, a[2]);
              a[3] = fmaf(xa[t], g[u].w, a[3]);
            }
          }
        }
      }
    }
  }
  if (!col_ok) return;
  float* out = part + (int64_t)blockIdx.x * k * n;
#pragma unroll
  for (int i = 0; i < kHalf; ++i) {
    const int f = i0 + i;
    if (f < k)
      *reinterpret_cast<float4*>(out + (int64_t)f * n + col) =
          make_float4(acc[i][0], acc[i][1], acc[i][2], acc[i][3]);
  }
}

}  // namespace

bool dw_skinny_ok(int64_t k, int64_t n) { return k >= 1 && k <= kMaxK && n >= 4 && n % 4 == 0; }

int64_t dw_skinny_max_parts() { return 4LL * sm_count(); }

int64_t dw_skinny_chunk(int64_t rows, int64_t n) {
  // enough chunks for ~4 CTAs per SM, each at least a few row blocks long
  const int64_t col_blocks = ceil_div(n, kCols);
  const int64_t want = std::max<int64_t>(1, dw_skinny_max_parts() / col_blocks);
  return std::max<int64_t>(4 * kRows, ceil_div(ceil_div(std::max<int64_t>(rows, 1), want), kRows) * kRows);
}

int dw_skinny_launch(const float* x, const float* dy, int64_t rows, int64_t k, int64_t n, float* part,
                     int* parts, cudaStream_t s) {
  SPO_CHECK_ARG(dw_skinny_ok(k, n), kErrUnsupported, "dw_skinny: k <= 32 and n % 4 == 0");
  SPO_CHECK_ARG(aligned16(dy) && aligned16(part), kErrAlign, "dw_skinny: dY and part must be 16-byte aligned");
  const int64_t chunk = dw_skinny_chunk(rows, n);
  const int64_t p = rows > 0 ? ceil_div(rows, chunk) : 0;
  if (parts) *parts = (int)p;
  if (p == 0) return kOk;
  dim3 grid((unsigned)p, (unsigned)ceil_div(n, kCols));
  dw_skinny_kernel<<<grid, kThreads, 0, s>>>(x, dy, rows, (int)k, n, chunk, part);
  SPO_LAUNCH_CHECK();
  return kOk;
}

}  // namespace spo
