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
// Every grid barrier wait is bounded (wait_ns); on expiry the CTA raises the abort bit of
// the arrival word, records a code in the learner's error word and goes to the exit; the
// others see the bit in the same word their waits poll. The last CTA to leave resets the
// barrier words for the next launch and, after a complete Adam phase, advances the step
// counter.
#include <algorithm>
#include <cmath>

#include "spo_common.cuh"
#include "kernels.cuh"
#include "small_step.cuh"
#include "tc_gemm.cuh"

namespace spo {

namespace {

constexpr int kT = 256;      // threads per CTA
constexpr int kW = kT / 32;  // warps per CTA
constexpr int kR = 32;       // rows held in shared memory at a time
constexpr int kLossIn = 28;  // per-row loss inputs in shared memory: mask | q | pi_old logits (9 each)
constexpr int kErrGridWait = 16;
constexpr int kErrWeightCopy = 17;

// SPO_SMALL_TRACE builds record %globaltimer at the phase boundaries of every CTA (thread
// 0) into small_trace[CTA][mark], read back with spo_small_trace_read; other builds
// compile the marks away.
#ifdef SPO_SMALL_TRACE
constexpr int kTraceMarks = 16;
__device__ unsigned long long small_trace[1024 * kTraceMarks];
#define SS_MARK(i)                                                                          \
  do {                                                                                      \
    if (threadIdx.x == 0) {                                                                 \
      unsigned long long t_;                                                                \
      asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t_));                                \
      small_trace[blockIdx.x * kTraceMarks + (i)] = t_;                                     \
      if ((i) == 0 || (i) == 8) small_trace[blockIdx.x * kTraceMarks + 14 + ((i) == 8)] = clock64(); \
    }                                                                                       \
  } while (0)
#define SS_SYNC_MARK(i) \
  do {                  \
    __syncthreads();    \
    SS_MARK(i);         \
  } while (0)
#else
#define SS_SYNC_MARK(i) \
  do {                  \
  } while (0)
#define SS_MARK(i) \
  do {             \
  } while (0)
#endif

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

__device__ __forceinline__ unsigned atom_add_acq_rel(unsigned* p, unsigned v) {
  unsigned old;
  asm volatile("atom.acq_rel.gpu.global.add.u32 %0, [%1], %2;" : "=r"(old) : "l"(p), "r"(v) : "memory");
  return old;
}

// Bit of the arrival word (sync[0]) that aborts the step. Arrivals count up to 3 * grid
// per launch, far below it. Set before the raising CTA's own arrival (same word, same
// thread order), so every CTA that sees a full count of arrivals also sees the bit.
constexpr unsigned kAbortBit = 1u << 30;

__device__ __forceinline__ void raise_abort(const SmallStepParams& P, int code) {
  atomicOr(P.sync + 0, kAbortBit);
  if (P.err) atomicCAS(P.err, 0, code);
}

// Data that other CTAs write during the launch (partials, gradients, parameters in the
// Adam phase) is read through L2 (.cg): never a stale L1 line. Weights are read before any
// write to them in the launch, through L1.
__device__ __forceinline__ float ldcg(const float* p) { return __ldcg(p); }

__device__ __forceinline__ float softplus_f(float x) { return log1pf(expf(-fabsf(x))) + fmaxf(x, 0.f); }

// Grid-wide barrier: every CTA arrives, then waits (bounded) until all have. false when
// the step was aborted. withhold: this CTA does not arrive (a test of the bounded wait: the
// others' waits then run out).
__device__ bool grid_barrier(unsigned& target, const SmallStepParams& P, bool withhold = false) {
  __shared__ int s_ok;
  __syncthreads();
  target += gridDim.x;
  if (threadIdx.x == 0) {
    // acq_rel arrival: the CTA's writes before the barrier (ordered before this thread by
    // the bar.sync above) are released to every CTA that acquires the count, and the
    // returned count acquires the others'; abort and completion are read from one word
    unsigned v = withhold ? ld_acquire(P.sync + 0) : atom_add_acq_rel(P.sync + 0, 1u) + 1u;
    if (!(v & kAbortBit) && v < target) {
      const uint64_t t0 = now_ns();
      for (;;) {
        v = ld_acquire(P.sync + 0);
        if ((v & kAbortBit) || v >= target) break;
        if (now_ns() - t0 > P.wait_ns) {
          raise_abort(P, kErrGridWait);
          v |= kAbortBit;
          break;
        }
      }
    }
    s_ok = !(v & kAbortBit);
  }
  __syncthreads();
  return s_ok != 0;
}

// ---------------------------------------------------------------- per-block steps
// Shared-memory rows: stride = width rounded up to 4 (float4 access).
__device__ __forceinline__ int pad4(int n) { return (n + 3) & ~3; }

// Dynamic shared memory of the kernel. The per-block steps below address it by float
// offsets (never through pointers held in arrays), so every access is a shared-memory
// instruction.
extern __shared__ __align__(16) float smem[];

__device__ __forceinline__ float4 lds4(int off) { return *reinterpret_cast<const float4*>(&smem[off]); }

// The weights of every layer stay in shared memory for the whole step of the CTA. A hidden
// layer's W_l [K x N] (N a multiple of 32) is held as N / 32 slabs of 32 columns, each
// [K x 32] with rows of 128 bytes, 128-byte swizzled: the 16-byte chunk q of row k sits at
// chunk q ^ (k & 7), so column n of row k is word (n & 31) ^ ((k & 7) << 2) of the row
// (w_at). A row read across 32 consecutive columns (the forward) then touches every bank
// once, and so does a float4 read of 8 consecutive rows at one column (dX). Each slab is
// one 2-D tensor copy (the copy engine applies the swizzle), with the first layer's rows
// past d0 zero-filled up to 32 (the input rows are 32 wide, zero past d0); the slabs start
// on 1024-byte boundaries, the period of the swizzle. The output layer (width 9 or 1) is
// stored as it is (one bulk copy): a column read by consecutive rows is conflict-free. The
// biases follow, each padded to a multiple of 4.
__host__ __device__ inline int wrows(int l, int k) { return l == 0 ? 32 : k; }

// Float offset of W[k][n] within a hidden layer's slabs (K rows each).
__device__ __forceinline__ int w_at(int K, int k, int n) { return (n >> 5) * K * 32 + k * 32 + ((n & 31) ^ ((k & 7) << 2)); }

// Register tiles of the row-block products. A warp owns TR rows (r = h + rg i, one row
// group h per warp, so the row operands are shared-memory broadcasts) and 32 TC columns
// (c = 32 TC g + lane + 32 j, consecutive lanes on consecutive columns, so the weight
// reads are conflict-free). Per 4 steps along the reduction a warp reads TR float4 row
// operands and 4 TC weights for 16 TR TC FMAs: shared-memory wavefronts, one per cycle
// per SM, bound these steps, and the tile shape is chosen to need the fewest.
struct Tile {
  int tr, tc;
};

// Row groups of a tile with cg column groups: the warps left per column group, rounded
// down to a power of two, so that a tile's rows h + rg i (i < TR, TR a power of two that
// covers R <= 32 rows) never pass the block's 32-row buffers.
__host__ __device__ inline int row_groups(int cg) {
  int rg = 1;
  while (2 * rg * cg <= kW) rg *= 2;
  return rg;
}

// The tile of an [R x N] output (N % 32 == 0) with the fewest wavefronts per step.
__device__ __forceinline__ Tile pick_tile(int R, int N) {
  Tile best{0, 0};
  int cost = 1 << 30;
  for (int tc = 1; tc <= 2; tc *= 2) {
    if (N % (32 * tc) != 0) continue;
    const int cg = N / (32 * tc);
    if (cg > kW) continue;
    const int rg = row_groups(cg);
    int tr = (R + rg - 1) / rg;
    tr = tr <= 1 ? 1 : tr <= 2 ? 2 : tr <= 4 ? 4 : tr <= 8 ? 8 : tr <= 16 ? 16 : 32;
    if (tc == 2 && (tr < 4 || tr > 16)) continue;   // instantiated: (1|2|4|8|16|32, 1), (4|8|16, 2)
    const int c = (cg * rg) * (tr + 4 * tc);
    if (c < cost) {
      cost = c;
      best = Tile{tr, tc};
    }
  }
  return best;
}

// out[R x N] = relu(in[R x K] W[K x N] + b) (in: stride ks, K % 4 == 0; out: stride N,
// N % 32 == 0), also to gout (the activation cache, stride N) when given.
template <int TR, int TC>
__device__ __noinline__ void block_forward_t(int in, int ks, int K, int w, int b, int N, int out, float* gout,
                                             int R) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int cg = N / (32 * TC), rg = row_groups(cg);
  if (warp >= cg * rg) return;
  const int g = warp % cg, h = warp / cg;
  const int c0 = 32 * TC * g + lane;
  const int ws = w + TC * g * K * 32;   // the warp's first slab: columns 32 TC g ..
  float acc[TR][TC];
#pragma unroll
  for (int i = 0; i < TR; ++i)
#pragma unroll
    for (int j = 0; j < TC; ++j) acc[i][j] = 0.f;
#pragma unroll 2
  for (int k = 0; k < K; k += 4) {
    // row k + u (k % 4 == 0): column lane at word lane ^ ((k & 4) << 2) ^ (u << 2) (w_at)
    const int wk = ws + k * 32, lx = lane ^ ((k & 4) << 2);
    float wv[4][TC];
#pragma unroll
    for (int u = 0; u < 4; ++u)
#pragma unroll
      for (int j = 0; j < TC; ++j) wv[u][j] = smem[wk + u * 32 + j * K * 32 + (lx ^ (u << 2))];
    float4 x[TR];   // rows past R read the block's unused buffer rows; never stored
#pragma unroll
    for (int i = 0; i < TR; ++i) x[i] = lds4(in + (h + rg * i) * ks + k);
#pragma unroll
    for (int i = 0; i < TR; ++i)
#pragma unroll
      for (int j = 0; j < TC; ++j) {
        float s = acc[i][j];
        s = fmaf(x[i].x, wv[0][j], s);
        s = fmaf(x[i].y, wv[1][j], s);
        s = fmaf(x[i].z, wv[2][j], s);
        s = fmaf(x[i].w, wv[3][j], s);
        acc[i][j] = s;
      }
  }
#pragma unroll
  for (int j = 0; j < TC; ++j) {
    const int c = c0 + 32 * j;
    const float bb = smem[b + c];
#pragma unroll
    for (int i = 0; i < TR; ++i) {
      const int r = h + rg * i;
      if (r < R) {
        const float y = fmaxf(acc[i][j] + bb, 0.f);
        smem[out + r * N + c] = y;
        if (gout) __stcg(gout + (int64_t)r * N + c, y);
      }
    }
  }
}

// out[R x K] = (dz[R x N] W[K x N]^T) * [act > 0] (dz: stride zs, a multiple of 4; act,
// out: stride K, K % 32 == 0); the columns of the tile are rows of W.
template <int TR, int TC>
__device__ __noinline__ void block_dx_t(int dz, int zs, int N, int w, int K, int act, int out, int R) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int cg = K / (32 * TC), rg = row_groups(cg);
  if (warp >= cg * rg) return;
  const int g = warp % cg, h = warp / cg;
  const int c0 = 32 * TC * g + lane;
  float acc[TR][TC];
#pragma unroll
  for (int i = 0; i < TR; ++i)
#pragma unroll
    for (int j = 0; j < TC; ++j) acc[i][j] = 0.f;
  if (N % 32 == 0) {   // swizzled slabs: one float4 of each of the TC rows per 4 n
    const int wc = w + c0 * 32, cx = (lane & 7) << 2;   // row c = c0 + 32 j: c & 7 == lane & 7
#pragma unroll 1
    for (int n = 0; n < N; n += 4) {
      const int off = wc + (n >> 5) * K * 32 + ((n & 31) ^ cx);   // w + w_at(K, c0, n); row c0 + 32 j: + 1024 j
      float4 wv[TC];
#pragma unroll
      for (int j = 0; j < TC; ++j) wv[j] = lds4(off + 32 * 32 * j);
      float4 z[TR];   // rows past R read the block's unused buffer rows; never stored
#pragma unroll
      for (int i = 0; i < TR; ++i) z[i] = lds4(dz + (h + rg * i) * zs + n);
#pragma unroll
      for (int i = 0; i < TR; ++i)
#pragma unroll
        for (int j = 0; j < TC; ++j) {
          float s = acc[i][j];
          s = fmaf(z[i].x, wv[j].x, s);
          s = fmaf(z[i].y, wv[j].y, s);
          s = fmaf(z[i].z, wv[j].z, s);
          s = fmaf(z[i].w, wv[j].w, s);
          acc[i][j] = s;
        }
    }
  } else {   // the output layer, stored as it is (odd width)
    for (int n = 0; n < N; ++n) {
      float wv[TC];
#pragma unroll
      for (int j = 0; j < TC; ++j) wv[j] = smem[w + (c0 + 32 * j) * N + n];
      float zv[TR];
#pragma unroll
      for (int i = 0; i < TR; ++i) zv[i] = smem[dz + (h + rg * i) * zs + n];
#pragma unroll
      for (int i = 0; i < TR; ++i)
#pragma unroll
        for (int j = 0; j < TC; ++j) acc[i][j] = fmaf(zv[i], wv[j], acc[i][j]);
    }
  }
#pragma unroll
  for (int j = 0; j < TC; ++j) {
    const int c = c0 + 32 * j;
#pragma unroll
    for (int i = 0; i < TR; ++i) {
      const int r = h + rg * i;
      if (r < R) smem[out + r * K + c] = smem[act + r * K + c] > 0.f ? acc[i][j] : 0.f;
    }
  }
}

#define SPO_TILE_DISPATCH(FN, ...)                          \
  do {                                                      \
    const int key_ = t.tc * 100 + t.tr;                     \
    switch (key_) {                                         \
      case 101: FN<1, 1>(__VA_ARGS__); break;               \
      case 102: FN<2, 1>(__VA_ARGS__); break;               \
      case 104: FN<4, 1>(__VA_ARGS__); break;               \
      case 108: FN<8, 1>(__VA_ARGS__); break;               \
      case 116: FN<16, 1>(__VA_ARGS__); break;              \
      case 132: FN<32, 1>(__VA_ARGS__); break;              \
      case 204: FN<4, 2>(__VA_ARGS__); break;               \
      case 208: FN<8, 2>(__VA_ARGS__); break;               \
      case 216: FN<16, 2>(__VA_ARGS__); break;              \
      default: break;                                       \
    }                                                       \
  } while (0)

__device__ void block_forward(int in, int ks, int K, int w, int b, int N, int out, float* gout, int R) {
  const Tile t = pick_tile(R, N);
  SPO_TILE_DISPATCH(block_forward_t, in, ks, K, w, b, N, out, gout, R);
}

__device__ void block_dx(int dz, int zs, int N, int w, int K, int act, int out, int R) {
  const Tile t = pick_tile(R, K);
  SPO_TILE_DISPATCH(block_dx_t, dz, zs, N, w, K, act, out, R);
}

// One row of a dW tile: its dz values (4 columns of the lane) and the KI float4 of its
// input that the warp's dW rows take.
template <int KI>
__device__ __forceinline__ void dw_load(int in, int dz, int c0, int nj, int warp, float (&z)[4], float4 (&a)[KI]) {
#pragma unroll
  for (int j = 0; j < 4; ++j) z[j] = j < nj ? smem[dz + c0 + 32 * j] : 0.f;
#pragma unroll
  for (int i = 0; i < KI; ++i) a[i] = lds4(in + 4 * warp + 4 * kW * i);
}

template <int KI>
__device__ __forceinline__ void dw_row(float (&acc)[KI][4][4], float (&db)[4], const float (&z)[4],
                                       const float4 (&a)[KI]) {
#pragma unroll
  for (int j = 0; j < 4; ++j) db[j] += z[j];
#pragma unroll
  for (int i = 0; i < KI; ++i) {
    const float av[4] = {a[i].x, a[i].y, a[i].z, a[i].w};
#pragma unroll
    for (int q = 0; q < 4; ++q)
#pragma unroll
      for (int j = 0; j < 4; ++j) acc[i][q][j] = fmaf(av[q], z[j], acc[i][q][j]);
  }
}

// pw[K x N] (+)= in[R x K]^T dz[R x N] and pb[N] (+)= sum of the rows of dz over this
// block's R rows (in: stride ks, zero past K up to a multiple of 4; dz: stride zs).
// N % 32 == 0: warp w owns the rows k = 4w + 4 kW i + q (q < 4, i < KI), lane the column
// lane + 32j; per row of the block, KI broadcast float4 of in and one dz feed 4 KI FMAs,
// and the partials are stored coalesced.
template <int KI>
__device__ __noinline__ void block_dw_t(int in, int ks, int K, int dz, int zs, int N, int R, float* pw, float* pb,
                                        bool first) {   // pb null: no bias gradient
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  for (int cb = 0; cb < N; cb += 128) {   // 4 columns per lane: c = cb + lane + 32 j
    const int nj = min(4, (N - cb) >> 5);
    const int c0 = cb + lane;
    float acc[KI][4][4];
#pragma unroll
    for (int i = 0; i < KI; ++i)
#pragma unroll
      for (int q = 0; q < 4; ++q)
#pragma unroll
        for (int j = 0; j < 4; ++j) acc[i][q][j] = 0.f;
    float db[4] = {0.f, 0.f, 0.f, 0.f};
    // two register sets of row operands: row r + 1's load under row r's FMAs
    float z0[4], z1[4];
    float4 a0[KI], a1[KI];
    dw_load<KI>(in, dz, c0, nj, warp, z0, a0);
#pragma unroll 1
    for (int r = 0; r < R; r += 2) {
      dw_load<KI>(in + min(r + 1, R - 1) * ks, dz + min(r + 1, R - 1) * zs, c0, nj, warp, z1, a1);
      dw_row<KI>(acc, db, z0, a0);
      if (r + 1 >= R) break;
      dw_load<KI>(in + min(r + 2, R - 1) * ks, dz + min(r + 2, R - 1) * zs, c0, nj, warp, z0, a0);
      dw_row<KI>(acc, db, z1, a1);
    }
    if (first) {   // stores only: no load may sit in front of them
#pragma unroll
      for (int i = 0; i < KI; ++i)
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          const int k = 4 * warp + 4 * kW * i + q;
#pragma unroll
          for (int j = 0; j < 4; ++j)
            if (k < K && j < nj) __stcg(pw + (int64_t)k * N + c0 + 32 * j, acc[i][q][j]);
        }
      if (warp == 0 && pb)
#pragma unroll
        for (int j = 0; j < 4; ++j)
          if (j < nj) __stcg(pb + c0 + 32 * j, db[j]);
    } else {
#pragma unroll
      for (int i = 0; i < KI; ++i)
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          const int k = 4 * warp + 4 * kW * i + q;
          float old[4];
#pragma unroll
          for (int j = 0; j < 4; ++j)
            old[j] = (k < K && j < nj) ? ldcg(pw + (int64_t)k * N + c0 + 32 * j) : 0.f;
#pragma unroll
          for (int j = 0; j < 4; ++j)
            if (k < K && j < nj) __stcg(pw + (int64_t)k * N + c0 + 32 * j, old[j] + acc[i][q][j]);
        }
      if (warp == 0 && pb)
#pragma unroll
        for (int j = 0; j < 4; ++j)
          if (j < nj) __stcg(pb + c0 + 32 * j, ldcg(pb + c0 + 32 * j) + db[j]);
    }
  }
}

// The output layer (N <= NA <= kSmallMaxA): thread t owns row k = t of dW and all N
// columns; thread 0 also sums the rows of dz for the bias.
template <int NA>
__device__ __noinline__ void block_dw_out_t(int in, int ks, int K, int dz, int zs, int N, int R, float* pw,
                                            float* pb, bool first) {
  for (int k = threadIdx.x; k < K; k += kT) {
    float acc[NA] = {}, db[NA] = {};
#pragma unroll 4
    for (int r = 0; r < R; ++r) {
      const float a = smem[in + r * ks + k];
      float z[NA];   // dz rows are zero past N up to their stride (a multiple of 4 >= N)
#pragma unroll
      for (int j = 0; j < NA; ++j) z[j] = j < zs ? smem[dz + r * zs + j] : 0.f;
#pragma unroll
      for (int j = 0; j < NA; ++j) {
        acc[j] = fmaf(a, z[j], acc[j]);
        db[j] += z[j];
      }
    }
    float* p = pw + (int64_t)k * N;
    if (first) {
#pragma unroll
      for (int j = 0; j < NA; ++j)
        if (j < N) __stcg(p + j, acc[j]);
      if (k == 0)
#pragma unroll
        for (int j = 0; j < NA; ++j)
          if (j < N) __stcg(pb + j, db[j]);
    } else {
      float old[NA], oldb[NA];
#pragma unroll
      for (int j = 0; j < NA; ++j) {
        old[j] = j < N ? ldcg(p + j) : 0.f;
        oldb[j] = (k == 0 && j < N) ? ldcg(pb + j) : 0.f;
      }
#pragma unroll
      for (int j = 0; j < NA; ++j)
        if (j < N) __stcg(p + j, old[j] + acc[j]);
      if (k == 0)
#pragma unroll
        for (int j = 0; j < NA; ++j)
          if (j < N) __stcg(pb + j, oldb[j] + db[j]);
    }
  }
}

__device__ void block_dw(int in, int ks, int K, int dz, int zs, int N, int R, float* pw, float* pb, bool first) {
  if (N % 32 != 0) {
    if (N == 1)
      block_dw_out_t<1>(in, ks, K, dz, zs, N, R, pw, pb, first);
    else
      block_dw_out_t<kSmallMaxA>(in, ks, K, dz, zs, N, R, pw, pb, first);
    return;
  }
  for (int k0 = 0; k0 < K; k0 += 128) {   // 128 rows of dW per pass
    float* w0 = pw + (int64_t)k0 * N;
    float* b0 = k0 == 0 ? pb : nullptr;
    switch (min(128 / (4 * kW), (K - k0 + 4 * kW - 1) / (4 * kW))) {
      case 1: block_dw_t<1>(in + k0, ks, K - k0, dz, zs, N, R, w0, b0, first); break;
      case 2: block_dw_t<2>(in + k0, ks, K - k0, dz, zs, N, R, w0, b0, first); break;
      case 3: block_dw_t<3>(in + k0, ks, K - k0, dz, zs, N, R, w0, b0, first); break;
      default: block_dw_t<4>(in + k0, ks, K - k0, dz, zs, N, R, w0, b0, first); break;
    }
  }
}

// Logits / V of rows [0, R) of the block (act: [R x H]; W: the output layer [H x A], b its
// bias), the row losses and dz (stride zs). The per-row inputs come from shared memory (li:
// mask or cells, q, pi_old logits, 9 each; the critic's target in the first column). Lane
// 0 of warp w adds the statistics of its rows to stw[w][..].
// Butterfly sums (max) of N values at once: the same xor order per value as warp_sum
// (warp_max), the N exchanges of a level issued together instead of N dependent chains.
template <int N>
__device__ __forceinline__ void warp_sum_n(float (&v)[N]) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1)
#pragma unroll
    for (int j = 0; j < N; ++j) v[j] += __shfl_xor_sync(0xffffffffu, v[j], o);
}
template <int N>
__device__ __forceinline__ void warp_max_n(float (&v)[N]) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1)
#pragma unroll
    for (int j = 0; j < N; ++j) v[j] = fmaxf(v[j], __shfl_xor_sync(0xffffffffu, v[j], o));
}

__device__ __noinline__ void block_loss(bool actor, bool has_mask, bool has_old, float scale, int H, int A, int act,
                                        int li, int R, int dz, int zs, int w, int b, float alpha, int stw) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const bool valid = lane < A;
  const float bias = valid ? smem[b + lane] : 0.f;
  float st[kStats] = {};
  if (!actor) {
    for (int r = warp; r < R; r += kW) {   // value head (A == 1): one row per warp at a time
      float p0 = 0.f;
      for (int h = lane; h < H; h += 32) p0 = fmaf(smem[act + r * H + h], smem[w + h], p0);
      const float v = warp_sum(p0);   // every lane takes part in the exchange
      const float z = (lane == 0 ? v : 0.f) + bias;
      const float d = z - smem[li + r * kLossIn];   // meaningful in lane 0
      if (lane < zs) smem[dz + r * zs + lane] = lane == 0 ? d * scale : 0.f;
      st[kStatCriticLoss] += 0.5f * d * d * scale;
    }
  } else {
    for (int r = warp; r < R; r += kW) {
      const int in_r = li + r * kLossIn;
      float part[kSmallMaxA] = {};
      for (int h = lane; h < H; h += 32) {
        const float a = smem[act + r * H + h];
#pragma unroll
        for (int j = 0; j < kSmallMaxA; ++j)
          if (j < A) part[j] = fmaf(a, smem[w + h * A + j], part[j]);
      }
      warp_sum_n(part);   // outputs j >= A stay 0
      float z = 0.f;
#pragma unroll
      for (int j = 0; j < kSmallMaxA; ++j)
        if (lane == j && j < A) z = part[j];
      z += bias;
      const float m_in = valid ? smem[in_r + lane] : 0.f;
      const float mk = valid ? (has_mask ? m_in : (m_in == 0.f ? 1.f : 0.f)) : 0.f;
      const bool legal = valid && mk != 0.f;
      const float qv = valid ? smem[in_r + 9 + lane] : 0.f;
      // the softmax of z and, with pi_old, of its logits: their reductions side by side
      float mxs[2] = {legal ? z : kNegInf, (has_old && legal) ? smem[in_r + 18 + lane] : kNegInf};
      const float zm = mxs[0], zo = mxs[1];
      warp_max_n(mxs);
      const float mx = mxs[0], mxo = mxs[1];
      float ss[2] = {valid ? expf(zm - mx) : 0.f, (has_old && valid) ? expf(zo - mxo) : 0.f};
      const float e = ss[0], eo = ss[1];
      warp_sum_n(ss);
      const float s = ss[0], so = ss[1];
      const float pi = e * (1.f / s);
      const float lp = zm - (mx + logf(s));
      float po = 0.f, klo_t = 0.f;
      if (has_old) {
        po = eo * (1.f / so);
        if (valid && po > 0.f) klo_t = po * ((zo - (mxo + logf(so))) - lp);
      }
      float sums[3] = {(valid && qv != 0.f) ? -qv * lp : 0.f, (valid && qv > 0.f) ? -qv * logf(qv) : 0.f, klo_t};
      warp_sum_n(sums);
      const float ce = sums[0], hq = sums[1], klo = sums[2];
      if (lane < zs) smem[dz + r * zs + lane] = legal ? ((pi - qv) + alpha * (pi - po)) * scale : 0.f;
      st[kStatActorLoss] += (ce + alpha * klo) * scale;
      st[kStatCE] += ce * scale;
      st[kStatEntropy] += hq * scale;
      st[kStatKLq] += (ce - hq) * scale;
      st[kStatKLold] += klo * scale;
    }
  }
  if (lane == 0)
#pragma unroll
    for (int k = 0; k < kStats; ++k) smem[stw + warp * kStats + k] += st[k];
}

// Shared memory of one network's row block, in floats: x [kR x 32] | loss inputs
// [kR x kLossIn] | per-warp statistics [kW x kStats] | a_0 .. a_{L-2} [kR x d_{l+1}] |
// dz ping-pong 2 x [kR x dmax] | up to 255 floats to the next 1024-byte boundary | W_0 ..
// W_{L-1} [wrows x d_{l+1}] | b_0 .. b_{L-1} [pad4(d_{l+1})]; every region starts on a
// 16-byte boundary, every hidden layer's W on a 1024-byte one (their sizes are multiples
// of 4096 bytes).
__host__ __device__ inline int small_dmax(const int* dims, int L) {
  int dmax = (dims[L] + 3) & ~3;
  for (int l = 1; l < L; ++l) dmax = dims[l] > dmax ? dims[l] : dmax;
  return dmax;
}
__host__ __device__ inline int small_acts_base() { return kR * 32 + kR * kLossIn + kW * kStats; }
// the end of the dz buffers (W_0 starts at the next 1024-byte boundary after it)
__host__ __device__ inline int small_w_base(const int* dims, int L) {
  int f = small_acts_base();
  for (int l = 1; l < L; ++l) f += kR * dims[l];
  return f + 2 * kR * small_dmax(dims, L);
}
__host__ __device__ inline int small_smem_floats(const int* dims, int L) {
  int f = small_w_base(dims, L) + 255;
  for (int l = 0; l < L; ++l) f += wrows(l, dims[l]) * dims[l + 1] + ((dims[l + 1] + 3) & ~3);
  return f;
}

__device__ __forceinline__ void cp4(float* dst, const float* src) {
  asm volatile("cp.async.ca.shared.global [%0], [%1], 4;" ::"r"(static_cast<uint32_t>(__cvta_generic_to_shared(dst))),
               "l"(src)
               : "memory");
}

__device__ __forceinline__ uint32_t smem_u32(int off) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(&smem[off]));
}

// One bulk copy (the copy engine, completion counted in bytes on the mbarrier bar).
__device__ __forceinline__ void bulk_copy(int dst, const float* src, uint32_t bytes, uint32_t bar) {
  asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
                   smem_u32(dst)),
               "l"(src), "r"(bytes), "r"(bar)
               : "memory");
}

__device__ __forceinline__ bool mbar_try(uint32_t bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(bar), "r"(parity)
      : "memory");
  return ok != 0;
}

// Bytes of layer l's weights and bias as staged (its copies' total; a hidden layer's slabs
// count their zero-filled rows).
__device__ __forceinline__ uint32_t staged_bytes(const SmallNet& n, int l) {
  return 4u * (wrows(l, n.dims[l]) * n.dims[l + 1] + ((n.dims[l + 1] + 3) & ~3));
}

// The first float offset at or after f whose shared-memory address is 1024-byte aligned.
__device__ __forceinline__ int align_1k(int f) { return f + (int)(((1024u - (smem_u32(f) & 1023u)) & 1023u) >> 2); }

// One 2-D tensor copy: the box at columns x.., rows y.. of the tensor map's array into
// shared memory at dst (completion counted in bytes on the mbarrier bar).
__device__ __forceinline__ void tensor_copy(int dst, const CUtensorMap* map, int x, int y, uint32_t bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];" ::"r"(
          smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(bar)
      : "memory");
}

// Bounded wait for the weight copies (parity phase of bar). On expiry: the step's abort
// word and the error word are set, and a second bounded wait lets the copies in flight
// land before the CTA goes on (its results are then discarded by the abort).
__device__ bool wait_staged(uint32_t bar, uint32_t parity, const SmallStepParams& P) {
  if (mbar_try(bar, parity)) return true;
  const uint64_t t0 = now_ns();
  while (!mbar_try(bar, parity)) {
    if (now_ns() - t0 > P.wait_ns) {
      raise_abort(P, kErrWeightCopy);
      const uint64_t t1 = now_ns();
      while (!mbar_try(bar, parity) && now_ns() - t1 < P.wait_ns) {
      }
      return false;
    }
  }
  return true;
}

// Every layer's weights (at wbase, the layout above) and biases (at bbase) into shared
// memory: a hidden layer's slabs by one tensor copy each (map wmap[l]: the layer's W with
// a box of 32 columns x wrows rows, 128-byte swizzle, zero fill past d_l), the output
// layer by one bulk copy, each bias by one bulk copy (the flat parameter buffer pads every
// tensor to 64 floats, so a bias padded to 4 is still inside it). Layer l's copies complete
// on the mbarrier bar0 + 8 l, which thread 0 has armed with that layer's bytes: the
// forward of a layer waits for its own weights only. Warp l issues layer l's slab copies.
__device__ void stage_weights(const SmallNet& n, const CUtensorMap* wmap, int wbase, int bbase, uint32_t bar0) {
  int w = wbase, b = bbase;
  for (int l = 0; l < n.L; ++l) {
    const int K = wrows(l, n.dims[l]), N = n.dims[l + 1];
    const uint32_t bar = bar0 + 8u * l;
    if (N % 32 == 0) {
      const int t = threadIdx.x - 32 * l;
      if (t >= 0 && t < N / 32) tensor_copy(w + t * K * 32, wmap + l, 32 * t, 0, bar);
    } else if (threadIdx.x == kT - 1) {
      bulk_copy(w, n.W[l], 4u * K * N, bar);
    }
    if (threadIdx.x == kT - 2 - l) bulk_copy(b, n.b[l], 4u * ((N + 3) & ~3), bar);
    w += K * N;
    b += (N + 3) & ~3;
  }
}

// One network over this CTA's rows [rb, re), 32 rows at a time.
// wmap: the tensor maps of its hidden layers' W; bar0: the CTA's mbarriers of the weight
// copies (one per layer, 8 bytes apart), phase their next parity.
__device__ void net_rows(const SmallStepParams& P, const SmallNet& n, const CUtensorMap* wmap, int64_t rb,
                         int64_t re, uint32_t bar0, uint32_t& phase) {
  const int L = n.L, d0 = n.dims[0];
  const int part = blockIdx.x;
  const bool actor = n.mode == 0;
  const int xs = 0, li = kR * 32, stw = li + kR * kLossIn, acts0 = small_acts_base();
  const int dmax = small_dmax(n.dims, L);
  int dzb0 = acts0;
  for (int l = 1; l < L; ++l) dzb0 += kR * n.dims[l];
  const int wbase = align_1k(small_w_base(n.dims, L));
  int bbase = wbase;
  for (int l = 0; l < L; ++l) bbase += wrows(l, n.dims[l]) * n.dims[l + 1];
  // log_alpha's load is issued here, its softplus taken at the first loss: the load's
  // latency stays off the path to the weight copies
  const bool has_kl = actor && P.z_old;
  const float log_alpha = has_kl ? *P.log_alpha : 0.f;
  float alpha = 0.f;
  for (int e = threadIdx.x; e < kW * kStats; e += kT) smem[stw + e] = 0.f;
  bool first = true;
  for (int64_t r0 = rb; r0 < re; r0 += kR, first = false) {
    const int R = (int)min((int64_t)kR, re - r0);
    // the weights first (the largest copy), then the loss inputs of the block's rows, all
    // asynchronous; the input rows' loads below overlap them
    if (first) {
      if (threadIdx.x == 0)
        for (int l = 0; l < L; ++l)
          asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(bar0 + 8u * l),
                       "r"(staged_bytes(n, l))
                       : "memory");
      __syncthreads();   // armed before any copy can complete; earlier reads of this memory done
      asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
      stage_weights(n, wmap, wbase, bbase, bar0);
    }
    for (int e = threadIdx.x; e < R * kLossIn; e += kT) {
      const int r = e / kLossIn, f = e - r * kLossIn;
      const int64_t row = r0 + r;
      const float* src = nullptr;
      if (!actor) {
        if (f == 0) src = P.target + row;
      } else if (f < 9) {
        src = P.mask ? P.mask + row * 9 + f : P.cells + row * 9 + f;
      } else if (f < 18) {
        src = P.q + row * 9 + (f - 9);
      } else if (f < 27 && P.z_old) {
        src = P.z_old + row * 9 + (f - 18);
      }
      if (src) cp4(&smem[li + e], src);
    }
    asm volatile("cp.async.commit_group;" ::: "memory");
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
        smem[xs + e] = x;
      }
    }
    SS_MARK(13);
    asm volatile("cp.async.commit_group;\n\tcp.async.wait_group 0;" ::: "memory");
    __syncthreads();
    SS_MARK(1);
    {
      int in = xs, ks = 32, a = acts0, w = wbase, b = bbase;
      for (int l = 0; l + 1 < L; ++l) {
        const int K = wrows(l, n.dims[l]), N = n.dims[l + 1];
        // the first block waits for each layer's weights just before using them (on
        // expiry the step is aborted and its results are not used)
        if (first) wait_staged(bar0 + 8u * l, phase, P);
        block_forward(in, ks, K, w, b, N, a, n.gact[l] ? n.gact[l] + r0 * N : nullptr, R);
        __syncthreads();
        in = a;
        ks = N;
        a += kR * N;
        w += K * N;
        b += (N + 3) & ~3;
      }
      SS_MARK(2);
      // in: the last hidden activations; w, b: the output layer
      if (first) {
        wait_staged(bar0 + 8u * (L - 1), phase, P);
        phase ^= 1u;   // every layer's barrier has completed this phase
      }
      int zs = (n.dims[L] + 3) & ~3;   // row stride of the gradient in the current dz buffer
      if (first && has_kl) alpha = softplus_f(log_alpha);
      block_loss(actor, P.mask != nullptr, P.z_old != nullptr, P.scale, n.dims[L - 1], n.dims[L], in, li, R, dzb0,
                 zs, w, b, alpha, stw);
      __syncthreads();
      SS_MARK(3);
      int cur = 0;
      for (int l = L - 1; l >= 0; --l) {
        const int N = n.dims[l + 1], K = l == 0 ? d0 : n.dims[l];
        const int dz = dzb0 + cur * kR * dmax, dzn = dzb0 + (cur ^ 1) * kR * dmax;
        const int act_in = l == 0 ? xs : in;   // the input of layer l
        block_dw(act_in, l == 0 ? 32 : K, K, dz, zs, N, R, n.pw[l] + (int64_t)part * K * N,
                 n.pb[l] + (int64_t)part * N, first);
        if (l == 1) SS_SYNC_MARK(12);
        if (l >= 1) block_dx(dz, zs, N, w, K, act_in, dzn, R);
        __syncthreads();
        zs = K;
        cur ^= 1;
        if (l >= 1) {   // step back one layer: its weights, its input activations
          w -= wrows(l - 1, n.dims[l - 1]) * K;
          in = l - 1 == 0 ? xs : in - kR * n.dims[l - 1];
        }
        SS_MARK(9 + l);
      }
    }
    SS_MARK(4);
  }
  // the statistics of this CTA's rows
  __syncthreads();
  if (threadIdx.x < kStats) {
    float v = 0.f;
#pragma unroll
    for (int w = 0; w < kW; ++w) v += smem[stw + w * kStats + threadIdx.x];
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

// sum over k < parts of src[k * stride], 32 loads in flight per round (the last round
// predicated): part k goes to partial sum k % 8 and the eight are combined in a fixed order
// (deterministic).
__device__ __forceinline__ float sum_parts(const float* src, int parts, int64_t stride) {
  constexpr int kU = 32;
  float a[8] = {};
  for (int k = 0; k < parts; k += kU) {
    float v[kU];
#pragma unroll
    for (int u = 0; u < kU; ++u) v[u] = k + u < parts ? ldcg(src + (int64_t)(k + u) * stride) : 0.f;
#pragma unroll
    for (int u = 0; u < kU; ++u) a[u & 7] += v[u];
  }
  return ((a[0] + a[1]) + (a[2] + a[3])) + ((a[4] + a[5]) + (a[6] + a[7]));
}

__global__ void __launch_bounds__(kT, 1) small_step_kernel(const __grid_constant__ SmallStepParams P) {
  __shared__ float s_clip[kMaxGroups], s_norm[kMaxGroups];
  __shared__ float s_sq[kW];
  unsigned target = 0;
  bool ok = true;
  const AdamParams& ap = P.adam;

  SS_MARK(0);
  // ---- rows: forward, loss, backward; per-CTA partial sums
  if (blockIdx.x < P.parts) {
    {   // the weight slabs' tensor maps into the copy engine's cache, ahead of the copies
      const int i = threadIdx.x / (kSmallMaxLayers - 1), l = threadIdx.x % (kSmallMaxLayers - 1);
      if (i < 2 && l + 1 < P.net[i].L)
        asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(P.wmap + i * (kSmallMaxLayers - 1) + l))
                     : "memory");
    }
    __shared__ __align__(8) unsigned long long s_wbar[kSmallMaxLayers];   // each layer's weight copies
    // Both networks' descriptors (dims, tensor addresses: read throughout the rows phase)
    // copied from the launch parameters into shared memory, one word per thread at once,
    // instead of a chain of dependent parameter reads.
    __shared__ __align__(8) SmallNet s_net[2];
    static_assert(sizeof(SmallNet) % 4 == 0, "SmallNet is copied as 4-byte words");
    {
      const uint32_t* src = reinterpret_cast<const uint32_t*>(&P.net[0]);
      uint32_t* dst = reinterpret_cast<uint32_t*>(&s_net[0]);
      for (int e = threadIdx.x; e < (int)(2 * sizeof(SmallNet) / 4); e += kT) dst[e] = src[e];
    }
    const uint32_t bar = static_cast<uint32_t>(__cvta_generic_to_shared(&s_wbar[0]));
    if (threadIdx.x == 0) {
      for (int l = 0; l < kSmallMaxLayers; ++l)
        asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;" ::"r"(bar + 8u * l) : "memory");
      asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    __syncthreads();
    uint32_t phase = 0;
    const int64_t rb = (int64_t)blockIdx.x * P.rows_per_cta;
    const int64_t re = min(rb + P.rows_per_cta, P.rows);
    for (int i = 0; i < 2; ++i)
      if (s_net[i].L) net_rows(P, s_net[i], P.wmap + i * (kSmallMaxLayers - 1), rb, re, bar, phase);
  }
  SS_MARK(5);
  ok = grid_barrier(target, P, P.withhold == blockIdx.x + 1u);
  SS_MARK(6);

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
      while (si + 1 < P.red.nseg && e >= P.seg_start[si + 1]) ++si;
      const int64_t i = e - P.seg_start[si];
      const int64_t fe = P.flat_index[si] + i;   // element of the flat buffers
      int gi = -1;
      if (fuse && fe >= 0) {
#pragma unroll
        for (int k = 0; k < kMaxGroups; ++k)
          if (k < ap.ngrp && fe >= ap.grp[k].begin && fe < ap.grp[k].end) gi = k;
      }
      // Adam's operands first: their loads overlap the partial sums'
      float p = 0.f, m = 0.f, v = 0.f;
      if (gi >= 0) {
        p = ldcg(ap.p + fe);
        m = ldcg(ap.m + fe);
        v = ldcg(ap.v + fe);
      }
      const ReduceSeg& sg = P.red.seg[si];
      const float g = sum_parts(sg.src + i, sg.parts, sg.part_stride);
      __stcg(sg.dst + i, g);
      if (gi < 0) continue;
      float gv = g;
      if (fe == ap.alpha_index) {
        // dual gradient: sigmoid(log_alpha) * (eps - mean KL(pi_old || pi)), the KL from the
        // actor's per-CTA statistics in the same order as its own reduced slot
        const float kl = sum_parts(P.net[0].pstats + kStatKLold, P.parts, kStats);
        gv = (1.f / (1.f + expf(-p))) * (ap.kl_eps - kl);
        __stcg(ap.g + fe, gv);
        if (ap.report) ap.report[kRepDlogAlpha] = gv;
      }
      adam_one(p, gv, m, v, ap.grp[gi].lr, ap.b1, ap.b2, ap.eps, bc1, bc2);
      __stcg(ap.p + fe, p);
      __stcg(ap.m + fe, m);
      __stcg(ap.v + fe, v);
    }
  }
  SS_MARK(7);
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
  // ---- exit: the last CTA out resets the barrier words (and advances the step). Nothing
  // after the reset needs a fence: the launch ends there, and its end makes every write
  // visible to the next kernel in the stream.
  __syncthreads();
  SS_MARK(8);
  if (threadIdx.x == 0) {
    // acq_rel: this CTA is done with the barrier words before the last one resets them
    const unsigned prev = atom_add_acq_rel(P.sync + 1, 1u);
    if (prev == gridDim.x - 1) {
      const unsigned arrivals = atomicExch(P.sync + 0, 0u);   // reset, reading the abort bit
      if (!(arrivals & kAbortBit) && P.apply) {
        *ap.step = t_step;
        if (ap.report) {
          for (int k = 0; k < kMaxGroups; ++k) {
            ap.report[kRepNorm0 + k] = s_norm[k];
            ap.report[kRepClip0 + k] = s_clip[k];
          }
          ap.report[kRepStep] = (float)t_step;
        }
      }
      P.sync[1] = 0u;
    }
  }
}

}  // namespace

#ifdef SPO_SMALL_TRACE
extern "C" __attribute__((visibility("default"))) int spo_small_trace_read(unsigned long long* host, int n) {
  return cudaMemcpyFromSymbol(host, small_trace, sizeof(unsigned long long) * std::min(n, 1024 * kTraceMarks)) ==
                 cudaSuccess
             ? 0
             : -5;
}
#endif

int small_weight_map(CUtensorMap* m, const float* W, int l, int rows, int cols) {
  return make_map(m, W, (uint64_t)cols, (uint64_t)rows, 32u, (uint32_t)wrows(l, rows), CU_TENSOR_MAP_SWIZZLE_128B);
}

size_t small_step_smem(const spo_mlp_desc* nets, int count) {
  size_t most = 0;
  for (int i = 0; i < count; ++i) {
    const spo_mlp_desc& d = nets[i];
    if (d.num_layers < 2) continue;
    most = std::max(most, (size_t)small_smem_floats(d.dims, d.num_layers) * sizeof(float));
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
