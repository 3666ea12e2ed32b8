// tcgen05 3xTF32 GEMM (see tc_gemm.cuh) — persistent, warp-specialised, sm_100a.
//
// CTA = warp 0 (TMA producer, one thread: hi/lo tiles of A and B into a STAGES-deep ring),
// warp 1 (TMEM allocator + MMA issuer, one thread: 3 tcgen05.mma per 8-wide k-step —
// lo.hi, hi.lo, hi.hi — into one of NACC fp32 TMEM accumulators) and 4 x (TBN / 64)
// epilogue warps: warp w reads TMEM lanes 32*(w%4)..+31 (= tile rows) and 64 of the
// tile's columns; it folds each accumulator into an fp32 running sum held in registers,
// releases the accumulator as soon as its tcgen05.ld has completed, and on the unit's
// last segment applies the fused bias/ReLU/mask/column sums, hi/lo split and stores to
// global memory. Tiles are 128 x TBN outputs (TBN = 128 or 256); k-blocks are 32 fp32
// (one 128-byte swizzle row). Operand tiles are written by TMA with 128-byte swizzling;
// K-major operands are read by the UMMA descriptors with SBO = 1024 B (8-row atoms) and a
// 32-byte start advance per k-step, MN-major operands (the dW products) are loaded as
// 32-element-wide boxes with LBO = 4096 B between boxes; TF32 MN-major operands need the
// 128-byte swizzle with 32-byte atoms (TMA SWIZZLE_128B_ATOM_32B, descriptor layout type
// 1), whose k-groups are 4 rows: SBO = 512 B.
//
// Every mbarrier wait is bounded (2 s of %globaltimer); on expiry the CTA sets an abort
// flag and the caller's error word, the producer waits (bounded) for its copies in
// flight, the MMA thread drains its issued MMAs (bounded), TMEM is freed and the kernel
// returns.
#include <cuda.h>
#include <cudaTypedefs.h>

#include <algorithm>
#include <mutex>
#include <set>
#include <utility>

#include "kernels.cuh"
#include "tc_gemm.cuh"

namespace spo {

namespace {

constexpr int BM = 128;                                  // output rows per CTA
constexpr int BK = 32;
constexpr int EPI_COLS = 64;                             // columns per epilogue warp
constexpr uint32_t A_TILE = BM * BK * 4;                 // 16 KB
constexpr int STAGES_MAX = 4;
constexpr int NACC_MAX = 4;
constexpr uint32_t TMEM_COLS = 512;                      // the whole TMEM of the SM
constexpr int ASTG_MAX = 4;

// Operands held in global memory as plain fp32 ("raw") instead of TF32 hi/lo pairs, split
// on chip by four split warps (one per TMEM lane quadrant). RAW bit 0: A, whose hi and lo
// halves the split warps write to tensor memory (tcgen05.st), from where the MMAs read A
// (no shared-memory traffic for A beyond the one read of the fp32 tile); bit 1: B (dW),
// split in shared memory (hi in place, lo in the stage's lo slot).
constexpr int kRawA = 1, kRawB = 2;
constexpr int kSplitWarps = 4;

// Geometry of one instantiation: PAIR = CTA pair (cta_group::2), TBN = output columns per
// tile (128, or 256 when N allows: one 128 x 256 MMA per k-step reads A once for twice the
// columns, and the per-k-block TMA refill and accumulator hand-offs are amortised over
// twice the work). Single CTA: A [128 x 32] and B [TBN x 32] hi/lo per k-block. CTA pair
// (256 x TBN output tile per pair): each CTA stages its own 128 rows of A and one half of B;
// the MMA issued by the pair's first CTA reads both CTAs' shared memory. The ring takes as
// many stages as fit in ~200 KB; TMEM holds 512 / TBN accumulators; the epilogue has one
// warp per (TMEM lane quadrant, 64-column group).
template <bool PAIR, int TBN, int RAW = 0>
struct Geo {
  static constexpr int BN = TBN;
  static constexpr int B_ROWS = PAIR ? BN / 2 : BN;
  static constexpr uint32_t B_TILE = B_ROWS * BK * 4;
  // A from tensor memory: a stage holds the fp32 A tile only (no lo slot)
  static constexpr bool TA = (RAW & kRawA) != 0;
  static constexpr uint32_t A_BYTES = TA ? A_TILE : 2 * A_TILE;   // A slots of a stage
  static constexpr uint32_t STAGE_BYTES = A_BYTES + 2 * B_TILE;
  static constexpr int STAGES = (200u * 1024u) / STAGE_BYTES < (uint32_t)STAGES_MAX
                                    ? (int)((200u * 1024u) / STAGE_BYTES)
                                    : STAGES_MAX;
  static constexpr int UNIT_M = PAIR ? 2 * BM : BM;                // output rows per unit
  // TMEM columns: accumulators first, then (A in TMEM) ASTG stages of A, 64 columns each
  // (32 hi, 32 lo): 2 x 128 + 4 x 64, or 1 x 256 + 4 x 64. Four A stages let the split
  // warps run up to three k-blocks ahead of the MMAs.
  static constexpr int NACC = TA ? (BN == 128 ? 2 : 1) : (int)(TMEM_COLS / BN);
  static constexpr int ASTG = TA ? (int)((TMEM_COLS - NACC * BN) / 64) : 0;
  static constexpr uint32_t ACOL0 = (uint32_t)(NACC * BN);
  static constexpr int EPI_WARPS = 4 * (BN / EPI_COLS);
  static constexpr int EPI_THREADS = 32 * EPI_WARPS;
  static constexpr int CONV_WARPS = RAW != 0 ? kSplitWarps : 0;
  static constexpr int THREADS = 64 + EPI_THREADS + 32 * CONV_WARPS;
};
// The tensor core's accumulation into TMEM is not exact fp32: its error grows with the
// number of MMAs summed into one accumulator. The epilogue therefore folds each
// accumulator into an fp32 running sum every SEG k-blocks; every fold is a TMEM read that
// the tensor pipe waits for, so SEG trades precision for speed per product:
//   forward  4 k-blocks: activations within 2.3e-6 of max (1e-6 at 2, 4e-6 at 8), their
//            ReLU decisions what decides the backward's branches
//   dX, dW   8 k-blocks: gradients within 6e-6 of max (4.5e-6 at 2), far inside the 1e-4
//            gradient tolerance (measured on the 27-256x3-9, 27-512x3-9 and 27-1024x4-9
//            actors against a float64 restatement)
#ifndef SPO_TC_SEG
#define SPO_TC_SEG 4
#endif
#ifndef SPO_TC_SEG_DX
#define SPO_TC_SEG_DX 8
#endif
#ifndef SPO_TC_SEG_DW
#define SPO_TC_SEG_DW 8
#endif
template <int KIND>
__host__ __device__ constexpr int seg_of() {
  return (KIND == 1 || KIND == 2) ? SPO_TC_SEG_DX : (KIND == 3 ? SPO_TC_SEG_DW : SPO_TC_SEG);
}

// Kernel-internal epilogue: the forward written as plain fp32 (TC_FWD with c_lo == null,
// for an activation that no tensor-core product reads), without the mask bits.
constexpr int kFwdF32 = 4;

constexpr uint64_t kWaitNs = 2000000000ull;              // 2 s: the limit of every wait
// (the drains on the exit path wait a quarter of it)
constexpr int kMaxColsumN = 1024;

enum WaitCode : int {
  kErrWaitEmpty = 1, kErrWaitFull = 2, kErrWaitTEmpty = 3, kErrWaitTFull = 4, kErrWaitLoaded = 5,
  kErrWaitAEmpty = 6
};

struct __align__(64) Ctl {
  uint64_t full[STAGES_MAX];     // operands ready for the MMAs
  uint64_t empty[STAGES_MAX];    // stage consumed by the MMAs
  uint64_t loaded[STAGES_MAX];   // raw operands: the stage's copies have landed
  uint64_t aempty[ASTG_MAX];     // A in TMEM: the stage's MMAs are done with it
  uint64_t tfull[NACC_MAX];
  uint64_t tempty[NACC_MAX];
  uint64_t drain;
  uint32_t tmem_base;
  int abort;
};

struct KParams {
  int kind;
  int a_mn, b_mn;
  int64_t M, N, K, k_chunk;
  int m_tiles, n_tiles, splits;
  int64_t units;
  const float* bias;
  const float* mask;
  float* c_hi;
  float* c_lo;
  float* c_part;
  float* colsum;
  int* err;
  const uint32_t* mask_bits;
  uint32_t* c_bits;
  uint64_t wait_ns;   // limit of every bounded wait
  uint32_t withhold;  // 1 + the k-block (in the producer's count) whose operands are never
                      // loaded, so that the MMA issuer's wait for them runs out (0: none)
};

// ---------------------------------------------------------------- PTX wrappers
__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ uint64_t now_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

__device__ __forceinline__ void mbar_init(uint32_t bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(bar), "r"(count) : "memory");
}

__device__ __forceinline__ void mbar_expect_tx(uint32_t bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(bar), "r"(bytes)
               : "memory");
}

__device__ __forceinline__ void mbar_arrive(uint32_t bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(bar) : "memory");
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

__device__ __forceinline__ bool mbar_try_cluster(uint32_t bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.acquire.cluster.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(bar), "r"(parity)
      : "memory");
  return ok != 0;
}

// Bounded wait. Returns false when this CTA aborted (another role gave up) or after
// limit ns, in which case it raises the abort flag and records `code` in *err.
template <bool CLUSTER = false>
__device__ bool mbar_wait(uint32_t bar, uint32_t parity, volatile int* abort_flag, int* err,
                          int code, uint64_t limit) {
  auto poll = [&]() { return CLUSTER ? mbar_try_cluster(bar, parity) : mbar_try(bar, parity); };
  if (poll()) return true;
  const uint64_t t0 = now_ns();
  while (true) {
    if (poll()) return true;
    if (*abort_flag) return false;
    if (now_ns() - t0 > limit) {
      *abort_flag = 1;
      if (err) atomicCAS(err, 0, code);
      return false;
    }
  }
}

// Bounded wait used on the exit path only (ignores the abort flag).
__device__ void mbar_drain(uint32_t bar, uint32_t parity, uint64_t limit) {
  const uint64_t t0 = now_ns();
  while (!mbar_try(bar, parity) && now_ns() - t0 < limit) {
  }
}

__device__ __forceinline__ void tma_load_2d(uint32_t dst, const CUtensorMap* map, uint32_t bar,
                                            int32_t x, int32_t y) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%3, %4}], [%2];" ::"r"(dst),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(bar), "r"(x), "r"(y)
      : "memory");
}

__device__ __forceinline__ void tc_fence_before() {
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tc_fence_after() {
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}

__device__ __forceinline__ void mma_tf32(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc,
                                         uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::tf32 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate));
}

// The same MMA with A read from tensor memory (a_tmem: lane 0, first column of the 8 K
// columns of this k-step; row i of A in lane i).
__device__ __forceinline__ void mma_tf32_ta(uint32_t d_tmem, uint32_t a_tmem, uint64_t bdesc,
                                            uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::tf32 [%0], [%1], %2, %3, p;\n\t}" ::"r"(d_tmem),
      "r"(a_tmem), "l"(bdesc), "r"(idesc), "r"(accumulate));
}

__device__ __forceinline__ void mma_tf32_ta_pair(uint32_t d_tmem, uint32_t a_tmem, uint64_t bdesc,
                                                 uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::2.kind::tf32 [%0], [%1], %2, %3, p;\n\t}" ::"r"(d_tmem),
      "r"(a_tmem), "l"(bdesc), "r"(idesc), "r"(accumulate));
}

// tcgen05.st.32x32b.x16: thread t of the warp writes 16 consecutive 32-bit columns of TMEM
// lane (quadrant base + t), starting at the column of taddr.
__device__ __forceinline__ void tmem_st16(uint32_t taddr, const float (&v)[16]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], "
      "{%1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, %16};" ::"r"(taddr),
      "r"(__float_as_uint(v[0])), "r"(__float_as_uint(v[1])), "r"(__float_as_uint(v[2])),
      "r"(__float_as_uint(v[3])), "r"(__float_as_uint(v[4])), "r"(__float_as_uint(v[5])),
      "r"(__float_as_uint(v[6])), "r"(__float_as_uint(v[7])), "r"(__float_as_uint(v[8])),
      "r"(__float_as_uint(v[9])), "r"(__float_as_uint(v[10])), "r"(__float_as_uint(v[11])),
      "r"(__float_as_uint(v[12])), "r"(__float_as_uint(v[13])), "r"(__float_as_uint(v[14])),
      "r"(__float_as_uint(v[15]))
      : "memory");
}

__device__ __forceinline__ void tmem_wait_st() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }

__device__ __forceinline__ void mma_commit(uint32_t bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
                   bar)
               : "memory");
}

// ---- CTA-pair forms (cta_group::2; the cluster is the pair)
__device__ __forceinline__ uint32_t cluster_rank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}

// shared::cluster address of the same shared-memory offset in CTA `rank` of the cluster
__device__ __forceinline__ uint32_t map_to_rank(uint32_t addr, uint32_t rank) {
  uint32_t r;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(addr), "r"(rank));
  return r;
}

// every thread of both CTAs; threads may arrive from divergent paths (no .aligned)
__device__ __forceinline__ void cluster_sync() {
  asm volatile("barrier.cluster.arrive.release;\n\tbarrier.cluster.wait.acquire;" ::: "memory");
}

// TMA load into this CTA's shared memory whose completion is counted on an mbarrier of the
// pair (here: the first CTA's). No multicast: every CTA loads its own operand halves.
__device__ __forceinline__ void tma_load_2d_pair(uint32_t dst, const CUtensorMap* map, uint32_t cluster_bar,
                                                 int32_t x, int32_t y) {
  asm volatile(
      "cp.async.bulk.tensor.2d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%3, %4}], [%2];" ::"r"(dst),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(cluster_bar), "r"(x), "r"(y)
      : "memory");
}

__device__ __forceinline__ void mma_tf32_pair(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc,
                                              uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::2.kind::tf32 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate));
}

// Arrive on the mbarrier at this shared-memory offset in both CTAs of the pair once the
// MMAs issued so far have completed.
__device__ __forceinline__ void mma_commit_pair(uint32_t bar) {
  asm volatile(
      "tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.multicast::cluster.b64 [%0], %1;" ::"r"(bar),
      "h"((unsigned short)3)
      : "memory");
}

__device__ __forceinline__ void mbar_arrive_cluster(uint32_t cluster_bar) {
  asm volatile("mbarrier.arrive.release.cluster.shared::cluster.b64 _, [%0];" ::"r"(cluster_bar) : "memory");
}

// tcgen05.ld.16x256b.x8 without its wait: 16 TMEM lanes (rows) x 64 columns. Register
// r[4g + i] of thread t holds row (t / 4) + 8 (i / 2), column 8 g + 2 (t % 4) + (i % 2),
// relative to the lane and column of taddr (the layout of an mma accumulator fragment).
// The registers hold the data only after tmem_wait_tie(r), which waits for this thread's
// loads and names the registers as its operands so that no use of them is scheduled
// above the wait.
__device__ __forceinline__ void tmem_ld16x256_x8(uint32_t taddr, uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.16x256b.x8.b32 "
      "{%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, %16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]), "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr));
}

// The same shape repeated 4 times: 16 lanes x 32 columns; r[4 g + i] as above, g < 4.
__device__ __forceinline__ void tmem_ld16x256_x4(uint32_t taddr, uint32_t (&r)[16]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.16x256b.x4.b32 "
      "{%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
      : "r"(taddr));
}

__device__ __forceinline__ void tmem_wait_tie16(uint32_t (&r)[16]) {
  asm volatile("tcgen05.wait::ld.sync.aligned;"
               : "+r"(r[0]), "+r"(r[1]), "+r"(r[2]), "+r"(r[3]), "+r"(r[4]), "+r"(r[5]), "+r"(r[6]), "+r"(r[7]),
                 "+r"(r[8]), "+r"(r[9]), "+r"(r[10]), "+r"(r[11]), "+r"(r[12]), "+r"(r[13]), "+r"(r[14]), "+r"(r[15])
               :
               : "memory");
}

__device__ __forceinline__ void tmem_wait_tie(uint32_t (&r)[32]) {
  asm volatile("tcgen05.wait::ld.sync.aligned;"
               : "+r"(r[0]), "+r"(r[1]), "+r"(r[2]), "+r"(r[3]), "+r"(r[4]), "+r"(r[5]), "+r"(r[6]), "+r"(r[7]), "+r"(r[8]), "+r"(r[9]), "+r"(r[10]), "+r"(r[11]), "+r"(r[12]), "+r"(r[13]), "+r"(r[14]), "+r"(r[15]), "+r"(r[16]), "+r"(r[17]), "+r"(r[18]), "+r"(r[19]), "+r"(r[20]), "+r"(r[21]), "+r"(r[22]), "+r"(r[23]), "+r"(r[24]), "+r"(r[25]), "+r"(r[26]), "+r"(r[27]), "+r"(r[28]), "+r"(r[29]), "+r"(r[30]), "+r"(r[31])
               :
               : "memory");
}

// UMMA shared-memory descriptor (sm100 version bits), 128-byte swizzle layouts.
__device__ __forceinline__ uint64_t make_desc(uint32_t saddr, uint32_t lbo, uint32_t sbo,
                                              uint32_t layout) {
  uint64_t d = 0;
  d |= (uint64_t)((saddr >> 4) & 0x3FFFu);
  d |= (uint64_t)((lbo >> 4) & 0x3FFFu) << 16;
  d |= (uint64_t)((sbo >> 4) & 0x3FFFu) << 32;
  d |= (uint64_t)1 << 46;
  d |= (uint64_t)layout << 61;  // 2 = SWIZZLE_128B, 1 = SWIZZLE_128B_BASE32B
  return d;
}

__device__ __forceinline__ void store2(float* p, float a, float b) {
  *reinterpret_cast<float2*>(p) = make_float2(a, b);
}

__device__ __forceinline__ void prefetch_l2(const void* p, uint32_t bytes) {
  asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(p), "r"(bytes) : "memory");
}

// TF32 hi/lo split of n4 float4 of a stage tile in place (hi) and into lo, threads t of nt.
__device__ __forceinline__ void split_tile(float4* hi, float4* lo, int n4, int t, int nt) {
#pragma unroll 4
  for (int i = t; i < n4; i += nt) {
    float4 v = hi[i], l;
    tf32_split(v.x, v.x, l.x);
    tf32_split(v.y, v.y, l.y);
    tf32_split(v.z, v.z, l.z);
    tf32_split(v.w, v.w, l.w);
    hi[i] = v;
    lo[i] = l;
  }
}

// Stores the packed ReLU bits of a warp's 64 columns (c0 = first column) for its 32 rows:
// the 4 threads of a row hold disjoint bits, OR them, one thread stores the two words.
__device__ __forceinline__ void store_bits(uint32_t (&bw)[2][4], const KParams& P, int64_t wrow0, int tr,
                                           int lane, int64_t c0) {
#pragma unroll
  for (int hh = 0; hh < 2; ++hh) {
#pragma unroll
    for (int o = 1; o <= 2; o <<= 1)
#pragma unroll
      for (int w = 0; w < 4; ++w) bw[hh][w] |= __shfl_xor_sync(0xffffffffu, bw[hh][w], o);
    const int64_t ra = wrow0 + 16 * hh + tr, rb = ra + 8;
    if ((lane & 3) == 0) {
      const int64_t wpr = P.N / 32, w0 = c0 / 32;
      if (ra < P.M) *reinterpret_cast<uint2*>(P.c_bits + ra * wpr + w0) = make_uint2(bw[hh][0], bw[hh][1]);
      if (rb < P.M) *reinterpret_cast<uint2*>(P.c_bits + rb * wpr + w0) = make_uint2(bw[hh][2], bw[hh][3]);
    }
  }
}

// ---------------------------------------------------------------- the kernel
// One instantiation per epilogue (KIND) and dX mask format (BITS: packed bits instead of
// fp32). 10 warps share the SM's four 16K-register files 3/3/2/2: at most 168 registers a
// thread.
template <int KIND, bool BITS, bool PAIR, int TBN, int RAW>
__global__ void __launch_bounds__(Geo<PAIR, TBN, RAW>::THREADS, 1)
tc_gemm_kernel(const __grid_constant__ CUtensorMap tm_ah, const __grid_constant__ CUtensorMap tm_al,
               const __grid_constant__ CUtensorMap tm_bh, const __grid_constant__ CUtensorMap tm_bl,
               const KParams P) {
  using G = Geo<PAIR, TBN, RAW>;
  constexpr int BN = G::BN;
  constexpr int NACC = G::NACC;
  constexpr int kEpiWarps = G::EPI_WARPS;
  constexpr int kEpiThreads = G::EPI_THREADS;
  constexpr int SEG = seg_of<KIND>();
  constexpr int STAGES = G::STAGES;
  constexpr uint32_t STAGE_BYTES = G::STAGE_BYTES;
  constexpr uint32_t B_TILE = G::B_TILE;
  constexpr bool TA = G::TA;                   // A from tensor memory
  constexpr int ASTG = G::ASTG;
  constexpr uint32_t B_OFF = G::A_BYTES;       // B's offset in a stage
  constexpr bool AMN = KIND == TC_DW;          // A (and B) MN-major: dW
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~uintptr_t(1023));
  Ctl* ctl = reinterpret_cast<Ctl*>(smem + STAGES * STAGE_BYTES);
  float* colacc = reinterpret_cast<float*>(reinterpret_cast<uint8_t*>(ctl) + sizeof(Ctl));
  volatile int* abort_flag = &ctl->abort;

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const uint32_t smem0 = smem_u32(smem);
  // CTA pair: rank 0 issues the MMAs of both CTAs and owns the operand-full and
  // accumulator-empty barriers; each CTA loads and stores its own 128 rows.
  const uint32_t rank = PAIR ? cluster_rank() : 0;
  const bool leader = rank == 0;
  const int64_t first_unit = PAIR ? (blockIdx.x >> 1) : blockIdx.x;
  const int64_t unit_step = PAIR ? (gridDim.x >> 1) : gridDim.x;

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      // raw operands: the split warps of both CTAs of a pair arrive on the first CTA's barrier
      mbar_init(smem_u32(&ctl->full[s]), RAW ? (PAIR ? 2 : 1) * G::CONV_WARPS : 1);
      mbar_init(smem_u32(&ctl->empty[s]), 1);
      mbar_init(smem_u32(&ctl->loaded[s]), 1);
    }
    for (int a = 0; a < NACC; ++a) {
      mbar_init(smem_u32(&ctl->tfull[a]), 1);
      mbar_init(smem_u32(&ctl->tempty[a]), PAIR ? 2 * kEpiWarps : kEpiWarps);
    }
    for (int j = 0; j < ASTG; ++j) mbar_init(smem_u32(&ctl->aempty[j]), 1);
    mbar_init(smem_u32(&ctl->drain), 1);
    ctl->abort = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  if (warp == 1) {
    __syncwarp();
    if constexpr (PAIR) {
      asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                       smem_u32(&ctl->tmem_base)),
                   "r"(TMEM_COLS));
      asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;");
    } else {
      asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                       smem_u32(&ctl->tmem_base)),
                   "r"(TMEM_COLS));
      asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
    }
  }
  tc_fence_before();
  if constexpr (PAIR)
    cluster_sync();  // the peer's barriers are initialised before anyone signals them
  else
    __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = ctl->tmem_base;
  // everything above is on-chip; global memory (operands, bias, masks, outputs) only below
  pdl_wait();
  pdl_trigger();

  const int64_t per_split = (int64_t)P.m_tiles * P.n_tiles;

  if (warp == 0 && lane == 0) {
    // ------------------------------------------------ TMA producer
    uint32_t it = 0;
    bool ok = true;
    for (int64_t u = first_unit; u < P.units && ok; u += unit_step) {
      const int64_t split = u / per_split, rem = u % per_split;
      const int32_t m0 = (int32_t)((rem / P.n_tiles) * G::UNIT_M + rank * BM);
      const int32_t n0 = (int32_t)((rem % P.n_tiles) * BN + rank * G::B_ROWS);
      const int64_t kbeg = split * P.k_chunk;
      const int64_t kend = min(P.K, kbeg + P.k_chunk);
      const int nkb = (int)((kend - kbeg + BK - 1) / BK);
      for (int kb = 0; kb < nkb; ++kb, ++it) {
        const uint32_t s = it % STAGES, ph = (it / STAGES) & 1;
        if (!mbar_wait(smem_u32(&ctl->empty[s]), ph ^ 1, abort_flag, P.err, kErrWaitEmpty, P.wait_ns)) {
          ok = false;
          break;
        }
        // a test of the timeout path withholds one stage: its barriers never complete
        if (it + 1 == P.withhold) continue;
        // Raw operands: every CTA's copies complete on its own `loaded` barrier (its split
        // warps wait there). Otherwise on `full`, a pair's (both CTAs') on the first CTA's.
        const uint32_t bar = smem_u32(RAW ? &ctl->loaded[s] : &ctl->full[s]);
        constexpr uint32_t kMyBytes = ((RAW & kRawA) ? A_TILE : 2 * A_TILE) + ((RAW & kRawB) ? B_TILE : 2 * B_TILE);
        if (RAW)
          mbar_expect_tx(bar, kMyBytes);
        else if (leader)
          mbar_expect_tx(bar, PAIR ? 2 * STAGE_BYTES : STAGE_BYTES);
        const uint32_t cbar = PAIR && !RAW ? map_to_rank(bar, 0) : bar;
        auto load = [&](uint32_t dst, const CUtensorMap* m, int32_t x, int32_t y) {
          if constexpr (PAIR && !RAW)
            tma_load_2d_pair(dst, m, cbar, x, y);
          else
            tma_load_2d(dst, m, bar, x, y);
        };
        const int32_t k0 = (int32_t)(kbeg + (int64_t)kb * BK);
        const uint32_t a_hi = smem0 + s * STAGE_BYTES, a_lo = a_hi + A_TILE;
        const uint32_t b_hi = a_hi + B_OFF, b_lo = b_hi + B_TILE;
        constexpr bool ra = (RAW & kRawA) != 0, rb = (RAW & kRawB) != 0;
        if (TA && AMN) {
          load(a_hi, &tm_ah, m0, k0);   // one unswizzled [32 k][128 m] box
        } else if (P.a_mn) {
#pragma unroll
          for (int j = 0; j < BM / 32; ++j) {
            load(a_hi + j * 4096, &tm_ah, m0 + 32 * j, k0);
            if (!ra) load(a_lo + j * 4096, &tm_al, m0 + 32 * j, k0);
          }
        } else {
          load(a_hi, &tm_ah, k0, m0);
          if (!ra) load(a_lo, &tm_al, k0, m0);
        }
        if (P.b_mn) {
#pragma unroll
          for (int j = 0; j < G::B_ROWS / 32; ++j) {
            load(b_hi + j * 4096, &tm_bh, n0 + 32 * j, k0);
            if (!rb) load(b_lo + j * 4096, &tm_bl, n0 + 32 * j, k0);
          }
        } else {
          load(b_hi, &tm_bh, k0, n0);
          if (!rb) load(b_lo, &tm_bl, k0, n0);
        }
      }
    }
    if (!ok) {
      // let the copies already issued land before the CTA's shared memory goes away
      if (RAW || leader) {
        const uint32_t first = it >= (uint32_t)STAGES ? it - STAGES : 0;
        for (uint32_t i = first; i < it; ++i)
          mbar_drain(smem_u32(RAW ? &ctl->loaded[i % STAGES] : &ctl->full[i % STAGES]), (i / STAGES) & 1,
                     P.wait_ns / 4);
      } else {
        // the second CTA's copies complete on the first CTA's barriers: give them time
        const uint64_t t0 = now_ns();
        while (now_ns() - t0 < 10000000ull) {
        }
      }
    }
  } else if (warp == 1 && lane == 0) {
    // ------------------------------------------------ MMA issuer
    if (leader) {
      // dW reads both operands MN-major, every other product K-major
      constexpr bool MN = KIND == TC_DW;
      constexpr uint32_t idesc = (1u << 4) | (2u << 7) | (2u << 10) | ((uint32_t)MN << 15) |
                                 ((uint32_t)MN << 16) | ((uint32_t)(BN >> 3) << 17) |
                                 ((uint32_t)(G::UNIT_M >> 4) << 24);
      constexpr uint32_t k_step = MN ? 1024u : 32u;  // bytes between 8-wide k-steps
      constexpr uint32_t lbo = MN ? 4096u : 16u, sbo = MN ? 512u : 1024u, lay = MN ? 1u : 2u;
      // Descriptors of stage 0, k-step 0. The start-address field is the low 14 bits of
      // the low word ((shared address) >> 4, every operand below 256 KB), so the
      // descriptor of another stage, half or k-step is the same high word and a low word
      // plus ((byte offset) >> 4): one add per descriptor in the loop.
      const uint64_t da0 = make_desc(smem0, lbo, sbo, lay);
      const uint64_t db0 = make_desc(smem0 + B_OFF, lbo, sbo, lay);
      // A from tensor memory is read in rows (lane = row of A): K-major whatever its layout in
      // global memory
      constexpr uint32_t idesc_ta = idesc & ~(1u << 15);
      const uint32_t da_lo = (uint32_t)da0, db_lo = (uint32_t)db0;
      const uint64_t d_hi = da0 & 0xFFFFFFFF00000000ull;  // equal for A and B
      // Each unit's k-range is cut into segments of at most SEG k-blocks; every segment
      // gets a fresh accumulator (round robin over NACC), which the epilogue folds into its
      // fp32 running sum. Few accumulations per TMEM accumulator keep the sum fp32-accurate.
      uint32_t it = 0, seg_i = 0;
      bool ok = true;
      for (int64_t u = first_unit; u < P.units && ok; u += unit_step) {
        const int64_t split = u / per_split;
        const int64_t kbeg = split * P.k_chunk;
        const int64_t kend = min(P.K, kbeg + P.k_chunk);
        const int nkb = (int)((kend - kbeg + BK - 1) / BK);
        for (int kb0 = 0; kb0 < nkb && ok; kb0 += SEG, ++seg_i) {
          const uint32_t acc = seg_i % NACC;
          if (!mbar_wait<PAIR>(smem_u32(&ctl->tempty[acc]), ((seg_i / NACC) & 1) ^ 1, abort_flag,
                               P.err, kErrWaitTEmpty, P.wait_ns)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t d = tmem_base + acc * BN;
          const int kb1 = min(nkb, kb0 + SEG);
          for (int kb = kb0; kb < kb1; ++kb, ++it) {
            const uint32_t s = it % STAGES, ph = (it / STAGES) & 1;
            if (!mbar_wait<(PAIR && RAW != 0)>(smem_u32(&ctl->full[s]), ph, abort_flag, P.err, kErrWaitFull,
                                              P.wait_ns)) {
              ok = false;
              break;
            }
            tc_fence_after();
            const uint32_t so = s * (STAGE_BYTES >> 4);
#pragma unroll
            for (int ks = 0; ks < BK / 8; ++ks) {
              const uint32_t ah = da_lo + so + ks * (k_step >> 4), bh = db_lo + so + ks * (k_step >> 4);
              const uint64_t adh = d_hi | ah, adl = d_hi | (ah + (A_TILE >> 4));
              const uint64_t bdh = d_hi | bh, bdl = d_hi | (bh + (B_TILE >> 4));
              const uint32_t accum = (kb > kb0 || ks > 0) ? 1u : 0u;
              if constexpr (TA) {
                const uint32_t th = tmem_base + G::ACOL0 + (it % ASTG) * 64 + 8 * ks, tl = th + 32;
                if constexpr (PAIR) {
                  mma_tf32_ta_pair(d, tl, bdh, idesc_ta, accum);
                  mma_tf32_ta_pair(d, th, bdl, idesc_ta, 1u);
                  mma_tf32_ta_pair(d, th, bdh, idesc_ta, 1u);
                } else {
                  mma_tf32_ta(d, tl, bdh, idesc_ta, accum);
                  mma_tf32_ta(d, th, bdl, idesc_ta, 1u);
                  mma_tf32_ta(d, th, bdh, idesc_ta, 1u);
                }
              } else if constexpr (PAIR) {
                mma_tf32_pair(d, adl, bdh, idesc, accum);
                mma_tf32_pair(d, adh, bdl, idesc, 1u);
                mma_tf32_pair(d, adh, bdh, idesc, 1u);
              } else {
                mma_tf32(d, adl, bdh, idesc, accum);
                mma_tf32(d, adh, bdl, idesc, 1u);
                mma_tf32(d, adh, bdh, idesc, 1u);
              }
            }
            if constexpr (PAIR)
              mma_commit_pair(smem_u32(&ctl->empty[s]));
            else
              mma_commit(smem_u32(&ctl->empty[s]));
            if constexpr (TA) {   // the A stage in TMEM is free once these MMAs complete
              if constexpr (PAIR)
                mma_commit_pair(smem_u32(&ctl->aempty[it % ASTG]));
              else
                mma_commit(smem_u32(&ctl->aempty[it % ASTG]));
            }
          }
          if (!ok) break;
          if constexpr (PAIR)
            mma_commit_pair(smem_u32(&ctl->tfull[acc]));
          else
            mma_commit(smem_u32(&ctl->tfull[acc]));
        }
      }
      // all MMAs issued by this thread complete before TMEM is released (in both CTAs:
      // the second CTA passes the final cluster barrier only after this thread)
      if constexpr (PAIR)
        mma_commit_pair(smem_u32(&ctl->drain));
      else
        mma_commit(smem_u32(&ctl->drain));
      mbar_drain(smem_u32(&ctl->drain), 0, P.wait_ns / 4);
    }
  } else if (RAW && warp >= 2 + kEpiWarps) {
    // ------------------------------------------------ operand split
    // Four warps, one per TMEM lane quadrant; thread t of the warp for quadrant q owns row
    // r = 32 q + t of A. Per k-block: the fp32 A row (32 k values) is read from the stage,
    // split into TF32 hi/lo and written to TMEM lane r, columns [hi 0..31 | lo 32..63] of
    // A stage it % ASTG (after the MMAs of that stage's previous use completed). A raw B
    // (dW) is split in shared memory by all four warps (hi in place, lo in the lo slot).
    // Then the stage is handed to the MMA issuer (in the first CTA of a pair).
    const int q = warp & 3;
    const int row = 32 * q + lane;
    const uint32_t lane_addr = (uint32_t)(32 * q) << 16;
    const int ct = (warp - 2 - kEpiWarps) * 32 + lane;
    constexpr int kCT = 32 * G::CONV_WARPS;
    const uint32_t full0 = smem_u32(&ctl->full[0]);
    const uint32_t full_at = PAIR ? map_to_rank(full0, 0) : full0;
    uint32_t it = 0;
    bool ok = true;
    for (int64_t u = first_unit; u < P.units && ok; u += unit_step) {
      const int64_t split = u / per_split;
      const int64_t kbeg = split * P.k_chunk;
      const int64_t kend = min(P.K, kbeg + P.k_chunk);
      const int nkb = (int)((kend - kbeg + BK - 1) / BK);
      for (int kb = 0; kb < nkb; ++kb, ++it) {
        const uint32_t s = it % STAGES, ph = (it / STAGES) & 1;
        if (!mbar_wait(smem_u32(&ctl->loaded[s]), ph, abort_flag, P.err, kErrWaitLoaded, P.wait_ns)) {
          ok = false;
          break;
        }
        uint8_t* st = smem + s * STAGE_BYTES;
        if constexpr (TA) {
          const uint32_t j = it % ASTG;
          if (!mbar_wait(smem_u32(&ctl->aempty[j]), ((it / ASTG) & 1) ^ 1, abort_flag, P.err, kErrWaitAEmpty,
                         P.wait_ns)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t ta = tmem_base + lane_addr + G::ACOL0 + j * 64;
#pragma unroll
          for (int h = 0; h < 2; ++h) {
            float v[16], lo[16];
            if constexpr (!AMN) {
              // K-major 128-byte-swizzled rows: 16-byte chunk c of row r sits at c ^ (r % 8)
              const float4* rp = reinterpret_cast<const float4*>(st + row * 128);
#pragma unroll
              for (int c4 = 0; c4 < 4; ++c4) {
                const float4 x = rp[(4 * h + c4) ^ (row & 7)];
                v[4 * c4] = x.x;
                v[4 * c4 + 1] = x.y;
                v[4 * c4 + 2] = x.z;
                v[4 * c4 + 3] = x.w;
              }
            } else {
              // MN-major, unswizzled [32 k][128 m]
              const float* cp = reinterpret_cast<const float*>(st) + row;
#pragma unroll
              for (int i = 0; i < 16; ++i) v[i] = cp[(16 * h + i) * 128];
            }
#pragma unroll
            for (int i = 0; i < 16; ++i) tf32_split(v[i], v[i], lo[i]);
            tmem_st16(ta + 16 * h, v);
            tmem_st16(ta + 32 + 16 * h, lo);
          }
        }
        if constexpr ((RAW & kRawB) != 0)
          split_tile(reinterpret_cast<float4*>(st + B_OFF), reinterpret_cast<float4*>(st + B_OFF + B_TILE),
                     B_TILE / 16, ct, kCT);
        if constexpr (TA) tmem_wait_st();
        if constexpr ((RAW & kRawB) != 0) asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
        tc_fence_before();
        __syncwarp();
        if (lane == 0) {
          if (PAIR && !leader)
            mbar_arrive_cluster(full_at + s * 8);
          else
            mbar_arrive(full0 + s * 8);
        }
      }
    }
  } else if (warp >= 2) {
    // ------------------------------------------------ epilogue
    // Warp w reads TMEM lanes 32 (w % 4) .. +31 (tile rows) and columns cb .. cb + 63.
    // Each 16-row half is read in the 16x256b layout: thread t holds, for column group g
    // (8 columns), rows t/4 and t/4 + 8 at columns 8g + 2(t%4) + {0, 1}. Rows of a store
    // instruction are then written 32 contiguous bytes each (4 threads x float2): whole
    // sectors, with no shared-memory staging.
    const int q = warp & 3;                  // TMEM lane quadrant this warp may access
    const int cgrp = (warp - 2) >> 2;        // which EPI_COLS columns of the tile
    const int cb = cgrp * EPI_COLS;
    const int tr = lane >> 2, tc = 2 * (lane & 3);
    constexpr bool dx = KIND == TC_DX || KIND == TC_DX_F32;
    if (dx)
      for (int c = lane; c < P.N; c += 32)
        if ((c / EPI_COLS) % (BN / EPI_COLS) == cgrp) colacc[q * P.N + c] = 0.f;
    __syncwarp();
    uint32_t seg_i = 0;
    bool ok = true;
    const uint32_t lane_addr = (uint32_t)(q * 32) << 16;
    float rs[2 * 32];                        // fp32 running sums: [16-row half][4 g + i]
    // where this warp signals that it has read an accumulator: the MMA issuer's CTA
    const uint32_t tempty0 = smem_u32(&ctl->tempty[0]);
    const uint32_t tempty_at = PAIR ? map_to_rank(tempty0, 0) : tempty0;
    for (int64_t u = first_unit; u < P.units && ok; u += unit_step) {
      const int64_t split = u / per_split, rem = u % per_split;
      const int64_t m0 = (rem / P.n_tiles) * G::UNIT_M + rank * BM;
      const int64_t n0 = (rem % P.n_tiles) * BN;
      const int64_t kbeg = split * P.k_chunk;
      const int64_t kend = min(P.K, kbeg + P.k_chunk);
      const int nkb = (int)((kend - kbeg + BK - 1) / BK);
      const int nseg = (nkb + SEG - 1) / SEG;
      const int64_t wrow0 = m0 + q * 32;     // first row of this warp
      // packed mask words of this thread's 4 rows (16-row half hh, row t/4 + 8 j), loaded
      // now so that they have arrived by the end of the tile
      uint2 mw[4] = {};
      if (dx && BITS) {
        const int64_t wpr = P.N / 32;
#pragma unroll
        for (int k = 0; k < 4; ++k) {
          const int64_t r = wrow0 + 16 * (k >> 1) + tr + 8 * (k & 1);
          if (r < P.M) mw[k] = __ldg(reinterpret_cast<const uint2*>(P.mask_bits + r * wpr + (n0 + cb) / 32));
        }
      } else if (dx) {
        // the mask rows this warp reads at the end of the tile: into L2 while the MMAs run
        const int64_t r = wrow0 + lane;
        if (r < P.M) prefetch_l2(P.mask + r * P.N + n0 + cb, EPI_COLS * 4);
      }
      for (int sg = 0; sg < nseg; ++sg, ++seg_i) {
        const uint32_t acc = seg_i % NACC;
        if (!mbar_wait(smem_u32(&ctl->tfull[acc]), (seg_i / NACC) & 1, abort_flag, P.err,
                       kErrWaitTFull, P.wait_ns)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t ta = tmem_base + lane_addr + acc * BN + cb;
        if constexpr (kEpiWarps <= 8) {
          // one 16-row half at a time (32 registers in flight)
#pragma unroll
          for (int hh = 0; hh < 2; ++hh) {
            uint32_t r[32];
            tmem_ld16x256_x8(ta + ((uint32_t)(16 * hh) << 16), r);
            tmem_wait_tie(r);
            float* v = rs + 32 * hh;
            if (sg == 0) {
#pragma unroll
              for (int j = 0; j < 32; ++j) v[j] = __uint_as_float(r[j]);
            } else {
#pragma unroll
              for (int j = 0; j < 32; ++j) v[j] = v[j] + __uint_as_float(r[j]);
            }
          }
        } else {
          // 16 epilogue warps share the register file 5/5/4/4 per scheduler (at most 96
          // registers a thread): 32 columns of one 16-row half at a time (16 in flight)
#pragma unroll
          for (int hq = 0; hq < 4; ++hq) {
            uint32_t r[16];
            tmem_ld16x256_x4(ta + ((uint32_t)(16 * (hq >> 1)) << 16) + 32 * (hq & 1), r);
            tmem_wait_tie16(r);
            float* v = rs + 32 * (hq >> 1) + 16 * (hq & 1);
            if (sg == 0) {
#pragma unroll
              for (int j = 0; j < 16; ++j) v[j] = __uint_as_float(r[j]);
            } else {
#pragma unroll
              for (int j = 0; j < 16; ++j) v[j] = v[j] + __uint_as_float(r[j]);
            }
          }
        }
        // the accumulator is free for the next segment's MMAs once the loads completed
        tc_fence_before();
        __syncwarp();
        if (lane == 0) {
          if (PAIR && !leader)
            mbar_arrive_cluster(tempty_at + acc * 8);
          else
            mbar_arrive(tempty0 + acc * 8);
        }
        if (sg != nseg - 1) continue;
        // Final epilogue, one 8-column group g at a time over both 16-row halves, so that
        // only a few values besides the running sums are live at once.
        const int64_t cbase = n0 + cb + tc;
        if constexpr (KIND == kFwdF32) {
          uint32_t bw[2][4] = {};  // [hh]: bits of rows ra, rb, columns 0-31 / 32-63
#pragma unroll
          for (int g = 0; g < 8; ++g) {
            const int64_t col = cbase + 8 * g;
            const float2 b2 = __ldg(reinterpret_cast<const float2*>(P.bias + col));
            const uint32_t sh = (8 * g + tc) & 31;
#pragma unroll
            for (int hh = 0; hh < 2; ++hh) {
              const float* v = rs + 32 * hh;
              const int64_t ra = wrow0 + 16 * hh + tr, rb = ra + 8;
              const float x0 = v[4 * g] + b2.x, x1 = v[4 * g + 1] + b2.y;
              const float x2 = v[4 * g + 2] + b2.x, x3 = v[4 * g + 3] + b2.y;
              if (ra < P.M) store2(P.c_hi + ra * P.N + col, x0 > 0.f ? x0 : 0.f, x1 > 0.f ? x1 : 0.f);
              if (rb < P.M) store2(P.c_hi + rb * P.N + col, x2 > 0.f ? x2 : 0.f, x3 > 0.f ? x3 : 0.f);
              if (BITS) {
                const uint32_t pa = (x0 > 0.f ? 1u : 0u) | (x1 > 0.f ? 2u : 0u);
                const uint32_t pb = (x2 > 0.f ? 1u : 0u) | (x3 > 0.f ? 2u : 0u);
                bw[hh][(g < 4 ? 0 : 1)] |= pa << sh;
                bw[hh][(g < 4 ? 2 : 3)] |= pb << sh;
              }
            }
          }
          if (BITS) store_bits(bw, P, wrow0, tr, lane, n0 + cb);
        } else if constexpr (KIND == TC_FWD) {
          uint32_t bw[2][4] = {};  // [hh]: bits of rows ra, rb, columns 0-31 / 32-63
#pragma unroll
          for (int g = 0; g < 8; ++g) {
            const int64_t col = cbase + 8 * g;
            const float2 b2 = __ldg(reinterpret_cast<const float2*>(P.bias + col));
            const uint32_t sh = (8 * g + tc) & 31;
#pragma unroll
            for (int hh = 0; hh < 2; ++hh) {
              const float* v = rs + 32 * hh;
              const int64_t ra = wrow0 + 16 * hh + tr, rb = ra + 8;
              const float x[4] = {v[4 * g] + b2.x, v[4 * g + 1] + b2.y, v[4 * g + 2] + b2.x,
                                  v[4 * g + 3] + b2.y};
              float h[4], l[4];
#pragma unroll
              for (int t = 0; t < 4; ++t) tf32_split_pos(x[t] > 0.f ? x[t] : 0.f, h[t], l[t]);
              if (ra < P.M) {
                store2(P.c_hi + ra * P.N + col, h[0], h[1]);
                store2(P.c_lo + ra * P.N + col, l[0], l[1]);
              }
              if (rb < P.M) {
                store2(P.c_hi + rb * P.N + col, h[2], h[3]);
                store2(P.c_lo + rb * P.N + col, l[2], l[3]);
              }
              const uint32_t pa = (h[0] > 0.f ? 1u : 0u) | (h[1] > 0.f ? 2u : 0u);
              const uint32_t pb = (h[2] > 0.f ? 1u : 0u) | (h[3] > 0.f ? 2u : 0u);
              bw[hh][(g < 4 ? 0 : 1)] |= pa << sh;
              bw[hh][(g < 4 ? 2 : 3)] |= pb << sh;
            }
          }
          if (P.c_bits) store_bits(bw, P, wrow0, tr, lane, n0 + cb);
        } else if constexpr (dx) {
#pragma unroll
          for (int g = 0; g < 8; ++g) {
            const int64_t col = cbase + 8 * g;
            const uint32_t sh = (8 * g + tc) & 31;
            float c0 = 0.f, c1 = 0.f;  // column sums of this thread's two columns
#pragma unroll
            for (int hh = 0; hh < 2; ++hh) {
              float* v = rs + 32 * hh;
              const int64_t ra = wrow0 + 16 * hh + tr, rb = ra + 8;
              const bool ina = ra < P.M, inb = rb < P.M;
              float2 ma, mb;
              if constexpr (BITS) {
                const uint2 wa = mw[2 * hh], wb = mw[2 * hh + 1];
                const uint32_t xa = (g < 4 ? wa.x : wa.y) >> sh, xb = (g < 4 ? wb.x : wb.y) >> sh;
                ma = make_float2((float)(xa & 1u), (float)((xa >> 1) & 1u));
                mb = make_float2((float)(xb & 1u), (float)((xb >> 1) & 1u));
              } else {
                ma = ina ? __ldg(reinterpret_cast<const float2*>(P.mask + ra * P.N + col)) : make_float2(0.f, 0.f);
                mb = inb ? __ldg(reinterpret_cast<const float2*>(P.mask + rb * P.N + col)) : make_float2(0.f, 0.f);
              }
              const float y0 = ma.x > 0.f ? v[4 * g] : 0.f, y1 = ma.y > 0.f ? v[4 * g + 1] : 0.f;
              const float y2 = mb.x > 0.f ? v[4 * g + 2] : 0.f, y3 = mb.y > 0.f ? v[4 * g + 3] : 0.f;
              if constexpr (KIND == TC_DX) {
                float h0, l0, h1, l1, h2, l2, h3, l3;
                tf32_split(y0, h0, l0);
                tf32_split(y1, h1, l1);
                tf32_split(y2, h2, l2);
                tf32_split(y3, h3, l3);
                if (ina) {
                  store2(P.c_hi + ra * P.N + col, h0, h1);
                  store2(P.c_lo + ra * P.N + col, l0, l1);
                }
                if (inb) {
                  store2(P.c_hi + rb * P.N + col, h2, h3);
                  store2(P.c_lo + rb * P.N + col, l2, l3);
                }
              } else {
                if (ina) store2(P.c_hi + ra * P.N + col, y0, y1);
                if (inb) store2(P.c_hi + rb * P.N + col, y2, y3);
              }
              c0 += y0 + y2;
              c1 += y1 + y3;
            }
            if (P.colsum) {
              // sum over the 8 threads sharing t % 4 (the warp's 32 rows); lanes 0-3 then
              // hold columns n0 + cb + 8 g + 2 lane + {0, 1}
#pragma unroll
              for (int o = 4; o <= 16; o <<= 1) {
                c0 += __shfl_xor_sync(0xffffffffu, c0, o);
                c1 += __shfl_xor_sync(0xffffffffu, c1, o);
              }
              if (lane < 4) {
                float* ca = colacc + q * P.N + n0 + cb + 8 * g + tc;
                ca[0] += c0;
                ca[1] += c1;
              }
            }
          }
        } else {  // TC_DW
          float* pc = P.c_part + split * P.M * P.N;
#pragma unroll
          for (int hh = 0; hh < 2; ++hh) {
            const float* v = rs + 32 * hh;
            const int64_t ra = wrow0 + 16 * hh + tr, rb = ra + 8;
#pragma unroll
            for (int g = 0; g < 8; ++g) {
              const int64_t col = cbase + 8 * g;
              if (ra < P.M) store2(pc + ra * P.N + col, v[4 * g], v[4 * g + 1]);
              if (rb < P.M) store2(pc + rb * P.N + col, v[4 * g + 2], v[4 * g + 3]);
            }
          }
        }
      }
    }
    if (dx && P.colsum) {
      asm volatile("bar.sync 1, %0;" ::"r"(kEpiThreads) : "memory");
      const int t = threadIdx.x - 2 * 32;
      for (int c = t; c < P.N; c += kEpiThreads)
        P.colsum[(int64_t)blockIdx.x * P.N + c] =
            ((colacc[c] + colacc[P.N + c]) + colacc[2 * P.N + c]) + colacc[3 * P.N + c];
    }
  }

  tc_fence_before();
  if constexpr (PAIR)
    cluster_sync();  // neither CTA leaves while the pair's MMAs or copies may touch it
  else
    __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    __syncwarp();
    if constexpr (PAIR)
      asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(tmem_base),
                   "r"(TMEM_COLS));
    else
      asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem_base),
                   "r"(TMEM_COLS));
  }
}

// ---------------------------------------------------------------- split kernels
__global__ void split_tf32_kernel(const float* __restrict__ x, float* __restrict__ hi,
                                  float* __restrict__ lo, int64_t n, int keep_positive) {
  const int64_t gs = (int64_t)gridDim.x * blockDim.x;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += gs) {
    float h, l;
    const float v = x[i];
    if (keep_positive && v == v)  // a NaN takes the general split, which keeps it
      tf32_split_pos(v, h, l);
    else
      tf32_split(v, h, l);
    hi[i] = h;
    lo[i] = l;
  }
}

__global__ void combine_tf32_kernel(float* __restrict__ hi, const float* __restrict__ lo, int64_t n) {
  const int64_t gs = (int64_t)gridDim.x * blockDim.x;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += gs) hi[i] += lo[i];
}

__global__ void split_weights_kernel(const float* __restrict__ w, int64_t K, int64_t N,
                                     float* __restrict__ wt_hi, float* __restrict__ wt_lo,
                                     float* __restrict__ w_hi, float* __restrict__ w_lo) {
  __shared__ float hs[32][33];
  __shared__ float ls[32][33];
  pdl_wait();
  pdl_trigger();
  const int64_t k0 = (int64_t)blockIdx.y * 32, n0 = (int64_t)blockIdx.x * 32;
  for (int i = threadIdx.y; i < 32; i += 8) {
    const int64_t k = k0 + i, n = n0 + threadIdx.x;
    float h = 0.f, l = 0.f;
    if (k < K && n < N) {
      tf32_split(w[k * N + n], h, l);
      w_hi[k * N + n] = h;
      w_lo[k * N + n] = l;
    }
    hs[i][threadIdx.x] = h;
    ls[i][threadIdx.x] = l;
  }
  __syncthreads();
  for (int i = threadIdx.y; i < 32; i += 8) {
    const int64_t n = n0 + i, k = k0 + threadIdx.x;
    if (k < K && n < N) {
      wt_hi[n * K + k] = hs[threadIdx.x][i];
      wt_lo[n * K + k] = ls[threadIdx.x][i];
    }
  }
}

// ---------------------------------------------------------------- host side
// CTA pairs (cta_group::2) for the dW products, unless built with SPO_TC_PAIR=0. Measured
// at 1048576 x 512 x 512 on B200: dW 2.89 ms paired vs 3.26 ms single; the forward and dX
// products run 5-10% slower paired (the pair advances at the pace of its slower CTA and
// the mainloop is bound by shared-memory bandwidth, which pairing barely relieves), so
// they stay on single CTAs.
#ifndef SPO_TC_PAIR
#define SPO_TC_PAIR 1
#endif
bool use_pair(int kind) { return SPO_TC_PAIR != 0 && kind == TC_DW && sm_count() >= 2; }

#ifndef SPO_TC_BN256
#define SPO_TC_BN256 1
#endif
// Output columns per tile: 256 for the epilogues that are light per element (dW partials,
// the plain fp32 forward) when N allows it, else 128. The hi/lo forward and the dX products
// keep 128: their final epilogue (split, masks, column sums, twice the stored bytes) must
// finish within the slack of four 128-column accumulators, which two 256-column ones do
// not give.
int tile_n(int kind, bool fp32_fwd, int64_t N) {
  const bool light = kind == TC_DW || (kind == TC_FWD && fp32_fwd);
  return (SPO_TC_BN256 != 0 && light && N % 256 == 0) ? 256 : 128;
}
// A plain fp32 A (split into tensor memory) takes 128-column tiles in the forward and dX:
// two 128-column accumulators and four A stages fill the 512 TMEM columns.
int tile_of(const TcGemmArgs& a) {
  if (a.a_lo == nullptr && a.kind != TC_DW) return 128;
  return tile_n(a.kind, a.c_lo == nullptr, a.N);
}

int threads_of(bool pair, int bn, int raw) {
  if (raw)
    return bn == 256 ? (pair ? Geo<true, 256, 3>::THREADS : Geo<false, 256, 3>::THREADS)
                     : (pair ? Geo<true, 128, 3>::THREADS : Geo<false, 128, 3>::THREADS);
  return bn == 256 ? (pair ? Geo<true, 256>::THREADS : Geo<false, 256>::THREADS)
                   : (pair ? Geo<true, 128>::THREADS : Geo<false, 128>::THREADS);
}

template <bool PAIR, int BN, int RAW>
constexpr size_t ring_of() { return (size_t)Geo<PAIR, BN, RAW>::STAGES * Geo<PAIR, BN, RAW>::STAGE_BYTES; }

size_t ring_bytes(bool pair, int bn, int raw) {
  if (raw)
    return bn == 256 ? (pair ? ring_of<true, 256, 3>() : ring_of<false, 256, 3>())
                     : (pair ? ring_of<true, 128, 3>() : ring_of<false, 128, 3>());
  return bn == 256 ? (pair ? ring_of<true, 256, 0>() : ring_of<false, 256, 0>())
                   : (pair ? ring_of<true, 128, 0>() : ring_of<false, 128, 0>());
}

// Dynamic shared memory of a launch; raw = -1: the most any variant of this geometry takes
// (the size every instantiation is opted in to).
size_t tc_smem_bytes(int kind, int64_t N, bool pair, int bn, int raw = -1) {
  const size_t ring = raw < 0 ? std::max(ring_bytes(pair, bn, 0), ring_bytes(pair, bn, 3)) : ring_bytes(pair, bn, raw);
  size_t b = 1024 + ring + sizeof(Ctl);
  if (kind == TC_DX || kind == TC_DX_F32) b += (size_t)4 * N * sizeof(float);
  return b;
}

using Kern = void (*)(const CUtensorMap, const CUtensorMap, const CUtensorMap, const CUtensorMap, const KParams);

// The instantiations. raw: kRawA / kRawB bits (fp32 operands split in the kernel); bits: the
// packed ReLU mask (read by dX, written by the fp32 forward); has_lo: the output is a hi/lo
// pair. 256-column tiles exist for the light epilogues only (tile_n): dW and the fp32
// forward.
template <int RAW>
Kern pick_fwd_dx(int kind, bool bits, bool has_lo, int bn) {
  if (bn == 256)
    return bits ? tc_gemm_kernel<kFwdF32, true, false, 256, RAW> : tc_gemm_kernel<kFwdF32, false, false, 256, RAW>;
  switch (kind) {
    case TC_FWD:
      if (has_lo) return tc_gemm_kernel<TC_FWD, false, false, 128, RAW>;
      return bits ? tc_gemm_kernel<kFwdF32, true, false, 128, RAW> : tc_gemm_kernel<kFwdF32, false, false, 128, RAW>;
    case TC_DX: return bits ? tc_gemm_kernel<TC_DX, true, false, 128, RAW> : tc_gemm_kernel<TC_DX, false, false, 128, RAW>;
    default:
      return bits ? tc_gemm_kernel<TC_DX_F32, true, false, 128, RAW> : tc_gemm_kernel<TC_DX_F32, false, false, 128, RAW>;
  }
}

template <int RAW>
Kern pick_dw(bool pair, int bn) {
  if (bn == 256) return pair ? tc_gemm_kernel<TC_DW, false, true, 256, RAW> : tc_gemm_kernel<TC_DW, false, false, 256, RAW>;
  return pair ? tc_gemm_kernel<TC_DW, false, true, 128, RAW> : tc_gemm_kernel<TC_DW, false, false, 128, RAW>;
}

Kern pick(int kind, bool pair, bool bits, bool has_lo, int bn, int raw) {
  if (kind == TC_DW) return raw ? pick_dw<kRawA | kRawB>(pair, bn) : pick_dw<0>(pair, bn);
  return raw ? pick_fwd_dx<kRawA>(kind, bits, has_lo, bn) : pick_fwd_dx<0>(kind, bits, has_lo, bn);
}

// Opt an instantiation in to its shared memory once per device (never while a stream is
// being captured: the first launch of each shape happens uncaptured).
int opt_in(Kern kern, bool pair, int bn) {
  static std::mutex mu;
  static std::set<std::pair<int, const void*>> opted;
  int dev = 0;
  SPO_CUDA_TRY(cudaGetDevice(&dev));
  std::lock_guard<std::mutex> lk(mu);
  if (!opted.count({dev, (const void*)kern})) {
    SPO_CUDA_TRY(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                      (int)tc_smem_bytes(TC_DX, kMaxColsumN, pair, bn)));
    opted.insert({dev, (const void*)kern});
  }
  return kOk;
}

// CTA pairs that fit on the device at once (one CTA per SM; both SMs of a pair in one
// GPC). A persistent grid larger than this would leave pairs waiting for a second wave.
int pair_slots_query(int bn) {
  cudaLaunchConfig_t cfg{};
  cfg.gridDim = dim3(2);
  cfg.blockDim = dim3(threads_of(true, bn, kRawA | kRawB));
  cfg.dynamicSmemBytes = tc_smem_bytes(TC_DX, kMaxColsumN, true, bn);  // the opt-in size of every launch
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = 2;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  Kern kern = pick(TC_DW, true, false, true, bn, kRawA | kRawB);  // the learner's dW
  int n = 0;
  if (opt_in(kern, true, bn) != kOk || cudaOccupancyMaxActiveClusters(&n, kern, &cfg) != cudaSuccess || n < 1) {
    (void)cudaGetLastError();
    n = sm_count() / 2;
  }
  return n;
}

int pair_slots(int bn) {
  static std::mutex mu;
  static int slots[64][2] = {};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return sm_count() / 2;
  const int k = bn == 256 ? 1 : 0;
  {
    std::lock_guard<std::mutex> lk(mu);
    if (slots[dev][k]) return slots[dev][k];
  }
  const int n = pair_slots_query(bn);
  std::lock_guard<std::mutex> lk(mu);
  slots[dev][k] = n;
  return n;
}

int64_t units_of(const TcGemmArgs& a, int* splits) {
  const int64_t mt = ceil_div(a.M, use_pair(a.kind) ? 2 * BM : BM), nt = a.N / tile_of(a);
  int sp = 1;
  if (a.kind == TC_DW) sp = (int)ceil_div(a.K, a.k_chunk);
  if (splits) *splits = sp;
  return mt * nt * sp;
}

}  // namespace

static PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  if (!fn) {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
  }
  return fn;
}

// 2-D fp32 map of a row-major [outer x inner] array, 128-byte swizzle (16-byte or
// 32-byte atoms), zero fill out of bounds.
int make_map(CUtensorMap* m, const float* ptr, uint64_t inner, uint64_t outer, uint32_t box_inner,
             uint32_t box_outer, CUtensorMapSwizzle swz) {
  auto fn = encode_fn();
  if (!fn) return set_error(kErrCuda, "cuTensorMapEncodeTiled unavailable");
  if (!aligned16(ptr) || (inner * 4) % 16 != 0)
    return set_error(kErrAlign, "tensor map: base and row pitch must be 16-byte aligned");
  cuuint64_t dims[2] = {inner, outer};
  cuuint64_t strides[1] = {inner * 4};
  cuuint32_t box[2] = {box_inner, box_outer};
  cuuint32_t es[2] = {1, 1};
  CUresult r = fn(m, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, const_cast<float*>(ptr), dims, strides, box,
                  es, CU_TENSOR_MAP_INTERLEAVE_NONE, swz,
                  CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS)
    return set_error(kErrCuda, "cuTensorMapEncodeTiled failed (" + std::to_string((int)r) + ")");
  return kOk;
}

bool tc_gemm_supported(int kind, int64_t M, int64_t N, int64_t K) {
  if (M < 1 || N < 1 || K < 1 || N % 128 != 0) return false;
  if (kind == TC_DW) return M % BM == 0 && M <= (1 << 20) && N <= (1 << 20);
  if (K % BK != 0) return false;
  if ((kind == TC_DX || kind == TC_DX_F32) && N > kMaxColsumN) return false;
  return M < (int64_t(1) << 31);
}

int64_t tc_gemm_tiles(int kind, int64_t M, int64_t N) {
  return ceil_div(M, use_pair(kind) ? 2 * BM : BM) * (N / tile_n(kind, false, N));
}

int tc_gemm_slots(int kind, int64_t N) {
  return use_pair(kind) ? pair_slots(tile_n(kind, false, N)) : sm_count();
}

int tc_gemm_splits(const TcGemmArgs& a) {
  int s = 1;
  units_of(a, &s);
  return s;
}

int tc_gemm_grid(const TcGemmArgs& a) {
  const int64_t u = units_of(a, nullptr);
  if (use_pair(a.kind)) return 2 * (int)std::max<int64_t>(1, std::min<int64_t>(u, pair_slots(tile_of(a))));
  return (int)std::max<int64_t>(1, std::min<int64_t>(u, sm_count()));
}

int tc_gemm_launch(const TcGemmArgs& a, cudaStream_t s) {
  SPO_CHECK_ARG(tc_gemm_supported(a.kind, a.M, a.N, a.K), kErrUnsupported,
                "tc_gemm: unsupported shape (N % 128, K % 32, dW M % 128)");
  // Operands: a_lo / b_lo null = the operand is plain fp32, split in the kernel. The forward
  // and dX products take B (the weights) as a pair; dW takes both pairs or both fp32.
  SPO_CHECK_ARG(a.a_hi && a.b_hi && (a.kind == TC_DW ? (a.a_lo == nullptr) == (a.b_lo == nullptr) : a.b_lo != nullptr),
                kErrArg, "tc_gemm: null operand (dW: both operands fp32 or both hi/lo pairs; forward and dX: B as a pair)");
  const int raw = a.a_lo == nullptr ? (a.kind == TC_DW ? kRawA | kRawB : kRawA) : 0;
  if (a.kind == TC_DW)
    SPO_CHECK_ARG(a.k_chunk >= BK && a.k_chunk % BK == 0 && a.c_part, kErrArg,
                  "tc_gemm: dW needs c_part and k_chunk a multiple of 32");
  else
    SPO_CHECK_ARG(a.c_hi && aligned16(a.c_hi) &&
                      (a.kind == TC_DX_F32 || (a.c_lo ? aligned16(a.c_lo) : a.kind == TC_FWD)),
                  kErrArg, "tc_gemm: null or misaligned output");
  if (a.kind == TC_FWD) SPO_CHECK_ARG(a.bias && aligned16(a.bias), kErrArg, "tc_gemm: bias");
  if (a.kind == TC_DX || a.kind == TC_DX_F32)
    SPO_CHECK_ARG(a.mask_bits ? reinterpret_cast<uintptr_t>(a.mask_bits) % 8 == 0
                              : (a.mask && aligned16(a.mask)),
                  kErrArg, "tc_gemm: mask (16-byte aligned) or mask_bits (8-byte aligned)");
  if (a.kind == TC_FWD && a.c_bits)
    SPO_CHECK_ARG(reinterpret_cast<uintptr_t>(a.c_bits) % 8 == 0, kErrArg, "tc_gemm: c_bits alignment");
  const bool mn = a.kind == TC_DW;
  const bool pair = use_pair(a.kind);
  const int bn = tile_of(a);
  const uint32_t b_rows = pair ? bn / 2 : bn;  // rows of B one CTA stages (K-major)
  CUtensorMap m_ah, m_al, m_bh, m_bl;
  int rc;
  if (mn) {  // A [K x M], B [K x N] row-major; boxes 32 wide (MN) x 32 deep (K)
    const CUtensorMapSwizzle sw = CU_TENSOR_MAP_SWIZZLE_128B_ATOM_32B;
    if (raw & kRawA) {   // fp32 A for tensor memory: one unswizzled [32 k][128 m] box
      if ((rc = make_map(&m_ah, a.a_hi, a.M, a.K, BM, BK, CU_TENSOR_MAP_SWIZZLE_NONE))) return rc;
      m_al = m_ah;
    } else {
      if ((rc = make_map(&m_ah, a.a_hi, a.M, a.K, 32, BK, sw))) return rc;
      if ((rc = make_map(&m_al, a.a_lo, a.M, a.K, 32, BK, sw))) return rc;
    }
    if ((rc = make_map(&m_bh, a.b_hi, a.N, a.K, 32, BK, sw))) return rc;
    if ((rc = make_map(&m_bl, a.b_lo ? a.b_lo : a.b_hi, a.N, a.K, 32, BK, sw))) return rc;
  } else {   // A [M x K], B [N x K] row-major; boxes 32 deep (K) x 128 (A) / b_rows (B) rows
    const CUtensorMapSwizzle sw = CU_TENSOR_MAP_SWIZZLE_128B;
    if ((rc = make_map(&m_ah, a.a_hi, a.K, a.M, BK, BM, sw))) return rc;
    if ((rc = make_map(&m_al, a.a_lo ? a.a_lo : a.a_hi, a.K, a.M, BK, BM, sw))) return rc;
    if ((rc = make_map(&m_bh, a.b_hi, a.K, a.N, BK, b_rows, sw))) return rc;
    if ((rc = make_map(&m_bl, a.b_lo, a.K, a.N, BK, b_rows, sw))) return rc;
  }
  KParams P{};
  P.kind = a.kind;
  P.a_mn = mn;
  P.b_mn = mn;
  P.M = a.M;
  P.N = a.N;
  P.K = a.K;
  P.k_chunk = mn ? a.k_chunk : align_up_i64(a.K, BK);
  P.m_tiles = (int)ceil_div(a.M, pair ? 2 * BM : BM);
  P.n_tiles = (int)(a.N / bn);
  P.units = units_of(a, &P.splits);
  P.bias = a.bias;
  P.mask = a.mask;
  P.c_hi = a.c_hi;
  P.c_lo = a.c_lo;
  P.c_part = a.c_part;
  P.colsum = a.colsum;
  P.err = a.err;
  P.mask_bits = a.kind == TC_DX || a.kind == TC_DX_F32 ? a.mask_bits : nullptr;
  P.c_bits = a.kind == TC_FWD ? a.c_bits : nullptr;
  P.wait_ns = a.wait_ns > 0 ? a.wait_ns : kWaitNs;
  P.withhold = a.withhold;
  const int grid = tc_gemm_grid(a);
  const size_t smem = tc_smem_bytes(a.kind, a.N, pair, bn, raw);
  const int threads = threads_of(pair, bn, raw);
  const bool bits = a.kind == TC_FWD ? P.c_bits != nullptr : P.mask_bits != nullptr;
  const Kern kern = pick(a.kind, pair, bits, a.c_lo != nullptr, bn, raw);
  if ((rc = opt_in(kern, pair, bn))) return rc;
  SPO_CUDA_TRY(launch_pdl(kern, dim3((unsigned)grid), dim3(threads), smem, s, pair ? 2u : 0u, m_ah, m_al, m_bh,
                          m_bl, P));
  return kOk;
}

int split_tf32_launch(const float* x, float* hi, float* lo, int64_t n, bool keep_positive,
                      cudaStream_t s) {
  if (n <= 0) return kOk;
  const int grid = (int)std::min<int64_t>(ceil_div(n, 256), 8LL * sm_count());
  split_tf32_kernel<<<grid, 256, 0, s>>>(x, hi, lo, n, keep_positive ? 1 : 0);
  SPO_LAUNCH_CHECK();
  return kOk;
}

int combine_tf32_launch(float* hi, const float* lo, int64_t n, cudaStream_t s) {
  if (n <= 0) return kOk;
  const int grid = (int)std::min<int64_t>(ceil_div(n, 256), 8LL * sm_count());
  combine_tf32_kernel<<<grid, 256, 0, s>>>(hi, lo, n);
  SPO_LAUNCH_CHECK();
  return kOk;
}

int split_weights_launch(const float* w, int64_t K, int64_t N, float* wt_hi, float* wt_lo,
                         float* w_hi, float* w_lo, cudaStream_t s) {
  if (K <= 0 || N <= 0) return kOk;
  SPO_CUDA_TRY(launch_pdl(split_weights_kernel, dim3((unsigned)ceil_div(N, 32), (unsigned)ceil_div(K, 32)),
                          dim3(32, 8), 0, s, 0u, w, K, N, wt_hi, wt_lo, w_hi, w_lo));
  return kOk;
}

}  // namespace spo
