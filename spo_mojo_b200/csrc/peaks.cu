// Compute peaks of this GPU for the learner's two arithmetic paths, measured rather than
// taken from a datasheet (the driver-measured peaks cover HBM and bf16 only):
//
// * tcgen05 TF32: one CTA per SM issues back-to-back tcgen05.mma.kind::tf32 128x256x8 with
//   both operands in shared memory (random data) into two TMEM accumulators; ends with a
//   commit and a bounded wait. The 256-wide shape is the faster one (it reads A once for
//   twice the columns; 128x128x8 reaches ~87 % of its rate), so this is the ceiling.
// * FP32 FMA: every thread runs 8 independent chains of packed FFMA2 (two fp32 fma.rn per
//   instruction, sm_100's widest FP32 issue), enough chains to cover the FMA latency.
//
// Timed with CUDA events on the caller's stream, one warm-up launch each.
#include <cuda.h>

#include "spo_common.cuh"

namespace spo {

namespace {

// A [128 x 32] + B [256 x 32] fp32 (48 KB) in a buffer above half the shared memory, so
// that one CTA (holding all 512 TMEM columns) runs per SM
constexpr int kMmaSmem = 120 * 1024;
constexpr uint64_t kWaitNs = 2000000000ull;

__device__ __forceinline__ uint64_t umma_desc(uint32_t saddr) {
  uint64_t d = 0;
  d |= (uint64_t)((saddr >> 4) & 0x3FFFu);
  d |= (uint64_t)(16 >> 4) << 16;    // LBO
  d |= (uint64_t)(1024 >> 4) << 32;  // SBO: 8 rows of 128 B
  d |= (uint64_t)1 << 46;            // sm100 descriptor version
  d |= (uint64_t)2 << 61;            // 128-byte swizzle
  return d;
}

__global__ void __launch_bounds__(128, 1) tf32_mma_peak_kernel(int iters, int* err) {
  extern __shared__ uint8_t sm_raw[];
  // 128-byte swizzle atoms start on 1 KB boundaries (the launch adds 1 KB of slack)
  uint8_t* sm = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(sm_raw) + 1023) & ~uintptr_t(1023));
  __shared__ uint32_t tbase;
  __shared__ __align__(8) uint64_t bar;
  const int warp = threadIdx.x >> 5;
  for (int i = threadIdx.x; i < kMmaSmem / 4; i += blockDim.x) {
    uint32_t h = (uint32_t)i * 2654435761u + blockIdx.x * 97u;
    h ^= h >> 13;
    h *= 0x5bd1e995u;
    h ^= h >> 15;
    reinterpret_cast<float*>(sm)[i] = (float)(h & 0xFFFFF) * (1.f / 1048576.f) - 0.5f;
  }
  const uint32_t bar_a = static_cast<uint32_t>(__cvta_generic_to_shared(&bar));
  if (threadIdx.x == 0) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;" ::"r"(bar_a));
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  if (warp == 0) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], 512;" ::"r"(
        static_cast<uint32_t>(__cvta_generic_to_shared(&tbase))));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
  }
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
  __syncthreads();
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
  if (threadIdx.x == 0) {
    const uint32_t s0 = static_cast<uint32_t>(__cvta_generic_to_shared(sm));
    const uint32_t a = s0, b = s0 + 32768;
    const uint32_t idesc = (1u << 4) | (2u << 7) | (2u << 10) | (32u << 17) | (8u << 24);  // N 256, M 128
    for (int i = 0; i < iters; ++i) {
      const uint64_t ad = umma_desc(a + (i & 3) * 32), bd = umma_desc(b + (i & 3) * 32);
      const uint32_t d = tbase + (uint32_t)(i & 1) * 256;
      asm volatile(
          "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
          "tcgen05.mma.cta_group::1.kind::tf32 [%0], %1, %2, %3, p;\n\t}" ::"r"(d),
          "l"(ad), "l"(bd), "r"(idesc), "r"(i >= 2 ? 1 : 0));
    }
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(bar_a)
                 : "memory");
    uint64_t t0;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t0));
    while (true) {
      uint32_t ok;
      asm volatile(
          "{\n\t.reg .pred p;\n\tmbarrier.try_wait.parity.shared::cta.b64 p, [%1], 0;\n\t"
          "selp.u32 %0, 1, 0, p;\n\t}"
          : "=r"(ok)
          : "r"(bar_a)
          : "memory");
      if (ok) break;
      uint64_t t;
      asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
      if (t - t0 > kWaitNs) {
        atomicExch(err, 1);
        break;
      }
    }
  }
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
  __syncthreads();
  if (warp == 0) {
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, 512;" ::"r"(tbase));
  }
}

__global__ void __launch_bounds__(256) fp32_ffma2_peak_kernel(int iters, float seed, float* sink) {
  float2 a[8];
#pragma unroll
  for (int j = 0; j < 8; ++j) a[j] = make_float2(seed + j + threadIdx.x, seed - j);
  const float2 m = make_float2(0.9999f, 1.0001f), c = make_float2(1e-7f, -1e-7f);
  for (int i = 0; i < iters; ++i) {
#pragma unroll
    for (int j = 0; j < 8; ++j) a[j] = __ffma2_rn(a[j], m, c);
  }
  float s = 0.f;
#pragma unroll
  for (int j = 0; j < 8; ++j) s += a[j].x + a[j].y;
  if (s == 12345.678f) sink[threadIdx.x] = s;  // keeps the chains alive
}

}  // namespace

// TF32 tensor FLOP/s (2 * 128 * 256 * 8 per MMA) and FP32 FLOP/s (4 per FFMA2).
int measure_peaks(double* tf32_flops, double* fp32_flops, cudaStream_t s) {
  const int sms = sm_count();
  int* err = nullptr;
  float* sink = nullptr;
  cudaEvent_t e0 = nullptr, e1 = nullptr;
  int rc = kOk;
  auto fail = [&](cudaError_t e, const char* what) {
    rc = set_error(kErrCuda, std::string(what) + ": " + cudaGetErrorString(e));
  };
  cudaError_t e;
  if ((e = cudaMalloc(&err, sizeof(int))) != cudaSuccess) fail(e, "peaks: cudaMalloc");
  if (!rc && (e = cudaMalloc(&sink, 256 * sizeof(float))) != cudaSuccess) fail(e, "peaks: cudaMalloc");
  if (!rc && (e = cudaMemsetAsync(err, 0, sizeof(int), s)) != cudaSuccess) fail(e, "peaks: memset");
  if (!rc && (e = cudaEventCreate(&e0)) != cudaSuccess) fail(e, "peaks: event");
  if (!rc && (e = cudaEventCreate(&e1)) != cudaSuccess) fail(e, "peaks: event");
  if (!rc && (e = cudaFuncSetAttribute(tf32_mma_peak_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       kMmaSmem + 1024)) != cudaSuccess)
    fail(e, "peaks: attribute");
  const int mma_iters = 100000, fma_iters = 20000;
  float ms = 0.f;
  if (!rc) {
    tf32_mma_peak_kernel<<<sms, 128, kMmaSmem + 1024, s>>>(1000, err);
    cudaEventRecord(e0, s);
    tf32_mma_peak_kernel<<<sms, 128, kMmaSmem + 1024, s>>>(mma_iters, err);
    cudaEventRecord(e1, s);
    if ((e = cudaEventSynchronize(e1)) != cudaSuccess) fail(e, "peaks: tf32 run");
  }
  if (!rc) {
    int h = 0;
    cudaMemcpy(&h, err, sizeof(int), cudaMemcpyDeviceToHost);
    if (h) rc = set_error(kErrTimeout, "peaks: the MMA loop's completion wait gave up");
  }
  if (!rc) {
    cudaEventElapsedTime(&ms, e0, e1);
    *tf32_flops = 2.0 * 128 * 256 * 8 * (double)mma_iters * sms / (ms * 1e-3);
    const int blocks = 8 * sms;
    fp32_ffma2_peak_kernel<<<blocks, 256, 0, s>>>(100, 1.f, sink);
    cudaEventRecord(e0, s);
    fp32_ffma2_peak_kernel<<<blocks, 256, 0, s>>>(fma_iters, 1.f, sink);
    cudaEventRecord(e1, s);
    if ((e = cudaEventSynchronize(e1)) != cudaSuccess) fail(e, "peaks: fp32 run");
  }
  if (!rc) {
    cudaEventElapsedTime(&ms, e0, e1);
    *fp32_flops = 4.0 * 8 * (double)fma_iters * 256.0 * 8 * sms / (ms * 1e-3);
  }
  if (e0) cudaEventDestroy(e0);
  if (e1) cudaEventDestroy(e1);
  if (err) cudaFree(err);
  if (sink) cudaFree(sink);
  return rc;
}

}  // namespace spo
