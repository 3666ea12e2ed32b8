// Shared definitions for the libspo_cuda kernels: error reporting, launch checks,
// the masking constant, and small device helpers.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>
#include <float.h>
#include <string>

namespace spo {

// ops/common.mojo:19-23 — the most negative FINITE float32 masks illegal logits.
constexpr float kNegInf = -FLT_MAX;

constexpr int kMaxLayers = 8;

// Status codes returned by every C-ABI entry point (mirrored in include/spo_cuda.h).
enum Status : int {
  kOk = 0,
  kErrArg = -1,
  kErrShape = -2,
  kErrAlign = -3,
  kErrWorkspace = -4,
  kErrCuda = -5,
  kErrNccl = -6,
  kErrUnsupported = -7,
  kErrTimeout = -8,
};

// Records the message for spo_last_error_string() (thread-local) and returns code.
int set_error(int code, const std::string& msg);
void clear_error();

#define SPO_CHECK_ARG(cond, code, msg)                                    \
  do {                                                                    \
    if (!(cond)) return ::spo::set_error((code), std::string(__func__) + ": " + (msg)); \
  } while (0)

#define SPO_CUDA_TRY(expr)                                                \
  do {                                                                    \
    cudaError_t _e = (expr);                                              \
    if (_e != cudaSuccess)                                                \
      return ::spo::set_error(::spo::kErrCuda, std::string(__func__) + ": " #expr ": " + \
                              cudaGetErrorString(_e));                    \
  } while (0)

// After a launch: report configuration errors (not asynchronous faults).
#define SPO_LAUNCH_CHECK()                                                \
  do {                                                                    \
    cudaError_t _e = cudaGetLastError();                                  \
    if (_e != cudaSuccess)                                                \
      return ::spo::set_error(::spo::kErrCuda, std::string(__func__) + ": launch: " + \
                              cudaGetErrorString(_e));                    \
  } while (0)

inline bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

inline int64_t ceil_div(int64_t a, int64_t b) { return (a + b - 1) / b; }
inline int64_t align_up_i64(int64_t n, int64_t a) { return (n + a - 1) / a * a; }

// Number of SMs of the current device (cached per device).
int sm_count();

// Programmatic dependent launch. The learner's kernels are launched with programmatic
// stream serialisation (launch_pdl), so a kernel may begin while the kernel before it in
// the stream still runs: its launch and its on-chip set-up (shared-memory barriers, TMEM,
// registers) overlap the previous kernel's last wave. Every kernel launched this way calls
// pdl_wait() before its first access to global memory (the instruction returns once the
// previous grid has completed and its writes are visible), then pdl_trigger(), which lets
// the next kernel in the stream begin launching. For a kernel launched without the
// attribute, both return at once. SPO_PDL=0 in the environment turns the attribute off.
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_trigger() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }

bool pdl_enabled();

// Launch `kernel` on s with programmatic stream serialisation (when pdl_enabled()), plus an
// optional cluster of cluster_x CTAs (0 = none).
template <typename... KArgs, typename... Args>
cudaError_t launch_pdl(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t s,
                       unsigned cluster_x, Args... args) {
  cudaLaunchConfig_t cfg{};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = s;
  cudaLaunchAttribute attr[2];
  unsigned na = 0;
  if (cluster_x > 0) {
    attr[na].id = cudaLaunchAttributeClusterDimension;
    attr[na].val.clusterDim.x = cluster_x;
    attr[na].val.clusterDim.y = 1;
    attr[na].val.clusterDim.z = 1;
    ++na;
  }
  if (pdl_enabled()) {
    attr[na].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[na].val.programmaticStreamSerializationAllowed = 1;
    ++na;
  }
  cfg.attrs = attr;
  cfg.numAttrs = na;
  return cudaLaunchKernelEx(&cfg, kernel, args...);
}

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}

// TF32 hi/lo split of an fp32 value (the operand format of the 3xTF32 tensor-core GEMM).
//
// Round to TF32 (10 explicit mantissa bits), to nearest with ties away from zero, on the
// integer pattern: add half a TF32 ulp to the magnitude and clear the 13 dropped bits (a
// carry into the exponent is the correct rounding up, to infinity past the largest TF32
// value). Equal to cvt.rna.tf32.f32 for every finite input (checked over all 2^32
// patterns) and for both infinities, in two integer ALU operations instead of a
// conversion-unit instruction. Not for NaN: for the patterns 0x7ffff000-0x7fffffff (CUDA's
// canonical NaN among them) and 0xfffff000-0xffffffff the carry runs into the sign bit or
// out of the word and the result is -0 or +0; tf32_split below keeps NaN itself.
__device__ __forceinline__ float tf32_rna(float x) {
  return __uint_as_float((__float_as_uint(x) + 0x1000u) & 0xffffe000u);
}

// Both halves are rounded to nearest and are exact TF32 values, so the tensor core sees
// them unchanged: hi = rna(v), lo = rna(v - hi) (v - hi is exact in fp32). The part
// dropped, v - hi - lo, is below 2^-22 |v| and unbiased. A NaN goes into hi unchanged (a
// NaN gradient or weight stays NaN through the products it enters; lo is then
// irrelevant); for an infinite v, hi carries it.
__device__ __forceinline__ void tf32_split(float v, float& hi, float& lo) {
  hi = v == v ? tf32_rna(v) : v;
  lo = tf32_rna(v - hi);
}

// Split of a ReLU output (v >= 0, computed as v > 0 ? v : 0, so never NaN): a positive
// value never maps to hi == 0 (the tiny subnormals that round to 0 keep their full value
// in hi, and lo = 0), so the mask of the layer below can be read from hi alone.
__device__ __forceinline__ void tf32_split_pos(float v, float& hi, float& lo) {
  const uint32_t u = __float_as_uint(v);
  const uint32_t h = (u + 0x1000u) & 0xffffe000u;
  hi = __uint_as_float(h != 0u ? h : u);
  lo = tf32_rna(v - hi);
}

}  // namespace spo
