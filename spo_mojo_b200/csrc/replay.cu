// The data formats on either side of the learner step, on the device:
//
// * Replay sampling and gather (rl_utils/buffer.mojo:133-211): sequence indices drawn with
//   the project's counter-based generator, index = rand_bits(seed, stream, i) % count
//   (ops/rng.mojo:43-58), and gathers of the sampled sequences' fields, in the order of the
//   indices, repeats allowed. The reference samples on the host and uploads the gathered
//   batch every update; here the buffer stays in HBM and only the indices are produced.
//   rand_bits cascades the "lowbias32" integer finaliser (xor-shift / multiply, Wellons'
//   hash-prospector constants, as the reference uses them) over counter, stream and seed.
//
// * Observation encoding and legal mask (envs/tictactoe.mojo:449-480, 577-597): board
//   cells coded +1 (agent) / -1 (rival) / 0 (empty) become the three plane-major 0/1
//   planes [empty | agent | rival] the learner's first layer reads (27 values per board)
//   and the legal mask (the empty plane). The reference's two-plane encoding is the same
//   without the empty plane; the 27-wide input is the configuration this library trains.
#include "spo_common.cuh"
#include "kernels.cuh"

namespace spo {

namespace {

__device__ __forceinline__ uint32_t mix32(uint32_t x) {
  x ^= x >> 16;
  x *= 0x7FEB352Du;
  x ^= x >> 15;
  x *= 0x846CA68Bu;
  x ^= x >> 16;
  return x;
}

__device__ __forceinline__ uint32_t rand_bits(uint32_t seed, uint32_t stream, uint32_t counter) {
  return mix32(seed ^ mix32(stream ^ mix32(counter)));
}

__global__ void replay_sample_kernel(int32_t* __restrict__ idx, int64_t n, uint32_t count, uint32_t seed,
                                     uint32_t stream) {
  const int64_t gs = (int64_t)gridDim.x * blockDim.x;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += gs)
    idx[i] = (int32_t)(rand_bits(seed, stream, (uint32_t)i) % count);
}

// One warp per gathered sequence (grid-stride); span floats per sequence. An index outside
// [0, count) yields a zero row and sets *err (the reference raises on the host).
template <bool VEC>
__global__ void replay_gather_kernel(float* __restrict__ dst, const float* __restrict__ src,
                                     const int32_t* __restrict__ idx, int64_t n, int64_t span, int64_t count,
                                     int* err) {
  const int lane = threadIdx.x & 31;
  const int64_t warps = (int64_t)gridDim.x * (blockDim.x >> 5);
  for (int64_t k = (int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5); k < n; k += warps) {
    const int64_t s = idx[k];
    const bool ok = s >= 0 && s < count;
    if (!ok && lane == 0 && err) atomicExch(err, 1);
    float* d = dst + k * span;
    const float* g = src + (ok ? s : 0) * span;
    if (VEC) {
      const int64_t v = span / 4;
      for (int64_t j = lane; j < v; j += 32)
        reinterpret_cast<float4*>(d)[j] =
            ok ? __ldg(reinterpret_cast<const float4*>(g) + j) : make_float4(0.f, 0.f, 0.f, 0.f);
    } else {
      for (int64_t j = lane; j < span; j += 32) d[j] = ok ? __ldg(g + j) : 0.f;
    }
  }
}

constexpr int kCells = 9;

__global__ void encode_obs_kernel(float* __restrict__ obs, float* __restrict__ mask,
                                  const float* __restrict__ cells, int64_t n) {
  const int64_t gs = (int64_t)gridDim.x * blockDim.x;
  for (int64_t e = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; e < n * kCells; e += gs) {
    const int64_t r = e / kCells;
    const int c = (int)(e - r * kCells);
    const float v = __ldg(cells + e);
    const float empty = v == 0.f ? 1.f : 0.f;
    float* o = obs + r * 3 * kCells;
    o[c] = empty;
    o[kCells + c] = v == 1.f ? 1.f : 0.f;
    o[2 * kCells + c] = v == -1.f ? 1.f : 0.f;
    if (mask) mask[e] = empty;
  }
}

int grid_for(int64_t work, int threads) {
  return (int)std::max<int64_t>(1, std::min<int64_t>(ceil_div(work, threads), 8LL * sm_count()));
}

}  // namespace

int replay_sample_launch(int32_t* idx, int64_t n, int64_t count, uint32_t seed, uint32_t stream,
                         cudaStream_t s) {
  SPO_CHECK_ARG(n >= 0 && (n == 0 || idx), kErrArg, "replay_sample: bad output");
  SPO_CHECK_ARG(count >= 1 && count <= 0xFFFFFFFFll, kErrArg,
                "replay_sample: the buffer is empty: there is nothing to sample");
  SPO_CHECK_ARG(n <= 0xFFFFFFFFll, kErrArg, "replay_sample: at most 2^32 draws (32-bit counter)");
  if (n == 0) return kOk;
  replay_sample_kernel<<<grid_for(n, 256), 256, 0, s>>>(idx, n, (uint32_t)count, seed, stream);
  SPO_LAUNCH_CHECK();
  return kOk;
}

int replay_gather_launch(float* dst, const float* src, const int32_t* idx, int64_t n, int64_t span,
                         int64_t count, int* err, cudaStream_t s) {
  SPO_CHECK_ARG(n >= 0 && span >= 1 && count >= 0, kErrArg, "replay_gather: bad sizes");
  if (n == 0) return kOk;
  SPO_CHECK_ARG(dst && src && idx, kErrArg, "replay_gather: null pointer");
  const bool vec = span % 4 == 0 && aligned16(dst) && aligned16(src);
  const int grid = grid_for(n * 32, 256);
  if (vec)
    replay_gather_kernel<true><<<grid, 256, 0, s>>>(dst, src, idx, n, span, count, err);
  else
    replay_gather_kernel<false><<<grid, 256, 0, s>>>(dst, src, idx, n, span, count, err);
  SPO_LAUNCH_CHECK();
  return kOk;
}

int encode_obs_launch(float* obs, float* mask, const float* cells, int64_t n, cudaStream_t s) {
  SPO_CHECK_ARG(n >= 0 && (n == 0 || (obs && cells)), kErrArg, "encode_obs: null pointer");
  if (n == 0) return kOk;
  encode_obs_kernel<<<grid_for(n * kCells, 256), 256, 0, s>>>(obs, mask, cells, n);
  SPO_LAUNCH_CHECK();
  return kOk;
}

}  // namespace spo
