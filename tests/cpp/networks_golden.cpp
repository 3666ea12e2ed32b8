// The reference's own actor-backward goldens (bw_small, bw_big: an 18-h-h-9 actor, the
// eq-11 loss, gradients from jax.grad at highest matmul precision) run through the C++
// mirror of its networks/ API: actor_probs, actor_log_probs, cross_entropy_rows and
// actor_backward, exactly as the reference's learner chains them
// (networks/actor.mojo:90-122, networks/actor_loss.mojo:68-79,194-214). Tolerances are the
// reference test's (tests/test_actor_backward.mojo:95,111,159-163): pi 2e-5 absolute,
// loss 2e-5, each gradient 1e-4 of its largest magnitude.
//
//   networks_golden <golden dir> <case> <batch> <hidden>
// Exit status: 0 all within tolerance, 1 a mismatch, 2 no usable CUDA device.
#include <cmath>
#include <cstdio>
#include <fstream>
#include <string>
#include <vector>

#include "spo_networks.hpp"

using namespace spo::networks;

namespace {

std::vector<float> read_f32(const std::string& path, size_t n) {
  std::ifstream f(path, std::ios::binary);
  if (!f) throw std::runtime_error("cannot open " + path);
  std::vector<float> v(n);
  f.read(reinterpret_cast<char*>(v.data()), static_cast<std::streamsize>(n * sizeof(float)));
  if (static_cast<size_t>(f.gcount()) != n * sizeof(float)) throw std::runtime_error("short file " + path);
  return v;
}

Buffer upload(DeviceContext& ctx, const std::vector<float>& h) {
  Buffer b = zero_buffer(ctx, h.size());
  ctx.enqueue_copy_from_host(b, h.data(), h.size());
  return b;
}

std::vector<float> download(DeviceContext& ctx, const float* dev, size_t n) {
  std::vector<float> h(n);
  check_cuda(cudaMemcpyAsync(h.data(), dev, n * sizeof(float), cudaMemcpyDeviceToHost, ctx.stream()),
             "cudaMemcpyAsync");
  ctx.synchronize();
  return h;
}

double max_abs_err(const std::vector<float>& got, const std::vector<float>& want) {
  double e = 0;
  for (size_t i = 0; i < want.size(); ++i) e = std::fmax(e, std::fabs((double)got[i] - (double)want[i]));
  return e;
}

double max_abs(const std::vector<float>& v) {
  double m = 0;
  for (float x : v) m = std::fmax(m, std::fabs((double)x));
  return m;
}

}  // namespace

int main(int argc, char** argv) {
  if (argc != 5) {
    std::fprintf(stderr, "usage: %s <golden dir> <case> <batch> <hidden>\n", argv[0]);
    return 1;
  }
  const std::string dir = argv[1], cs = argv[2];
  const int m = std::stoi(argv[3]), h = std::stoi(argv[4]);
  const int in = 18, A = NUM_ACTIONS;
  auto file = [&](const std::string& name) { return dir + "/" + cs + "_" + name + ".bin"; };

  int device_count = 0;
  if (cudaGetDeviceCount(&device_count) != cudaSuccess || device_count == 0) {
    std::printf("no CUDA device\n");
    return 2;
  }
  try {
    DeviceContext ctx(0);
    const std::vector<int> dims{in, h, h, A};
    ActorParams params(ctx, dims);
    const std::vector<std::vector<float>> w = {read_f32(file("w1"), (size_t)in * h), read_f32(file("w2"), (size_t)h * h),
                                               read_f32(file("w3"), (size_t)h * A)};
    const std::vector<std::vector<float>> b = {read_f32(file("b1"), h), read_f32(file("b2"), h),
                                               read_f32(file("b3"), A)};
    for (int l = 1; l <= 3; ++l) params.load(ctx, l, w[l - 1].data(), b[l - 1].data());

    Buffer x = upload(ctx, read_f32(file("x"), (size_t)m * in));
    Buffer mask = upload(ctx, read_f32(file("mask"), (size_t)m * A));
    Buffer q = upload(ctx, read_f32(file("q"), (size_t)m * A));
    ActorCache cache(ctx, m, dims);
    Buffer pi = zero_buffer(ctx, (size_t)m * A), log_pi = zero_buffer(ctx, (size_t)m * A);
    Buffer ce = zero_buffer(ctx, m);

    actor_log_probs(ctx, params, cache, x, mask, log_pi, m);
    cross_entropy_rows(ctx, ce, q, log_pi, m, A);
    actor_probs(ctx, params, cache, x, mask, pi, m);  // leaves the cache of this forward
    CriticGrads grads(ctx, dims);
    CriticScratch scratch(ctx, m, dims);
    actor_backward(ctx, params, cache, grads, scratch, x, pi, q, mask, m);

    int bad = 0;
    const double pi_err = max_abs_err(download(ctx, pi.unsafe_ptr(), (size_t)m * A),
                                      read_f32(file("pi"), (size_t)m * A));
    std::printf("%s pi max abs err %.3g\n", cs.c_str(), pi_err);
    bad += pi_err > 2e-5;
    const std::vector<float> ce_h = download(ctx, ce.unsafe_ptr(), m);
    double loss = 0;
    for (float v : ce_h) loss += v;
    loss /= m;
    const double want_loss = read_f32(file("loss"), 1)[0];
    std::printf("%s loss %.8f want %.8f\n", cs.c_str(), loss, want_loss);
    bad += std::fabs(loss - want_loss) > 2e-5;
    const size_t sizes[3][2] = {{(size_t)in * h, (size_t)h}, {(size_t)h * h, (size_t)h}, {(size_t)h * A, (size_t)A}};
    for (int l = 1; l <= 3; ++l) {
      for (int wb = 0; wb < 2; ++wb) {
        const std::string name = std::string(wb ? "db" : "dw") + std::to_string(l);
        const std::vector<float> want = read_f32(file(name), sizes[l - 1][wb]);
        const std::vector<float> got = download(ctx, wb ? grads.db(l) : grads.dw(l), sizes[l - 1][wb]);
        const double rel = max_abs_err(got, want) / std::fmax(max_abs(want), 1e-30);
        std::printf("%s %s rel err of max %.3g\n", cs.c_str(), name.c_str(), rel);
        bad += rel > 1e-4;
      }
    }
    return bad ? 1 : 0;
  } catch (const std::exception& e) {
    std::printf("error: %s\n", e.what());
    return 1;
  }
}
