// Host-side checks of the C++ mirror of the reference's networks/ API (spo_networks.hpp)
// that need no GPU: the flat parameter layout, capacity errors raised before anything is
// enqueued, the library's own errors surfacing as spo::networks::Error, and the pure host
// functions. Device pointers are borrowed fakes that nothing dereferences.
//
// Output: one "layout" line per network shape (checked against the Python layout by the
// test that builds this program), then "ok <check>" per passed check; exit status 1 on the
// first failed check.
#include <cmath>
#include <cstdio>
#include <string>
#include <vector>

#include "spo_networks.hpp"

using namespace spo::networks;

namespace {

int failures = 0;

void expect(bool cond, const char* name, const std::string& detail = "") {
  if (cond) {
    std::printf("ok %s\n", name);
  } else {
    std::printf("FAIL %s %s\n", name, detail.c_str());
    ++failures;
  }
}

// the Error thrown by f, or code 0 when nothing was thrown
template <class F>
Error thrown_by(F f) {
  try {
    f();
  } catch (const Error& e) {
    return e;
  }
  return Error(0, "");
}

Buffer fake(uintptr_t addr, size_t n) { return Buffer::borrow(reinterpret_cast<float*>(addr), n); }

}  // namespace

int main() {
  const std::vector<std::vector<int>> shapes = {{27, 128, 128, 9}, {27, 512, 512, 512, 1}, {18, 5, 3}};
  for (const auto& dims : shapes) {
    int64_t total = 0;
    const auto offs = MLPParams::layout(dims, &total);
    std::printf("layout");
    for (int d : dims) std::printf(" %d", d);
    std::printf(" :");
    for (const auto& o : offs) std::printf(" %lld %lld", (long long)o.first, (long long)o.second);
    std::printf(" total %lld\n", (long long)total);
  }

  // an MLP with no layer, or more than the library's maximum, is refused
  expect(thrown_by([] { MLPParams::desc_of({27}); }).code() == SPO_ERR_SHAPE, "desc_of_too_short");
  expect(thrown_by([] { MLPParams::desc_of(std::vector<int>(SPO_MAX_LAYERS + 2, 8)); }).code() == SPO_ERR_SHAPE,
         "desc_of_too_long");

  // the reference's capacity error (networks/actor.mojo:156-165), same wording
  {
    const Error e = thrown_by([] { check_batch(4, 5, "actor", "boards"); });
    expect(e.code() == SPO_ERR_SHAPE &&
               std::string(e.what()) == "the actor was reserved for 4 boards and is being asked for 5",
           "actor_capacity_message", e.what());
    expect(thrown_by([] { check_batch(4, 4, "actor", "boards"); }).code() == 0, "actor_capacity_exact_fits");
  }

  DeviceContext ctx(0, nullptr);  // borrows the legacy stream: no CUDA call is made here

  // buffer capacities are checked before anything reaches the library
  {
    Buffer y = fake(0x10000, 100), x = fake(0x20000, 4 * 27), w = fake(0x30000, 27 * 128),
           b = fake(0x40000, 128);
    const Error e = thrown_by([&] { linear_forward(ctx, y, x, w, b, 4, 27, 128); });
    expect(e.code() == SPO_ERR_SHAPE && std::string(e.what()).find("linear_forward: y") == 0,
           "linear_forward_short_output", e.what());
    Buffer dw = fake(0x50000, 27 * 128), db = fake(0x60000, 128), dx, dy = fake(0x70000, 3 * 128);
    const Error e2 = thrown_by([&] { linear_backward(ctx, dw, db, dx, x, w, dy, 4, 27, 128); });
    expect(e2.code() == SPO_ERR_SHAPE && std::string(e2.what()).find("linear_backward: dy") == 0,
           "linear_backward_short_dy", e2.what());
    Buffer empty;
    expect(thrown_by([&] { relu(ctx, empty, 1); }).code() == SPO_ERR_SHAPE, "relu_empty_buffer");
    expect(thrown_by([&] { relu(ctx, empty, 0); }).code() == 0, "relu_nothing_to_do");
  }

  // an error found by the library itself carries its status and message
  {
    Buffer p = fake(0x100000, 64), g = fake(0x200000, 64);
    AdamState st{ctx, 0};  // zero-sized: no allocation
    st.m = fake(0x300000, 64);
    st.v = fake(0x400000, 64);
    const Error e = thrown_by([&] { adam_step(ctx, p, g, st, 64, 3e-4f, 1.f, 0); });
    expect(e.code() == SPO_ERR_ARG && std::string(e.what()).find("step starts at 1") != std::string::npos,
           "adam_step_zero_is_refused_by_the_library", e.what());
  }

  // pure host function: global_clip_scale (networks/optim.mojo:133-142), norm 13 -> 0.5 / 13
  {
    const float s = global_clip_scale(169.f, 0.5f);
    expect(std::fabs(s - 0.5f / 13.f) < 1e-7f, "global_clip_scale_known_answer", std::to_string(s));
    expect(global_clip_scale(0.01f, 0.5f) == 1.f, "global_clip_scale_no_clip");
  }

  // borrowed buffers are views: moving one moves the view, destroying it frees nothing
  {
    Buffer a = fake(0x500000, 7);
    Buffer b2 = std::move(a);
    expect(a.unsafe_ptr() == nullptr && a.size() == 0 && b2.size() == 7, "borrowed_move");
  }

  // the search models' weight-sync shape test (envs/tictactoe_actor.mojo:121-140)
  {
    const Error e = thrown_by([] { check_sync_shape({27, 64, 64, 9}, {27, 128, 128, 9}, "actor being copied"); });
    expect(e.code() == SPO_ERR_SHAPE &&
               std::string(e.what()) == "the actor being copied does not have the model's shape: 27x64x64x9",
           "sync_shape_message", e.what());
    expect(thrown_by([] { check_sync_shape({27, 128, 128, 1}, {27, 128, 128, 1}, "critic"); }).code() == 0,
           "sync_shape_equal");
  }

  return failures ? 1 : 0;
}
