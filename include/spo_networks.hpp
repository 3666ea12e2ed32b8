/*
 * spo_networks.hpp — C++ host mirror of the reference's networks/ API over libspo_cuda.
 *
 * The reference (josedanielchg/spo-mojo) is Mojo: its learner calls the functions of
 * networks/ (linear.mojo, mlp.mojo, actor.mojo, actor_loss.mojo, optim.mojo) with a
 * DeviceContext and DeviceBuffer[float32] handles, and they raise Error on bad shapes.
 * This header keeps those names, argument orders and meanings for C++ callers, and
 * enqueues the library's kernels through the C ABI of spo_cuda.h on the context's
 * stream. Nothing here computes on the CPU.
 *
 *   - DeviceContext: one device and one in-order stream (networks/mlp.mojo:109-110).
 *   - DeviceBuffer<T>: n elements of device memory, owned (cudaMalloc, zero-filled, freed
 *     on destruction; movable, not copyable, like the reference's buffers) or borrowed
 *     from memory the caller owns (DeviceBuffer<T>::borrow).
 *   - Errors: a failed call throws spo::networks::Error carrying the library's status and
 *     message (the reference raises Error in the same places). Buffer capacities are
 *     checked on the host before anything is enqueued.
 *   - Parameter containers keep the reference's field numbering (w(1), b(1), ...) but are
 *     views into ONE flat buffer (the layout of spo_mlp_param_layout), so that Adam runs
 *     over all of a network's tensors in one launch. W is stored [in, out].
 *
 * Link with -lspo_cuda -lcudart. C++17.
 */
#ifndef SPO_NETWORKS_HPP_
#define SPO_NETWORKS_HPP_

#include <cuda_runtime_api.h>

#include <cstddef>
#include <cstdint>
#include <stdexcept>
#include <string>
#include <utility>
#include <vector>

#include "spo_cuda.h"

namespace spo {
namespace networks {

constexpr int OBS_DIM = 27;        // three planes [empty | agent | rival] x 9 cells
constexpr int NUM_ACTIONS = 9;
constexpr float ADAM_EPS = 1e-5f;  // networks/optim.mojo:41-45 (Stoix's value)
constexpr float BETA1 = 0.9f;
constexpr float BETA2 = 0.999f;

// ------------------------------------------------------------------ errors

class Error : public std::runtime_error {
 public:
  Error(int code, const std::string& msg) : std::runtime_error(msg), code_(code) {}
  int code() const { return code_; }

 private:
  int code_;
};

// A nonzero library status becomes an Error with the library's own message.
inline void check(int status) {
  if (status != SPO_OK) throw Error(status, spo_last_error_string());
}

inline void check_cuda(cudaError_t e, const char* what) {
  if (e != cudaSuccess) throw Error(SPO_ERR_CUDA, std::string(what) + ": " + cudaGetErrorString(e));
}

// ------------------------------------------------------------------ buffers and context

template <class T>
class DeviceBuffer {
 public:
  DeviceBuffer() = default;

  // n zero-filled elements on the current device, the fill enqueued on `stream`
  DeviceBuffer(size_t n, cudaStream_t stream) : n_(n), owned_(true) {
    if (n == 0) return;
    check_cuda(cudaMalloc(reinterpret_cast<void**>(&ptr_), n * sizeof(T)), "cudaMalloc");
    const cudaError_t e = cudaMemsetAsync(ptr_, 0, n * sizeof(T), stream);
    if (e != cudaSuccess) {
      cudaFree(ptr_);
      ptr_ = nullptr;
      check_cuda(e, "cudaMemsetAsync");
    }
  }

  // A view of n elements of device memory the caller owns and keeps alive.
  static DeviceBuffer borrow(T* ptr, size_t n) {
    DeviceBuffer b;
    b.ptr_ = ptr;
    b.n_ = n;
    b.owned_ = false;
    return b;
  }

  DeviceBuffer(const DeviceBuffer&) = delete;
  DeviceBuffer& operator=(const DeviceBuffer&) = delete;
  DeviceBuffer(DeviceBuffer&& o) noexcept : ptr_(o.ptr_), n_(o.n_), owned_(o.owned_) {
    o.ptr_ = nullptr;
    o.n_ = 0;
    o.owned_ = false;
  }
  DeviceBuffer& operator=(DeviceBuffer&& o) noexcept {
    if (this != &o) {
      release();
      ptr_ = o.ptr_;
      n_ = o.n_;
      owned_ = o.owned_;
      o.ptr_ = nullptr;
      o.n_ = 0;
      o.owned_ = false;
    }
    return *this;
  }
  ~DeviceBuffer() { release(); }

  T* unsafe_ptr() const { return ptr_; }
  size_t size() const { return n_; }

 private:
  void release() {
    if (owned_ && ptr_) cudaFree(ptr_);  // cudaFree waits for the device's work on it
    ptr_ = nullptr;
  }
  T* ptr_ = nullptr;
  size_t n_ = 0;
  bool owned_ = false;
};

using Buffer = DeviceBuffer<float>;

// Host-side capacity check: `buf` must hold at least `need` elements.
template <class T>
inline void require(const DeviceBuffer<T>& buf, int64_t need, const char* what) {
  if (need < 0 || (need > 0 && buf.unsafe_ptr() == nullptr) || static_cast<uint64_t>(need) > buf.size())
    throw Error(SPO_ERR_SHAPE, std::string(what) + ": needs " + std::to_string(need) + " elements, the buffer holds " +
                                   std::to_string(buf.size()));
}

class DeviceContext {
 public:
  // Device `device` with a stream of its own.
  explicit DeviceContext(int device = 0) : device_(device), owns_stream_(true) {
    check_cuda(cudaSetDevice(device), "cudaSetDevice");
    check_cuda(cudaStreamCreateWithFlags(&stream_, cudaStreamNonBlocking), "cudaStreamCreate");
  }
  // Device `device` enqueuing on the caller's stream (which the caller keeps alive).
  DeviceContext(int device, cudaStream_t stream) : device_(device), stream_(stream), owns_stream_(false) {}
  DeviceContext(const DeviceContext&) = delete;
  DeviceContext& operator=(const DeviceContext&) = delete;
  ~DeviceContext() {
    ws_ = DeviceBuffer<unsigned char>();
    if (owns_stream_ && stream_) cudaStreamDestroy(stream_);
  }

  int device() const { return device_; }
  cudaStream_t stream() const { return stream_; }
  spo_stream_t handle() const { return reinterpret_cast<spo_stream_t>(stream_); }
  void synchronize() const { check_cuda(cudaStreamSynchronize(stream_), "cudaStreamSynchronize"); }

  template <class T>
  DeviceBuffer<T> enqueue_create_buffer(size_t n) const {
    return DeviceBuffer<T>(n, stream_);
  }

  // Scratch for the calls that need it, grown on demand and reused.
  DeviceBuffer<unsigned char>& workspace(size_t nbytes) {
    if (nbytes < 256) nbytes = 256;
    if (ws_.size() < nbytes) {
      synchronize();  // the old scratch may still be in use by enqueued work
      ws_ = DeviceBuffer<unsigned char>(nbytes, stream_);
    }
    return ws_;
  }

  template <class T>
  void enqueue_copy_from_host(DeviceBuffer<T>& dst, const T* src, size_t n) const {
    require(dst, static_cast<int64_t>(n), "enqueue_copy_from_host");
    check_cuda(cudaMemcpyAsync(dst.unsafe_ptr(), src, n * sizeof(T), cudaMemcpyHostToDevice, stream_),
               "cudaMemcpyAsync");
  }
  template <class T>
  void enqueue_copy_to_host(T* dst, const DeviceBuffer<T>& src, size_t n) const {
    require(src, static_cast<int64_t>(n), "enqueue_copy_to_host");
    check_cuda(cudaMemcpyAsync(dst, src.unsafe_ptr(), n * sizeof(T), cudaMemcpyDeviceToHost, stream_),
               "cudaMemcpyAsync");
  }

 private:
  int device_ = 0;
  cudaStream_t stream_ = nullptr;
  bool owns_stream_ = false;
  DeviceBuffer<unsigned char> ws_;
};

// ops/buffers.mojo:21-34
inline Buffer zero_buffer(const DeviceContext& ctx, size_t n) { return ctx.enqueue_create_buffer<float>(n); }

// ------------------------------------------------------------------ Linear (networks/linear.mojo)

// y[m x n] = x[m x k] W[k x n] + b  (networks/linear.mojo:86-95); relu = true fuses
// networks/mlp.mojo:34-46.
inline void linear_forward(DeviceContext& ctx, Buffer& y, const Buffer& x, const Buffer& w, const Buffer& bias,
                           int64_t m, int64_t k, int64_t n, bool relu = false) {
  require(y, m * n, "linear_forward: y");
  require(x, m * k, "linear_forward: x");
  require(w, k * n, "linear_forward: w");
  require(bias, n, "linear_forward: bias");
  check(spo_linear_fwd(ctx.handle(), y.unsafe_ptr(), x.unsafe_ptr(), w.unsafe_ptr(), bias.unsafe_ptr(), m, k, n,
                       relu ? SPO_ACT_RELU : SPO_ACT_NONE));
}

// dW = x^T dy, db = sum_rows dy, dx = dy W^T  (networks/linear.mojo:170-193); dx may be
// an empty buffer (the first layer drops it, :176-178); relu_src, when given, masks dx
// with (relu_src > 0) (relu_backward_kernel, networks/mlp.mojo:155-166).
inline void linear_backward(DeviceContext& ctx, Buffer& dw, Buffer& db, Buffer& dx, const Buffer& x, const Buffer& w,
                            const Buffer& dy, int64_t m, int64_t k, int64_t n, const Buffer* relu_src = nullptr) {
  require(dw, k * n, "linear_backward: dw");
  require(db, n, "linear_backward: db");
  if (dx.unsafe_ptr()) require(dx, m * k, "linear_backward: dx");
  require(x, m * k, "linear_backward: x");
  require(w, k * n, "linear_backward: w");
  require(dy, m * n, "linear_backward: dy");
  if (relu_src) require(*relu_src, m * k, "linear_backward: relu_src");
  const size_t nbytes = spo_linear_bwd_workspace_size(m, k, n);
  if (nbytes == 0) check(SPO_ERR_SHAPE);
  auto& ws = ctx.workspace(nbytes);
  check(spo_linear_bwd(ctx.handle(), dw.unsafe_ptr(), db.unsafe_ptr(), dx.unsafe_ptr(), x.unsafe_ptr(),
                       w.unsafe_ptr(), dy.unsafe_ptr(), relu_src ? relu_src->unsafe_ptr() : nullptr, m, k, n,
                       ws.unsafe_ptr(), ws.size()));
}

// In-place ReLU (networks/mlp.mojo:42-46) and grad *= (activation > 0) (:155-166).
inline void relu(DeviceContext& ctx, Buffer& a, int64_t n) {
  require(a, n, "relu");
  check(spo_relu(ctx.handle(), a.unsafe_ptr(), n));
}
inline void relu_backward(DeviceContext& ctx, Buffer& grad, const Buffer& activation, int64_t n) {
  require(grad, n, "relu_backward: grad");
  require(activation, n, "relu_backward: activation");
  check(spo_relu_bwd(ctx.handle(), grad.unsafe_ptr(), activation.unsafe_ptr(), n));
}

// ------------------------------------------------------------------ MLP (networks/mlp.mojo)

// Weights of an MLP with dims d0..dL (CriticParams, networks/mlp.mojo:50-68, generalised
// to L layers) as views into one flat buffer; w(l), b(l) for l = 1..L as in the
// reference's w1, b1, w2, ...
class MLPParams {
 public:
  // The flat layout of `dims` without allocating: offsets[l-1] = {w offset, b offset}.
  static std::vector<std::pair<int64_t, int64_t>> layout(const std::vector<int>& dims, int64_t* total) {
    const spo_mlp_desc d = desc_of(dims);
    int64_t wo[SPO_MAX_LAYERS] = {}, bo[SPO_MAX_LAYERS] = {};
    check(spo_mlp_param_layout(&d, wo, bo, total));
    std::vector<std::pair<int64_t, int64_t>> out;
    for (int l = 0; l < d.num_layers; ++l) out.emplace_back(wo[l], bo[l]);
    return out;
  }

  static spo_mlp_desc desc_of(const std::vector<int>& dims) {
    if (dims.size() < 2 || dims.size() > SPO_MAX_LAYERS + 1)
      throw Error(SPO_ERR_SHAPE, "an MLP needs 1 to " + std::to_string(SPO_MAX_LAYERS) + " layers");
    spo_mlp_desc d{};
    d.num_layers = static_cast<int32_t>(dims.size() - 1);
    for (size_t i = 0; i < dims.size(); ++i) d.dims[i] = dims[i];
    return d;
  }

  MLPParams(DeviceContext& ctx, std::vector<int> dims) : dims_(std::move(dims)) {
    int64_t total = 0;
    offsets_ = layout(dims_, &total);
    flat_ = zero_buffer(ctx, static_cast<size_t>(total));
  }

  const std::vector<int>& dims() const { return dims_; }
  int num_layers() const { return static_cast<int>(dims_.size()) - 1; }
  int in_dim() const { return dims_.front(); }
  int hidden() const { return dims_[1]; }
  int out_dim() const { return dims_.back(); }
  spo_mlp_desc desc() const { return desc_of(dims_); }
  Buffer& flat() { return flat_; }
  const Buffer& flat() const { return flat_; }
  int64_t size() const { return static_cast<int64_t>(flat_.size()); }

  // W_l [d_{l-1} x d_l] and b_l [d_l], l = 1..L
  float* w(int l) const { return flat_.unsafe_ptr() + offsets_.at(l - 1).first; }
  float* b(int l) const { return flat_.unsafe_ptr() + offsets_.at(l - 1).second; }

  // Copy layer l's weights and bias from host memory.
  void load(DeviceContext& ctx, int l, const float* host_w, const float* host_b) {
    const int64_t k = dims_.at(l - 1), n = dims_.at(l);
    check_cuda(cudaMemcpyAsync(w(l), host_w, sizeof(float) * k * n, cudaMemcpyHostToDevice, ctx.stream()),
               "cudaMemcpyAsync");
    check_cuda(cudaMemcpyAsync(b(l), host_b, sizeof(float) * n, cudaMemcpyHostToDevice, ctx.stream()),
               "cudaMemcpyAsync");
  }

 private:
  std::vector<int> dims_;
  std::vector<std::pair<int64_t, int64_t>> offsets_;
  Buffer flat_;
};

using CriticParams = MLPParams;
using ActorParams = MLPParams;  // networks/actor.mojo:39-40

// networks/mlp.mojo:71-81 (depth = number of hidden layers, 2 in the reference)
inline MLPParams zero_critic_params(DeviceContext& ctx, int in_dim, int hidden, int out_dim, int depth = 2) {
  std::vector<int> dims{in_dim};
  for (int i = 0; i < depth; ++i) dims.push_back(hidden);
  dims.push_back(out_dim);
  return MLPParams(ctx, dims);
}
// networks/actor.mojo:45-47
inline MLPParams zero_actor_params(DeviceContext& ctx, int hidden, int in_dim = OBS_DIM, int depth = 2) {
  return zero_critic_params(ctx, in_dim, hidden, NUM_ACTIONS, depth);
}

// Raises like the reference's capacity checks (networks/actor.mojo:156-165).
inline void check_batch(int64_t max_batch, int64_t m, const char* who, const char* unit) {
  if (m < 0 || m > max_batch)
    throw Error(SPO_ERR_SHAPE, std::string("the ") + who + " was reserved for " + std::to_string(max_batch) + " " +
                                   unit + " and is being asked for " + std::to_string(m));
}

// One forward's post-ReLU activations a1..a_{L-1} and output (networks/mlp.mojo:84-102).
class CriticCache {
 public:
  CriticCache(DeviceContext& ctx, int64_t max_batch, std::vector<int> dims)
      : dims_(std::move(dims)), max_batch_(max_batch) {
    const spo_mlp_desc d = MLPParams::desc_of(dims_);
    const int64_t n_act = spo_mlp_acts_size(&d, max_batch);
    if (n_act < 0) check(SPO_ERR_SHAPE);
    acts = zero_buffer(ctx, static_cast<size_t>(n_act > 0 ? n_act : 1));
    value = zero_buffer(ctx, static_cast<size_t>(max_batch * dims_.back()));
  }
  void check(int64_t m) const { check_batch(max_batch_, m, "cache", "rows"); }
  int64_t max_batch() const { return max_batch_; }
  const std::vector<int>& dims() const { return dims_; }
  // a_i of the last forward with m rows, [m x d_i], i = 1..L-1
  float* act(int i, int64_t m) const {
    int64_t off = 0;
    for (int j = 1; j < i; ++j) off += m * dims_.at(j);
    return acts.unsafe_ptr() + off;
  }

  Buffer acts;   // a1 .. a_{L-1}, layer after layer
  Buffer value;  // [max_batch x dL]: V, or the actor's (masked) logits

 private:
  std::vector<int> dims_;
  int64_t max_batch_;
};
using ActorCache = CriticCache;

// V(s) for m inputs, activations kept in cache (networks/mlp.mojo:105-123).
inline void critic_forward(DeviceContext& ctx, const MLPParams& params, CriticCache& cache, const Buffer& x,
                           int64_t m) {
  cache.check(m);
  require(x, m * params.in_dim(), "critic_forward: x");
  const spo_mlp_desc d = params.desc();
  check(spo_mlp_fwd(ctx.handle(), &d, params.flat().unsafe_ptr(), x.unsafe_ptr(), m, cache.acts.unsafe_ptr(),
                    cache.value.unsafe_ptr()));
}

// Gradients with the parameters' layout (networks/mlp.mojo:169-186): dw(l), db(l).
class CriticGrads {
 public:
  CriticGrads(DeviceContext& ctx, std::vector<int> dims) : p_(ctx, std::move(dims)) {}
  float* dw(int l) const { return p_.w(l); }
  float* db(int l) const { return p_.b(l); }
  Buffer& flat() { return p_.flat(); }
  const Buffer& flat() const { return p_.flat(); }

 private:
  MLPParams p_;
};

// dvalue and the backward's working memory (networks/mlp.mojo:189-209).
class CriticScratch {
 public:
  CriticScratch(DeviceContext& ctx, int64_t max_batch, const std::vector<int>& dims) : max_batch_(max_batch) {
    dvalue = zero_buffer(ctx, static_cast<size_t>(max_batch * dims.back()));
    const spo_mlp_desc d = MLPParams::desc_of(dims);
    const size_t nbytes = spo_mlp_bwd_workspace_size(&d, max_batch);
    if (nbytes == 0) check(SPO_ERR_SHAPE);
    ws = ctx.enqueue_create_buffer<unsigned char>(nbytes);
  }
  int64_t max_batch() const { return max_batch_; }

  Buffer dvalue;                   // dL/d(out) [max_batch x dL]
  DeviceBuffer<unsigned char> ws;  // spo_mlp_bwd's workspace

 private:
  int64_t max_batch_;
};

// All gradients from scratch.dvalue (networks/mlp.mojo:236-275). The cache must come from
// a forward with the same x and params (:218-221).
inline void backward_from_dvalue(DeviceContext& ctx, const MLPParams& params, const CriticCache& cache,
                                 CriticGrads& grads, CriticScratch& scratch, const Buffer& x, int64_t m) {
  cache.check(m);
  check_batch(scratch.max_batch(), m, "scratch", "rows");
  require(x, m * params.in_dim(), "backward_from_dvalue: x");
  const spo_mlp_desc d = params.desc();
  check(spo_mlp_bwd(ctx.handle(), &d, params.flat().unsafe_ptr(), x.unsafe_ptr(), cache.acts.unsafe_ptr(),
                    scratch.dvalue.unsafe_ptr(), m, grads.flat().unsafe_ptr(), scratch.ws.unsafe_ptr(),
                    scratch.ws.size()));
}

// Gradients of L = mean 0.5 (V - target)^2 (networks/mlp.mojo:212-233).
inline void critic_backward(DeviceContext& ctx, const MLPParams& params, const CriticCache& cache, CriticGrads& grads,
                            CriticScratch& scratch, const Buffer& x, const Buffer& target, int64_t m) {
  const int64_t n_out = m * params.out_dim();
  cache.check(m);
  require(target, n_out, "critic_backward: target");
  check(spo_value_loss_grad(ctx.handle(), scratch.dvalue.unsafe_ptr(), cache.value.unsafe_ptr(), target.unsafe_ptr(),
                            n_out, n_out > 0 ? 1.0f / static_cast<float>(n_out) : 0.0f));
  backward_from_dvalue(ctx, params, cache, grads, scratch, x, m);
}

// ------------------------------------------------------------------ softmax (ops/softmax.mojo:58-135)

inline void softmax_rows(DeviceContext& ctx, Buffer& out, const Buffer& a, int64_t rows, int row_size) {
  require(out, rows * row_size, "softmax_rows: out");
  require(a, rows * row_size, "softmax_rows: a");
  check(spo_softmax_rows(ctx.handle(), out.unsafe_ptr(), a.unsafe_ptr(), rows, row_size));
}
inline void log_softmax_rows(DeviceContext& ctx, Buffer& out, const Buffer& a, int64_t rows, int row_size) {
  require(out, rows * row_size, "log_softmax_rows: out");
  require(a, rows * row_size, "log_softmax_rows: a");
  check(spo_log_softmax_rows(ctx.handle(), out.unsafe_ptr(), a.unsafe_ptr(), rows, row_size));
}
inline void logsumexp_rows(DeviceContext& ctx, Buffer& out, const Buffer& a, int64_t rows, int row_size) {
  require(out, rows, "logsumexp_rows: out");
  require(a, rows * row_size, "logsumexp_rows: a");
  check(spo_logsumexp_rows(ctx.handle(), out.unsafe_ptr(), a.unsafe_ptr(), rows, row_size));
}

// ------------------------------------------------------------------ actor (networks/actor.mojo)

// Masked logits into cache.value (networks/actor.mojo:74-87).
inline void actor_logits(DeviceContext& ctx, const MLPParams& params, CriticCache& cache, const Buffer& obs,
                         const Buffer& mask, int64_t m) {
  require(mask, m * params.out_dim(), "actor_logits: mask");
  critic_forward(ctx, params, cache, obs, m);
  check(spo_mask_logits(ctx.handle(), cache.value.unsafe_ptr(), mask.unsafe_ptr(), m * params.out_dim()));
}
// pi(a|s) (networks/actor.mojo:90-103)
inline void actor_probs(DeviceContext& ctx, const MLPParams& params, CriticCache& cache, const Buffer& obs,
                        const Buffer& mask, Buffer& probs_out, int64_t m) {
  require(probs_out, m * params.out_dim(), "actor_probs: probs_out");
  actor_logits(ctx, params, cache, obs, mask, m);
  check(spo_softmax_rows(ctx.handle(), probs_out.unsafe_ptr(), cache.value.unsafe_ptr(), m, params.out_dim()));
}
// log pi(a|s), computed directly (networks/actor.mojo:106-122)
inline void actor_log_probs(DeviceContext& ctx, const MLPParams& params, CriticCache& cache, const Buffer& obs,
                            const Buffer& mask, Buffer& log_probs_out, int64_t m) {
  require(log_probs_out, m * params.out_dim(), "actor_log_probs: log_probs_out");
  actor_logits(ctx, params, cache, obs, mask, m);
  check(spo_log_softmax_rows(ctx.handle(), log_probs_out.unsafe_ptr(), cache.value.unsafe_ptr(), m,
                             params.out_dim()));
}

// The actor with its buffers for up to max_batch boards (networks/actor.mojo:125-194).
// `state` is the boards [m x 9], +1 agent / -1 rival / 0 empty; `obs` their encoding
// [m x in_dim] (the environment computes it, as in the reference).
class Actor {
 public:
  Actor(DeviceContext& ctx, int64_t max_batch, int hidden, int in_dim = OBS_DIM, int depth = 2)
      : params(zero_actor_params(ctx, hidden, in_dim, depth)),
        cache(ctx, max_batch, params.dims()),
        mask(zero_buffer(ctx, static_cast<size_t>(max_batch * NUM_ACTIONS))),
        probs(zero_buffer(ctx, static_cast<size_t>(max_batch * NUM_ACTIONS))),
        log_probs(zero_buffer(ctx, static_cast<size_t>(max_batch * NUM_ACTIONS))),
        hidden(hidden),
        max_batch(max_batch),
        obs_scratch_(zero_buffer(ctx, static_cast<size_t>(max_batch * OBS_DIM))) {}

  // A loud error instead of an out-of-range write (networks/actor.mojo:156-165).
  void _check(int64_t m) const { check_batch(max_batch, m, "actor", "boards"); }

  // The legal mask from the boards: the empty cells (networks/actor.mojo:167-174).
  void mask_from_state(DeviceContext& ctx, const Buffer& state, int64_t m) {
    _check(m);
    require(state, m * NUM_ACTIONS, "mask_from_state: state");
    check(spo_encode_obs(ctx.handle(), obs_scratch_.unsafe_ptr(), mask.unsafe_ptr(), state.unsafe_ptr(), m));
  }
  // Board -> policy: mask, MLP, masking and softmax (networks/actor.mojo:176-186).
  void forward(DeviceContext& ctx, const Buffer& state, const Buffer& obs, int64_t m) {
    _check(m);
    mask_from_state(ctx, state, m);
    actor_probs(ctx, params, cache, obs, mask, probs, m);
  }
  // Board -> log pi (networks/actor.mojo:188-194).
  void forward_log(DeviceContext& ctx, const Buffer& state, const Buffer& obs, int64_t m) {
    _check(m);
    mask_from_state(ctx, state, m);
    actor_log_probs(ctx, params, cache, obs, mask, log_probs, m);
  }

  ActorParams params;
  ActorCache cache;
  Buffer mask;       // [max_batch x 9] 1 legal, 0 occupied
  Buffer probs;      // [max_batch x 9] pi after the masked softmax
  Buffer log_probs;  // [max_batch x 9] log pi
  int hidden;
  int64_t max_batch;

 private:
  Buffer obs_scratch_;  // the encoding spo_encode_obs writes beside the mask
};

// ------------------------------------------------------------------ loss (networks/actor_loss.mojo)

// -sum_{q > 0} q log pi per row (networks/actor_loss.mojo:68-79)
inline void cross_entropy_rows(DeviceContext& ctx, Buffer& loss_out, const Buffer& q, const Buffer& log_pi,
                               int64_t n_rows, int num_actions) {
  require(loss_out, n_rows, "cross_entropy_rows: loss_out");
  require(q, n_rows * num_actions, "cross_entropy_rows: q");
  require(log_pi, n_rows * num_actions, "cross_entropy_rows: log_pi");
  check(spo_cross_entropy_rows(ctx.handle(), loss_out.unsafe_ptr(), q.unsafe_ptr(), log_pi.unsafe_ptr(), n_rows,
                               num_actions));
}
// H(q) per row (networks/actor_loss.mojo:133-139)
inline void entropy_rows(DeviceContext& ctx, Buffer& h_out, const Buffer& q, int64_t n_rows, int num_actions) {
  require(h_out, n_rows, "entropy_rows: h_out");
  require(q, n_rows * num_actions, "entropy_rows: q");
  check(spo_entropy_rows(ctx.handle(), h_out.unsafe_ptr(), q.unsafe_ptr(), n_rows, num_actions));
}
// KL(q || pi) = CE - H per row (networks/actor_loss.mojo:142-148)
inline void kl_rows(DeviceContext& ctx, Buffer& kl_out, const Buffer& cross_entropy, const Buffer& entropy,
                    int64_t n_rows) {
  require(kl_out, n_rows, "kl_rows: kl_out");
  require(cross_entropy, n_rows, "kl_rows: cross_entropy");
  require(entropy, n_rows, "kl_rows: entropy");
  check(spo_kl_rows(ctx.handle(), kl_out.unsafe_ptr(), cross_entropy.unsafe_ptr(), entropy.unsafe_ptr(), n_rows));
}

// Gradients of the equation-11 loss: dz = (pi - q) / m, 0 on illegal cells, then the
// MLP backward (networks/actor_loss.mojo:194-214).
inline void actor_backward(DeviceContext& ctx, const MLPParams& params, const CriticCache& cache, CriticGrads& grads,
                           CriticScratch& scratch, const Buffer& x, const Buffer& pi, const Buffer& q,
                           const Buffer& mask, int64_t m) {
  const int64_t n_out = m * params.out_dim();
  cache.check(m);
  require(pi, n_out, "actor_backward: pi");
  require(q, n_out, "actor_backward: q");
  require(mask, n_out, "actor_backward: mask");
  check(spo_logits_grad(ctx.handle(), scratch.dvalue.unsafe_ptr(), pi.unsafe_ptr(), q.unsafe_ptr(),
                        mask.unsafe_ptr(), n_out, m > 0 ? 1.0f / static_cast<float>(m) : 0.0f));
  backward_from_dvalue(ctx, params, cache, grads, scratch, x, m);
}

// ------------------------------------------------------------------ optimiser (networks/optim.mojo)

// The two moments of one tensor or one flat buffer, starting at zero (:102-112).
class AdamState {
 public:
  AdamState(DeviceContext& ctx, int64_t size)
      : m(zero_buffer(ctx, static_cast<size_t>(size))), v(zero_buffer(ctx, static_cast<size_t>(size))), size(size) {}
  Buffer m;
  Buffer v;
  int64_t size;
};

// sum x^2, returned to the host like the reference (:115-130); synchronises ctx's stream.
inline float sum_squares(DeviceContext& ctx, const Buffer& x, int64_t n) {
  require(x, n, "sum_squares: x");
  Buffer out = zero_buffer(ctx, 1);
  auto& ws = ctx.workspace(spo_sum_squares_workspace_size());
  check(spo_sum_squares(ctx.handle(), x.unsafe_ptr(), n, out.unsafe_ptr(), ws.unsafe_ptr(), ws.size()));
  float host = 0.f;
  ctx.enqueue_copy_to_host(&host, out, 1);
  ctx.synchronize();
  return host;
}

// min(1, max_norm / ||g||) (:133-142)
inline float global_clip_scale(float total_sq, float max_norm) { return spo_global_clip_scale(total_sq, max_norm); }

// One Adam step over n elements, `step` from 1 (:172-187).
inline void adam_step(DeviceContext& ctx, Buffer& param, const Buffer& grad, AdamState& state, int64_t n, float lr,
                      float grad_scale, int step, float eps = ADAM_EPS, float b1 = BETA1, float b2 = BETA2) {
  require(param, n, "adam_step: param");
  require(grad, n, "adam_step: grad");
  require(state.m, n, "adam_step: state.m");
  require(state.v, n, "adam_step: state.v");
  check(spo_adam_flat(ctx.handle(), param.unsafe_ptr(), grad.unsafe_ptr(), state.m.unsafe_ptr(), state.v.unsafe_ptr(),
                      n, lr, b1, b2, eps, step, grad_scale));
}

// target <- tau * online + (1 - tau) * target (:163-169)
inline void ema_update(DeviceContext& ctx, Buffer& target, const Buffer& online, int64_t n, float tau) {
  require(target, n, "ema_update: target");
  require(online, n, "ema_update: online");
  check(spo_ema(ctx.handle(), target.unsafe_ptr(), online.unsafe_ptr(), n, tau));
}

// rl_utils/multistep.mojo:72-82, batch-major [batch x t_len]
inline void truncated_gae(DeviceContext& ctx, Buffer& adv, Buffer& targets, const Buffer& reward,
                          const Buffer& discount, const Buffer& v_tm1, const Buffer& v_t, const Buffer& truncation,
                          int64_t batch, int t_len, float lambda) {
  const int64_t n = batch * t_len;
  require(adv, n, "truncated_gae: adv");
  require(targets, n, "truncated_gae: targets");
  require(reward, n, "truncated_gae: reward");
  require(discount, n, "truncated_gae: discount");
  require(v_tm1, n, "truncated_gae: v_tm1");
  require(v_t, n, "truncated_gae: v_t");
  require(truncation, n, "truncated_gae: truncation");
  check(spo_truncated_gae(ctx.handle(), adv.unsafe_ptr(), targets.unsafe_ptr(), reward.unsafe_ptr(),
                          discount.unsafe_ptr(), v_tm1.unsafe_ptr(), v_t.unsafe_ptr(), truncation.unsafe_ptr(),
                          batch, t_len, lambda));
}

// ------------------------------------------------------------------ search heads (envs/)

// The weight-sync shape test of the search models (envs/tictactoe_actor.mojo:108-140,
// envs/tictactoe_critic.mojo:145-155): a network is copied only into one of the same
// shape; here every width must match (the reference compares input, hidden and output).
inline void check_sync_shape(const std::vector<int>& src, const std::vector<int>& want, const char* what) {
  if (src != want) {
    std::string dims;
    for (size_t i = 0; i < src.size(); ++i) dims += (i ? "x" : "") + std::to_string(src[i]);
    throw Error(SPO_ERR_SHAPE, std::string("the ") + what + " does not have the model's shape: " + dims);
  }
}

inline void copy_params(DeviceContext& ctx, MLPParams& dst, const MLPParams& src) {
  check_cuda(cudaMemcpyAsync(dst.flat().unsafe_ptr(), src.flat().unsafe_ptr(), sizeof(float) * dst.size(),
                             cudaMemcpyDeviceToDevice, ctx.stream()),
             "cudaMemcpyAsync");
}

// The network part of the search's actor model (envs/tictactoe_actor.mojo:64-191): frozen
// copies of the trained actor and critic, refreshed from the learner with sync_from /
// sync_critic_from, and their batched forward over m boards (m = envs x particles in the
// search). The environment's dynamics and the bootstrap around them are not part of this
// library.
class TicTacToeActorHead {
 public:
  TicTacToeActorHead(DeviceContext& ctx, int64_t max_batch, int hidden, int depth = 2)
      : params(zero_actor_params(ctx, hidden, OBS_DIM, depth)),
        cache(ctx, max_batch, params.dims()),
        obs(zero_buffer(ctx, static_cast<size_t>(max_batch * OBS_DIM))),
        mask(zero_buffer(ctx, static_cast<size_t>(max_batch * NUM_ACTIONS))),
        critic(zero_critic_params(ctx, OBS_DIM, hidden, 1, depth)),
        ccache(ctx, max_batch, critic.dims()),
        hidden(hidden),
        max_batch(max_batch) {}

  // the trained actor's weights into the model's (:121-140)
  void sync_from(DeviceContext& ctx, const MLPParams& src) {
    check_sync_shape(src.dims(), params.dims(), "actor being copied");
    copy_params(ctx, params, src);
  }
  // the trained critic's weights into the model's (:108-119)
  void sync_critic_from(DeviceContext& ctx, const MLPParams& src) {
    check_sync_shape(src.dims(), critic.dims(), "critic");
    copy_params(ctx, critic, src);
  }
  // Masked logits over m boards into out_logits; the mask and the observation come from
  // the boards (state [m x 9], +1 agent / -1 rival / 0 empty) (:148-171).
  void _prior(DeviceContext& ctx, const Buffer& state, Buffer& out_logits, int64_t m) {
    check_batch(max_batch, m, "model", "boards");
    require(state, m * NUM_ACTIONS, "_prior: state");
    require(out_logits, m * NUM_ACTIONS, "_prior: out_logits");
    check(spo_encode_obs(ctx.handle(), obs.unsafe_ptr(), mask.unsafe_ptr(), state.unsafe_ptr(), m));
    actor_logits(ctx, params, cache, obs, mask, m);
    check_cuda(cudaMemcpyAsync(out_logits.unsafe_ptr(), cache.value.unsafe_ptr(), sizeof(float) * m * NUM_ACTIONS,
                               cudaMemcpyDeviceToDevice, ctx.stream()),
               "cudaMemcpyAsync");
  }
  // The prior, then V from the critic on the observation _prior encoded (eval_root,
  // :173-191).
  void eval_root(DeviceContext& ctx, const Buffer& state, Buffer& logits_out, Buffer& value_out, int64_t m) {
    require(value_out, m, "eval_root: value_out");
    _prior(ctx, state, logits_out, m);
    critic_forward(ctx, critic, ccache, obs, m);
    check_cuda(cudaMemcpyAsync(value_out.unsafe_ptr(), ccache.value.unsafe_ptr(), sizeof(float) * m,
                               cudaMemcpyDeviceToDevice, ctx.stream()),
               "cudaMemcpyAsync");
  }

  ActorParams params;
  ActorCache cache;
  Buffer obs;   // [max_batch x 27] encoding of the last boards
  Buffer mask;  // [max_batch x 9] their legal cells
  CriticParams critic;
  CriticCache ccache;
  int hidden;
  int64_t max_batch;
};

// The network part of the search's critic model (envs/tictactoe_critic.mojo:98-192).
class TicTacToeCriticHead {
 public:
  TicTacToeCriticHead(DeviceContext& ctx, int64_t max_batch, int hidden, int depth = 2)
      : params(zero_critic_params(ctx, OBS_DIM, hidden, 1, depth)),
        cache(ctx, max_batch, params.dims()),
        obs(zero_buffer(ctx, static_cast<size_t>(max_batch * OBS_DIM))),
        hidden(hidden),
        max_batch(max_batch) {}

  // :145-162
  void sync_from(DeviceContext& ctx, const MLPParams& src) {
    check_sync_shape(src.dims(), params.dims(), "critic being copied");
    copy_params(ctx, params, src);
  }
  // V over m boards (the network half of eval_root, :170-192)
  void value(DeviceContext& ctx, const Buffer& state, Buffer& value_out, int64_t m) {
    check_batch(max_batch, m, "model", "boards");
    require(state, m * NUM_ACTIONS, "value: state");
    require(value_out, m, "value: value_out");
    check(spo_encode_obs(ctx.handle(), obs.unsafe_ptr(), nullptr, state.unsafe_ptr(), m));
    critic_forward(ctx, params, cache, obs, m);
    check_cuda(cudaMemcpyAsync(value_out.unsafe_ptr(), cache.value.unsafe_ptr(), sizeof(float) * m,
                               cudaMemcpyDeviceToDevice, ctx.stream()),
               "cudaMemcpyAsync");
  }

  CriticParams params;
  CriticCache cache;
  Buffer obs;
  int hidden;
  int64_t max_batch;
};

}  // namespace networks
}  // namespace spo

#endif  // SPO_NETWORKS_HPP_
