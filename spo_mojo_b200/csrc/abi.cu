// C-ABI entry points of libspo_cuda (declared in include/spo_cuda.h) and the
// learner-step plan that sequences the fused kernels.
//
// Learner step for one network with L Linear layers (dims d0..dL), rows B:
//   forward   a_l = relu(a_{l-1} W_l + b_l), l = 0..L-2          gemm_simt (EPI_BIAS_RELU)
//   head      last layer + loss + dz + dW_{L-1}, db_{L-1},
//             dZ_{L-2} = (dz W^T) * [a_{L-2} > 0] and its column sums      head_kernel
//   backward  for l = L-2..0:
//               dW_l = in_l^T dZ_l (split over rows, partial tiles)       gemm_simt (OP_COL x OP_ROW)
//               dZ_{l-1} = (dZ_l W_l^T) * [a_{l-1} > 0] + column sums     gemm_simt (EPI_RELU_MASK)
//   reduce    all per-CTA partials -> flat gradient buffer (fixed order)  reduce_kernel
// then (spo_learner_apply) optional grouped sum of squares and one flat Adam.
#include <algorithm>
#include <chrono>
#include <cmath>
#include <cstdlib>
#include <cstring>
#include <mutex>
#include <string>
#include <thread>
#include <vector>

#include <nccl.h>

#include "spo_cuda.h"
#include "gemm_simt.cuh"
#include "kernels.cuh"
#include "tc_gemm.cuh"
#include "small_step.cuh"

namespace spo {

namespace {
thread_local std::string g_last_error;
}

int set_error(int code, const std::string& msg) {
  g_last_error = msg;
  return code;
}

void clear_error() { g_last_error.clear(); }

bool pdl_enabled() {
  static const bool on = [] {
    const char* e = std::getenv("SPO_PDL");
    return !(e && e[0] == '0');
  }();
  return on;
}

int sm_count() {
  static int cached[64] = {0};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return 148;
  if (cached[dev] == 0) {
    int n = 0;
    if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n <= 0)
      n = 148;
    cached[dev] = n;
  }
  return cached[dev];
}

namespace {

constexpr int64_t kAlignFloats = SPO_ALIGN_FLOATS;
inline int64_t align_up(int64_t n, int64_t a) { return (n + a - 1) / a * a; }

// Bump allocator over a caller-provided workspace (or a size probe when base == null).
struct Carve {
  char* base;
  size_t off = 0;
  explicit Carve(void* b) : base(static_cast<char*>(b)) {}
  template <class T>
  T* take(size_t count) {
    off = (off + 255) & ~size_t(255);
    T* p = base ? reinterpret_cast<T*>(base + off) : nullptr;
    off += count * sizeof(T);
    return p;
  }
};

bool desc_ok(const spo_mlp_desc* d) {
  if (!d || d->num_layers < 1 || d->num_layers > SPO_MAX_LAYERS) return false;
  for (int i = 0; i <= d->num_layers; ++i)
    if (d->dims[i] < 1 || d->dims[i] > (1 << 16)) return false;
  return true;
}

void mlp_layout(const spo_mlp_desc& d, int64_t* w_off, int64_t* b_off, int64_t* total) {
  int64_t off = 0;
  for (int l = 0; l < d.num_layers; ++l) {
    w_off[l] = off;
    off = align_up(off + (int64_t)d.dims[l] * d.dims[l + 1], kAlignFloats);
    b_off[l] = off;
    off = align_up(off + d.dims[l + 1], kAlignFloats);
  }
  *total = off;
}

int target_ctas() { return 2 * sm_count(); }

// ---------------------------------------------------------------- GEMM launch plans
struct FwdCfg {
  int tile;
  dim3 grid;
};

FwdCfg fwd_cfg(int64_t rows, int64_t n) {
  FwdCfg c;
  c.tile = gemm_pick_tile(rows, n);
  const GemmShape s = gemm_shape(c.tile);
  const int64_t nt = ceil_div(n, s.bn), mt = ceil_div(rows, s.bm);
  const int64_t mg = std::max<int64_t>(1, std::min<int64_t>(mt, ceil_div(target_ctas(), nt)));
  c.grid = dim3((unsigned)nt, (unsigned)(rows > 0 ? mg : 0), 1);
  return c;
}

int64_t fwd_parts_bound(int64_t n) {
  // m_groups <= ceil(target / n_tiles) for either tile shape
  return std::max<int64_t>(1, ceil_div(target_ctas(), ceil_div(n, 128)));
}

struct DwCfg {
  int tile;
  dim3 grid;
  int64_t k_chunk;
  int parts;
};

DwCfg dw_cfg(int64_t k_in, int64_t n_out, int64_t rows) {
  DwCfg c;
  c.tile = gemm_pick_tile(k_in, n_out);
  const GemmShape s = gemm_shape(c.tile);
  const int64_t tiles = ceil_div(k_in, s.bm) * ceil_div(n_out, s.bn);
  int64_t S = std::min<int64_t>(ceil_div(target_ctas(), tiles), std::max<int64_t>(1, rows / 256));
  S = std::max<int64_t>(S, 1);
  c.k_chunk = std::max<int64_t>(16, align_up(ceil_div(std::max<int64_t>(rows, 1), S), 16));
  c.parts = rows > 0 ? (int)ceil_div(rows, c.k_chunk) : 0;
  c.grid = dim3((unsigned)ceil_div(n_out, s.bn), (unsigned)ceil_div(k_in, s.bm), (unsigned)c.parts);
  return c;
}

int64_t dw_parts_bound(int64_t k_in, int64_t n_out) {
  // parts <= ceil(target / tiles) with the smaller tile count of the two shapes
  const int64_t tiles = ceil_div(k_in, 128) * ceil_div(n_out, 128);
  const int64_t simt = std::max<int64_t>(1, ceil_div(target_ctas(), tiles));
  return dw_skinny_ok(k_in, n_out) ? std::max(simt, dw_skinny_max_parts()) : simt;
}

int gemm_fwd(cudaStream_t s, float* y, const float* x, const float* w, const float* b,
             int64_t rows, int64_t k, int64_t n, bool relu) {
  if (rows == 0) return kOk;
  FwdCfg c = fwd_cfg(rows, n);
  GemmParams p{};
  p.A = x; p.B = w; p.C = y; p.bias = b;
  p.M = rows; p.N = n; p.K = k;
  p.lda = k; p.ldb = n; p.ldc = n;
  p.k_chunk = align_up(std::max<int64_t>(k, 1), 16);
  return gemm_simt_launch(c.tile, OP_ROW, OP_ROW, relu ? EPI_BIAS_RELU : EPI_BIAS, p, c.grid, s);
}

// dX = (dY W^T) [* mask > 0]; dY [rows x n], W [k x n], dX [rows x k]. Column sums of dX
// to colsum[parts][k] when colsum != null; returns the number of parts in *parts.
int gemm_dx(cudaStream_t s, float* dx, const float* dy, const float* w, const float* mask,
            int64_t rows, int64_t k, int64_t n, float* colsum, int* parts) {
  FwdCfg c = fwd_cfg(rows, k);
  if (parts) *parts = (int)c.grid.y;
  if (rows == 0) return kOk;
  GemmParams p{};
  p.A = dy; p.B = w; p.C = dx; p.mask = mask; p.colsum = colsum;
  p.M = rows; p.N = k; p.K = n;
  p.lda = n; p.ldb = n; p.ldc = k; p.ldm = k;
  p.k_chunk = align_up(n, 16);
  return gemm_simt_launch(c.tile, OP_ROW, OP_COL, mask ? EPI_RELU_MASK : EPI_STORE, p, c.grid, s);
}

// dW partials: part[z][k x n] = sum over rows of chunk z of x^T dY.
int gemm_dw(cudaStream_t s, float* part, const float* x, const float* dy, int64_t rows,
            int64_t k, int64_t n, int* parts) {
  if (dw_skinny_ok(k, n) && aligned16(dy) && aligned16(part))
    return dw_skinny_launch(LayerInput{x, nullptr}, dy, rows, k, n, part, parts, s);
  DwCfg c = dw_cfg(k, n, rows);
  if (parts) *parts = c.parts;
  if (c.parts == 0) return kOk;
  GemmParams p{};
  p.A = x; p.B = dy; p.C = part;
  p.M = k; p.N = n; p.K = rows;
  p.lda = k; p.ldb = n; p.ldc = n;
  p.k_chunk = c.k_chunk;
  p.c_split_stride = k * n;
  return gemm_simt_launch(c.tile, OP_COL, OP_ROW, EPI_STORE, p, c.grid, s);
}

// Column sums of a [rows x n] matrix: per-chunk partials, then one reduction.
constexpr int64_t kColsumChunks = 256;

int colsum(cudaStream_t s, float* out, const float* x, int64_t rows, int64_t n, float* scratch) {
  const int64_t chunks = std::max<int64_t>(1, std::min<int64_t>(kColsumChunks, ceil_div(rows, 256)));
  int rc = colsum_part_launch(x, rows, n, chunks, scratch, s);
  if (rc) return rc;
  ReduceParams q{};
  ReduceSeg& sg = q.seg[q.nseg++];
  sg.src = scratch;
  sg.dst = out;
  sg.count = n;
  sg.part_stride = n;
  sg.parts = (int32_t)chunks;
  return reduce_launch(q, s);
}

void add_seg(ReduceParams& p, const float* src, float* dst, int64_t count, int64_t stride, int parts) {
  ReduceSeg& sg = p.seg[p.nseg++];
  sg.src = src;
  sg.dst = dst;
  sg.count = count;
  sg.part_stride = stride;
  sg.parts = parts;
}

// Zero the alignment gaps of a flat MLP buffer (so Adam sees zero gradients there).
void add_gap_segs(ReduceParams& p, const spo_mlp_desc& d, const int64_t* w_off, const int64_t* b_off,
                  int64_t total, float* grads) {
  for (int l = 0; l < d.num_layers; ++l) {
    const int64_t wend = w_off[l] + (int64_t)d.dims[l] * d.dims[l + 1];
    if (b_off[l] > wend) add_seg(p, nullptr, grads + wend, b_off[l] - wend, 0, 0);
    const int64_t bend = b_off[l] + d.dims[l + 1];
    const int64_t next = (l + 1 < d.num_layers) ? w_off[l + 1] : total;
    if (next > bend) add_seg(p, nullptr, grads + bend, next - bend, 0, 0);
  }
}

}  // namespace

// ====================================================================== learner plan
struct NetPlan {
  bool present = false;
  spo_mlp_desc d{};
  int64_t w_off[SPO_MAX_LAYERS], b_off[SPO_MAX_LAYERS], size = 0, offset = 0;
  int64_t max_hidden = 0;
  // Tensor-core mode: hidden x hidden products on tcgen05 (3xTF32). Activations and the
  // gradients between hidden layers are then stored as TF32 hi/lo pairs (acts/acts_lo,
  // dz/dz_lo); dz0 is the plain fp32 gradient of layer 0's output (its dW stays on the
  // CUDA cores: the 27-wide input has no 16-byte-aligned rows for TMA).
  bool tc = false;
  // workspace carve-outs
  float* acts[SPO_MAX_LAYERS] = {};     // a_l, l = 0..L-2: [rows x d_{l+1}] (hi in TC mode)
  float* acts_lo[SPO_MAX_LAYERS] = {};  // TC mode, l <= L-3: lo halves (a_{L-2} is fp32)
  uint32_t* acts_bits[SPO_MAX_LAYERS] = {};  // TC mode, l <= L-3: a_l > 0 packed [rows x d_{l+1}/32]
  float* dz[2] = {};                    // ping-pong [rows x max_hidden] (hi in TC mode)
  float* dz_lo[2] = {};                 // TC mode
  float* dz0 = nullptr;                 // TC mode: [rows x d_1] fp32
  // TC mode with a first layer at most 32 wide and d_1 % 128 == 0: that layer's forward
  // runs on tensor cores too, from the input padded to 32 columns (hi/lo) and W_0^T padded
  bool tc0 = false;
  float* x0[2] = {};                    // [rows x 32] hi, lo
  float* w0t[2] = {};                   // [d_1 x 32] hi, lo
  float* wsplit[SPO_MAX_LAYERS][4] = {};  // TC mode, hidden l: W^T hi, W^T lo, W hi, W lo
  float* head_dw = nullptr;          // [Gh][d_{L-1} x d_L]
  float* head_db = nullptr;          // [Gh][d_L]
  float* head_dbx = nullptr;         // [Gh][d_{L-1}]
  float* head_stats = nullptr;       // [Gh][kStats]
  float* dw_part[SPO_MAX_LAYERS] = {};
  int64_t dw_part_cap[SPO_MAX_LAYERS] = {};  // partials dw_part[l] holds
  float* db_part[SPO_MAX_LAYERS] = {};  // column sums of dZ_{l} from layer l+1's dX GEMM
  // the one-launch small-batch step (small_step.cu): its partial sums
  bool small = false;                   // the network's shape fits the small step
  float* sm_pw[SPO_MAX_LAYERS] = {};   // [grid][d_l x d_{l+1}]
  float* sm_pb[SPO_MAX_LAYERS] = {};   // [grid][d_{l+1}]
  float* sm_pstats = nullptr;          // [grid][kStats]
  // the tensor maps of the hidden layers' W (encoded for the parameter buffer at sm_wmap_of)
  CUtensorMap sm_wmap[kSmallMaxLayers - 1] = {};
  const float* sm_wmap_of = nullptr;
};

}  // namespace spo

struct spo_learner {
  spo_learner_desc desc;
  spo_learner_layout layout;
  spo::NetPlan net[2];  // 0 actor, 1 critic
  float* sumsq_part = nullptr;
  unsigned* ticket = nullptr;
  int* err = nullptr;  // device error word of the tensor-core kernels' bounded waits
  size_t ws_bytes = 0;
  // one-launch step for batches of at most small_rows rows (0: never)
  int64_t small_rows = 0;
  int sm_grid = 0;
  float* sm_sumsq = nullptr;            // [kMaxGroups][sm_grid]
  CUtensorMap* sm_wmap = nullptr;       // [2][kSmallMaxLayers - 1]: the networks' weight maps
  unsigned* sm_sync = nullptr;          // barrier words, zero between launches
  bool last_small = false;              // the last forward ran in the small step
};

namespace spo {
namespace {

int64_t head_parts_bound() { return 2LL * sm_count(); }

// Tensor-core mode when every hidden width is a multiple of 128 (the tcgen05 tile) and at
// most 1024 (the fused head and the dX column sums), with at least one hidden x hidden
// layer to put on the tensor cores.
bool net_uses_tc(const spo_mlp_desc& d, int engine) {
  if (engine == 1 || d.num_layers < 3) return false;
  for (int l = 1; l < d.num_layers; ++l)
    if (d.dims[l] % 128 != 0 || d.dims[l] > 1024) return false;
  return true;
}

// Upper bound of the row splits of a tensor-core dW launch for `rows` rows.
// At least kDwMinKBlocks k-blocks (32 rows each) per unit of a split dW product. Large
// batches split far less than this allows (the rule below stops at the first S that fills
// the slots); it binds for batches of a few thousand to ~100 k rows, where a longer minimum
// left most CTA pairs idle while a few walked their rows serially (4,096 rows: 2 splits of
// 64 k-blocks, 46 us; with 8, 16 splits).
constexpr int64_t kDwMinKBlocks = 8;

int64_t tc_dw_splits_max(int64_t rows) {
  return std::max<int64_t>(1, std::min<int64_t>(ceil_div(rows, 32) / kDwMinKBlocks, 4LL * sm_count()));
}

// Row splits S of a tensor-core dW product whose unit grid has `tiles` output tiles per
// split and `slots` units running at once: at least kDwMinKBlocks k-blocks per unit, and
// the smallest S whose tiles*S units fill the slots in whole waves (>= 95% of the last
// wave busy), else the best such fill. S <= min(tc_dw_splits_max(rows), slots): S = slots
// always fills whole waves.
int64_t tc_dw_splits(int64_t tiles, int64_t slots, int64_t rows) {
  const int64_t smax = tc_dw_splits_max(rows);
  int64_t best = 1;
  double best_eff = -1.0;
  for (int64_t S = 1; S <= smax; ++S) {
    const int64_t units = tiles * S;
    const double eff = (double)units / (double)(ceil_div(units, slots) * slots);
    if (units >= slots && eff >= 0.95) return S;
    if (eff > best_eff + 1e-9) {
      best_eff = eff;
      best = S;
    }
  }
  return best;
}

void carve_net(NetPlan& n, Carve& c, int64_t rows) {
  const spo_mlp_desc& d = n.d;
  const int L = d.num_layers;
  for (int l = 0; l + 1 < L; ++l) {
    n.acts[l] = c.take<float>((size_t)rows * d.dims[l + 1]);
    // the last hidden activation is read only by the fused head: plain fp32
    if (n.tc && l + 2 < L) n.acts_lo[l] = c.take<float>((size_t)rows * d.dims[l + 1]);
    // packed for the dX GEMM of layer l + 1 (the last hidden layer's mask is read by the
    // head); layer 0's is written by the input-layer forward when its shape allows
    const bool packs = l >= 1 || (fwd_skinny_ok(d.dims[0], d.dims[1]) && d.dims[1] % 32 == 0);
    if (n.tc && packs && l + 2 < L) n.acts_bits[l] = c.take<uint32_t>((size_t)rows * (d.dims[l + 1] / 32));
  }
  for (int i = 0; i < 2; ++i) {
    n.dz[i] = c.take<float>((size_t)rows * n.max_hidden);
    if (n.tc) n.dz_lo[i] = c.take<float>((size_t)rows * n.max_hidden);
  }
  if (n.tc) {
    n.dz0 = c.take<float>((size_t)rows * d.dims[1]);
    if (n.tc0)
      for (int k = 0; k < 2; ++k) {
        n.x0[k] = c.take<float>((size_t)rows * 32);
        n.w0t[k] = c.take<float>((size_t)d.dims[1] * 32);
      }
    for (int l = 1; l + 1 < L; ++l)
      for (int k = 0; k < 4; ++k) n.wsplit[l][k] = c.take<float>((size_t)d.dims[l] * d.dims[l + 1]);
  }
  const int64_t gh = head_parts_bound();
  const int64_t hl = d.dims[L - 1], al = d.dims[L];
  n.head_dw = c.take<float>((size_t)(gh * hl * al));
  n.head_db = c.take<float>((size_t)(gh * al));
  n.head_dbx = c.take<float>((size_t)(gh * hl));
  n.head_stats = c.take<float>((size_t)(gh * kStats));
  for (int l = 0; l + 1 < L; ++l) {
    const int64_t parts = (n.tc && l >= 1) ? std::min<int64_t>(tc_dw_splits_max(rows),
                                                               tc_gemm_slots(TC_DW, d.dims[l + 1]))
                                           : dw_parts_bound(d.dims[l], d.dims[l + 1]);
    n.dw_part[l] = c.take<float>((size_t)(parts * d.dims[l] * d.dims[l + 1]));
    n.dw_part_cap[l] = parts;
  }
  for (int l = 0; l + 2 < L; ++l) {  // db of layer l comes from layer l+1's dX GEMM
    const int64_t parts = std::max<int64_t>(fwd_parts_bound(d.dims[l + 1]), n.tc ? sm_count() : 0);
    n.db_part[l] = c.take<float>((size_t)(parts * d.dims[l + 1]));
  }
}

int check_net_desc(const spo_mlp_desc& d, int out_dim, const char* which) {
  if (!desc_ok(&d))
    return set_error(kErrShape, std::string("learner: bad ") + which + " dimensions");
  if (d.num_layers < 2)
    return set_error(kErrUnsupported, std::string("learner: ") + which + " needs at least 2 layers");
  if (d.dims[d.num_layers] != out_dim)
    return set_error(kErrUnsupported, std::string("learner: ") + which + " output width must be " +
                                          std::to_string(out_dim));
  const int hl = d.dims[d.num_layers - 1];
  if (hl % 4 != 0 || hl > 1024)
    return set_error(kErrUnsupported, std::string("learner: ") + which +
                                          " last hidden width must be a multiple of 4, <= 1024");
  for (int l = 1; l < d.num_layers; ++l)
    if (d.dims[l] % 4 != 0)
      return set_error(kErrUnsupported, std::string("learner: ") + which +
                                            " hidden widths must be multiples of 4");
  return kOk;
}

// Shapes of the one-launch small-batch step: 2 to 4 Linear layers, input at most 32 wide,
// hidden widths multiples of 32 up to 256, output 9 (actor) or 1 (critic).
bool small_net_ok(const spo_mlp_desc& d) {
  if (d.num_layers < 2 || d.num_layers > kSmallMaxLayers || d.dims[0] > kSmallMaxIn) return false;
  int64_t params = 0;
  for (int l = 0; l < d.num_layers; ++l) params += (int64_t)d.dims[l] * d.dims[l + 1] + d.dims[l + 1];
  for (int l = 1; l < d.num_layers; ++l)
    if (d.dims[l] % 32 != 0 || d.dims[l] > kSmallMaxHidden) return false;
  const int a = d.dims[d.num_layers];
  return (a == 1 || a == kSmallMaxA) && params <= kSmallMaxParams && small_step_smem(&d, 1) <= kSmallMaxSmem;
}

int build_plan(const spo_learner_desc* desc, spo_learner* L, void* ws, size_t* bytes) {
  SPO_CHECK_ARG(desc != nullptr, kErrArg, "null descriptor");
  SPO_CHECK_ARG(desc->actor.num_layers > 0 || desc->critic.num_layers > 0, kErrArg,
                "learner needs an actor or a critic");
  SPO_CHECK_ARG(desc->max_rows >= 1, kErrShape, "max_rows must be >= 1");
  if (desc->actor.num_layers > 0) {
    int rc = check_net_desc(desc->actor, 9, "actor");
    if (rc) return rc;
  }
  if (desc->critic.num_layers > 0) {
    int rc = check_net_desc(desc->critic, 1, "critic");
    if (rc) return rc;
    if (desc->actor.num_layers > 0 && desc->actor.dims[0] != desc->critic.dims[0])
      return set_error(kErrShape, "learner: actor and critic must read the same observation width");
  }
  std::memset(&L->layout, 0, sizeof(L->layout));
  L->desc = *desc;
  int64_t off = 0;
  for (int i = 0; i < 2; ++i) {
    NetPlan& n = L->net[i];
    const spo_mlp_desc& d = i == 0 ? desc->actor : desc->critic;
    n = NetPlan{};
    n.present = d.num_layers > 0;
    if (!n.present) continue;
    n.d = d;
    mlp_layout(d, n.w_off, n.b_off, &n.size);
    n.offset = off;
    off += n.size;
    for (int l = 1; l < d.num_layers; ++l) n.max_hidden = std::max<int64_t>(n.max_hidden, d.dims[l]);
    n.tc = net_uses_tc(d, desc->engine);
    n.tc0 = n.tc && d.dims[0] <= 32 && d.dims[1] % 128 == 0;
  }
  spo_learner_layout& lay = L->layout;
  lay.actor_offset = L->net[0].offset;
  lay.actor_size = L->net[0].present ? L->net[0].size : 0;
  lay.critic_offset = L->net[1].offset;
  lay.critic_size = L->net[1].present ? L->net[1].size : 0;
  for (int l = 0; l < SPO_MAX_LAYERS; ++l) {
    lay.actor_w_off[l] = L->net[0].present && l < L->net[0].d.num_layers ? L->net[0].offset + L->net[0].w_off[l] : -1;
    lay.actor_b_off[l] = L->net[0].present && l < L->net[0].d.num_layers ? L->net[0].offset + L->net[0].b_off[l] : -1;
    lay.critic_w_off[l] = L->net[1].present && l < L->net[1].d.num_layers ? L->net[1].offset + L->net[1].w_off[l] : -1;
    lay.critic_b_off[l] = L->net[1].present && l < L->net[1].d.num_layers ? L->net[1].offset + L->net[1].b_off[l] : -1;
  }
  lay.alpha_index = off;
  off += kAlignFloats;
  lay.stats_offset = off;
  off += kAlignFloats;
  lay.total = off;

  Carve c(ws);
  for (int i = 0; i < 2; ++i)
    if (L->net[i].present) carve_net(L->net[i], c, desc->max_rows);
  L->sumsq_part = c.take<float>(kMaxGroups * kSumsqParts);
  L->ticket = c.take<unsigned>(4);
  L->err = c.take<int>(4);
  L->sm_sync = c.take<unsigned>(4);
  // The one-launch small-batch step: every present network must fit it.
  bool small = true;
  for (int i = 0; i < 2; ++i)
    if (L->net[i].present) small = small && (L->net[i].small = small_net_ok(L->net[i].d));
  L->small_rows = small ? std::min<int64_t>(kSmallDefaultRows, desc->max_rows) : 0;
  if (small) {
    const int G = sm_count();   // one CTA per SM
    L->sm_grid = G;
    for (int i = 0; i < 2; ++i) {
      NetPlan& n = L->net[i];
      if (!n.present) continue;
      for (int l = 0; l < n.d.num_layers; ++l) {
        n.sm_pw[l] = c.take<float>((size_t)G * n.d.dims[l] * n.d.dims[l + 1]);
        n.sm_pb[l] = c.take<float>((size_t)G * n.d.dims[l + 1]);
      }
      n.sm_pstats = c.take<float>((size_t)G * kStats);
    }
    L->sm_sumsq = c.take<float>((size_t)kMaxGroups * G);
    L->sm_wmap = c.take<CUtensorMap>(2 * (kSmallMaxLayers - 1));
  }
  *bytes = c.off + 256;
  return kOk;
}


// Layer 0 forward with the activation written as a TF32 hi/lo pair.
int gemm_fwd_split(cudaStream_t s, float* y_hi, float* y_lo, const float* x, const float* w,
                   const float* b, int64_t rows, int64_t k, int64_t n) {
  if (rows == 0) return kOk;
  FwdCfg c = fwd_cfg(rows, n);
  GemmParams p{};
  p.A = x; p.B = w; p.C = y_hi; p.C2 = y_lo; p.bias = b;
  p.M = rows; p.N = n; p.K = k;
  p.lda = k; p.ldb = n; p.ldc = n;
  p.k_chunk = align_up(std::max<int64_t>(k, 1), 16);
  return gemm_simt_launch(c.tile, OP_ROW, OP_ROW, EPI_BIAS_RELU_SPLIT, p, c.grid, s);
}

constexpr int64_t kTc0MinRows = 16384;

// Forward of layers 0..L-2 (ReLU) into the activation cache. In tensor-core mode the
// hidden weights are first split into TF32 hi/lo pairs (W^T for the forward, W for dX).
int net_forward_hidden(const NetPlan& n, cudaStream_t s, const float* params, LayerInput in,
                       int64_t rows, int* err) {
  const spo_mlp_desc& d = n.d;
  SPO_CHECK_ARG(!in.cells || fwd_skinny_ok(d.dims[0], d.dims[1]), kErrUnsupported,
                "board cells need a 27-wide input layer");
  if (!n.tc) {
    const float* h = in.x;
    for (int l = 0; l + 1 < d.num_layers; ++l) {
      const float* w = params + n.w_off[l];
      const float* b = params + n.b_off[l];
      int rc = l == 0 && fwd_skinny_ok(d.dims[0], d.dims[1])
                   ? fwd_skinny_launch(in, w, b, rows, d.dims[0], d.dims[1], n.acts[0], nullptr, nullptr, s)
                   : gemm_fwd(s, n.acts[l], h, w, b, rows, d.dims[l], d.dims[l + 1], true);
      if (rc) return rc;
      h = n.acts[l];
    }
    return kOk;
  }
  for (int l = 1; l + 1 < d.num_layers; ++l) {
    int rc = split_weights_launch(params + n.w_off[l], d.dims[l], d.dims[l + 1], n.wsplit[l][0],
                                  n.wsplit[l][1], n.wsplit[l][2], n.wsplit[l][3], s);
    if (rc) return rc;
  }
  int rc;
  // The input layer on tensor cores costs three launches (W_0^T and input splits, GEMM) of
  // mostly fixed latency; below kTc0MinRows rows the one-launch CUDA-core kernel, which
  // writes the same hi/lo pair and packed mask, is faster (256 rows, 27 -> 128: ~16 us of
  // launches -> ~6 us).
  if (n.tc0 && rows >= kTc0MinRows) {
    rc = split_weights_t_pad_launch(params + n.w_off[0], d.dims[0], d.dims[1], n.w0t[0], n.w0t[1], s);
    if (rc) return rc;
    rc = pad_split_input_launch(in, d.dims[0], rows, n.x0[0], n.x0[1], s);
    if (rc) return rc;
    if (rows > 0) {
      TcGemmArgs a{};
      a.kind = TC_FWD;
      a.a_hi = n.x0[0];
      a.a_lo = n.x0[1];
      a.b_hi = n.w0t[0];
      a.b_lo = n.w0t[1];
      a.M = rows;
      a.N = d.dims[1];
      a.K = 32;
      a.bias = params + n.b_off[0];
      a.c_hi = n.acts[0];
      a.c_lo = n.acts_lo[0];
      a.c_bits = n.acts_bits[0];
      a.err = err;
      rc = tc_gemm_launch(a, s);
    }
  } else {
    rc = fwd_skinny_ok(d.dims[0], d.dims[1])
             ? fwd_skinny_launch(in, params + n.w_off[0], params + n.b_off[0], rows, d.dims[0], d.dims[1],
                                 n.acts[0], n.acts_lo[0], n.acts_bits[0], s)
             : gemm_fwd_split(s, n.acts[0], n.acts_lo[0], in.x, params + n.w_off[0], params + n.b_off[0],
                              rows, d.dims[0], d.dims[1]);
  }
  if (rc) return rc;
  if (rows == 0) return kOk;
  for (int l = 1; l + 1 < d.num_layers; ++l) {
    TcGemmArgs a{};
    a.kind = TC_FWD;
    a.a_hi = n.acts[l - 1];
    a.a_lo = n.acts_lo[l - 1];
    a.b_hi = n.wsplit[l][0];
    a.b_lo = n.wsplit[l][1];
    a.M = rows;
    a.N = d.dims[l + 1];
    a.K = d.dims[l];
    a.bias = params + n.b_off[l];
    a.c_hi = n.acts[l];
    a.c_lo = n.acts_lo[l];
    a.c_bits = n.acts_bits[l];
    a.err = err;
    rc = tc_gemm_launch(a, s);
    if (rc) return rc;
  }
  return kOk;
}

// Backward of the hidden layers L-2..1 on the tensor cores (dW split over rows; dX with
// the ReLU mask and the bias-gradient column sums fused), then layer 0's dW on the CUDA
// cores from the fp32 dz0.
int net_backward_tc(const NetPlan& n, cudaStream_t s, const float* /*params: the hidden weights
                    come from their TF32 splits, made by the forward*/, LayerInput in,
                    int64_t rows, float* grads, ReduceParams& red, int* err) {
  const spo_mlp_desc& d = n.d;
  const int L = d.num_layers;
  int cur = 0;
  int rc;
  for (int l = L - 2; l >= 1; --l) {
    const int64_t kin = d.dims[l], nout = d.dims[l + 1];
    int parts = 0;
    if (rows > 0) {
      TcGemmArgs w{};
      w.kind = TC_DW;
      w.a_hi = n.acts[l - 1];
      w.a_lo = n.acts_lo[l - 1];
      w.b_hi = n.dz[cur];
      w.b_lo = n.dz_lo[cur];
      w.M = kin;
      w.N = nout;
      w.K = rows;
      const int64_t S = std::min(tc_dw_splits(tc_gemm_tiles(TC_DW, kin, nout), tc_gemm_slots(TC_DW, nout), rows),
                                 n.dw_part_cap[l]);
      w.k_chunk = align_up(ceil_div(ceil_div(rows, 32), S), 1) * 32;
      w.c_part = n.dw_part[l];
      w.err = err;
      parts = tc_gemm_splits(w);
      rc = tc_gemm_launch(w, s);
      if (rc) return rc;
    }
    add_seg(red, n.dw_part[l], grads + n.w_off[l], kin * nout, kin * nout, parts);

    int cparts = 0;
    if (rows > 0) {
      TcGemmArgs x{};
      const bool last = l == 1;
      x.kind = last ? TC_DX_F32 : TC_DX;
      x.a_hi = n.dz[cur];
      x.a_lo = n.dz_lo[cur];
      x.b_hi = n.wsplit[l][2];
      x.b_lo = n.wsplit[l][3];
      x.M = rows;
      x.N = kin;
      x.K = nout;
      x.mask = n.acts[l - 1];
      x.mask_bits = n.acts_bits[l - 1];  // packed by the forward of layer l - 1, when it was
      x.c_hi = last ? n.dz0 : n.dz[cur ^ 1];
      x.c_lo = last ? nullptr : n.dz_lo[cur ^ 1];
      x.colsum = n.db_part[l - 1];
      x.err = err;
      cparts = tc_gemm_grid(x);
      rc = tc_gemm_launch(x, s);
      if (rc) return rc;
    }
    add_seg(red, n.db_part[l - 1], grads + n.b_off[l - 1], kin, kin, cparts);
    cur ^= 1;
  }
  int parts = 0;
  rc = in.cells ? dw_skinny_launch(in, n.dz0, rows, d.dims[0], d.dims[1], n.dw_part[0], &parts, s)
                : gemm_dw(s, n.dw_part[0], in.x, n.dz0, rows, d.dims[0], d.dims[1], &parts);
  if (rc) return rc;
  add_seg(red, n.dw_part[0], grads + n.w_off[0], (int64_t)d.dims[0] * d.dims[1],
          (int64_t)d.dims[0] * d.dims[1], parts);
  return kOk;
}

// Forward, head and backward of one network; appends its reduction segments.
// params/grads point at the network's slice of the flat buffers.
int net_backward(const spo_learner* Lr, int which, cudaStream_t s, const float* params,
                 const float* log_alpha, const spo_batch& b, float scale, float* grads,
                 ReduceParams& red, const float** stats_src, int* stats_parts) {
  const NetPlan& n = Lr->net[which];
  const spo_mlp_desc& d = n.d;
  const int L = d.num_layers;
  const int64_t rows = b.rows;
  const LayerInput in{b.obs, b.obs ? nullptr : b.cells};
  int rc = net_forward_hidden(n, s, params, in, rows, Lr->err);
  if (rc) return rc;

  const int hl = d.dims[L - 1], al = d.dims[L];
  HeadParams hp{};
  hp.act = n.acts[L - 2];
  hp.act_lo = n.tc ? n.acts_lo[L - 2] : nullptr;
  hp.dX_lo = n.tc ? n.dz_lo[0] : nullptr;
  hp.W = params + n.w_off[L - 1];
  hp.b = params + n.b_off[L - 1];
  hp.M = rows;
  hp.H = hl;
  hp.A = al;
  hp.scale = scale;
  hp.dX = n.dz[0];
  hp.dW_part = n.head_dw;
  hp.db_part = n.head_db;
  hp.dbx_part = n.head_dbx;
  hp.stats_part = n.head_stats;
  if (which == 0) {
    hp.mode = kHeadActor;
    hp.mask = b.mask;
    hp.cells = b.mask ? nullptr : b.cells;
    hp.q = b.q;
    hp.z_old = Lr->desc.use_kl ? b.logits_old : nullptr;
    hp.log_alpha = Lr->desc.use_kl ? log_alpha : nullptr;
  } else {
    hp.mode = kHeadCritic;
    hp.target = b.target;
  }
  const int gh = head_grid(hp);
  if (rows > 0) {
    rc = head_launch(hp, gh, s);
    if (rc) return rc;
  }
  const int ghp = rows > 0 ? gh : 0;
  add_seg(red, n.head_dw, grads + n.w_off[L - 1], (int64_t)hl * al, (int64_t)hl * al, ghp);
  add_seg(red, n.head_db, grads + n.b_off[L - 1], al, al, ghp);
  add_seg(red, n.head_dbx, grads + n.b_off[L - 2], hl, hl, ghp);
  *stats_src = n.head_stats;
  *stats_parts = ghp;

  if (n.tc) {
    rc = net_backward_tc(n, s, params, in, rows, grads, red, Lr->err);
    if (rc) return rc;
    add_gap_segs(red, d, n.w_off, n.b_off, n.size, grads);
    return kOk;
  }
  int cur = 0;
  for (int l = L - 2; l >= 0; --l) {
    const float* x = l == 0 ? b.obs : n.acts[l - 1];
    int parts = 0;
    rc = l == 0 && in.cells
             ? dw_skinny_launch(in, n.dz[cur], rows, d.dims[0], d.dims[1], n.dw_part[0], &parts, s)
             : gemm_dw(s, n.dw_part[l], x, n.dz[cur], rows, d.dims[l], d.dims[l + 1], &parts);
    if (rc) return rc;
    add_seg(red, n.dw_part[l], grads + n.w_off[l], (int64_t)d.dims[l] * d.dims[l + 1],
            (int64_t)d.dims[l] * d.dims[l + 1], parts);
    if (l >= 1) {
      int cparts = 0;
      rc = gemm_dx(s, n.dz[cur ^ 1], n.dz[cur], params + n.w_off[l], n.acts[l - 1], rows, d.dims[l],
                   d.dims[l + 1], n.db_part[l - 1], &cparts);
      if (rc) return rc;
      add_seg(red, n.db_part[l - 1], grads + n.b_off[l - 1], d.dims[l], d.dims[l], rows > 0 ? cparts : 0);
      cur ^= 1;
    }
  }
  add_gap_segs(red, d, n.w_off, n.b_off, n.size, grads);
  return kOk;
}

// The loss statistics' segments of the reduction: the actor's slots and the critic's loss
// slot from their per-CTA partials, the dual-gradient slot zeroed (Adam sets it).
void add_stats_segs(ReduceParams& red, const spo_learner* Lr, float* grads, const float* const* src,
                    const int* parts) {
  const spo_learner_layout& lay = Lr->layout;
  float* stats = grads + lay.stats_offset;
  if (Lr->net[0].present && Lr->net[1].present) {
    add_seg(red, src[0], stats, kStatCriticLoss, kStats, parts[0]);
    add_seg(red, src[1] + kStatCriticLoss, stats + kStatCriticLoss, 1, kStats, parts[1]);
    add_seg(red, src[0] + kStatCriticLoss + 1, stats + kStatCriticLoss + 1,
            kStats - kStatCriticLoss - 1, kStats, parts[0]);
  } else {
    const int i = Lr->net[0].present ? 0 : 1;
    add_seg(red, src[i], stats, kStats, kStats, parts[i]);
  }
  add_seg(red, nullptr, grads + lay.alpha_index, kAlignFloats, 0, 0);  // dual gradient: set by Adam
}

// Adam over the learner's flat buffers: one group per network (its lr and clip) and, with
// the dual, the log_alpha slot. *clip: whether a global-norm clip applies.
int build_adam(const spo_learner* Lr, const spo_train_state* st, AdamParams& ap, bool* clip) {
  SPO_CHECK_ARG(st && st->params && st->grads && st->adam_m && st->adam_v && st->step, kErrArg,
                "null train state");
  const spo_learner_layout& lay = Lr->layout;
  const spo_learner_desc& d = Lr->desc;
  ap = AdamParams{};
  ap.p = st->params;
  ap.g = st->grads;
  ap.m = st->adam_m;
  ap.v = st->adam_v;
  ap.b1 = d.beta1;
  ap.b2 = d.beta2;
  ap.eps = d.adam_eps;
  ap.grad_scale = 1.f;
  ap.step = st->step;
  ap.ticket = Lr->ticket;
  ap.alpha_index = -1;
  ap.report = st->report;
  *clip = d.max_grad_norm > 0.f && std::isfinite(d.max_grad_norm);
  if (Lr->net[0].present)
    ap.grp[ap.ngrp++] = AdamGroup{lay.actor_offset, lay.actor_offset + lay.actor_size, d.lr_actor,
                                  *clip ? d.max_grad_norm : 0.f};
  else
    ap.grp[ap.ngrp++] = AdamGroup{0, 0, 0.f, 0.f};
  if (Lr->net[1].present)
    ap.grp[ap.ngrp++] = AdamGroup{lay.critic_offset, lay.critic_offset + lay.critic_size,
                                  d.lr_critic, *clip ? d.max_grad_norm : 0.f};
  else
    ap.grp[ap.ngrp++] = AdamGroup{0, 0, 0.f, 0.f};
  if (Lr->net[0].present && d.dual && d.use_kl) {
    ap.grp[ap.ngrp++] = AdamGroup{lay.alpha_index, lay.alpha_index + 4, d.lr_actor, 0.f};
    ap.alpha_index = lay.alpha_index;
    ap.kl_stat = st->grads + lay.stats_offset + kStatKLold;
    ap.kl_eps = d.kl_eps;
  }
  return kOk;
}

int learner_apply(spo_learner* Lr, cudaStream_t s, const spo_train_state* st) {
  AdamParams ap{};
  bool clip = false;
  int rc = build_adam(Lr, st, ap, &clip);
  if (rc) return rc;
  if (clip) {
    rc = sumsq_groups_launch(st->grads, ap.grp, 2, Lr->sumsq_part, s);
    if (rc) return rc;
    ap.sumsq_part = Lr->sumsq_part;
  }
  return adam_launch(ap, Lr->layout.total, s);
}

// The whole step of a small batch in one launch (small_step.cu); with apply, the clip and
// Adam too.
// wait_ns: the limit of every barrier wait; withhold: 1 + the CTA whose first barrier
// arrival is withheld (a test of the bounded waits), 0 in every other launch.
int small_step(spo_learner* Lr, cudaStream_t s, const spo_batch* b, float scale, const spo_train_state* st,
               bool apply, uint64_t wait_ns = 2000000000ull, uint32_t withhold = 0) {
  SmallStepParams p{};
  const spo_learner_layout& lay = Lr->layout;
  const int G = Lr->sm_grid;
  SPO_CHECK_ARG(G >= 1 && G <= small_step_grid(), kErrUnsupported, "small step: grid is not co-resident");
  // rows per CTA: a multiple of 4, enough CTAs to spread the rows over the SMs (measured at
  // 256 rows: 4 rows on 64 CTAs 33-34 us per step, 8 on 32 CTAs 38-39 us, 2 on 128 CTAs
  // 38 us: more partials to write and add)
  p.rows = b->rows;
  p.rows_per_cta = std::max<int64_t>(4, align_up(ceil_div(b->rows, G), 4));
  p.parts = (int)ceil_div(b->rows, p.rows_per_cta);
  const float* stats_src[2] = {nullptr, nullptr};
  int stats_parts[2] = {0, 0};
  bool upload = false;   // a network's weight maps were encoded anew
  for (int i = 0; i < 2; ++i) {
    NetPlan& n = Lr->net[i];
    SmallNet& sn = p.net[i];
    if (!n.present) continue;
    const spo_mlp_desc& d = n.d;
    const float* prm = st->params + n.offset;
    float* grads = st->grads + n.offset;
    sn.L = d.num_layers;
    sn.mode = i;
    for (int l = 0; l <= d.num_layers; ++l) sn.dims[l] = d.dims[l];
    for (int l = 0; l < d.num_layers; ++l) {
      sn.W[l] = prm + n.w_off[l];
      sn.b[l] = prm + n.b_off[l];
      sn.pw[l] = n.sm_pw[l];
      sn.pb[l] = n.sm_pb[l];
      add_seg(p.red, n.sm_pw[l], grads + n.w_off[l], (int64_t)d.dims[l] * d.dims[l + 1],
              (int64_t)d.dims[l] * d.dims[l + 1], p.parts);
      add_seg(p.red, n.sm_pb[l], grads + n.b_off[l], d.dims[l + 1], d.dims[l + 1], p.parts);
    }
    sn.pstats = n.sm_pstats;
    for (int l = 0; l + 1 < d.num_layers; ++l) sn.gact[l] = n.acts[l];   // the activation cache
    if (n.sm_wmap_of != prm) {   // a new parameter buffer: encode its hidden layers' maps
      for (int l = 0; l + 1 < d.num_layers; ++l) {
        int rc = small_weight_map(&n.sm_wmap[l], prm + n.w_off[l], l, d.dims[l], d.dims[l + 1]);
        if (rc) {
          n.sm_wmap_of = nullptr;
          return rc;
        }
      }
      n.sm_wmap_of = prm;
      upload = true;
    }
    add_gap_segs(p.red, d, n.w_off, n.b_off, n.size, grads);
    stats_src[i] = n.sm_pstats;
    stats_parts[i] = p.parts;
  }
  add_stats_segs(p.red, Lr, st->grads, stats_src, stats_parts);
  SPO_CHECK_ARG(p.red.nseg <= kMaxSegs, kErrUnsupported, "too many reduction segments");
  if (upload) {   // the maps into device memory, ahead of the launch on the same stream
    cudaStreamCaptureStatus cs = cudaStreamCaptureStatusNone;
    cudaStreamIsCapturing(s, &cs);
    if (cs != cudaStreamCaptureStatusNone) {
      for (int i = 0; i < 2; ++i) Lr->net[i].sm_wmap_of = nullptr;
      return set_error(kErrUnsupported, "small step: the first step on a parameter buffer must run outside "
                                        "stream capture (it uploads the weights' tensor maps)");
    }
    CUtensorMap maps[2][kSmallMaxLayers - 1] = {};
    for (int i = 0; i < 2; ++i)
      for (int l = 0; Lr->net[i].present && l + 1 < Lr->net[i].d.num_layers; ++l) maps[i][l] = Lr->net[i].sm_wmap[l];
    // pageable source: staged before the call returns, so the local array may go
    cudaError_t ce = cudaMemcpyAsync(Lr->sm_wmap, maps, sizeof(maps), cudaMemcpyHostToDevice, s);
    if (ce != cudaSuccess) {
      for (int i = 0; i < 2; ++i) Lr->net[i].sm_wmap_of = nullptr;
      return set_error(kErrCuda, std::string("small step: tensor maps: ") + cudaGetErrorString(ce));
    }
  }
  p.wmap = Lr->sm_wmap;
  int64_t e = 0;
  for (int k = 0; k < p.red.nseg; ++k) {
    p.seg_start[k] = e;
    p.flat_index[k] = p.red.seg[k].dst - st->grads;
    e += p.red.seg[k].count;
  }
  p.total_red = e;
  p.obs = b->obs;
  p.cells = b->obs ? nullptr : b->cells;
  p.mask = b->mask;
  p.q = b->q;
  p.z_old = Lr->desc.use_kl ? b->logits_old : nullptr;
  p.target = b->target;
  p.log_alpha = st->params + lay.alpha_index;
  p.scale = scale;
  p.apply = apply ? 1 : 0;
  if (apply) {
    bool clip = false;
    int rc = build_adam(Lr, st, p.adam, &clip);
    if (rc) return rc;
    p.clip = clip ? 1 : 0;
  }
  p.total = lay.total;
  p.sumsq = Lr->sm_sumsq;
  p.sync = Lr->sm_sync;
  p.err = Lr->err;
  p.wait_ns = wait_ns;
  p.withhold = withhold;
  Lr->last_small = true;
  return small_step_launch(p, G, kSmallMaxSmem, s);
}

// Forward, loss and backward (gradients and statistics into st->grads). When `applied` is
// given and the batch takes the one-launch small step, that launch also applies the
// optimiser and *applied is set.
int learner_backward(spo_learner* Lr, cudaStream_t s, const spo_batch* b, float scale,
                     const spo_train_state* st, bool* applied = nullptr) {
  if (applied) *applied = false;
  SPO_CHECK_ARG(b != nullptr && st != nullptr && st->params && st->grads, kErrArg, "null argument");
  SPO_CHECK_ARG(b->rows >= 0 && b->rows <= Lr->desc.max_rows, kErrShape,
                "batch rows " + std::to_string(b->rows) + " exceed the learner's max_rows " +
                    std::to_string(Lr->desc.max_rows));
  SPO_CHECK_ARG(b->rows == 0 || b->obs != nullptr || b->cells != nullptr, kErrArg,
                "batch.obs (or batch.cells) is null");
  if (Lr->net[0].present) {
    SPO_CHECK_ARG(b->rows == 0 || (b->q && (b->mask || (!b->obs && b->cells))), kErrArg,
                  "actor needs batch.q and batch.mask (or batch.cells)");
    SPO_CHECK_ARG(b->rows == 0 || !Lr->desc.use_kl || b->logits_old, kErrArg,
                  "use_kl needs batch.logits_old");
  }
  if (Lr->net[1].present)
    SPO_CHECK_ARG(b->rows == 0 || b->target, kErrArg, "critic needs batch.target");
  SPO_CHECK_ARG(aligned16(st->params) && aligned16(st->grads), kErrAlign,
                "params/grads must be 16-byte aligned");
  if (b->rows >= 1 && b->rows <= Lr->small_rows && (b->obs || (b->cells && (Lr->net[0].present ? Lr->net[0].d.dims[0] : Lr->net[1].d.dims[0]) == 27))) {
    int rc = small_step(Lr, s, b, scale, st, applied != nullptr);
    if (rc == kOk && applied) *applied = true;
    return rc;
  }
  Lr->last_small = false;
  ReduceParams red{};
  const float* stats_src[2] = {nullptr, nullptr};
  int stats_parts[2] = {0, 0};
  const spo_learner_layout& lay = Lr->layout;
  for (int i = 0; i < 2; ++i) {
    if (!Lr->net[i].present) continue;
    const int64_t off = Lr->net[i].offset;
    int rc = net_backward(Lr, i, s, st->params + off, st->params + lay.alpha_index, *b, scale,
                          st->grads + off, red, &stats_src[i], &stats_parts[i]);
    if (rc) return rc;
  }
  add_stats_segs(red, Lr, st->grads, stats_src, stats_parts);
  if (red.nseg > kMaxSegs) return set_error(kErrUnsupported, "too many reduction segments");
  return reduce_launch(red, s);
}

}  // namespace
}  // namespace spo

using namespace spo;

#define SPO_ENTRY(body)                                                   \
  do {                                                                    \
    try {                                                                 \
      body                                                                \
    } catch (const std::exception& e) {                                   \
      return set_error(kErrArg, std::string("exception: ") + e.what());   \
    } catch (...) {                                                       \
      return set_error(kErrArg, "unknown exception");                     \
    }                                                                     \
  } while (0)

static inline cudaStream_t S(spo_stream_t s) { return reinterpret_cast<cudaStream_t>(s); }

extern "C" {

int32_t spo_abi_version(void) { return SPO_ABI_VERSION; }

const char* spo_last_error_string(void) { return g_last_error.c_str(); }

// ---------------------------------------------------------------- Linear
int spo_linear_fwd(spo_stream_t stream, float* y, const float* x, const float* w, const float* b,
                   int64_t m, int64_t k, int64_t n, int32_t act) {
  SPO_CHECK_ARG(m >= 0 && k >= 1 && n >= 1, kErrShape, "bad shape");
  SPO_CHECK_ARG(m == 0 || (y && x && w && b), kErrArg, "null pointer");
  SPO_CHECK_ARG(act == SPO_ACT_NONE || act == SPO_ACT_RELU, kErrArg, "bad activation");
  return gemm_fwd(S(stream), y, x, w, b, m, k, n, act == SPO_ACT_RELU);
}

size_t spo_linear_bwd_workspace_size(int64_t /*m: the bound holds for any row count*/, int64_t k,
                                      int64_t n) {
  Carve c(nullptr);
  c.take<float>((size_t)(dw_parts_bound(k, n) * k * n));
  c.take<float>((size_t)(kColsumChunks * n));
  return c.off + 256;
}

int spo_linear_bwd(spo_stream_t stream, float* dw, float* db, float* dx, const float* x,
                   const float* w, const float* dy, const float* relu_src, int64_t m, int64_t k,
                   int64_t n, void* workspace, size_t workspace_bytes) {
  SPO_CHECK_ARG(m >= 0 && k >= 1 && n >= 1, kErrShape, "bad shape");
  SPO_CHECK_ARG(dw && db && (m == 0 || (x && dy)) && (!dx || w), kErrArg, "null pointer");
  SPO_CHECK_ARG(workspace && workspace_bytes >= spo_linear_bwd_workspace_size(m, k, n),
                kErrWorkspace, "workspace too small");
  Carve c(workspace);
  float* part = c.take<float>((size_t)(dw_parts_bound(k, n) * k * n));
  float* cs = c.take<float>((size_t)(kColsumChunks * n));
  cudaStream_t s = S(stream);
  int parts = 0;
  int rc = gemm_dw(s, part, x, dy, m, k, n, &parts);
  if (rc) return rc;
  ReduceParams red{};
  add_seg(red, part, dw, k * n, k * n, parts);
  rc = reduce_launch(red, s);
  if (rc) return rc;
  rc = colsum(s, db, dy, m, n, cs);
  if (rc) return rc;
  if (dx) return gemm_dx(s, dx, dy, w, relu_src, m, k, n, nullptr, nullptr);
  return kOk;
}

int spo_relu(spo_stream_t stream, float* a, int64_t n) {
  SPO_CHECK_ARG(n >= 0 && (n == 0 || a), kErrArg, "bad argument");
  return relu_launch(a, n, S(stream));
}

int spo_relu_bwd(spo_stream_t stream, float* grad, const float* act, int64_t n) {
  SPO_CHECK_ARG(n >= 0 && (n == 0 || (grad && act)), kErrArg, "bad argument");
  return relu_bwd_launch(grad, act, n, S(stream));
}

// ---------------------------------------------------------------- MLP
int spo_mlp_param_layout(const spo_mlp_desc* desc, int64_t* w_off, int64_t* b_off, int64_t* total) {
  SPO_CHECK_ARG(desc_ok(desc), kErrShape, "bad MLP descriptor");
  SPO_CHECK_ARG(w_off && b_off && total, kErrArg, "null output");
  mlp_layout(*desc, w_off, b_off, total);
  return kOk;
}

int64_t spo_mlp_acts_size(const spo_mlp_desc* desc, int64_t m) {
  if (!desc_ok(desc) || m < 0) return -1;
  int64_t t = 0;
  for (int l = 0; l + 1 < desc->num_layers; ++l) t += m * desc->dims[l + 1];
  return t;
}

int spo_mlp_fwd(spo_stream_t stream, const spo_mlp_desc* desc, const float* params, const float* x,
                int64_t m, float* acts, float* out) {
  SPO_CHECK_ARG(desc_ok(desc), kErrShape, "bad MLP descriptor");
  SPO_CHECK_ARG(m >= 0, kErrShape, "bad row count");
  SPO_CHECK_ARG(m == 0 || (params && x && out && (desc->num_layers == 1 || acts)), kErrArg,
                "null pointer");
  int64_t w_off[SPO_MAX_LAYERS], b_off[SPO_MAX_LAYERS], total;
  mlp_layout(*desc, w_off, b_off, &total);
  const float* h = x;
  float* a = acts;
  cudaStream_t s = S(stream);
  for (int l = 0; l < desc->num_layers; ++l) {
    const bool last = l + 1 == desc->num_layers;
    float* y = last ? out : a;
    int rc = gemm_fwd(s, y, h, params + w_off[l], params + b_off[l], m, desc->dims[l],
                      desc->dims[l + 1], !last);
    if (rc) return rc;
    if (!last) {
      h = a;
      a += m * desc->dims[l + 1];
    }
  }
  return kOk;
}

size_t spo_mlp_bwd_workspace_size(const spo_mlp_desc* desc, int64_t m) {
  if (!desc_ok(desc) || m < 0) return 0;
  Carve c(nullptr);
  int64_t mh = 1;
  for (int l = 1; l < desc->num_layers; ++l) mh = std::max<int64_t>(mh, desc->dims[l]);
  c.take<float>((size_t)(2 * m * mh));
  for (int l = 0; l < desc->num_layers; ++l) {
    c.take<float>((size_t)(dw_parts_bound(desc->dims[l], desc->dims[l + 1]) * desc->dims[l] *
                           desc->dims[l + 1]));
    c.take<float>((size_t)(std::max(fwd_parts_bound(desc->dims[l + 1]), kColsumChunks) *
                           desc->dims[l + 1]));
  }
  return c.off + 256;
}

int spo_mlp_bwd(spo_stream_t stream, const spo_mlp_desc* desc, const float* params, const float* x,
                const float* acts, const float* dout, int64_t m, float* grads, void* workspace,
                size_t workspace_bytes) {
  SPO_CHECK_ARG(desc_ok(desc), kErrShape, "bad MLP descriptor");
  SPO_CHECK_ARG(m >= 0, kErrShape, "bad row count");
  SPO_CHECK_ARG(grads && params && (m == 0 || (x && dout && (desc->num_layers == 1 || acts))),
                kErrArg, "null pointer");
  SPO_CHECK_ARG(workspace && workspace_bytes >= spo_mlp_bwd_workspace_size(desc, m), kErrWorkspace,
                "workspace too small");
  const int L = desc->num_layers;
  int64_t w_off[SPO_MAX_LAYERS], b_off[SPO_MAX_LAYERS], total;
  mlp_layout(*desc, w_off, b_off, &total);
  const float* act[SPO_MAX_LAYERS];
  {
    const float* a = acts;
    for (int l = 0; l + 1 < L; ++l) {
      act[l] = a;
      a += m * desc->dims[l + 1];
    }
  }
  Carve c(workspace);
  int64_t mh = 1;
  for (int l = 1; l < L; ++l) mh = std::max<int64_t>(mh, desc->dims[l]);
  float* dzb = c.take<float>((size_t)(2 * m * mh));
  float* dz[2] = {dzb, dzb + m * mh};
  float* dwp[SPO_MAX_LAYERS];
  float* dbp[SPO_MAX_LAYERS];
  for (int l = 0; l < L; ++l) {
    dwp[l] = c.take<float>((size_t)(dw_parts_bound(desc->dims[l], desc->dims[l + 1]) * desc->dims[l] *
                                    desc->dims[l + 1]));
    dbp[l] = c.take<float>((size_t)(std::max(fwd_parts_bound(desc->dims[l + 1]), kColsumChunks) *
                                    desc->dims[l + 1]));
  }
  cudaStream_t s = S(stream);
  ReduceParams red{};
  // db of the top layer: column sums of dout
  int rc = colsum(s, grads + b_off[L - 1], dout, m, desc->dims[L], dbp[L - 1]);
  if (rc) return rc;
  const float* cur = dout;
  int pp = 0;
  for (int l = L - 1; l >= 0; --l) {
    const float* in = l == 0 ? x : act[l - 1];
    int parts = 0;
    rc = gemm_dw(s, dwp[l], in, cur, m, desc->dims[l], desc->dims[l + 1], &parts);
    if (rc) return rc;
    add_seg(red, dwp[l], grads + w_off[l], (int64_t)desc->dims[l] * desc->dims[l + 1],
            (int64_t)desc->dims[l] * desc->dims[l + 1], parts);
    if (l >= 1) {
      int cparts = 0;
      rc = gemm_dx(s, dz[pp], cur, params + w_off[l], act[l - 1], m, desc->dims[l], desc->dims[l + 1],
                   dbp[l - 1], &cparts);
      if (rc) return rc;
      add_seg(red, dbp[l - 1], grads + b_off[l - 1], desc->dims[l], desc->dims[l], m > 0 ? cparts : 0);
      cur = dz[pp];
      pp ^= 1;
    }
  }
  add_gap_segs(red, *desc, w_off, b_off, total, grads);
  return reduce_launch(red, s);
}

// ---------------------------------------------------------------- softmax / actor / losses
int spo_mask_logits(spo_stream_t stream, float* logits, const float* mask, int64_t n) {
  SPO_CHECK_ARG(n >= 0 && (n == 0 || (logits && mask)), kErrArg, "bad argument");
  return mask_logits_launch(logits, mask, n, S(stream));
}

int spo_softmax_rows(spo_stream_t stream, float* out, const float* in, int64_t rows, int32_t cols) {
  SPO_CHECK_ARG(rows >= 0 && cols >= 1 && (rows == 0 || (out && in)), kErrArg, "bad argument");
  return softmax_rows_launch(out, in, rows, cols, 0, S(stream));
}

int spo_log_softmax_rows(spo_stream_t stream, float* out, const float* in, int64_t rows,
                         int32_t cols) {
  SPO_CHECK_ARG(rows >= 0 && cols >= 1 && (rows == 0 || (out && in)), kErrArg, "bad argument");
  return softmax_rows_launch(out, in, rows, cols, 1, S(stream));
}

int spo_logsumexp_rows(spo_stream_t stream, float* out, const float* in, int64_t rows, int32_t cols) {
  SPO_CHECK_ARG(rows >= 0 && cols >= 1 && (rows == 0 || (out && in)), kErrArg, "bad argument");
  return softmax_rows_launch(out, in, rows, cols, 2, S(stream));
}

int spo_cross_entropy_rows(spo_stream_t stream, float* loss, const float* q, const float* log_pi,
                           int64_t rows, int32_t cols) {
  SPO_CHECK_ARG(rows >= 0 && cols >= 1 && (rows == 0 || (loss && q && log_pi)), kErrArg, "bad argument");
  return ce_rows_launch(loss, q, log_pi, rows, cols, S(stream));
}

int spo_entropy_rows(spo_stream_t stream, float* h, const float* q, int64_t rows, int32_t cols) {
  SPO_CHECK_ARG(rows >= 0 && cols >= 1 && (rows == 0 || (h && q)), kErrArg, "bad argument");
  return entropy_rows_launch(h, q, rows, cols, S(stream));
}

int spo_kl_rows(spo_stream_t stream, float* kl, const float* ce, const float* h, int64_t rows) {
  SPO_CHECK_ARG(rows >= 0 && (rows == 0 || (kl && ce && h)), kErrArg, "bad argument");
  return kl_rows_launch(kl, ce, h, rows, S(stream));
}

int spo_logits_grad(spo_stream_t stream, float* dz, const float* pi, const float* q,
                    const float* mask, int64_t n, float scale) {
  SPO_CHECK_ARG(n >= 0 && (n == 0 || (dz && pi && q)), kErrArg, "bad argument");
  return logits_grad_launch(dz, pi, q, mask, n, scale, S(stream));
}

int spo_value_loss_grad(spo_stream_t stream, float* dv, const float* v, const float* target,
                        int64_t n, float scale) {
  SPO_CHECK_ARG(n >= 0 && (n == 0 || (dv && v && target)), kErrArg, "bad argument");
  return value_grad_launch(dv, v, target, n, scale, S(stream));
}

size_t spo_head_workspace_size(int64_t m, int32_t h, int32_t a) {
  if (m < 0 || h < 1 || a < 1) return 0;
  Carve c(nullptr);
  const int64_t g = head_parts_bound();
  c.take<float>((size_t)(g * h * a));
  c.take<float>((size_t)(g * a));
  c.take<float>((size_t)(g * h));
  c.take<float>((size_t)(g * kStats));
  return c.off + 256;
}

static int head_common(cudaStream_t s, HeadParams hp, float* dw, float* db, float* dbact,
                       float* stats, void* workspace, size_t workspace_bytes) {
  SPO_CHECK_ARG(dw && db && stats, kErrArg, "dw, db and stats are required");
  SPO_CHECK_ARG(hp.M >= 0, kErrShape, "bad row count");
  SPO_CHECK_ARG(hp.M == 0 || (hp.act && hp.W && hp.b), kErrArg, "null pointer");
  SPO_CHECK_ARG(workspace && workspace_bytes >= spo_head_workspace_size(hp.M, hp.H, hp.A),
                kErrWorkspace, "workspace too small");
  Carve c(workspace);
  const int64_t g = head_parts_bound();
  hp.dW_part = c.take<float>((size_t)(g * hp.H * hp.A));
  hp.db_part = c.take<float>((size_t)(g * hp.A));
  hp.dbx_part = c.take<float>((size_t)(g * hp.H));
  hp.stats_part = c.take<float>((size_t)(g * kStats));
  const int grid = head_grid(hp);
  const int parts = hp.M > 0 ? grid : 0;
  if (hp.M > 0) {
    int rc = head_launch(hp, grid, s);
    if (rc) return rc;
  } else {
    SPO_CHECK_ARG(hp.H % 4 == 0 && hp.H <= 1024 && (hp.A == 1 || hp.A == 9), kErrUnsupported,
                  "head: unsupported shape");
  }
  ReduceParams red{};
  add_seg(red, hp.dW_part, dw, (int64_t)hp.H * hp.A, (int64_t)hp.H * hp.A, parts);
  add_seg(red, hp.db_part, db, hp.A, hp.A, parts);
  if (dbact) add_seg(red, hp.dbx_part, dbact, hp.H, hp.H, parts);
  add_seg(red, hp.stats_part, stats, kStats, kStats, parts);
  return reduce_launch(red, s);
}

int spo_actor_head_fwd_bwd(spo_stream_t stream, const float* act, const float* w, const float* b,
                           int64_t m, int32_t h, int32_t a, const float* mask, const float* q,
                           const float* logits_old, const float* log_alpha, float scale,
                           float* logits_out, float* pi_out, float* dz_out, float* dact, float* dw,
                           float* db, float* dbact, float* stats, void* workspace,
                           size_t workspace_bytes) {
  SPO_CHECK_ARG(m == 0 || q, kErrArg, "q is required");
  SPO_CHECK_ARG(!logits_old || log_alpha, kErrArg, "logits_old needs log_alpha");
  HeadParams hp{};
  hp.act = act; hp.W = w; hp.b = b; hp.M = m; hp.H = h; hp.A = a;
  hp.mode = kHeadActor;
  hp.mask = mask; hp.q = q; hp.z_old = logits_old; hp.log_alpha = logits_old ? log_alpha : nullptr;
  hp.scale = scale;
  hp.out_logits = logits_out; hp.out_pi = pi_out; hp.dz_out = dz_out; hp.dX = dact;
  return head_common(S(stream), hp, dw, db, dbact, stats, workspace, workspace_bytes);
}

int spo_critic_head_fwd_bwd(spo_stream_t stream, const float* act, const float* w, const float* b,
                            int64_t m, int32_t h, const float* target, float scale, float* v_out,
                            float* dv_out, float* dact, float* dw, float* db, float* dbact,
                            float* stats, void* workspace, size_t workspace_bytes) {
  SPO_CHECK_ARG(m == 0 || target, kErrArg, "target is required");
  HeadParams hp{};
  hp.act = act; hp.W = w; hp.b = b; hp.M = m; hp.H = h; hp.A = 1;
  hp.mode = kHeadCritic;
  hp.target = target;
  hp.scale = scale;
  hp.out_logits = v_out; hp.dz_out = dv_out; hp.dX = dact;
  return head_common(S(stream), hp, dw, db, dbact, stats, workspace, workspace_bytes);
}

size_t spo_loss_workspace_size(void) { return sizeof(float) * (size_t)(loss_parts_max() * kStats) + 256; }

int spo_actor_loss_fwd_bwd(spo_stream_t stream, const float* logits, const float* mask, const float* q,
                           const float* logits_old, const float* log_alpha, float eps_kl, int64_t rows,
                           int32_t a, float scale, float* dz, float* loss_stats, float* dlog_alpha,
                           void* workspace, size_t workspace_bytes) {
  SPO_CHECK_ARG(rows >= 0 && a >= 1 && a <= 32, kErrShape, "rows >= 0 and 1 <= a <= 32 required");
  SPO_CHECK_ARG(loss_stats != nullptr, kErrArg, "loss_stats is required");
  SPO_CHECK_ARG(rows == 0 || (logits && q && dz), kErrArg, "logits, q and dz are required");
  SPO_CHECK_ARG(!logits_old || log_alpha, kErrArg, "logits_old needs log_alpha");
  SPO_CHECK_ARG(workspace && workspace_bytes >= spo_loss_workspace_size(), kErrWorkspace,
                "workspace too small");
  return actor_loss_launch(logits, mask, q, logits_old, log_alpha, eps_kl, rows, a, scale, dz, loss_stats,
                           dlog_alpha, static_cast<float*>(workspace), S(stream));
}

int spo_value_loss_fwd_bwd(spo_stream_t stream, const float* v, const float* target, int64_t n, float scale,
                           float* dv, float* loss_stats, void* workspace, size_t workspace_bytes) {
  SPO_CHECK_ARG(n >= 0, kErrShape, "n >= 0 required");
  SPO_CHECK_ARG(loss_stats != nullptr, kErrArg, "loss_stats is required");
  SPO_CHECK_ARG(n == 0 || (v && target && dv), kErrArg, "v, target and dv are required");
  SPO_CHECK_ARG(workspace && workspace_bytes >= spo_loss_workspace_size(), kErrWorkspace,
                "workspace too small");
  return value_loss_launch(v, target, n, scale, dv, loss_stats, static_cast<float*>(workspace), S(stream));
}

// ---------------------------------------------------------------- optimiser
size_t spo_sum_squares_workspace_size(void) { return sizeof(float) * kSumsqParts + 256; }

int spo_sum_squares(spo_stream_t stream, const float* x, int64_t n, float* out, void* workspace,
                    size_t workspace_bytes) {
  SPO_CHECK_ARG(n >= 0 && out && (n == 0 || x), kErrArg, "bad argument");
  SPO_CHECK_ARG(workspace && workspace_bytes >= spo_sum_squares_workspace_size(), kErrWorkspace,
                "workspace too small");
  return sumsq_launch(x, n, static_cast<float*>(workspace), out, S(stream));
}

float spo_global_clip_scale(float total_sq, float max_norm) {
  const float norm = std::sqrt(total_sq);
  if (!(max_norm > 0.f) || !std::isfinite(max_norm) || norm <= max_norm) return 1.f;
  return max_norm / norm;
}

int spo_adam_flat(spo_stream_t stream, float* p, const float* g, float* m, float* v, int64_t n,
                  float lr, float b1, float b2, float eps, int32_t step, float grad_scale) {
  SPO_CHECK_ARG(n >= 0 && (n == 0 || (p && g && m && v)), kErrArg, "bad argument");
  SPO_CHECK_ARG(step >= 1, kErrArg, "step starts at 1");
  if (n == 0) return kOk;
  AdamParams ap{};
  ap.p = p; ap.g = const_cast<float*>(g); ap.m = m; ap.v = v;
  ap.grp[0] = AdamGroup{0, n, lr, 0.f};
  ap.ngrp = 1;
  ap.b1 = b1; ap.b2 = b2; ap.eps = eps;
  ap.grad_scale = grad_scale;
  ap.host_step = step;
  ap.alpha_index = -1;
  return adam_launch(ap, n, S(stream));
}

int spo_ema(spo_stream_t stream, float* target, const float* online, int64_t n, float tau) {
  SPO_CHECK_ARG(n >= 0 && (n == 0 || (target && online)), kErrArg, "bad argument");
  return ema_launch(target, online, n, tau, S(stream));
}

int spo_truncated_gae(spo_stream_t stream, float* adv, float* targets, const float* reward,
                      const float* discount, const float* v_tm1, const float* v_t,
                      const float* truncation, int64_t batch, int32_t t_len, float lambda) {
  SPO_CHECK_ARG(batch >= 0 && t_len >= 1, kErrShape, "bad shape");
  SPO_CHECK_ARG(batch == 0 || (adv && targets && reward && discount && v_tm1 && v_t && truncation),
                kErrArg, "null pointer");
  return gae_launch(adv, targets, reward, discount, v_tm1, v_t, truncation, batch, t_len, lambda,
                    S(stream));
}

int spo_measure_peaks(spo_stream_t stream, double* tf32_flops, double* fp32_flops) {
  SPO_CHECK_ARG(tf32_flops && fp32_flops, kErrArg, "null output");
  return measure_peaks(tf32_flops, fp32_flops, S(stream));
}

int spo_replay_sample(spo_stream_t stream, int32_t* idx, int64_t n, int64_t count, uint32_t seed,
                      uint32_t stream_id) {
  return replay_sample_launch(idx, n, count, seed, stream_id, S(stream));
}

int spo_replay_gather(spo_stream_t stream, float* dst, const float* src, const int32_t* idx, int64_t n,
                      int64_t span, int64_t count, int32_t* err) {
  return replay_gather_launch(dst, src, idx, n, span, count, err, S(stream));
}

int spo_encode_obs(spo_stream_t stream, float* obs, float* mask, const float* cells, int64_t n) {
  return encode_obs_launch(obs, mask, cells, n, S(stream));
}

// ---------------------------------------------------------------- learner
int spo_learner_layout_of(const spo_learner_desc* desc, spo_learner_layout* out) {
  SPO_CHECK_ARG(out != nullptr, kErrArg, "null output");
  spo_learner tmp{};
  size_t bytes = 0;
  int rc = build_plan(desc, &tmp, nullptr, &bytes);
  if (rc) return rc;
  *out = tmp.layout;
  return kOk;
}

size_t spo_learner_workspace_size(const spo_learner_desc* desc) {
  spo_learner tmp{};
  size_t bytes = 0;
  if (build_plan(desc, &tmp, nullptr, &bytes)) return 0;
  return bytes;
}

int spo_learner_create(const spo_learner_desc* desc, void* workspace, size_t workspace_bytes,
                       spo_learner_t* out) {
  SPO_CHECK_ARG(out && workspace, kErrArg, "null argument");
  SPO_CHECK_ARG(aligned16(workspace), kErrAlign, "workspace must be 16-byte aligned");
  SPO_ENTRY({
    spo_learner* L = new spo_learner{};
    size_t need = 0;
    int rc = build_plan(desc, L, nullptr, &need);
    if (rc == kOk && workspace_bytes < need)
      rc = set_error(kErrWorkspace, "learner workspace too small: need " + std::to_string(need) +
                                        " bytes");
    if (rc == kOk) rc = build_plan(desc, L, workspace, &need);
    if (rc == kOk) {
      L->ws_bytes = need;
      cudaError_t e = cudaMemset(L->ticket, 0, 4 * sizeof(unsigned));
      if (e == cudaSuccess) e = cudaMemset(L->err, 0, 4 * sizeof(int));
      if (e == cudaSuccess) e = cudaMemset(L->sm_sync, 0, 4 * sizeof(unsigned));
      if (e != cudaSuccess) rc = set_error(kErrCuda, std::string("memset: ") + cudaGetErrorString(e));
    }
    if (rc != kOk) {
      delete L;
      return rc;
    }
    *out = L;
    return kOk;
  });
}

int spo_learner_destroy(spo_learner_t learner) {
  delete learner;
  return kOk;
}

int spo_learner_backward(spo_learner_t learner, spo_stream_t stream, const spo_batch* batch,
                         float grad_scale, const spo_train_state* state) {
  SPO_CHECK_ARG(learner != nullptr, kErrArg, "null learner");
  return learner_backward(learner, S(stream), batch, grad_scale, state);
}

int spo_learner_apply(spo_learner_t learner, spo_stream_t stream, const spo_train_state* state) {
  SPO_CHECK_ARG(learner != nullptr, kErrArg, "null learner");
  return learner_apply(learner, S(stream), state);
}

int spo_learner_cache(spo_learner_t learner, int32_t which, int32_t layer, const float** hi,
                      const float** lo) {
  SPO_CHECK_ARG(learner && hi && lo, kErrArg, "null argument");
  SPO_CHECK_ARG((which == 0 || which == 1) && learner->net[which].present, kErrArg,
                "no such network");
  const NetPlan& n = learner->net[which];
  SPO_CHECK_ARG(layer >= 0 && layer + 1 < n.d.num_layers, kErrArg, "no such hidden layer");
  *hi = n.acts[layer];
  *lo = n.tc && !learner->last_small ? n.acts_lo[layer] : nullptr;
  return kOk;
}

int spo_learner_status(spo_learner_t learner, int32_t* device_error) {
  SPO_CHECK_ARG(learner && device_error, kErrArg, "null argument");
  int v = 0;
  SPO_CUDA_TRY(cudaMemcpy(&v, learner->err, sizeof(int), cudaMemcpyDeviceToHost));
  if (v != 0) SPO_CUDA_TRY(cudaMemset(learner->err, 0, sizeof(int)));
  *device_error = v;
  return kOk;
}

int spo_learner_step(spo_learner_t learner, spo_stream_t stream, const spo_batch* batch,
                     const spo_train_state* state) {
  SPO_CHECK_ARG(learner && batch, kErrArg, "null argument");
  const float scale = batch->rows > 0 ? 1.f / (float)batch->rows : 0.f;
  bool applied = false;
  int rc = learner_backward(learner, S(stream), batch, scale, state, &applied);
  if (rc || applied) return rc;
  return learner_apply(learner, S(stream), state);
}

int spo_learner_set_small_rows(spo_learner_t learner, int64_t max_rows) {
  SPO_CHECK_ARG(learner != nullptr, kErrArg, "null learner");
  SPO_CHECK_ARG(max_rows >= 0, kErrShape, "max_rows must be >= 0");
  bool fits = true;
  for (int i = 0; i < 2; ++i)
    if (learner->net[i].present) fits = fits && learner->net[i].small;
  SPO_CHECK_ARG(max_rows == 0 || fits, kErrUnsupported,
                "the one-launch step needs 2-4 layers, input <= 32, hidden widths multiples of 32 up to 256");
  learner->small_rows = std::min<int64_t>(max_rows, learner->desc.max_rows);
  return kOk;
}

int spo_learner_step_withheld(spo_learner_t learner, spo_stream_t stream, const spo_batch* batch,
                              const spo_train_state* state, int64_t wait_us) {
  SPO_CHECK_ARG(learner && batch && state && state->params && state->grads, kErrArg, "null argument");
  SPO_CHECK_ARG(wait_us >= 1 && wait_us <= 2000000, kErrArg, "wait_us must be in [1, 2000000]");
  SPO_CHECK_ARG(learner->err != nullptr, kErrArg, "learner has no error word");
  SPO_CHECK_ARG(batch->rows >= 1 && batch->rows <= learner->small_rows, kErrUnsupported,
                "spo_learner_step_withheld: the batch does not take the one-launch step");
  SPO_CHECK_ARG(aligned16(state->params) && aligned16(state->grads), kErrAlign,
                "params and grads must be 16-byte aligned");
  const float scale = 1.0f / (float)batch->rows;
  return small_step(learner, S(stream), batch, scale, state, true, (uint64_t)wait_us * 1000u, 1u);
}

int spo_learner_forward(spo_learner_t learner, spo_stream_t stream, int32_t which,
                        const float* params, const float* obs, const float* mask, int64_t rows,
                        float* out, float* pi_out) {
  SPO_CHECK_ARG(learner && params && (rows == 0 || (obs && out)), kErrArg, "null argument");
  SPO_CHECK_ARG(which == 0 || which == 1, kErrArg, "which must be 0 (actor) or 1 (critic)");
  SPO_CHECK_ARG(learner->net[which].present, kErrArg, "that network is not part of the learner");
  SPO_CHECK_ARG(rows >= 0 && rows <= learner->desc.max_rows, kErrShape, "rows exceed max_rows");
  const NetPlan& n = learner->net[which];
  const float* p = params + n.offset;
  cudaStream_t s = S(stream);
  int rc = net_forward_hidden(n, s, p, LayerInput{obs, nullptr}, rows, learner->err);
  if (rc) return rc;
  const int L = n.d.num_layers;
  if (n.tc && n.acts_lo[L - 2]) {  // the last layer reads plain fp32: fold lo into hi
    rc = combine_tf32_launch(n.acts[L - 2], n.acts_lo[L - 2], rows * n.d.dims[L - 1], s);
    if (rc) return rc;
  }
  rc = gemm_fwd(s, out, n.acts[L - 2], p + n.w_off[L - 1], p + n.b_off[L - 1], rows, n.d.dims[L - 1],
                n.d.dims[L], false);
  if (rc) return rc;
  if (which == 0 && mask) {
    rc = mask_logits_launch(out, mask, rows * n.d.dims[L], s);
    if (rc) return rc;
  }
  if (which == 0 && pi_out) return softmax_rows_launch(pi_out, out, rows, n.d.dims[L], 0, s);
  return kOk;
}

// ---------------------------------------------------------------- data parallel (NCCL)
struct spo_comm {
  ncclComm_t comm;
};

int spo_comm_get_unique_id(void* id_out) {
  SPO_CHECK_ARG(id_out != nullptr, kErrArg, "null output");
  static_assert(sizeof(ncclUniqueId) == SPO_COMM_ID_BYTES, "unique id size");
  ncclUniqueId id;
  ncclResult_t r = ncclGetUniqueId(&id);
  if (r != ncclSuccess) return set_error(kErrNccl, std::string("ncclGetUniqueId: ") + ncclGetErrorString(r));
  std::memcpy(id_out, &id, sizeof(id));
  return kOk;
}

// Non-blocking init polled against a deadline, so a rank that never joins ends in an
// error status (after ncclCommAbort) instead of a hang.
int spo_comm_init(spo_comm_t* out, const void* id, int32_t nranks, int32_t rank) {
  SPO_CHECK_ARG(out && id, kErrArg, "null argument");
  SPO_CHECK_ARG(nranks >= 1 && rank >= 0 && rank < nranks, kErrArg, "bad rank");
  ncclUniqueId uid;
  std::memcpy(&uid, id, sizeof(uid));
  ncclConfig_t cfg = NCCL_CONFIG_INITIALIZER;
  cfg.blocking = 0;
  ncclComm_t comm = nullptr;
  ncclResult_t r = ncclCommInitRankConfig(&comm, nranks, uid, rank, &cfg);
  const char* env = std::getenv("SPO_COMM_TIMEOUT_MS");
  const long timeout_ms = env ? std::atol(env) : 120000;
  const auto t0 = std::chrono::steady_clock::now();
  while (r == ncclInProgress || r == ncclSuccess) {
    ncclResult_t st = ncclInProgress;
    if (comm) ncclCommGetAsyncError(comm, &st);
    if (st == ncclSuccess) break;
    if (st != ncclInProgress) { r = st; break; }
    const long el = (long)std::chrono::duration_cast<std::chrono::milliseconds>(
                        std::chrono::steady_clock::now() - t0).count();
    if (el > timeout_ms) {
      if (comm) ncclCommAbort(comm);
      return set_error(kErrTimeout, "spo_comm_init: peers did not join within " +
                                        std::to_string(timeout_ms) + " ms");
    }
    std::this_thread::sleep_for(std::chrono::milliseconds(1));
  }
  if (r != ncclSuccess && r != ncclInProgress) {
    if (comm) ncclCommAbort(comm);
    return set_error(kErrNccl, std::string("ncclCommInitRankConfig: ") + ncclGetErrorString(r));
  }
  *out = new spo_comm{comm};
  return kOk;
}

int spo_comm_destroy(spo_comm_t comm) {
  if (!comm) return kOk;
  ncclCommDestroy(comm->comm);
  delete comm;
  return kOk;
}

int spo_allreduce_sum(spo_comm_t comm, spo_stream_t stream, float* buf, int64_t n) {
  SPO_CHECK_ARG(comm && (n == 0 || buf), kErrArg, "bad argument");
  ncclResult_t r = ncclAllReduce(buf, buf, (size_t)n, ncclFloat32, ncclSum, comm->comm, S(stream));
  if (r == ncclInProgress) {
    const auto t0 = std::chrono::steady_clock::now();
    do {
      ncclCommGetAsyncError(comm->comm, &r);
      if (std::chrono::steady_clock::now() - t0 > std::chrono::seconds(120)) {
        ncclCommAbort(comm->comm);
        return set_error(kErrTimeout, "spo_allreduce_sum: enqueue did not complete");
      }
    } while (r == ncclInProgress);
  }
  if (r != ncclSuccess) return set_error(kErrNccl, std::string("ncclAllReduce: ") + ncclGetErrorString(r));
  return kOk;
}

}  // extern "C"

// ---------------------------------------------------------------- tensor-core GEMM

static int tc_args_of(const spo_tc_gemm_desc* d, TcGemmArgs* a) {
  SPO_CHECK_ARG(d != nullptr, kErrArg, "null descriptor");
  SPO_CHECK_ARG(d->kind >= SPO_TC_FWD && d->kind <= SPO_TC_DW, kErrArg, "bad kind");
  *a = TcGemmArgs{};
  a->kind = d->kind;
  a->a_hi = d->a_hi; a->a_lo = d->a_lo; a->b_hi = d->b_hi; a->b_lo = d->b_lo;
  a->M = d->m; a->N = d->n; a->K = d->k; a->k_chunk = d->k_chunk;
  a->bias = d->bias; a->mask = d->mask;
  a->c_hi = d->c_hi; a->c_lo = d->c_lo; a->c_part = d->c_part; a->colsum = d->colsum;
  a->err = d->err;
  a->mask_bits = d->mask_bits; a->c_bits = d->c_bits;
  if (a->kind == TC_DW) {
    SPO_CHECK_ARG(a->k_chunk >= 32 && a->k_chunk % 32 == 0, kErrArg, "k_chunk must be a multiple of 32");
  }
  SPO_CHECK_ARG(tc_gemm_supported(a->kind, a->M, a->N, a->K), kErrUnsupported,
                "tensor-core GEMM: unsupported shape");
  return kOk;
}

extern "C" {

int spo_tc_gemm_shape(const spo_tc_gemm_desc* desc, int32_t* grid, int32_t* splits) {
  TcGemmArgs a;
  int rc = tc_args_of(desc, &a);
  if (rc) return rc;
  if (grid) *grid = tc_gemm_grid(a);
  if (splits) *splits = tc_gemm_splits(a);
  return kOk;
}

int spo_tc_gemm(spo_stream_t stream, const spo_tc_gemm_desc* desc) {
  TcGemmArgs a;
  int rc = tc_args_of(desc, &a);
  if (rc) return rc;
  return tc_gemm_launch(a, S(stream));
}

int spo_tc_gemm_withheld(spo_stream_t stream, const spo_tc_gemm_desc* desc, int64_t wait_us) {
  TcGemmArgs a;
  int rc = tc_args_of(desc, &a);
  if (rc) return rc;
  SPO_CHECK_ARG(a.err != nullptr, kErrArg, "the failure test needs desc->err");
  SPO_CHECK_ARG(wait_us >= 1 && wait_us <= 2000000, kErrArg, "wait_us must be in [1, 2000000]");
  a.wait_ns = (uint64_t)wait_us * 1000u;
  a.withhold = 1;  // the first k-block of every CTA is never loaded
  return tc_gemm_launch(a, S(stream));
}

int spo_split_tf32(spo_stream_t stream, float* hi, float* lo, const float* x, int64_t n,
                   int32_t keep_positive) {
  SPO_CHECK_ARG(n >= 0 && (n == 0 || (hi && lo && x)), kErrArg, "bad argument");
  return split_tf32_launch(x, hi, lo, n, keep_positive != 0, S(stream));
}

}  // extern "C"

// ---------------------------------------------------------------- allocation-free variant
// spo_linear_bwd without a caller workspace, for callers that cannot allocate device
// memory: a host framework that pre-reserves nearly all of the GPU's memory for its own
// pool (JAX does by default) leaves cudaMalloc nothing to give, and some embedders forbid
// allocation outside their arena. Its scratch (split-K partials of dW and the column-sum
// chunks of db) lives in one file-scope device array, resident on every GPU that loads
// this library until the process exits.
namespace {

constexpr int64_t kStaticScratchFloats = 2 * 1024 * 1024;  // 8 MiB per device
static __device__ __align__(256) float g_static_scratch[kStaticScratchFloats];

std::mutex g_static_mu;
float* g_static_ptr[64] = {};

// Device address of g_static_scratch on the current device. The host-side name of the
// array is only a stand-in and must never reach a kernel; the address comes from
// cudaGetSymbolAddress, looked up once per device with that device current.
int static_scratch(float** out) {
  int dev = 0;
  SPO_CUDA_TRY(cudaGetDevice(&dev));
  SPO_CHECK_ARG(dev >= 0 && dev < 64, kErrUnsupported, "device index out of range");
  std::lock_guard<std::mutex> lock(g_static_mu);
  if (g_static_ptr[dev] == nullptr) {
    void* p = nullptr;
    SPO_CUDA_TRY(cudaGetSymbolAddress(&p, g_static_scratch));
    g_static_ptr[dev] = static_cast<float*>(p);
  }
  *out = g_static_ptr[dev];
  return kOk;
}

}  // namespace

extern "C" int spo_linear_bwd_noalloc(spo_stream_t stream, float* dw, float* db, float* dx,
                                      const float* x, const float* w, const float* dy,
                                      const float* relu_src, int64_t m, int64_t k, int64_t n) {
  SPO_CHECK_ARG(m >= 0 && k >= 1 && n >= 1, kErrShape, "bad shape");
  SPO_CHECK_ARG(dw && db && (m == 0 || (x && dy)) && (!dx || w), kErrArg, "null pointer");
  // bound n, then k, before forming k*n, so that no product of caller sizes can wrap
  const bool fits = n <= kStaticScratchFloats / (kColsumChunks + 1) &&
                    k <= (kStaticScratchFloats - kColsumChunks * n) / n;
  SPO_CHECK_ARG(fits, kErrWorkspace,
                "spo_linear_bwd_noalloc: k*n + 256*n exceeds its static scratch of " +
                    std::to_string(kStaticScratchFloats) + " floats (k = " + std::to_string(k) +
                    ", n = " + std::to_string(n) + "); use spo_linear_bwd with a workspace");
  const int64_t cs_floats = kColsumChunks * n;
  float* scratch = nullptr;
  int rc = static_scratch(&scratch);
  if (rc) return rc;
  float* cs = scratch;                 // [kColsumChunks][n]
  float* part = scratch + cs_floats;   // [parts][k x n]
  const int64_t max_parts = (kStaticScratchFloats - cs_floats) / (k * n);
  cudaStream_t s = S(stream);

  // dW: split-K over rows as spo_linear_bwd does, with the split count capped so that the
  // partials fit the static array. Every split writes its whole partial tile, so nothing
  // has to be cleared between calls.
  DwCfg c = dw_cfg(k, n, m);
  int parts = c.parts;
  if (parts > max_parts) {
    c.k_chunk = std::max<int64_t>(16, align_up(ceil_div(m, max_parts), 16));
    parts = (int)ceil_div(m, c.k_chunk);
    c.grid.z = (unsigned)parts;
  }
  if (parts > 0) {
    GemmParams p{};
    p.A = x; p.B = dy; p.C = part;
    p.M = k; p.N = n; p.K = m;
    p.lda = k; p.ldb = n; p.ldc = n;
    p.k_chunk = c.k_chunk;
    p.c_split_stride = k * n;
    rc = gemm_simt_launch(c.tile, OP_COL, OP_ROW, EPI_STORE, p, c.grid, s);
    if (rc) return rc;
  }
  ReduceParams red{};
  add_seg(red, part, dw, k * n, k * n, parts);
  rc = reduce_launch(red, s);
  if (rc) return rc;
  rc = colsum(s, db, dy, m, n, cs);
  if (rc) return rc;
  if (dx) return gemm_dx(s, dx, dy, w, relu_src, m, k, n, nullptr, nullptr);
  return kOk;
}
